from .config import DSALTConfig
from .dsalt_lm import DSALTLMHeadModel

__all__ = ["DSALTConfig", "DSALTLMHeadModel"]
