from .dsalt_attention import DSALTAttention
from .dsalt_transformer import DSALTTransformerBlock, SwiGLUFFN

__all__ = ["DSALTAttention", "DSALTTransformerBlock", "SwiGLUFFN"]
