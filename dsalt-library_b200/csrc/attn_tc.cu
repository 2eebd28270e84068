// tcgen05 / TMEM / TMA attention kernels for sm_100a (placeholder until the
// tensor-core kernels land; the dispatcher then uses the SIMT kernels).
#include "common.cuh"

namespace dsalt {
bool tc_supported(const DsaltAttnParams&) { return false; }
cudaError_t tc_attention_stage(int, const DsaltAttnParams&, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace dsalt
