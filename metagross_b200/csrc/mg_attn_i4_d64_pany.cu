// Decode-attention kernel instantiations: packed-INT4 pages, head_dim 64, any other page size.
#include "mg_attention_kernel.cuh"

namespace mg {
template mg_status launch_p<true, 64, false>(const DecodeParams&, const DecodePlan&, cudaStream_t);
}  // namespace mg
