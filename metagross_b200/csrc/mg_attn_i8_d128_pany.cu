// Decode-attention kernel instantiations: INT8 pages, head_dim 128, any other page size.
#include "mg_attention_kernel.cuh"

namespace mg {
template mg_status launch_p<false, 128, false>(const DecodeParams&, const DecodePlan&, cudaStream_t);
}  // namespace mg
