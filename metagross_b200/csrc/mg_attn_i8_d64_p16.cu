// Decode-attention kernel instantiations: INT8 pages, head_dim 64, page size 16.
#include "mg_attention_kernel.cuh"

namespace mg {
template mg_status launch_p<false, 64, true>(const DecodeParams&, const DecodePlan&, cudaStream_t);
}  // namespace mg
