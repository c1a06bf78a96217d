// Bulk-copy decode-attention kernel instantiations: INT8 pages, head_dim 128.
#include "mg_attention_tma_kernel.cuh"

namespace mg {
template mg_status launch_tma<false, 128>(const DecodeParams&, const DecodePlan&, const CUtensorMap&, const CUtensorMap&,
                                       cudaStream_t, bool);
}  // namespace mg
