// Bulk-copy decode-attention kernel instantiations: INT4 pages, head_dim 64.
#include "mg_attention_tma_kernel.cuh"

namespace mg {
template mg_status launch_tma<true, 64>(const DecodeParams&, const DecodePlan&, const CUtensorMap&, const CUtensorMap&,
                                       cudaStream_t, bool);
}  // namespace mg
