// Packed-INT4-page instantiations of the fused paged decode-attention kernel.
#include "mg_attention_kernel.cuh"

namespace mg {
mg_status launch_decode_i4(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s, int hd) {
    return launch_kv<true>(p, pl, s, hd);
}
}  // namespace mg
