// INT8-page instantiations of the fused paged decode-attention kernel.
#include "mg_attention_kernel.cuh"

namespace mg {
mg_status launch_decode_i8(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s, int hd) {
    return launch_kv<false>(p, pl, s, hd);
}
}  // namespace mg
