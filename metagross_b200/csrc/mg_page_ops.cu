// Single-page quantize / dequantize ops and the sanity add: the C-ABI
// counterparts of the reference's csrc/quantize.cu, csrc/quantize_int4.cu,
// csrc/dequantize.cu, csrc/dequantize_int4.cu and csrc/sanity_add.cu.
//
// Unlike the reference (a one-CTA absmax kernel, a device->host copy of the
// absmax, then a second quantize kernel), the new-scale ops are one kernel:
// the CTA reduces the absmax, derives the scale on the device in double and
// quantizes, so nothing synchronises the host.  The scale is left in a device
// word for the caller.
#include "mg_common.cuh"

namespace mg {
namespace {

constexpr int kPageThreads = 1024;

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o,
                           int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        o[i] = a[i] + b[i];
}

// One CTA: absmax over input[0, n), scale, then codes into out[out_base + i].
template <bool INT4>
__global__ void __launch_bounds__(kPageThreads) quantize_new_scale_kernel(const float* __restrict__ in, int64_t n,
                                                                          void* __restrict__ out, int64_t out_base,
                                                                          double* __restrict__ scale_out) {
    __shared__ float red[32];
    float a = 0.0f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) a = fmaxf(a, fabsf(in[i]));
    a = block_max(a, red);
    const double s = n == 0 ? 1e-8 : scale_from_absmax(a, INT4 ? 7.0 : 127.0);
    if (threadIdx.x == 0 && scale_out) *scale_out = s;
    const float sf = static_cast<float>(s);
    if (!INT4) {
        int8_t* o = static_cast<int8_t*>(out) + out_base;
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) o[i] = static_cast<int8_t>(quant_code(in[i], sf, 127.0f));
    } else {
        uint8_t* o = static_cast<uint8_t*>(out) + out_base;
        for (int64_t i = threadIdx.x; i < n / 2; i += blockDim.x) {
            const int q0 = quant_code(in[2 * i], sf, 7.0f);
            const int q1 = quant_code(in[2 * i + 1], sf, 7.0f);
            o[i] = static_cast<uint8_t>((q0 & 0xF) | ((q1 & 0xF) << 4));
        }
    }
}

__global__ void quantize_fixed_kernel(const float* __restrict__ in, int64_t n, int8_t* __restrict__ out, float sf) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = static_cast<int8_t>(quant_code(in[i], sf, 127.0f));
}

__global__ void dequantize_int8_kernel(const int8_t* __restrict__ in, int64_t n, float* __restrict__ out, float sf) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = static_cast<float>(in[i]) * sf;
}

__device__ __forceinline__ int sext4(uint32_t nib) { return static_cast<int>(static_cast<int8_t>(nib << 4)) >> 4; }

__global__ void dequantize_int4_kernel(const uint8_t* __restrict__ in, int64_t nbytes, float* __restrict__ out,
                                       float sf) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nbytes;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t b = in[i];
        out[2 * i] = static_cast<float>(sext4(b & 0xFu)) * sf;
        out[2 * i + 1] = static_cast<float>(sext4((b >> 4) & 0xFu)) * sf;
    }
}

inline unsigned grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return static_cast<unsigned>(g);
}

inline bool finite_positive(double s) { return s > 0.0 && s < 1.0 / 0.0 && s == s; }

}  // namespace
}  // namespace mg

using namespace mg;

extern "C" mg_status mg_add_f32(const float* a, const float* b, float* out, int64_t n, mg_stream_t stream) {
    MG_REQUIRE(n >= 0, "n must be >= 0, got %lld", (long long)n);
    if (n == 0) return MG_OK;
    MG_REQUIRE(a && b && out, "null pointer");
    add_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(a, b, out, n);
    return check_launch("add_kernel");
}

extern "C" mg_status mg_quantize_int8_new_scale(const float* input, int64_t num_tokens, int64_t row, int8_t* page,
                                                int64_t page_tokens, int64_t token_offset, double* scale_out,
                                                mg_stream_t stream) {
    MG_REQUIRE(token_offset >= 0, "token_offset_in_page must be >= 0, got %lld", (long long)token_offset);
    MG_REQUIRE(num_tokens >= 0 && row >= 0, "negative size");
    MG_REQUIRE(token_offset + num_tokens <= page_tokens,
               "write would overflow the page (offset=%lld, num_tokens=%lld, page_size=%lld)",
               (long long)token_offset, (long long)num_tokens, (long long)page_tokens);
    MG_REQUIRE(scale_out != nullptr, "scale_out must be a device pointer");
    const int64_t n = num_tokens * row;
    MG_REQUIRE(n == 0 || (input && page), "null pointer");
    quantize_new_scale_kernel<false><<<1, kPageThreads, 0, as_stream(stream)>>>(input, n, page, token_offset * row,
                                                                                scale_out);
    return check_launch("quantize_new_scale_kernel<int8>");
}

extern "C" mg_status mg_quantize_int8_fixed_scale(const float* input, int64_t num_tokens, int64_t row, int8_t* page,
                                                  int64_t page_tokens, int64_t token_offset, double scale,
                                                  mg_stream_t stream) {
    MG_REQUIRE(finite_positive(scale), "scale must be a positive finite number, got %g", scale);
    MG_REQUIRE(token_offset >= 0, "token_offset_in_page must be >= 0, got %lld", (long long)token_offset);
    MG_REQUIRE(num_tokens >= 0 && row >= 0, "negative size");
    MG_REQUIRE(token_offset + num_tokens <= page_tokens,
               "write would overflow the page (offset=%lld, num_tokens=%lld, page_size=%lld)",
               (long long)token_offset, (long long)num_tokens, (long long)page_tokens);
    const int64_t n = num_tokens * row;
    if (n == 0) return MG_OK;
    MG_REQUIRE(input && page, "null pointer");
    quantize_fixed_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(input, n, page + token_offset * row,
                                                                            static_cast<float>(scale));
    return check_launch("quantize_fixed_kernel");
}

extern "C" mg_status mg_dequantize_int8_page(const int8_t* page, int64_t page_tokens, int64_t row,
                                             int64_t token_offset, int64_t num_tokens, double scale, float* out,
                                             mg_stream_t stream) {
    MG_REQUIRE(token_offset >= 0, "token_offset_in_page must be >= 0, got %lld", (long long)token_offset);
    MG_REQUIRE(num_tokens >= 0, "num_tokens must be >= 0, got %lld", (long long)num_tokens);
    MG_REQUIRE(finite_positive(scale), "scale must be a positive finite number, got %g", scale);
    MG_REQUIRE(token_offset + num_tokens <= page_tokens,
               "read would overflow the page (offset=%lld, num_tokens=%lld, page_size=%lld)",
               (long long)token_offset, (long long)num_tokens, (long long)page_tokens);
    const int64_t n = num_tokens * row;
    if (n == 0) return MG_OK;
    MG_REQUIRE(page && out, "null pointer");
    dequantize_int8_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(page + token_offset * row, n, out,
                                                                             static_cast<float>(scale));
    return check_launch("dequantize_int8_kernel");
}

extern "C" mg_status mg_quantize_int4_new_scale(const float* input, int64_t num_tokens, int64_t num_heads,
                                                int64_t head_dim, uint8_t* packed, int64_t page_tokens,
                                                int64_t token_offset, double* scale_out, mg_stream_t stream) {
    MG_REQUIRE(head_dim > 0, "head_dim must be positive, got %lld", (long long)head_dim);
    MG_REQUIRE(head_dim % 2 == 0, "head_dim must be even for INT4 packing, got %lld", (long long)head_dim);
    MG_REQUIRE(token_offset >= 0, "token_offset_in_page must be >= 0, got %lld", (long long)token_offset);
    MG_REQUIRE(num_tokens >= 0 && num_heads >= 0, "negative size");
    MG_REQUIRE(token_offset + num_tokens <= page_tokens,
               "write would overflow the page (offset=%lld, num_tokens=%lld, page_size=%lld)",
               (long long)token_offset, (long long)num_tokens, (long long)page_tokens);
    MG_REQUIRE(scale_out != nullptr, "scale_out must be a device pointer");
    const int64_t n = num_tokens * num_heads * head_dim;
    MG_REQUIRE(n == 0 || (input && packed), "null pointer");
    const int64_t half_row = num_heads * head_dim / 2;
    quantize_new_scale_kernel<true><<<1, kPageThreads, 0, as_stream(stream)>>>(input, n, packed,
                                                                               token_offset * half_row, scale_out);
    return check_launch("quantize_new_scale_kernel<int4>");
}

extern "C" mg_status mg_dequantize_int4_page(const uint8_t* packed, int64_t page_tokens, int64_t half_row,
                                             int64_t token_offset, int64_t num_tokens, double scale, float* out,
                                             mg_stream_t stream) {
    MG_REQUIRE(token_offset >= 0, "token_offset_in_page must be >= 0, got %lld", (long long)token_offset);
    MG_REQUIRE(num_tokens >= 0, "num_tokens must be >= 0, got %lld", (long long)num_tokens);
    MG_REQUIRE(finite_positive(scale), "scale must be a positive finite number, got %g", scale);
    MG_REQUIRE(token_offset + num_tokens <= page_tokens,
               "read would overflow the page (offset=%lld, num_tokens=%lld, page_size=%lld)",
               (long long)token_offset, (long long)num_tokens, (long long)page_tokens);
    const int64_t nbytes = num_tokens * half_row;
    if (nbytes == 0) return MG_OK;
    MG_REQUIRE(packed && out, "null pointer");
    dequantize_int4_kernel<<<grid_for(nbytes, 256), 256, 0, as_stream(stream)>>>(packed + token_offset * half_row,
                                                                                  nbytes, out,
                                                                                  static_cast<float>(scale));
    return check_launch("dequantize_int4_kernel");
}
