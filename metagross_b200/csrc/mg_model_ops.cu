// Dense-side helpers of a Llama decode step (fp16): RMSNorm, the rotary
// embedding of q / k with the q|k|v split, and the SwiGLU gate.  Each replaces
// a chain of small torch elementwise kernels in a captured decode step, and
// writes q / k / v contiguous so the append and attention calls take them as
// they are.  Semantics follow the reference model's Hugging Face Llama modules
// (LlamaRMSNorm; rotate-half rotary embedding, metagross/generate_llama.py:20-37;
// SiLU-gated MLP): fp32 math, fp16 storage.
#include "mg_common.cuh"

namespace mg {
namespace {

constexpr int kOpThreads = 256;

__device__ __forceinline__ float block_sum_f(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

// RMSNorm of rows whose cols (a multiple of 8, <= kOpThreads * 8 * NV) fit in
// registers: one pass, 16-byte loads and stores.
template <int NV>
__global__ void __launch_bounds__(kOpThreads) rmsnorm_reg_kernel(const __half* x, const __half* w, __half* y,
                                                                 int cols, float eps) {
    __shared__ float red[32];
    const int64_t r = blockIdx.x;
    uint4 u[NV];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c = (i * kOpThreads + threadIdx.x) * 8;
        u[i] = c < cols ? *reinterpret_cast<const uint4*>(x + r * cols + c) : make_uint4(0u, 0u, 0u, 0u);
        const __half2* h = reinterpret_cast<const __half2*>(&u[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h[j]);
            ss += f.x * f.x + f.y * f.y;
        }
    }
    const float inv = rsqrtf(block_sum_f(ss, red) / static_cast<float>(cols) + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c = (i * kOpThreads + threadIdx.x) * 8;
        if (c >= cols) continue;
        const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
        const __half2* h = reinterpret_cast<const __half2*>(&u[i]);
        const __half2* wh = reinterpret_cast<const __half2*>(&wv);
        uint4 o;
        __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h[j]);
            oh[j] = __hmul2(__floats2half2_rn(f.x * inv, f.y * inv), wh[j]);
        }
        *reinterpret_cast<uint4*>(y + r * cols + c) = o;
    }
}

// y[r] = fp16(x[r] * rsqrt(mean(x[r]^2) + eps)) * w, one CTA per row.
__global__ void __launch_bounds__(kOpThreads) rmsnorm_kernel(const __half* x, const __half* w, __half* y,
                                                             int64_t cols, float eps) {
    __shared__ float red[32];
    const int64_t r = blockIdx.x;
    const __half* xr = x + r * cols;
    float ss = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        const float v = __half2float(xr[c]);
        ss += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    const float inv = rsqrtf(tot / static_cast<float>(cols) + eps);
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
        y[r * cols + c] = __hmul(__float2half(__half2float(xr[c]) * inv), w[c]);
}

// qkv [B, (Hq + 2 Hkv) * D] -> q [B, Hq, D], k [B, Hkv, D] rotated at position
// pos[b] (cos / sin tables [*, D/2]), v [B, Hkv, D] copied.  One thread per
// rotated pair (b, head, j < D/2), then one per v element.
__global__ void __launch_bounds__(kOpThreads) rope_qkv_kernel(const __half* qkv, const int64_t* pos,
                                                              const float* cosb, const float* sinb, __half* q,
                                                              __half* k, __half* v, int B, int Hq, int Hkv, int D) {
    const int half = D / 2;
    const int64_t row = static_cast<int64_t>(Hq + 2 * Hkv) * D;
    const int64_t nrot = static_cast<int64_t>(B) * (Hq + Hkv) * half;
    const int64_t nv = static_cast<int64_t>(B) * Hkv * D;
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i < nrot) {
        const int64_t bh = i / half;
        const int j = static_cast<int>(i - bh * half);
        const int b = static_cast<int>(bh / (Hq + Hkv)), h = static_cast<int>(bh - static_cast<int64_t>(b) * (Hq + Hkv));
        const __half* src = qkv + b * row + static_cast<int64_t>(h) * D;
        const int64_t p = pos[b];
        const float c = cosb[p * half + j], s = sinb[p * half + j];
        const float x1 = __half2float(src[j]), x2 = __half2float(src[j + half]);
        __half* dst = h < Hq ? q + (static_cast<int64_t>(b) * Hq + h) * D : k + (static_cast<int64_t>(b) * Hkv + h - Hq) * D;
        // products rounded separately (no FMA contraction), as mg_kv_append_rope does
        dst[j] = __float2half_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
        dst[j + half] = __float2half_rn(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
    } else if (i < nrot + nv) {
        const int64_t e = i - nrot;
        const int64_t b = e / (static_cast<int64_t>(Hkv) * D);
        v[e] = qkv[b * row + static_cast<int64_t>(Hq + Hkv) * D + (e - b * Hkv * D)];
    }
}

// h[r, j] = fp16(silu(gu[r, j])) * gu[r, F + j], 8 at a time (F % 8 == 0, 16-byte aligned)
__global__ void __launch_bounds__(kOpThreads) silu_mul8_kernel(const __half* gu, __half* h, int64_t rows, int64_t F) {
    const int64_t n8 = rows * F / 8;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = i * 8, r = e / F, j = e - r * F;
        const uint4 gv = *reinterpret_cast<const uint4*>(gu + r * 2 * F + j);
        const uint4 uv = *reinterpret_cast<const uint4*>(gu + r * 2 * F + F + j);
        const __half* g8 = reinterpret_cast<const __half*>(&gv);
        const __half* u8 = reinterpret_cast<const __half*>(&uv);
        uint4 o;
        __half* o8 = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float g = __half2float(g8[k]);
            o8[k] = __hmul(__float2half(g / (1.0f + expf(-g))), u8[k]);
        }
        *reinterpret_cast<uint4*>(h + e) = o;
    }
}

// h[r, j] = fp16(silu(gu[r, j])) * gu[r, F + j]
__global__ void __launch_bounds__(kOpThreads) silu_mul_kernel(const __half* gu, __half* h, int64_t rows, int64_t F) {
    const int64_t n = rows * F;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / F, j = i - r * F;
        const float g = __half2float(gu[r * 2 * F + j]);
        const __half a = __float2half(g / (1.0f + expf(-g)));
        h[i] = __hmul(a, gu[r * 2 * F + F + j]);
    }
}

}  // namespace
}  // namespace mg

using namespace mg;

extern "C" mg_status mg_rmsnorm_f16(const void* x, const void* w, void* y, int64_t rows, int64_t cols, float eps,
                                    mg_stream_t stream) {
    MG_REQUIRE(rows >= 0 && cols > 0, "rows must be >= 0 and cols > 0");
    if (rows == 0) return MG_OK;
    MG_REQUIRE(x && w && y, "null pointer");
    MG_REQUIRE(rows < (1ll << 31), "too many rows");
    const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) &
                     15u) == 0;
    const auto xh = static_cast<const __half*>(x);
    const auto wh = static_cast<const __half*>(w);
    const auto yh = static_cast<__half*>(y);
    cudaStream_t s = as_stream(stream);
    if (al && cols % 8 == 0 && cols <= kOpThreads * 8)
        rmsnorm_reg_kernel<1><<<static_cast<unsigned>(rows), kOpThreads, 0, s>>>(xh, wh, yh, static_cast<int>(cols), eps);
    else if (al && cols % 8 == 0 && cols <= kOpThreads * 8 * 4)
        rmsnorm_reg_kernel<4><<<static_cast<unsigned>(rows), kOpThreads, 0, s>>>(xh, wh, yh, static_cast<int>(cols), eps);
    else
        rmsnorm_kernel<<<static_cast<unsigned>(rows), kOpThreads, 0, s>>>(xh, wh, yh, cols, eps);
    return check_launch("rmsnorm_kernel");
}

extern "C" mg_status mg_rope_qkv_f16(const void* qkv, const int64_t* pos, const float* cos_table,
                                     const float* sin_table, void* q, void* k, void* v, int32_t batch,
                                     int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                     mg_stream_t stream) {
    MG_REQUIRE(batch >= 0 && num_q_heads > 0 && num_kv_heads > 0 && head_dim > 0 && head_dim % 2 == 0,
               "bad rope shape");
    if (batch == 0) return MG_OK;
    MG_REQUIRE(qkv && pos && cos_table && sin_table && q && k && v, "null pointer");
    const int64_t n = static_cast<int64_t>(batch) * ((num_q_heads + num_kv_heads) * (head_dim / 2) +
                                                      static_cast<int64_t>(num_kv_heads) * head_dim);
    rope_qkv_kernel<<<static_cast<unsigned>((n + kOpThreads - 1) / kOpThreads), kOpThreads, 0, as_stream(stream)>>>(
        static_cast<const __half*>(qkv), pos, cos_table, sin_table, static_cast<__half*>(q), static_cast<__half*>(k),
        static_cast<__half*>(v), batch, num_q_heads, num_kv_heads, head_dim);
    return check_launch("rope_qkv_kernel");
}

extern "C" mg_status mg_silu_mul_f16(const void* gu, void* h, int64_t rows, int64_t ffn, mg_stream_t stream) {
    MG_REQUIRE(rows >= 0 && ffn > 0, "rows must be >= 0 and ffn > 0");
    if (rows == 0) return MG_OK;
    MG_REQUIRE(gu && h, "null pointer");
    const bool al = ((reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(h)) & 15u) == 0;
    const bool v8 = al && ffn % 8 == 0;
    const int64_t n = rows * ffn / (v8 ? 8 : 1);
    const int64_t blocks = (n + kOpThreads - 1) / kOpThreads;
    const unsigned grid = static_cast<unsigned>(blocks < 148 * 16 ? blocks : 148 * 16);
    if (v8)
        silu_mul8_kernel<<<grid, kOpThreads, 0, as_stream(stream)>>>(static_cast<const __half*>(gu),
                                                                     static_cast<__half*>(h), rows, ffn);
    else
        silu_mul_kernel<<<grid, kOpThreads, 0, as_stream(stream)>>>(static_cast<const __half*>(gu),
                                                                    static_cast<__half*>(h), rows, ffn);
    return check_launch("silu_mul_kernel");
}
