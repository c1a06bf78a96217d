// Shared device/host helpers for the sm_100a kernels of the paged KV-cache path.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "metagross_b200.h"

namespace mg {

// ---------------------------------------------------------------------------
// host-side error reporting (thread-local message behind mg_last_error)
// ---------------------------------------------------------------------------
mg_status set_error(mg_status s, const char* fmt, ...);
mg_status check_launch(const char* what);
int sm_count();  // multiprocessors of the current device (cached per device)

#define MG_REQUIRE(cond, ...)                                                  \
    do {                                                                       \
        if (!(cond)) return ::mg::set_error(MG_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)

inline cudaStream_t as_stream(mg_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// device-side status word
// ---------------------------------------------------------------------------
__device__ __forceinline__ void flag(int32_t* status, int32_t bits) {
    if (status) atomicOr(status, bits);
}

// ---------------------------------------------------------------------------
// quantization arithmetic, bit-exact with the reference kernels:
//   code = NaN ? 0 : (int)roundf(fminf(qmax, fmaxf(-qmax, x / s)))
// (csrc/quantize.cu:51-57, csrc/quantize_int4.cu:57-58).  x / s is the IEEE
// round-to-nearest quotient (the reference builds without fast-math), made
// explicit with __fdiv_rn so no compiler flag can turn it into a reciprocal.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int quant_code(float x, float s, float qmax) {
    if (isnan(x)) return 0;
    float k = fminf(qmax, fmaxf(-qmax, __fdiv_rn(x, s)));
    return static_cast<int>(roundf(k));
}

// quant_code of 8 values with the quotients formed as x * inv, inv = 1 / s
// rounded once.  x * inv is within 2^-23 |x / s| (plus its own rounding) of
// the correctly rounded x / s, so the two round to the same integer unless the
// quotient lies within a few ulps of a half-integer: one test for the group,
// and the IEEE quotient for all 8 only when one of them lies near a
// half-integer or is not finite (the test is false for NaN quotients, and an
// infinite x gives a NaN fractional part).  Away from half-integers round-to-
// nearest-even and round-half-away agree, so the fast codes are one
// conversion each.  The clamp commutes: |x / s| <= qmax + 1 ulp whenever
// s = absmax / qmax covers x, and a clamped quotient stays clamped.  Codes
// equal quant_code's for every input.
__device__ __forceinline__ void quant_codes8(const float (&v)[8], float s, float inv, float qmax, int (&out)[8]) {
    float q[8];
    bool slow = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        q[i] = v[i] * inv;
        const float f = fabsf(q[i] - truncf(q[i]));
        slow |= !(fabsf(f - 0.5f) > fabsf(q[i]) * 4.8e-7f);
    }
    if (slow) {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = quant_code(v[i], s, qmax);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = __float2int_rn(fminf(qmax, fmaxf(-qmax, q[i])));
    }
}

// scale = absmax / qmax in double (csrc/quantize.cu:108-109), 1e-8 when the
// absmax is not finite or <= 1e-12.
__device__ __forceinline__ double scale_from_absmax(float a, double qmax) {
    bool ok = isfinite(a) && a > 1e-12f;
    return ok ? __ddiv_rn(static_cast<double>(a), qmax) : 1e-8;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide max of non-negative values (absmax); every thread gets the result.
// scratch: >= 32 floats of shared memory.
__device__ __forceinline__ float block_max(float v, float* scratch) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    float r = lane < nw ? scratch[lane] : 0.0f;
    r = warp_max(r);
    return r;
}

// Block-wide exclusive scan of one int per thread; returns the exclusive
// prefix, *total receives the block sum.  scratch >= 33 ints.
__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) scratch[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nw ? scratch[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) scratch[lane] = w;  // inclusive per-warp offsets
        if (lane == nw - 1) scratch[32] = w;
    }
    __syncthreads();
    const int warp_off = warp == 0 ? 0 : scratch[warp - 1];
    *total = scratch[32];
    return warp_off + x - v;
}

// ---------------------------------------------------------------------------
// int8 / int4 -> fp16 conversion without I2F.
// fp16 0x6400 is 1024.0 with a 10-bit mantissa of unit weight, so the half
// with bit pattern 0x6400 | u (u in 0..255 after a sign flip, or a nibble) is
// exactly 1024 + u; subtracting 1024 + bias gives the signed code exactly.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
    // (a & b) ^ c in one LOP3 (immediate 0x6A = (A & B) ^ C)
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    // (a & b) | c, immediate 0xEA
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// Bytes b_lo (bits 0-7) and b_hi (bits 16-23) of x, each a two's-complement
// int8, to half2 (lo, hi).  Other bits of x are ignored.
__device__ __forceinline__ uint32_t s8pair_to_half2(uint32_t x) {
    const uint32_t h = lop3_and_xor(x, 0x00FF00FFu, 0x64806480u);  // 1024 + (b ^ 0x80) = 1152 + b
    return hsub2_u32(h, 0x64806480u);                                // - 1152 (fp16 0x6480)
}
// Nibbles at bits 0-3 and 16-19 (two's complement int4) to half2.
__device__ __forceinline__ uint32_t s4pair_lo_to_half2(uint32_t x_xored) {
    // x_xored = x ^ 0x88888888 (offset binary); 0x6408 = 1032.0
    const uint32_t h = lop3_and_or(x_xored, 0x000F000Fu, 0x64006400u);
    return hsub2_u32(h, 0x64086408u);
}
// Nibbles at bits 4-7 and 20-23 to half2: (1024 + 16 u) / 16 - (64 + 8).
__device__ __forceinline__ uint32_t s4pair_hi_to_half2(uint32_t x_xored) {
    const uint32_t h = lop3_and_or(x_xored, 0x00F000F0u, 0x64006400u);
    // fma(h, 1/16, -72): 0x2C00 = 0.0625, 0xD480 = -72.0
    return hfma2_u32(h, 0x2C002C00u, 0xD480D480u);
}

// ---------------------------------------------------------------------------
// warp-level tensor-core primitives (sm_80+ PTX, valid on sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 8x8 b16 transpose across the warp: lane 4r+c holds row r cols (2c, 2c+1);
// afterwards it holds row r of the transpose.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t r;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
    return r;
}

__device__ __forceinline__ float ex2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// mbarrier + bulk (TMA, non-tensor) copies, global -> shared
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// One bounded attempt; true when the phase with the given parity completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after max_tries attempts (each attempt itself is
// time-limited by the hardware), so a lost copy can never hang the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t max_tries) {
    for (uint32_t i = 0; i < max_tries; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// 1-D bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// completing on `bar` (complete_tx).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 16-byte asynchronous global -> shared copy (both addresses 16-byte aligned);
// completion is awaited per thread with cp_async_wait_all().
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src_gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}
// 4-byte form (both addresses 4-byte aligned), through L1
__device__ __forceinline__ void cp_async4(void* dst_smem, const void* src_gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
// Wait until at most N of this thread's most recent cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// Non-blocking hint: bring the line holding ptr into L1.
__device__ __forceinline__ void prefetch_l1(const void* ptr) { asm volatile("prefetch.global.L1 [%0];" ::"l"(ptr)); }
// Non-blocking hint: bring the line holding ptr into L2 (coherent with every writer).
__device__ __forceinline__ void prefetch_l2(const void* ptr) { asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr)); }
// Non-blocking hint: bring [ptr, ptr + bytes) into L2; ptr 16-byte aligned,
// bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* ptr, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}
// Barrier among the nthreads (a multiple of 32) threads that use barrier id.
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Programmatic dependent launch: block until the grids this one depends on
// have completed (a no-op when launched without the attribute), and let the
// next kernel in the stream start its launch early.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// Fast unsigned division by a runtime divisor d in [1, 2^16): magic
// m = ceil(2^32 / d) = (2^32 + e) / d with 0 <= e < d, q = umulhi(n, m).  Exact
// while n * e < 2^32, i.e. for every n < 2^32 / d (n < 2^16 for any d < 2^16).
struct FastDiv {
    uint32_t d, m;
    __host__ __device__ FastDiv() : d(1), m(0) {}
    __host__ explicit FastDiv(uint32_t div) : d(div), m(div == 1 ? 0u : (uint32_t)((0x100000000ull + div - 1) / div)) {}
    __device__ __forceinline__ uint32_t div(uint32_t n) const { return d == 1 ? n : __umulhi(n, m); }
};

}  // namespace mg
