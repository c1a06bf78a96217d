/*
 * mg_oracle.c -- CPU restatement of the reference's byte/integer arithmetic
 * for the paged quantized KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: the product path never
 * links it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg load it.
 *
 * Semantics follow the reference's CUDA ops (the bit-exact target), not the
 * numpy helper tests/reference.py (which rounds half-to-even and lets NaN
 * poison the absmax):
 *   - absmax      csrc/quantize.cu:10-31   fmaxf(acc, fabsf(x)), acc starts 0,
 *                                          so NaN is ignored and Inf propagates
 *   - INT8 scale  csrc/quantize.cu:105-109 isfinite(a) && a > 1e-12
 *                                          ? (double)a / 127.0 : 1e-8
 *   - INT8 code   csrc/quantize.cu:51-57   NaN -> 0, else
 *                                          (int)roundf(fminf(127, fmaxf(-127, x / (float)s)))
 *   - INT8 write  csrc/quantize.cu:59      page[(offset + t) * H*D + hd]
 *   - INT8 deq    csrc/dequantize.cu:9-26  (float)code * (float)scale
 *   - INT4 scale  csrc/quantize_int4.cu:109-113  absmax / 7.0 in double
 *   - INT4 code   csrc/quantize_int4.cu:55-61   clamp to +-7, roundf, NaN -> 0,
 *                                               byte = (q0 & 0xF) | (q1 & 0xF) << 4
 *                                               (element 2j in the low nibble)
 *   - INT4 deq    csrc/dequantize_int4.cu:9-36  sign-extend each nibble, * scale
 *   - allocator   metagross/allocator.py:1-33   LIFO free list, pop() from the end
 *
 * Compiled with -O2 -fno-fast-math -ffp-contract=off so float division is
 * IEEE round-to-nearest (as CUDA's '/' without fast-math) and no FMA
 * contraction changes any product.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define MGO_API __attribute__((visibility("default")))

/* absmax with fmaxf semantics: NaN ignored, Inf kept (csrc/quantize.cu:14-17). */
MGO_API float mgo_absmax(const float* x, int64_t n) {
    float a = 0.0f;
    for (int64_t i = 0; i < n; ++i) a = fmaxf(a, fabsf(x[i]));
    return a;
}

/* Scale chosen from an absmax (csrc/quantize.cu:108-109, quantize_int4.cu:112-113). */
MGO_API double mgo_scale_from_absmax(float absmax, double qmax) {
    int ok = isfinite(absmax) && absmax > 1e-12f;
    return ok ? ((double)absmax / qmax) : 1e-8;
}

static inline int32_t code_of(float v, float s, float qmax) {
    if (isnan(v)) return 0;
    float k = fminf(qmax, fmaxf(-qmax, v / s));
    return (int32_t)roundf(k);
}

/*
 * INT8 page quantize.  input [num_tokens, row] fp32 (row = H*D), written into
 * page[(offset + t) * row + i].  new_scale != 0: compute the scale from the
 * input's absmax (csrc/quantize.cu:65-120); otherwise use fixed_scale
 * (csrc/quantize.cu:122-167).  Returns the scale as double.  Zero tokens:
 * page untouched, returns 1e-8 (csrc/quantize.cu:96-98).
 */
MGO_API double mgo_quantize_int8(const float* input, int64_t num_tokens, int64_t row,
                                 int8_t* page, int64_t offset, int new_scale,
                                 double fixed_scale) {
    int64_t n = num_tokens * row;
    if (n == 0) return new_scale ? 1e-8 : fixed_scale;
    double scale = new_scale ? mgo_scale_from_absmax(mgo_absmax(input, n), 127.0) : fixed_scale;
    float s = (float)scale;
    for (int64_t i = 0; i < n; ++i) page[offset * row + i] = (int8_t)code_of(input[i], s, 127.0f);
    return scale;
}

/* INT8 dequantize of tokens [offset, offset+num_tokens) (csrc/dequantize.cu:9-26). */
MGO_API void mgo_dequantize_int8(const int8_t* page, int64_t offset, int64_t num_tokens,
                                 int64_t row, double scale, float* out) {
    float s = (float)scale;
    for (int64_t i = 0; i < num_tokens * row; ++i) out[i] = (float)page[offset * row + i] * s;
}

/*
 * INT4 packed quantize with a fresh scale (csrc/quantize_int4.cu:33-125).
 * input [num_tokens, H, D] fp32 with D even; packed [*, H, D/2] uint8, element
 * 2j in the low nibble of byte j.
 */
MGO_API double mgo_quantize_int4(const float* input, int64_t num_tokens, int64_t heads,
                                 int64_t head_dim, uint8_t* packed, int64_t offset,
                                 int new_scale, double fixed_scale) {
    int64_t n = num_tokens * heads * head_dim;
    if (n == 0) return new_scale ? 1e-8 : fixed_scale;
    double scale = new_scale ? mgo_scale_from_absmax(mgo_absmax(input, n), 7.0) : fixed_scale;
    float w = (float)scale;
    int64_t half_row = heads * head_dim / 2;
    for (int64_t i = 0; i < n / 2; ++i) {
        int32_t q0 = code_of(input[2 * i], w, 7.0f);
        int32_t q1 = code_of(input[2 * i + 1], w, 7.0f);
        packed[offset * half_row + i] = (uint8_t)(((uint32_t)q0 & 0xFu) | (((uint32_t)q1 & 0xFu) << 4));
    }
    return scale;
}

static inline int32_t sext4(uint32_t nib) { return (int32_t)((int8_t)(nib << 4) >> 4); }

/* INT4 dequantize (csrc/dequantize_int4.cu:9-36): out has 2 floats per byte. */
MGO_API void mgo_dequantize_int4(const uint8_t* packed, int64_t offset, int64_t num_tokens,
                                 int64_t half_row, double scale, float* out) {
    float s = (float)scale;
    for (int64_t i = 0; i < num_tokens * half_row; ++i) {
        uint8_t b = packed[offset * half_row + i];
        out[2 * i] = (float)sext4(b & 0xFu) * s;
        out[2 * i + 1] = (float)sext4((b >> 4) & 0xFu) * s;
    }
}

/*
 * Allocator replay (metagross/allocator.py:1-33).  State: free list of
 * n_free ids (initially 0..num_pages-1).  ops[i] >= 0 frees page ops[i];
 * ops[i] == -1 allocates.  out[i] receives the page id allocated (or freed),
 * or a negative error: -1 exhausted (RuntimeError), -2 double free
 * (RuntimeError), -3 out of range (ValueError).  Returns the final n_free.
 */
MGO_API int64_t mgo_allocator_replay(int32_t* free_list, int64_t n_free, int64_t num_pages,
                                     const int32_t* ops, int64_t n_ops, int32_t* out) {
    for (int64_t i = 0; i < n_ops; ++i) {
        int32_t op = ops[i];
        if (op == -1) {
            if (n_free == 0) { out[i] = -1; continue; }
            out[i] = free_list[--n_free];
        } else {
            if (op < 0 || op >= num_pages) { out[i] = -3; continue; }
            int dup = 0;
            for (int64_t j = 0; j < n_free; ++j) if (free_list[j] == op) { dup = 1; break; }
            if (dup) { out[i] = -2; continue; }
            free_list[n_free++] = op;
            out[i] = op;
        }
    }
    return n_free;
}
