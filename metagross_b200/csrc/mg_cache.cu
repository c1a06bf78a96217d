// Device-resident paged cache: page allocator, step planner, KV append with
// page commit (quantize), block gather/dequantize, sequence free.
//
// Semantics are those of the reference's per-sequence Python cache
// (metagross/cache.py:45-85) and allocator (metagross/allocator.py:1-33),
// batched: one pool and one LIFO allocator serve every sequence of the batch
// and every layer (all layers commit at the same token counts, so one block
// table per sequence serves them all -- the reference's 2*num_layers
// allocators of one sequence all hand out the same ids).
#include <type_traits>

#include "mg_alloc_step.cuh"
#include "mg_common.cuh"

namespace mg {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kAppendThreads = 256;
constexpr int kGatherThreads = 256;

__global__ void alloc_init_kernel(int32_t* free_stack, int32_t* n_free, int32_t* in_use, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        free_stack[i] = static_cast<int32_t>(i);
        in_use[i] = 0;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *n_free = static_cast<int32_t>(n);
}

// One CTA: the step's allocation (mg_alloc_step.cuh).
__global__ void __launch_bounds__(kPlanThreads) plan_append_kernel(AllocStep a) { alloc_step(a); }

// Frees the listed sequences' pages beyond new_lens (0 when new_lens is
// null) in (list order, block-table order): the order in which the
// reference's BlockAllocator.free would be called.  One CTA.  With distinct
// sequence ids and the bookkeeping in shared memory (sm_words > 0), every
// listed sequence is checked at once, the pages to free are numbered by a
// prefix sum over the list, and the whole flattened page list is freed in
// block-wide rounds; a list that names a sequence twice takes the sequential
// walk, which sees each entry's effect on the next.
__global__ void __launch_bounds__(kPlanThreads) free_sequences_kernel(int32_t* free_stack, int32_t* n_free_p,
                                                                      int32_t* in_use, int64_t num_pages,
                                                                      const int32_t* block_tables,
                                                                      int32_t max_blocks, int32_t* seq_lens,
                                                                      int32_t batch, const int32_t* seq_ids,
                                                                      const int32_t* new_lens, int32_t num_seqs,
                                                                      int32_t P, int32_t* status, int32_t sm_words) {
    extern __shared__ int fsm[];
    __shared__ int scratch[33];
    __shared__ int s_dup;
    int top = *n_free_p;
    auto free_page = [&](const int32_t* row, int j, bool live, int32_t& page) -> int {
        if (!live) return 0;
        page = row[j];
        if (page < 0 || page >= num_pages) {
            flag(status, MG_DEV_BAD_PAGE_ID);
            return 0;
        }
        if (atomicExch(&in_use[page], 0) != 1) {
            flag(status, MG_DEV_DOUBLE_FREE);
            return 0;
        }
        return 1;
    };
    bool sequential = sm_words == 0;
    if (!sequential) {
        int* base = fsm;                  // [num_seqs + 1] first flattened page of entry i
        int* keep = base + num_seqs + 1;  // [num_seqs] first page freed, -1: entry skipped
        unsigned* seen = reinterpret_cast<unsigned*>(keep + num_seqs);  // [batch / 32 + 1] bitmap
        const int nbits = batch / 32 + 1;
        if (threadIdx.x == 0) s_dup = 0;
        for (int w = threadIdx.x; w < nbits; w += blockDim.x) seen[w] = 0u;
        __syncthreads();
        for (int i = threadIdx.x; i < num_seqs; i += blockDim.x) {
            const int sq = seq_ids[i];
            int cnt = 0, kp = -1;
            if (sq < 0 || sq >= batch) {
                flag(status, MG_DEV_BAD_ARGUMENT);
            } else {
                if (atomicOr(&seen[sq >> 5], 1u << (sq & 31)) & (1u << (sq & 31))) s_dup = 1;
                const int old_len = seq_lens[sq];
                const int new_len = new_lens ? new_lens[i] : 0;
                const int committed = (old_len / P) * P;
                if (new_len < 0 || new_len > old_len || (new_len % P != 0 && new_len < committed)) {
                    flag(status, MG_DEV_BAD_ARGUMENT);
                } else {
                    const int npages = old_len / P < max_blocks ? old_len / P : max_blocks;
                    kp = new_len / P;
                    cnt = npages > kp ? npages - kp : 0;
                }
            }
            base[i] = cnt;
            keep[i] = kp;
        }
        __syncthreads();
        sequential = s_dup != 0;
        if (!sequential) {
            // exclusive prefix of the counts, in place
            int run = 0;
            for (int start = 0; start < num_seqs; start += blockDim.x) {
                const int i = start + threadIdx.x;
                const int v = i < num_seqs ? base[i] : 0;
                int tot;
                const int ex = block_exclusive_scan(v, scratch, &tot);
                __syncthreads();
                if (i < num_seqs) base[i] = run + ex;
                run += tot;
                __syncthreads();
            }
            if (threadIdx.x == 0) base[num_seqs] = run;
            __syncthreads();
            const int total = run;
            for (int t0 = 0; t0 < total; t0 += blockDim.x) {
                const int t = t0 + threadIdx.x;
                int ok = 0;
                int32_t page = -1;
                if (t < total) {
                    int lo = 0, hi = num_seqs - 1;  // last entry i with base[i] <= t
                    while (lo < hi) {
                        const int mid = (lo + hi + 1) >> 1;
                        if (base[mid] <= t) lo = mid;
                        else hi = mid - 1;
                    }
                    const int32_t* row = block_tables + static_cast<int64_t>(seq_ids[lo]) * max_blocks;
                    ok = free_page(row, keep[lo] + (t - base[lo]), true, page);
                }
                int cnt;
                const int excl = block_exclusive_scan(ok, scratch, &cnt);
                if (ok) free_stack[top + excl] = page;
                top += cnt;
            }
            __syncthreads();
            for (int i = threadIdx.x; i < num_seqs; i += blockDim.x)
                if (keep[i] >= 0) seq_lens[seq_ids[i]] = new_lens ? new_lens[i] : 0;
        }
    }
    if (sequential) {
        for (int i = 0; i < num_seqs; ++i) {
            const int sq = seq_ids[i];
            if (sq < 0 || sq >= batch) {
                if (threadIdx.x == 0) flag(status, MG_DEV_BAD_ARGUMENT);
                continue;
            }
            const int old_len = seq_lens[sq];
            const int new_len = new_lens ? new_lens[i] : 0;
            const int committed = (old_len / P) * P;
            if (new_len < 0 || new_len > old_len || (new_len % P != 0 && new_len < committed)) {
                if (threadIdx.x == 0) flag(status, MG_DEV_BAD_ARGUMENT);
                continue;
            }
            int npages = old_len / P;
            if (npages > max_blocks) npages = max_blocks;
            const int kp = new_len / P;
            const int32_t* row = block_tables + static_cast<int64_t>(sq) * max_blocks;
            for (int start = kp; start < npages; start += blockDim.x) {
                const int j = start + threadIdx.x;
                int32_t page = -1;
                const int ok = free_page(row, j, j < npages, page);
                int cnt;
                const int excl = block_exclusive_scan(ok, scratch, &cnt);
                if (ok) free_stack[top + excl] = page;
                top += cnt;
            }
            __syncthreads();
            if (threadIdx.x == 0) seq_lens[sq] = new_len;
            __syncthreads();  // the next entry may name the same sequence
        }
    }
    if (threadIdx.x == 0) *n_free_p = top;
}

// ---------------------------------------------------------------------------
// KV append: one CTA per (sequence, touched page, K|V).
// ---------------------------------------------------------------------------
template <typename T>
struct Vec8;  // 8 consecutive elements
template <>
struct Vec8<float> {
    static __device__ __forceinline__ void load(const float* p, float (&v)[8]) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        const float4 b = *reinterpret_cast<const float4*>(p + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    static __device__ __forceinline__ void store(float* p, const float (&v)[8]) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
};
template <>
struct Vec8<__half> {
    static __device__ __forceinline__ void load(const __half* p, float (&v)[8]) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    static __device__ __forceinline__ void store(__half* p, const float (&v)[8]) {
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        *reinterpret_cast<uint4*>(p) = u;
    }
};

struct AppendParams {
    const void* k_new;
    const void* v_new;
    int32_t max_new;
    void* k_pool;
    void* v_pool;
    float* k_scales;
    float* v_scales;
    void* staging_k;
    void* staging_v;
    const int32_t* block_tables;
    int32_t max_blocks;
    const int32_t* seq_lens;
    const int32_t* n_new;
    int32_t P;
    int32_t row;  // Hkv * D elements per token
    int32_t D;
    int32_t scale_th;  // scales [N, P, Hkv] (one per token and head) instead of [N]
    int64_t num_pages;
    int32_t* status;
    int64_t new_stride;     // elements from one new token's row to the next (row, or (Hq + 2 Hkv) D in a qkv buffer)
    const float* rope_cos;  // non-null: rotate K (and q) by these tables [rope_rows, D / 2] (rotate-half)
    const float* rope_sin;
    int32_t rope_rows;
    int32_t Hq;
    const __half* q_src;  // q heads of the new tokens, row stride new_stride
    __half* q_out;        // [batch, max_new, Hq, D] rotated q
    int32_t release_early;  // MG_APPEND_EARLY_LAUNCH: release the next launch at the start
    FastDiv rowdiv;         // division by row (element offsets within a page are below 2^20)
};

// Rotate-half rotary embedding of one element pair at position pos (fp32
// products, one rounding to fp16 each, as the reference's rotary embedding of
// fp16 activations): (x1, x2) -> (x1 c - x2 s, x2 c + x1 s); own / partner are
// this element and the one D/2 away, lower says which half this one is in.
__device__ __forceinline__ float rope_elem(float own, float partner, float c, float s, bool lower) {
    const float r = lower ? __fsub_rn(__fmul_rn(own, c), __fmul_rn(partner, s))
                          : __fadd_rn(__fmul_rn(own, c), __fmul_rn(partner, s));
    return __half2float(__float2half_rn(r));
}

// Code of 8 consecutive elements into the pool at element e of a page (INT8:
// 8 bytes, INT4: 4 bytes of nibbles, the even element in the low nibble),
// through quant_codes8 (the same codes as the IEEE quotient x / sf).
template <bool INT4>
__device__ __forceinline__ void store_codes(uint8_t* page_base, int64_t e, const float (&v)[8], float sf) {
    const float inv = 1.0f / sf;
    int q[8];
    quant_codes8(v, sf, inv, INT4 ? 7.0f : 127.0f, q);
    if (!INT4) {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w0 |= (static_cast<uint32_t>(q[i]) & 0xFFu) << (8 * i);
            w1 |= (static_cast<uint32_t>(q[4 + i]) & 0xFFu) << (8 * i);
        }
        *reinterpret_cast<uint2*>(page_base + e) = make_uint2(w0, w1);
    } else {
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) w |= (static_cast<uint32_t>(q[i]) & 0xFu) << (4 * i);
        *reinterpret_cast<uint32_t*>(page_base + e / 2) = w;
    }
}

// KEEP: groups of 8 elements a commit thread keeps in registers (2 for pages of
// up to 4096 elements, which then leaves room for 4 CTAs per SM; 8 otherwise).
template <bool INT4, typename ST, typename NT, int KEEP>
__global__ void __launch_bounds__(kAppendThreads, KEEP <= 2 ? 4 : 2) kv_append_kernel(AppendParams p) {
    constexpr int kKeep = KEEP;
    __shared__ float red[32];
    const int b = blockIdx.x, jj = blockIdx.y, kv = blockIdx.z;
    // with MG_APPEND_EARLY_LAUNCH a programmatic dependent launch (the wait is a
    // no-op otherwise): the new tokens come from the previous launch.  Only then
    // is the next launch released at once, so that an attention launch reads its
    // plan while this one runs; released early after a plain launch, the
    // attention measured slower in the TinyLlama decode step (1.35 against 1.22
    // ms a step), so a plain launch releases it at its end.
    grid_dependency_wait();
    if (p.release_early) grid_launch_dependents();
    // status, length and count in one round trip
    const int32_t stat = p.status ? *(volatile int32_t*)p.status : 0;
    const int new_len = p.seq_lens[b], add = p.n_new[b];
    if (stat & kStopBits) return;
    if (add <= 0) return;
    if (add > p.max_new || add > new_len) {
        if (jj == 0 && kv == 0 && threadIdx.x == 0) flag(p.status, MG_DEV_BAD_ARGUMENT);
        return;
    }
    const int old = new_len - add;
    if (kv == 2) {
        // rotary q of this sequence's new tokens (the rotary variant's third grid slice)
        if (jj != 0) return;
        const int half = p.D / 2;
        const int64_t npairs = static_cast<int64_t>(add) * p.Hq * half;
        for (int64_t i = threadIdx.x; i < npairs; i += blockDim.x) {
            const int64_t th = i / half;  // (token, head)
            const int jd = static_cast<int>(i - th * half);
            const int t = static_cast<int>(th / p.Hq), h = static_cast<int>(th - static_cast<int64_t>(t) * p.Hq);
            const int pos = old + t;
            if (pos >= p.rope_rows) {
                flag(p.status, MG_DEV_BAD_ARGUMENT);
                continue;
            }
            const __half* src = p.q_src + (static_cast<int64_t>(b) * p.max_new + t) * p.new_stride + h * p.D;
            const float c = p.rope_cos[static_cast<int64_t>(pos) * half + jd];
            const float sn = p.rope_sin[static_cast<int64_t>(pos) * half + jd];
            const float x1 = __half2float(src[jd]), x2 = __half2float(src[jd + half]);
            __half* dst = p.q_out + ((static_cast<int64_t>(b) * p.max_new + t) * p.Hq + h) * p.D;
            dst[jd] = __float2half_rn(rope_elem(x1, x2, c, sn, true));
            dst[jd + half] = __float2half_rn(rope_elem(x2, x1, c, sn, false));
        }
        return;
    }
    const int P = p.P, row = p.row;
    const int j0 = old / P, jlast = (new_len - 1) / P;
    const int j = j0 + jj;
    if (j > jlast) return;
    const int64_t pe = static_cast<int64_t>(P) * row;  // elements per page
    ST* staging = static_cast<ST*>(kv ? p.staging_v : p.staging_k) + static_cast<int64_t>(b) * pe;
    const NT* src_new =
        static_cast<const NT*>(kv ? p.v_new : p.k_new) + static_cast<int64_t>(b) * p.max_new * p.new_stride;
    const int page_start = j * P;

    // 8 consecutive elements at element c of new token t (step-relative); K
    // rotated at position old + t when the call carries rotary tables
    auto load_new8 = [&](int t, int64_t c, float (&v)[8]) {
        const NT* src = src_new + static_cast<int64_t>(t) * p.new_stride;
        Vec8<NT>::load(src + c, v);
        if (p.rope_cos != nullptr && kv == 0) {
            const int half = p.D / 2;
            const int d = static_cast<int>(c) % p.D;
            const bool lower = d < half;
            float w[8];
            Vec8<NT>::load(src + c + (lower ? half : -half), w);
            int pos = old + t;
            if (pos >= p.rope_rows) {
                flag(p.status, MG_DEV_BAD_ARGUMENT);
                pos = 0;
            }
            const int64_t ti = static_cast<int64_t>(pos) * half + (lower ? d : d - half);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = rope_elem(v[i], w[i], p.rope_cos[ti + i], p.rope_sin[ti + i], lower);
        }
    };
    // 8 consecutive elements at element e of page j: staged rows, then this step's tokens
    auto load8 = [&](int64_t e, float (&v)[8]) {
        const int t = static_cast<int>(p.rowdiv.div(static_cast<uint32_t>(e)));
        const int tok = page_start + t;
        const int64_t c = static_cast<int>(e) - t * row;
        if (tok < old) Vec8<ST>::load(staging + static_cast<int64_t>(t) * row + c, v);
        else load_new8(tok - old, c, v);
    };
    if (page_start + P <= new_len) {  // page j fills during this step: commit it
        const int32_t page = j < p.max_blocks ? p.block_tables[static_cast<int64_t>(b) * p.max_blocks + j] : -1;
        uint8_t* pool = static_cast<uint8_t*>(kv ? p.v_pool : p.k_pool);
        float* scales = kv ? p.v_scales : p.k_scales;
        const bool bad_page = page < 0 || page >= p.num_pages;
        if (!p.scale_th && pe <= static_cast<int64_t>(kAppendThreads) * 8 * kKeep) {
            // the whole page in registers (up to kKeep groups of 8 per thread): every
            // load in flight at once, one pass over the staged and new rows; the
            // loads do not wait for the page id (only the stores need it)
            float v[kKeep][8];
            float a = 0.0f;
#pragma unroll
            for (int u = 0; u < kKeep; ++u) {
                const int64_t e = (static_cast<int64_t>(u) * kAppendThreads + threadIdx.x) * 8;
#pragma unroll
                for (int i = 0; i < 8; ++i) v[u][i] = 0.0f;
                if (e < pe) load8(e, v[u]);
#pragma unroll
                for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[u][i]));
            }
            a = block_max(a, red);
            if (bad_page) {
                if (threadIdx.x == 0) flag(p.status, MG_DEV_BAD_PAGE_ID);
            } else {
                const float sf = static_cast<float>(scale_from_absmax(a, INT4 ? 7.0 : 127.0));
                if (threadIdx.x == 0) scales[page] = sf;
                uint8_t* base = pool + static_cast<int64_t>(page) * (INT4 ? pe / 2 : pe);
#pragma unroll
                for (int u = 0; u < kKeep; ++u) {
                    const int64_t e = (static_cast<int64_t>(u) * kAppendThreads + threadIdx.x) * 8;
                    if (e < pe) store_codes<INT4>(base, e, v[u], sf);
                }
            }
        } else if (bad_page) {
            if (threadIdx.x == 0) flag(p.status, MG_DEV_BAD_PAGE_ID);
        } else if (p.scale_th) {
            // one fresh scale per (token, head) D-vector, the reference's
            // quantize_new_scale of a [1, 1, D] slice: the D / 8 consecutive
            // threads holding a vector reduce its absmax by shuffles (every
            // thread runs every round, so the shuffles never diverge)
            const int gl = p.D >> 3;
            uint8_t* base = pool + static_cast<int64_t>(page) * (INT4 ? pe / 2 : pe);
            for (int64_t r0 = 0; r0 < pe; r0 += static_cast<int64_t>(kAppendThreads) * 8 * kKeep) {
                float v[kKeep][8];
#pragma unroll
                for (int u = 0; u < kKeep; ++u) {
                    const int64_t e = r0 + (static_cast<int64_t>(u) * kAppendThreads + threadIdx.x) * 8;
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[u][i] = 0.0f;
                    if (e < pe) load8(e, v[u]);
                }
#pragma unroll
                for (int u = 0; u < kKeep; ++u) {
                    const int64_t e = r0 + (static_cast<int64_t>(u) * kAppendThreads + threadIdx.x) * 8;
                    float a = 0.0f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[u][i]));
                    for (int o = gl >> 1; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
                    if (e < pe) {
                        const int t = static_cast<int>(e / row);
                        const int64_t c = e - static_cast<int64_t>(t) * row;
                        const float sf = static_cast<float>(scale_from_absmax(a, INT4 ? 7.0 : 127.0));
                        if ((threadIdx.x & (gl - 1)) == 0)
                            scales[(static_cast<int64_t>(page) * P + t) * (row / p.D) + c / p.D] = sf;
                        store_codes<INT4>(base, e, v[u], sf);
                    }
                }
            }
        } else {
            // larger pages: absmax pass, then a second pass that quantizes
            float a = 0.0f;
            for (int64_t e = threadIdx.x * 8; e < pe; e += kAppendThreads * 8) {
                float v[8];
                load8(e, v);
#pragma unroll
                for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[i]));
            }
            a = block_max(a, red);
            const double s = scale_from_absmax(a, INT4 ? 7.0 : 127.0);
            const float sf = static_cast<float>(s);
            if (threadIdx.x == 0) scales[page] = sf;
            uint8_t* base = pool + static_cast<int64_t>(page) * (INT4 ? pe / 2 : pe);
            for (int64_t e = threadIdx.x * 8; e < pe; e += kAppendThreads * 8) {
                float v[8];
                load8(e, v);
                store_codes<INT4>(base, e, v, sf);
            }
        }
    }
    // The first touched page's CTA is the only one that reads the old staged
    // rows, so it also writes the new partial page's rows (after its reads).
    if (jj == 0 && (jlast + 1) * P > new_len) {
        __syncthreads();
        const int first = old > jlast * P ? old : jlast * P;
        const int64_t e0 = static_cast<int64_t>(first - jlast * P) * row;
        const int64_t e1 = static_cast<int64_t>(new_len - jlast * P) * row;
        for (int64_t e = e0 + threadIdx.x * 8; e < e1; e += kAppendThreads * 8) {
            const int t = static_cast<int>(e / row);
            const int64_t c = e - static_cast<int64_t>(t) * row;
            float v[8];
            load_new8(jlast * P + t - old, c, v);
            Vec8<ST>::store(staging + e, v);
        }
    }
}

// ---------------------------------------------------------------------------
// gather + dequantize: one CTA per (logical page slot, sequence, K|V)
// ---------------------------------------------------------------------------
struct GatherParams {
    const void* k_pool;
    const void* v_pool;
    const float* k_scales;
    const float* v_scales;
    const void* staging_k;
    const void* staging_v;
    const int32_t* block_tables;
    int32_t max_blocks;
    const int32_t* seq_lens;
    const int32_t* cu_seqlens;
    int32_t P;
    int32_t row;
    int32_t D;
    int32_t scale_th;  // scales [N, P, Hkv] instead of [N]
    int64_t num_pages;
    int32_t include_staging;
    void* out_k;
    void* out_v;
    int32_t* status;
};

template <bool INT4, typename ST, typename OT>
__global__ void __launch_bounds__(kGatherThreads) gather_dequant_kernel(GatherParams p) {
    const int j = blockIdx.x, b = blockIdx.y, kv = blockIdx.z;
    const int len = p.seq_lens[b];
    const int P = p.P, row = p.row;
    const int npages = len / P, tail = len % P;
    const int64_t pe = static_cast<int64_t>(P) * row;
    const int expect = p.include_staging ? len : npages * P;
    if (p.cu_seqlens[b + 1] - p.cu_seqlens[b] != expect || npages > p.max_blocks) {
        if (j == 0 && kv == 0 && threadIdx.x == 0) flag(p.status, MG_DEV_BAD_ARGUMENT);
        return;
    }
    OT* out = static_cast<OT*>(kv ? p.out_v : p.out_k) + (static_cast<int64_t>(p.cu_seqlens[b]) + static_cast<int64_t>(j) * P) * row;
    if (j < npages) {
        int32_t page = p.block_tables[static_cast<int64_t>(b) * p.max_blocks + j];
        if (page < 0 || page >= p.num_pages) {
            if (threadIdx.x == 0) flag(p.status, MG_DEV_BAD_PAGE_ID);
            page = 0;
        }
        const float* scales = kv ? p.v_scales : p.k_scales;
        const float sf_page = p.scale_th ? 0.0f : scales[page];
        const uint8_t* pool = static_cast<const uint8_t*>(kv ? p.v_pool : p.k_pool);
        for (int64_t e = threadIdx.x * 8; e < pe; e += kGatherThreads * 8) {
            float v[8];
            float sf = sf_page;
            if (p.scale_th) {  // the scale of this (token, head) D-vector
                const int t = static_cast<int>(e / row);
                sf = scales[(static_cast<int64_t>(page) * P + t) * (row / p.D) + (e - static_cast<int64_t>(t) * row) / p.D];
            }
            if (!INT4) {
                const uint2 w = *reinterpret_cast<const uint2*>(pool + static_cast<int64_t>(page) * pe + e);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    v[i] = static_cast<float>(static_cast<int8_t>(w.x >> (8 * i))) * sf;
                    v[4 + i] = static_cast<float>(static_cast<int8_t>(w.y >> (8 * i))) * sf;
                }
            } else {
                const uint32_t w = *reinterpret_cast<const uint32_t*>(pool + static_cast<int64_t>(page) * (pe / 2) + e / 2);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    v[i] = static_cast<float>(static_cast<int>(static_cast<int8_t>((w >> (4 * i)) << 4)) >> 4) * sf;
            }
            Vec8<OT>::store(out + e, v);
        }
    } else if (j == npages && p.include_staging && tail > 0) {
        const ST* st = static_cast<const ST*>(kv ? p.staging_v : p.staging_k) + static_cast<int64_t>(b) * pe;
        for (int64_t e = threadIdx.x * 8; e < static_cast<int64_t>(tail) * row; e += kGatherThreads * 8) {
            float v[8];
            Vec8<ST>::load(st + e, v);
            Vec8<OT>::store(out + e, v);
        }
    }
}

inline bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

mg_status check_layout(const mg_cache_layout* L) {
    MG_REQUIRE(L != nullptr, "null layout");
    MG_REQUIRE(L->kv_dtype == MG_KV_INT8 || L->kv_dtype == MG_KV_INT4, "kv_dtype must be MG_KV_INT8 or MG_KV_INT4");
    MG_REQUIRE(L->staging_dtype == MG_F32 || L->staging_dtype == MG_F16, "staging_dtype must be MG_F32 or MG_F16");
    MG_REQUIRE(L->page_size >= 1 && L->page_size <= 64, "page_size must be in [1, 64], got %d", L->page_size);
    MG_REQUIRE(L->num_kv_heads >= 1, "num_kv_heads must be positive");
    MG_REQUIRE(L->head_dim >= 8 && L->head_dim % 8 == 0, "head_dim must be a positive multiple of 8, got %d",
               L->head_dim);
    MG_REQUIRE(L->kv_dtype == MG_KV_INT8 || L->head_dim % 32 == 0,
               "INT4 pools need head_dim % 32 == 0 (16-byte rows), got %d", L->head_dim);
    MG_REQUIRE(L->max_blocks >= 1, "max_blocks must be positive");
    MG_REQUIRE(L->num_pages >= 1 && L->num_pages < (1ll << 31), "num_pages out of range");
    MG_REQUIRE(L->scale_layout == MG_SCALE_PAGE || L->scale_layout == MG_SCALE_TOKEN_HEAD,
               "scale_layout must be MG_SCALE_PAGE or MG_SCALE_TOKEN_HEAD");
    MG_REQUIRE(L->scale_layout == MG_SCALE_PAGE || (L->head_dim <= 256 && (L->head_dim & (L->head_dim - 1)) == 0),
               "MG_SCALE_TOKEN_HEAD needs head_dim a power of two <= 256, got %d", L->head_dim);
    return MG_OK;
}

}  // namespace

mg_status check_cache_layout(const mg_cache_layout* L) { return check_layout(L); }

}  // namespace mg

using namespace mg;

extern "C" mg_status mg_alloc_init(const mg_allocator* a, mg_stream_t stream) {
    MG_REQUIRE(a && a->free_stack && a->n_free && a->in_use, "null allocator pointer");
    MG_REQUIRE(a->num_pages >= 1 && a->num_pages < (1ll << 31), "num_pages out of range");
    const unsigned g = static_cast<unsigned>((a->num_pages + 255) / 256 > 4096 ? 4096 : (a->num_pages + 255) / 256);
    alloc_init_kernel<<<g, 256, 0, as_stream(stream)>>>(a->free_stack, a->n_free, a->in_use, a->num_pages);
    return check_launch("alloc_init_kernel");
}

extern "C" mg_status mg_plan_append(const mg_allocator* a, int32_t* block_tables, int32_t max_blocks,
                                    int32_t* seq_lens, const int32_t* n_new, int32_t batch, int32_t page_size,
                                    int32_t* dev_status, mg_stream_t stream) {
    MG_REQUIRE(a && a->free_stack && a->n_free && a->in_use, "null allocator pointer");
    MG_REQUIRE(batch >= 0, "batch must be >= 0");
    if (batch == 0) return MG_OK;
    MG_REQUIRE(block_tables && seq_lens && n_new, "null pointer");
    MG_REQUIRE(page_size >= 1 && max_blocks >= 1, "page_size and max_blocks must be positive");
    const AllocStep st{a->free_stack, a->n_free, a->in_use, block_tables, max_blocks, seq_lens, n_new, batch,
                       page_size, dev_status};
    plan_append_kernel<<<1, kPlanThreads, 0, as_stream(stream)>>>(st);
    return check_launch("plan_append_kernel");
}

extern "C" mg_status mg_truncate_sequences(const mg_allocator* a, const int32_t* block_tables, int32_t max_blocks,
                                           int32_t* seq_lens, int32_t batch, const int32_t* seq_ids,
                                           const int32_t* new_lens, int32_t num_seqs, int32_t page_size,
                                           int32_t* dev_status, mg_stream_t stream) {
    MG_REQUIRE(a && a->free_stack && a->n_free && a->in_use, "null allocator pointer");
    MG_REQUIRE(num_seqs >= 0, "num_seqs must be >= 0");
    if (num_seqs == 0) return MG_OK;
    MG_REQUIRE(block_tables && seq_lens && seq_ids, "null pointer");
    MG_REQUIRE(page_size >= 1 && max_blocks >= 1 && batch >= 1, "page_size, max_blocks and batch must be positive");
    // shared memory of the parallel walk: prefix [n + 1], keep [n], bitmap [batch / 32 + 1]
    const int64_t words = 2ll * num_seqs + 1 + batch / 32 + 1;
    const bool fits = words * 4 <= 48 * 1024;
    free_sequences_kernel<<<1, kPlanThreads, fits ? static_cast<size_t>(words * 4) : 0, as_stream(stream)>>>(
        a->free_stack, a->n_free, a->in_use, a->num_pages, block_tables, max_blocks, seq_lens, batch, seq_ids,
        new_lens, num_seqs, page_size, dev_status, fits ? static_cast<int32_t>(words) : 0);
    return check_launch("free_sequences_kernel");
}

extern "C" mg_status mg_free_sequences(const mg_allocator* a, const int32_t* block_tables, int32_t max_blocks,
                                       int32_t* seq_lens, int32_t batch, const int32_t* seq_ids, int32_t num_seqs,
                                       int32_t page_size, int32_t* dev_status, mg_stream_t stream) {
    return mg_truncate_sequences(a, block_tables, max_blocks, seq_lens, batch, seq_ids, nullptr, num_seqs,
                                 page_size, dev_status, stream);
}

namespace mg {
namespace {

// The append proper: checks, parameters and the launch.  new_stride: elements
// between consecutive new-token rows (row for k_new / v_new tensors).  With
// rotary tables (fp16 tokens and staging only) K is rotated on the way in and
// a third grid slice writes the rotated q of q_src to q_out.
mg_status append_launch(const mg_cache_layout* L, const mg_layer_ptrs* lp, const int32_t* block_tables,
                        const int32_t* seq_lens, const int32_t* n_new, int32_t batch, const void* k_new,
                        const void* v_new, int32_t new_dtype, int32_t max_new, int64_t new_stride,
                        const float* rope_cos, const float* rope_sin, int32_t rope_rows, int32_t num_q_heads,
                        const void* q_src, void* q_out, int32_t* dev_status, mg_stream_t stream,
                        bool early_launch = false) {
    mg_status st = check_layout(L);
    if (st != MG_OK) return st;
    MG_REQUIRE(lp != nullptr, "null layer pointers");
    MG_REQUIRE(batch >= 0 && max_new >= 0, "batch and max_new must be >= 0");
    if (batch == 0 || max_new == 0) return MG_OK;
    MG_REQUIRE(new_dtype == MG_F32 || new_dtype == MG_F16, "new_dtype must be MG_F32 or MG_F16");
    MG_REQUIRE(!(new_dtype == MG_F32 && L->staging_dtype == MG_F16),
               "fp32 tokens cannot be staged in an fp16 staging buffer without rounding");
    MG_REQUIRE(lp->k_pool && lp->v_pool && lp->k_scales && lp->v_scales && lp->staging_k && lp->staging_v,
               "null layer pointer");
    MG_REQUIRE(k_new && v_new && block_tables && seq_lens && n_new, "null pointer");
    MG_REQUIRE(aligned16(k_new) && aligned16(v_new) && aligned16(lp->staging_k) && aligned16(lp->staging_v) &&
                   aligned16(lp->k_pool) && aligned16(lp->v_pool),
               "k_new, v_new, staging and pools must be 16-byte aligned");
    const int64_t row = static_cast<int64_t>(L->num_kv_heads) * L->head_dim;
    MG_REQUIRE(new_stride >= row && new_stride % 8 == 0, "new-token row stride must be >= %lld and a multiple of 8",
               (long long)row);
    AppendParams p;
    p.k_new = k_new;
    p.v_new = v_new;
    p.max_new = max_new;
    p.k_pool = lp->k_pool;
    p.v_pool = lp->v_pool;
    p.k_scales = lp->k_scales;
    p.v_scales = lp->v_scales;
    p.staging_k = lp->staging_k;
    p.staging_v = lp->staging_v;
    p.block_tables = block_tables;
    p.max_blocks = L->max_blocks;
    p.seq_lens = seq_lens;
    p.n_new = n_new;
    p.P = L->page_size;
    // element offsets within a page (< 64 * row) divide exactly by the FastDiv of row while row <= 8192
    MG_REQUIRE(row <= 8192, "num_kv_heads * head_dim must be at most 8192 for the append, got %lld", (long long)row);
    p.row = static_cast<int32_t>(row);
    p.rowdiv = FastDiv(static_cast<uint32_t>(row));
    p.D = L->head_dim;
    p.scale_th = L->scale_layout == MG_SCALE_TOKEN_HEAD;
    p.num_pages = L->num_pages;
    p.status = dev_status;
    p.new_stride = new_stride;
    p.rope_cos = rope_cos;
    p.rope_sin = rope_sin;
    p.rope_rows = rope_rows;
    p.Hq = num_q_heads;
    p.q_src = static_cast<const __half*>(q_src);
    p.q_out = static_cast<__half*>(q_out);
    const int64_t touch = (static_cast<int64_t>(max_new) + L->page_size - 1) / L->page_size + 1;
    MG_REQUIRE(touch <= 65535,
               "max_new %d spans %lld pages of %d tokens; one append takes at most 65534 pages per sequence "
               "(split the prefill into several steps)",
               max_new, (long long)touch - 1, L->page_size);
    dim3 grid(batch, static_cast<unsigned>(touch), rope_cos ? 3 : 2);
    const bool i4 = L->kv_dtype == MG_KV_INT4;
    const bool s16 = L->staging_dtype == MG_F16, n16 = new_dtype == MG_F16;
    cudaStream_t s = as_stream(stream);
    const bool small = static_cast<int64_t>(L->page_size) * p.row <= static_cast<int64_t>(kAppendThreads) * 8 * 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAppendThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = early_launch ? 1 : 0;
    p.release_early = early_launch ? 1 : 0;
    auto go = [&](auto keep) {
        constexpr int K = decltype(keep)::value;
        if (!i4 && s16 && n16) cudaLaunchKernelEx(&cfg, kv_append_kernel<false, __half, __half, K>, p);
        else if (!i4 && !s16 && n16) cudaLaunchKernelEx(&cfg, kv_append_kernel<false, float, __half, K>, p);
        else if (!i4 && !s16 && !n16) cudaLaunchKernelEx(&cfg, kv_append_kernel<false, float, float, K>, p);
        else if (i4 && s16 && n16) cudaLaunchKernelEx(&cfg, kv_append_kernel<true, __half, __half, K>, p);
        else if (i4 && !s16 && n16) cudaLaunchKernelEx(&cfg, kv_append_kernel<true, float, __half, K>, p);
        else cudaLaunchKernelEx(&cfg, kv_append_kernel<true, float, float, K>, p);
    };
    if (small) go(std::integral_constant<int, 2>{});
    else go(std::integral_constant<int, 8>{});
    return check_launch("kv_append_kernel");
}

}  // namespace
}  // namespace mg

extern "C" mg_status mg_kv_append(const mg_cache_layout* L, const mg_layer_ptrs* lp, const int32_t* block_tables,
                                  const int32_t* seq_lens, const int32_t* n_new, int32_t batch, const void* k_new,
                                  const void* v_new, int32_t new_dtype, int32_t max_new, int32_t* dev_status,
                                  mg_stream_t stream) {
    const int64_t row = L ? static_cast<int64_t>(L->num_kv_heads) * L->head_dim : 0;
    return mg::append_launch(L, lp, block_tables, seq_lens, n_new, batch, k_new, v_new, new_dtype, max_new, row,
                             nullptr, nullptr, 0, 0, nullptr, nullptr, dev_status, stream);
}

extern "C" mg_status mg_kv_append_flags(const mg_cache_layout* L, const mg_layer_ptrs* lp,
                                        const int32_t* block_tables, const int32_t* seq_lens, const int32_t* n_new,
                                        int32_t batch, const void* k_new, const void* v_new, int32_t new_dtype,
                                        int32_t max_new, uint32_t flags, int32_t* dev_status, mg_stream_t stream) {
    MG_REQUIRE((flags & ~MG_APPEND_EARLY_LAUNCH) == 0, "unknown append flags 0x%x", flags);
    const int64_t row = L ? static_cast<int64_t>(L->num_kv_heads) * L->head_dim : 0;
    return mg::append_launch(L, lp, block_tables, seq_lens, n_new, batch, k_new, v_new, new_dtype, max_new, row,
                             nullptr, nullptr, 0, 0, nullptr, nullptr, dev_status, stream,
                             (flags & MG_APPEND_EARLY_LAUNCH) != 0);
}

extern "C" mg_status mg_kv_append_rope(const mg_cache_layout* L, const mg_layer_ptrs* lp,
                                       const int32_t* block_tables, const int32_t* seq_lens, const int32_t* n_new,
                                       int32_t batch, const void* qkv, int32_t num_q_heads, const float* cos_table,
                                       const float* sin_table, int32_t table_rows, void* q_out, int32_t max_new,
                                       int32_t* dev_status, mg_stream_t stream) {
    MG_REQUIRE(L != nullptr, "null layout");
    MG_REQUIRE(L->staging_dtype == MG_F16, "the rotary append takes fp16 tokens into fp16 staging");
    MG_REQUIRE(num_q_heads >= 1 && L->head_dim % 16 == 0, "num_q_heads must be positive and head_dim % 16 == 0");
    MG_REQUIRE(qkv && cos_table && sin_table && q_out && table_rows >= 1, "null pointer or empty rotary table");
    MG_REQUIRE(aligned16(q_out), "q_out must be 16-byte aligned");
    const int64_t D = L->head_dim, hkv = L->num_kv_heads;
    const int64_t stride = (num_q_heads + 2 * hkv) * D;
    const __half* base = static_cast<const __half*>(qkv);
    return mg::append_launch(L, lp, block_tables, seq_lens, n_new, batch, base + num_q_heads * D,
                             base + (num_q_heads + hkv) * D, MG_F16, max_new, stride, cos_table, sin_table,
                             table_rows, num_q_heads, qkv, q_out, dev_status, stream);
}

extern "C" mg_status mg_gather_dequant(const mg_cache_layout* L, const mg_layer_ptrs* lp, const int32_t* block_tables,
                                       const int32_t* seq_lens, const int32_t* cu_seqlens, int32_t batch,
                                       int32_t max_context, int32_t include_staging, void* out_k, void* out_v,
                                       int32_t out_dtype, int32_t* dev_status, mg_stream_t stream) {
    mg_status st = check_layout(L);
    if (st != MG_OK) return st;
    MG_REQUIRE(lp != nullptr, "null layer pointers");
    MG_REQUIRE(batch >= 0 && max_context >= 0, "batch and max_context must be >= 0");
    if (batch == 0 || max_context == 0) return MG_OK;
    MG_REQUIRE(out_dtype == MG_F32 || out_dtype == MG_F16, "out_dtype must be MG_F32 or MG_F16");
    MG_REQUIRE(block_tables && seq_lens && cu_seqlens && out_k && out_v, "null pointer");
    MG_REQUIRE(aligned16(out_k) && aligned16(out_v), "outputs must be 16-byte aligned");
    GatherParams p;
    p.k_pool = lp->k_pool;
    p.v_pool = lp->v_pool;
    p.k_scales = lp->k_scales;
    p.v_scales = lp->v_scales;
    p.staging_k = lp->staging_k;
    p.staging_v = lp->staging_v;
    p.block_tables = block_tables;
    p.max_blocks = L->max_blocks;
    p.seq_lens = seq_lens;
    p.cu_seqlens = cu_seqlens;
    p.P = L->page_size;
    p.row = L->num_kv_heads * L->head_dim;
    p.D = L->head_dim;
    p.scale_th = L->scale_layout == MG_SCALE_TOKEN_HEAD;
    p.num_pages = L->num_pages;
    p.include_staging = include_staging;
    p.out_k = out_k;
    p.out_v = out_v;
    p.status = dev_status;
    dim3 grid(max_context / L->page_size + 1, batch, 2);
    const bool i4 = L->kv_dtype == MG_KV_INT4;
    const bool s16 = L->staging_dtype == MG_F16, o16 = out_dtype == MG_F16;
    cudaStream_t s = as_stream(stream);
    if (!i4) {
        if (s16 && o16) gather_dequant_kernel<false, __half, __half><<<grid, kGatherThreads, 0, s>>>(p);
        else if (s16) gather_dequant_kernel<false, __half, float><<<grid, kGatherThreads, 0, s>>>(p);
        else if (o16) gather_dequant_kernel<false, float, __half><<<grid, kGatherThreads, 0, s>>>(p);
        else gather_dequant_kernel<false, float, float><<<grid, kGatherThreads, 0, s>>>(p);
    } else {
        if (s16 && o16) gather_dequant_kernel<true, __half, __half><<<grid, kGatherThreads, 0, s>>>(p);
        else if (s16) gather_dequant_kernel<true, __half, float><<<grid, kGatherThreads, 0, s>>>(p);
        else if (o16) gather_dequant_kernel<true, float, __half><<<grid, kGatherThreads, 0, s>>>(p);
        else gather_dequant_kernel<true, float, float><<<grid, kGatherThreads, 0, s>>>(p);
    }
    return check_launch("gather_dequant_kernel");
}
