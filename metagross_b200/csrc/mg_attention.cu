// Fused paged decode attention over quantized pages (INT8 or packed INT4) plus
// the exact staged tail, for a batch of sequences.
//
// Reference semantics: csrc/paged_attention.cu:25-135 (committed pages, two
// passes, one warp per query head) + metagross/attention.py:62-134 (staging
// tail in torch, log-sum-exp merge, normalisation).  Here everything is one
// kernel with one online softmax:
//
//   grid  = (num_splits, batch); CTA = NW warps; warp w owns kv heads
//           w, w+NW, ... (all q heads of each head's GQA group)
//   pages = whole physical pages ([P, Hkv, row] contiguous, K then V) are
//           staged in shared memory by 1-D bulk copies (cp.async.bulk,
//           mbarrier complete_tx), NSTAGES deep
//   math  = per 16-token tile and kv head, S^T = K Q^T and O^T += V^T P^T on
//           the tensor cores (mma.sync m16n8k16, fp16 in, fp32 accumulate).
//           Codes are exact in fp16 (|q| <= 127) and converted in registers
//           with the 0x6400 exponent trick (no I2F); the page scale is applied
//           to the fp32 scores (K) and folded into P (V).  fp32 queries and
//           all small groups (G <= 4) carry q and P as hi+lo fp16 pairs in
//           two mma columns, which keeps ~22 mantissa bits.
//   tail  = the r < P staged tokens of the split that owns them are merged in
//           fp32 on the CUDA cores into the same running softmax state.
//   split = splits write (m, l, acc) partials; the last CTA of a sequence
//           (atomic ticket, no waiting) merges them and writes the output.
#include "mg_common.cuh"

namespace mg {
namespace {

constexpr int kMaxStages = 16;
constexpr int kMaxPagesPerStage = 16;
constexpr uint32_t kWaitTries = 1u << 20;

struct DecodeParams {
    const void* q;
    int q_f16;
    const uint8_t* k_pool;
    const uint8_t* v_pool;
    const float* k_scales;
    const float* v_scales;
    const void* staging_k;
    const void* staging_v;
    int st_f16;
    int has_staging;
    const int32_t* block_tables;
    int32_t max_blocks;
    const int32_t* seq_lens;
    int32_t uniform_len;  // >= 0: every sequence has this many committed tokens (legacy op)
    int Hq, Hkv, G, P;
    FastDiv pdiv;
    int page_bytes;
    int pages_per_split, num_splits;
    int pages_per_stage, nstages;
    int nwarps;
    float sm_scale_log2;
    int64_t num_pages;
    void* out;
    int out_f16;
    float* out_wv;  // unnormalised outputs (legacy op) when non-null
    float* out_l;
    float* out_m;
    float* ws_acc;
    float* ws_m;
    float* ws_l;
    uint32_t* tickets;
    int32_t* status;
};

template <bool KV4, int HD, int NT>
struct Cfg {
    static constexpr int KSTEPS = HD / 16;
    static constexpr int MTILES = HD / 16;
    static constexpr int ROWB = KV4 ? HD / 2 : HD;  // bytes per (token, head) row
    static constexpr int KCHB = ROWB / 4;           // K bytes per lane per row
    static constexpr int VCHB = ROWB / 8;           // V bytes per lane per token
    static constexpr int VE = HD / 8;               // d values per lane
    static constexpr int MAXHPW = (HD == 64 && NT == 1) ? 4 : ((HD == 128 && NT == 2) ? 1 : 2);
};

template <int BYTES>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t (&w)[BYTES / 4]) {
    if constexpr (BYTES == 4) {
        w[0] = *reinterpret_cast<const uint32_t*>(p);
    } else if constexpr (BYTES == 8) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        w[0] = v.x; w[1] = v.y;
    } else if constexpr (BYTES == 16) {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else {
        static_assert(BYTES == 32, "row chunk");
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        const uint4 u = *reinterpret_cast<const uint4*>(p + 16);
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
        w[4] = u.x; w[5] = u.y; w[6] = u.z; w[7] = u.w;
    }
}

// d index (within the head) of K-fragment slot s (0: k=2c, 1: 2c+1, 2: 2c+8,
// 3: 2c+9) of k-step kk for lane column c.  Must match k_frag() below.
template <bool KV4, int HD>
__device__ __forceinline__ int k_slot_d(int kk, int c, int s) {
    if (!KV4) {
        // word kk of the lane's 16/32-byte chunk; a0 = bytes (0,2), a2 = bytes (1,3)
        const int off[4] = {0, 2, 1, 3};
        return (HD / 4) * c + 4 * kk + off[s];
    } else {
        // word kk>>1 (8 nibbles); h = kk&1 picks nibbles (2h,2h+4) and (2h+1,2h+5)
        const int off[4] = {0, 4, 1, 5};
        return (HD / 4) * c + 8 * (kk >> 1) + 2 * (kk & 1) + off[s];
    }
}

// K A-fragment registers (a0/a2 for one row) of k-step kk from the row's words.
template <bool KV4>
__device__ __forceinline__ void k_frag_row(const uint32_t* w, int kk, uint32_t& lo, uint32_t& hi) {
    if (!KV4) {
        const uint32_t x = w[kk];
        lo = s8pair_to_half2(x);       // bytes 0, 2
        hi = s8pair_to_half2(x >> 8);  // bytes 1, 3
    } else {
        const uint32_t x = w[kk >> 1] ^ 0x88888888u;
        const uint32_t y = (kk & 1) ? (x >> 8) : x;
        lo = s4pair_lo_to_half2(y);  // nibbles (2h, 2h+4)
        hi = s4pair_hi_to_half2(y);  // nibbles (2h+1, 2h+5)
    }
}

// V A-fragment pairs for one token pair (A at k-slot 2c[+8], B at 2c+1[+9]).
// Produces, for each m-tile mt, (row d0 = VE*g + 2mt, row d1 = d0 + 1) half2s
// holding (A, B) codes.
template <bool KV4, int HD>
__device__ __forceinline__ void v_pairs(const uint32_t* wa, const uint32_t* wb, uint32_t (&r0)[HD / 16],
                                        uint32_t (&r1)[HD / 16]) {
    if (!KV4) {
#pragma unroll
        for (int wi = 0; wi < HD / 32; ++wi) {  // VE/4 words per token
            const uint32_t X = __byte_perm(wa[wi], wb[wi], 0x5410);  // A0 A1 B0 B1
            const uint32_t Y = __byte_perm(wa[wi], wb[wi], 0x7632);  // A2 A3 B2 B3
            r0[2 * wi] = s8pair_to_half2(X);
            r1[2 * wi] = s8pair_to_half2(X >> 8);
            r0[2 * wi + 1] = s8pair_to_half2(Y);
            r1[2 * wi + 1] = s8pair_to_half2(Y >> 8);
        }
    } else {
#pragma unroll
        for (int wi = 0; wi < HD / 64; ++wi) {  // 8 nibbles per word
            const uint32_t X = __byte_perm(wa[wi], wb[wi], 0x5410) ^ 0x88888888u;
            const uint32_t Y = __byte_perm(wa[wi], wb[wi], 0x7632) ^ 0x88888888u;
            r0[4 * wi + 0] = s4pair_lo_to_half2(X);
            r1[4 * wi + 0] = s4pair_hi_to_half2(X);
            r0[4 * wi + 1] = s4pair_lo_to_half2(X >> 8);
            r1[4 * wi + 1] = s4pair_hi_to_half2(X >> 8);
            r0[4 * wi + 2] = s4pair_lo_to_half2(Y);
            r1[4 * wi + 2] = s4pair_hi_to_half2(Y);
            r0[4 * wi + 3] = s4pair_lo_to_half2(Y >> 8);
            r1[4 * wi + 3] = s4pair_hi_to_half2(Y >> 8);
        }
    }
}

__device__ __forceinline__ float load_f(const void* p, int64_t i, int f16) {
    return f16 ? __half2float(static_cast<const __half*>(p)[i]) : static_cast<const float*>(p)[i];
}

template <bool KV4, int HD, int NT, bool SPLIT>
__global__ void __launch_bounds__(256) paged_decode_kernel(const DecodeParams p) {
    using C = Cfg<KV4, HD, NT>;
    constexpr int MAXHPW = C::MAXHPW;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[kMaxStages];
    __shared__ float sm_ks[kMaxStages][kMaxPagesPerStage];
    __shared__ float sm_vs[kMaxStages][kMaxPagesPerStage];
    __shared__ int sm_flag;

    const int split = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int P = p.P;

    if (p.status && (*(volatile int32_t*)p.status & (MG_DEV_OUT_OF_PAGES | MG_DEV_BLOCK_TABLE_FULL))) return;

    // ---- work of this CTA --------------------------------------------------
    const int len = p.uniform_len >= 0 ? p.uniform_len : p.seq_lens[b];
    const int n_pages = len / P;
    const int tail = p.has_staging ? len - n_pages * P : 0;
    const int pps = p.pages_per_split, S = p.num_splits;
    const int with_pages = (n_pages + pps - 1) / pps;
    const int s_tail = min(n_pages / pps, S - 1);
    const int nwork = tail > 0 ? max(with_pages, s_tail + 1) : with_pages;
    const int64_t out_row0 = static_cast<int64_t>(b) * p.Hq;

    if (nwork == 0) {  // empty sequence: zeros (normalised) / (0, 0, -inf) (unnormalised)
        if (split == 0) {
            for (int i = tid; i < p.Hq * HD; i += blockDim.x) {
                if (p.out_wv) {
                    p.out_wv[out_row0 * HD + i] = 0.0f;
                } else if (p.out_f16) {
                    static_cast<__half*>(p.out)[out_row0 * HD + i] = __float2half(0.0f);
                } else {
                    static_cast<float*>(p.out)[out_row0 * HD + i] = 0.0f;
                }
            }
            if (p.out_wv)
                for (int i = tid; i < p.Hq; i += blockDim.x) {
                    p.out_l[out_row0 + i] = 0.0f;
                    p.out_m[out_row0 + i] = -INFINITY;
                }
        }
        return;
    }
    if (with_pages > S) {  // max_context given to the launch was too small for this sequence
        if (split == 0 && tid == 0) flag(p.status, MG_DEV_CONTEXT_OVERFLOW);
        return;
    }
    if (split >= nwork) return;
    const int p0 = split * pps;
    const int p1 = min(p0 + pps, n_pages);
    const int n_lp = max(p1 - p0, 0);
    const bool has_tail = tail > 0 && split == s_tail;

    const int Hkv = p.Hkv, G = p.G;
    const int page_bytes = p.page_bytes;
    const int PPS = p.pages_per_stage, NST = p.nstages;
    const int stage_bytes = PPS * 2 * page_bytes;
    const int n_st = (n_lp + PPS - 1) / PPS;
    const int32_t* bt = p.block_tables + static_cast<int64_t>(b) * p.max_blocks;

    if (tid == 0) {
        for (int i = 0; i < NST; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();

    auto issue = [&](int si) {
        const int slot = si % NST;
        const int pa = p0 + si * PPS;
        const int np = min(PPS, p1 - pa);
        uint8_t* dst = smem + static_cast<int64_t>(slot) * stage_bytes;
        for (int k = 0; k < np; ++k) {
            int32_t pid = bt[pa + k];
            if (pid < 0 || pid >= p.num_pages) {
                flag(p.status, MG_DEV_BAD_PAGE_ID);
                pid = 0;
            }
            sm_ks[slot][k] = p.k_scales[pid];
            sm_vs[slot][k] = p.v_scales[pid];
        }
        mbar_arrive_expect_tx(&bars[slot], static_cast<uint32_t>(np) * 2u * page_bytes);
        for (int k = 0; k < np; ++k) {
            int32_t pid = bt[pa + k];
            if (pid < 0 || pid >= p.num_pages) pid = 0;
            const int64_t off = static_cast<int64_t>(pid) * page_bytes;
            bulk_g2s(dst + static_cast<int64_t>(k) * 2 * page_bytes, p.k_pool + off, page_bytes, &bars[slot]);
            bulk_g2s(dst + static_cast<int64_t>(k) * 2 * page_bytes + page_bytes, p.v_pool + off, page_bytes,
                     &bars[slot]);
        }
    };
    if (tid == 0)
        for (int si = 0; si < min(NST, n_st); ++si) issue(si);

    // ---- per-warp state -----------------------------------------------------
    const int nw = p.nwarps;
    uint32_t qf[MAXHPW][NT][C::KSTEPS][2];
    float acc[MAXHPW][C::MTILES][NT][4];
    float mrun[MAXHPW][NT][2], lpart[MAXHPW][NT][2];

#pragma unroll
    for (int hh = 0; hh < MAXHPW; ++hh) {
        const int h = warp + hh * nw;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            // B-fragment column g of n-tile nt
            const int gi = SPLIT ? nt * 4 + (g >> 1) : nt * 8 + g;
            const bool live = h < Hkv && gi < G;
            const int64_t qrow = (out_row0 + static_cast<int64_t>(h) * G + gi) * HD;
#pragma unroll
            for (int kk = 0; kk < C::KSTEPS; ++kk) {
                float v[4];
#pragma unroll
                for (int s = 0; s < 4; ++s) v[s] = live ? load_f(p.q, qrow + k_slot_d<KV4, HD>(kk, c, s), p.q_f16) : 0.0f;
                if (SPLIT) {
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const float hi = __half2float(__float2half_rn(v[s]));
                        v[s] = (g & 1) ? (v[s] - hi) : hi;  // column pair (hi, lo)
                    }
                }
                qf[hh][nt][kk][0] = pack_half2(v[0], v[1]);
                qf[hh][nt][kk][1] = pack_half2(v[2], v[3]);
            }
            mrun[hh][nt][0] = mrun[hh][nt][1] = -INFINITY;
            lpart[hh][nt][0] = lpart[hh][nt][1] = 0.0f;
#pragma unroll
            for (int mt = 0; mt < C::MTILES; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[hh][mt][nt][i] = 0.0f;
        }
    }

    // ---- main loop over staged pages ----------------------------------------
    const float sscale = p.sm_scale_log2;
    bool timed_out = false;
    for (int si = 0; si < n_st; ++si) {
        const int slot = si % NST;
        const bool ok = mbar_wait_bounded(&bars[slot], (si / NST) & 1, kWaitTries);
        if (__syncthreads_or(!ok)) {
            timed_out = true;
            break;
        }
        const uint8_t* stage = smem + static_cast<int64_t>(slot) * stage_bytes;
        const int np = min(PPS, p1 - (p0 + si * PPS));
        const int ntok = np * P;
        const int ntiles = (ntok + 15) >> 4;

#pragma unroll
        for (int hh = 0; hh < MAXHPW; ++hh) {
            const int h = warp + hh * nw;
            if (h >= Hkv) continue;
            for (int tt = 0; tt < ntiles; ++tt) {
                // K rows g and g+8 of the tile
                const int x0 = tt * 16 + g, x1 = x0 + 8;
                const bool v0 = x0 < ntok, v1 = x1 < ntok;
                const int k0 = p.pdiv.div(v0 ? x0 : 0), k1 = p.pdiv.div(v1 ? x1 : 0);
                const int t0 = (v0 ? x0 : 0) - k0 * P, t1 = (v1 ? x1 : 0) - k1 * P;
                const uint8_t* kr0 = stage + (2 * k0) * page_bytes + (t0 * Hkv + h) * C::ROWB;
                const uint8_t* kr1 = stage + (2 * k1) * page_bytes + (t1 * Hkv + h) * C::ROWB;
                uint32_t w0[C::KCHB / 4], w1[C::KCHB / 4];
                lds_words<C::KCHB>(kr0 + c * C::KCHB, w0);
                lds_words<C::KCHB>(kr1 + c * C::KCHB, w1);
                float sc[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) sc[nt][i] = 0.0f;
#pragma unroll
                for (int kk = 0; kk < C::KSTEPS; ++kk) {
                    uint32_t a[4];
                    k_frag_row<KV4>(w0, kk, a[0], a[2]);
                    k_frag_row<KV4>(w1, kk, a[1], a[3]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) mma_16816(sc[nt], a, qf[hh][nt][kk][0], qf[hh][nt][kk][1]);
                }
                const float ks0 = v0 ? sm_ks[slot][k0] * sscale : 0.0f;
                const float ks1 = v1 ? sm_ks[slot][k1] * sscale : 0.0f;
                const float vs0 = sm_vs[slot][k0], vs1 = sm_vs[slot][k1];

                // online softmax update, P^T fragments
                uint32_t pb[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float s_g[2], s_g8[2];
                    if (SPLIT) {
                        s_g[0] = v0 ? (sc[nt][0] + sc[nt][1]) * ks0 : -INFINITY;
                        s_g8[0] = v1 ? (sc[nt][2] + sc[nt][3]) * ks1 : -INFINITY;
                    } else {
                        s_g[0] = v0 ? sc[nt][0] * ks0 : -INFINITY;
                        s_g[1] = v0 ? sc[nt][1] * ks0 : -INFINITY;
                        s_g8[0] = v1 ? sc[nt][2] * ks1 : -INFINITY;
                        s_g8[1] = v1 ? sc[nt][3] * ks1 : -INFINITY;
                    }
                    float pr_g[2], pr_g8[2];
#pragma unroll
                    for (int col = 0; col < (SPLIT ? 1 : 2); ++col) {
                        float mx = fmaxf(s_g[col], s_g8[col]);
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                        const float m_old = mrun[hh][nt][col];
                        const float m_new = fmaxf(m_old, mx);
                        const float alpha = ex2(m_old - m_new);
                        pr_g[col] = ex2(s_g[col] - m_new);
                        pr_g8[col] = ex2(s_g8[col] - m_new);
                        lpart[hh][nt][col] = lpart[hh][nt][col] * alpha + pr_g[col] + pr_g8[col];
                        mrun[hh][nt][col] = m_new;
                        if (SPLIT) {
#pragma unroll
                            for (int mt = 0; mt < C::MTILES; ++mt)
#pragma unroll
                                for (int i = 0; i < 4; ++i) acc[hh][mt][nt][i] *= alpha;
                        } else {
#pragma unroll
                            for (int mt = 0; mt < C::MTILES; ++mt) {
                                acc[hh][mt][nt][col] *= alpha;
                                acc[hh][mt][nt][col + 2] *= alpha;
                            }
                        }
                    }
                    uint32_t h_g, h_g8;
                    if (SPLIT) {
                        const float a0 = pr_g[0] * vs0, a1 = pr_g8[0] * vs1;
                        const float a0h = __half2float(__float2half_rn(a0));
                        const float a1h = __half2float(__float2half_rn(a1));
                        h_g = pack_half2(a0h, a0 - a0h);
                        h_g8 = pack_half2(a1h, a1 - a1h);
                    } else {
                        h_g = pack_half2(pr_g[0] * vs0, pr_g[1] * vs0);
                        h_g8 = pack_half2(pr_g8[0] * vs1, pr_g8[1] * vs1);
                    }
                    pb[nt][0] = movmatrix_trans(h_g);
                    pb[nt][1] = movmatrix_trans(h_g8);
                }

                // V tokens 2c, 2c+1, 2c+8, 2c+9 of the tile
                uint32_t wv[4][C::VCHB / 4 > 0 ? C::VCHB / 4 : 1];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int x = tt * 16 + 2 * c + (r & 1) + (r >> 1) * 8;
                    const int xx = x < ntok ? x : 0;
                    const int kq = p.pdiv.div(xx);
                    const int tq = xx - kq * P;
                    const uint8_t* vr = stage + (2 * kq + 1) * page_bytes + (tq * Hkv + h) * C::ROWB + g * C::VCHB;
                    lds_words<C::VCHB>(vr, wv[r]);
                }
                uint32_t r0a[C::MTILES], r1a[C::MTILES], r0b[C::MTILES], r1b[C::MTILES];
                v_pairs<KV4, HD>(wv[0], wv[1], r0a, r1a);
                v_pairs<KV4, HD>(wv[2], wv[3], r0b, r1b);
#pragma unroll
                for (int mt = 0; mt < C::MTILES; ++mt) {
                    const uint32_t a[4] = {r0a[mt], r1a[mt], r0b[mt], r1b[mt]};
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) mma_16816(acc[hh][mt][nt], a, pb[nt][0], pb[nt][1]);
                }
            }
        }
        __syncthreads();
        if (tid == 0 && si + NST < n_st) {
            fence_proxy_async_smem();
            issue(si + NST);
        }
    }
    if (timed_out) {
        if (tid == 0) {
            flag(p.status, MG_DEV_TIMEOUT);
            // bounded drain of the copies this CTA still has in flight
            for (int sj = 0; sj < n_st; ++sj) (void)mbar_wait_bounded(&bars[sj % NST], (sj / NST) & 1, 1024);
        }
        return;
    }

    // ---- exact staged tail (fp32, CUDA cores), merged into the same state -----
    if (has_tail) {
        const int64_t st_base = static_cast<int64_t>(b) * P * Hkv * HD;
#pragma unroll
        for (int hh = 0; hh < MAXHPW; ++hh) {
            const int h = warp + hh * nw;
            if (h >= Hkv) continue;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int col = 0; col < (SPLIT ? 1 : 2); ++col) {
                    const int gi = SPLIT ? nt * 4 + c : nt * 8 + 2 * c + col;
                    const bool live = gi < G;
                    const int64_t qrow = (out_row0 + static_cast<int64_t>(h) * G + (live ? gi : 0)) * HD;
                    float qv[C::VE];
#pragma unroll
                    for (int e = 0; e < C::VE; ++e) qv[e] = load_f(p.q, qrow + C::VE * g + e, p.q_f16);
                    for (int t = 0; t < tail; ++t) {
                        const int64_t rbase = st_base + (static_cast<int64_t>(t) * Hkv + h) * HD + C::VE * g;
                        float part = 0.0f;
#pragma unroll
                        for (int e = 0; e < C::VE; ++e) part += qv[e] * load_f(p.staging_k, rbase + e, p.st_f16);
                        part += __shfl_xor_sync(0xffffffffu, part, 4);
                        part += __shfl_xor_sync(0xffffffffu, part, 8);
                        part += __shfl_xor_sync(0xffffffffu, part, 16);
                        const float s = part * sscale;
                        const float m_old = mrun[hh][nt][col];
                        const float m_new = fmaxf(m_old, s);
                        const float alpha = ex2(m_old - m_new);
                        const float pr = ex2(s - m_new);
                        lpart[hh][nt][col] = lpart[hh][nt][col] * alpha + (g == 0 ? pr : 0.0f);
                        mrun[hh][nt][col] = m_new;
                        // acc columns of this head: SPLIT -> (0,1) [+2 rows], else col [+2]
#pragma unroll
                        for (int mt = 0; mt < C::MTILES; ++mt) {
                            const float vd0 = load_f(p.staging_v, rbase + 2 * mt, p.st_f16);
                            const float vd1 = load_f(p.staging_v, rbase + 2 * mt + 1, p.st_f16);
                            if (SPLIT) {
                                acc[hh][mt][nt][0] = acc[hh][mt][nt][0] * alpha + pr * vd0;
                                acc[hh][mt][nt][1] *= alpha;
                                acc[hh][mt][nt][2] = acc[hh][mt][nt][2] * alpha + pr * vd1;
                                acc[hh][mt][nt][3] *= alpha;
                            } else {
                                acc[hh][mt][nt][col] = acc[hh][mt][nt][col] * alpha + pr * vd0;
                                acc[hh][mt][nt][col + 2] = acc[hh][mt][nt][col + 2] * alpha + pr * vd1;
                            }
                        }
                    }
                }
            }
        }
    }

    // ---- epilogue: per-head (m, l, acc) -> output or split partial ------------
    const bool single = nwork == 1;
    const float ln2 = 0.6931471805599453f;
#pragma unroll
    for (int hh = 0; hh < MAXHPW; ++hh) {
        const int h = warp + hh * nw;
        if (h >= Hkv) continue;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int col = 0; col < (SPLIT ? 1 : 2); ++col) {
                float l = lpart[hh][nt][col];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                const int gi = SPLIT ? nt * 4 + c : nt * 8 + 2 * c + col;
                if (gi >= G) continue;
                const int hq = h * G + gi;
                float o[C::VE];
#pragma unroll
                for (int mt = 0; mt < C::MTILES; ++mt) {
                    if (SPLIT) {
                        o[2 * mt] = acc[hh][mt][nt][0] + acc[hh][mt][nt][1];
                        o[2 * mt + 1] = acc[hh][mt][nt][2] + acc[hh][mt][nt][3];
                    } else {
                        o[2 * mt] = acc[hh][mt][nt][col];
                        o[2 * mt + 1] = acc[hh][mt][nt][col + 2];
                    }
                }
                const float m = mrun[hh][nt][col];
                if (single) {
                    const int64_t base = (out_row0 + hq) * HD + C::VE * g;
                    if (p.out_wv) {
#pragma unroll
                        for (int e = 0; e < C::VE; ++e) p.out_wv[base + e] = o[e];
                        if (g == 0) {
                            p.out_l[out_row0 + hq] = l;
                            p.out_m[out_row0 + hq] = m * ln2;
                        }
                    } else {
                        const float inv = 1.0f / l;
                        if (p.out_f16) {
                            __half* op = static_cast<__half*>(p.out) + base;
#pragma unroll
                            for (int e = 0; e < C::VE; e += 2)
                                *reinterpret_cast<__half2*>(op + e) = __floats2half2_rn(o[e] * inv, o[e + 1] * inv);
                        } else {
                            float* op = static_cast<float*>(p.out) + base;
#pragma unroll
                            for (int e = 0; e < C::VE; e += 4)
                                *reinterpret_cast<float4*>(op + e) =
                                    make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
                        }
                    }
                } else {
                    const int64_t prow = (static_cast<int64_t>(b) * S + split) * p.Hq + hq;
                    float* wp = p.ws_acc + prow * HD + C::VE * g;
#pragma unroll
                    for (int e = 0; e < C::VE; e += 4)
                        __stcg(reinterpret_cast<float4*>(wp + e), make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]));
                    if (g == 0) {
                        __stcg(p.ws_m + prow, m);
                        __stcg(p.ws_l + prow, l);
                    }
                }
            }
        }
    }
    if (single) return;

    // ---- split merge by the last CTA of this sequence (no waiting) -----------
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const uint32_t prev = atomicAdd(&p.tickets[b], 1u);
        sm_flag = (prev == static_cast<uint32_t>(nwork - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!sm_flag) return;
    __threadfence();
    const int Hq = p.Hq;
    for (int it = tid; it < Hq * (HD / 4); it += blockDim.x) {
        const int hq = it / (HD / 4), d4 = (it - hq * (HD / 4)) * 4;
        float M = -INFINITY;
        for (int j = 0; j < nwork; ++j) M = fmaxf(M, __ldcg(p.ws_m + (static_cast<int64_t>(b) * S + j) * Hq + hq));
        float L = 0.0f;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < nwork; ++j) {
            const int64_t prow = (static_cast<int64_t>(b) * S + j) * Hq + hq;
            const float mj = __ldcg(p.ws_m + prow);
            const float f = (mj == -INFINITY) ? 0.0f : ex2(mj - M);
            L += __ldcg(p.ws_l + prow) * f;
            const float4 v = __ldcg(reinterpret_cast<const float4*>(p.ws_acc + prow * HD + d4));
            a.x += v.x * f;
            a.y += v.y * f;
            a.z += v.z * f;
            a.w += v.w * f;
        }
        const int64_t base = (out_row0 + hq) * HD + d4;
        if (p.out_wv) {
            *reinterpret_cast<float4*>(p.out_wv + base) = a;
            if (d4 == 0) {
                p.out_l[out_row0 + hq] = L;
                p.out_m[out_row0 + hq] = M * ln2;
            }
        } else {
            const float inv = 1.0f / L;
            if (p.out_f16) {
                __half2* op = reinterpret_cast<__half2*>(static_cast<__half*>(p.out) + base);
                op[0] = __floats2half2_rn(a.x * inv, a.y * inv);
                op[1] = __floats2half2_rn(a.z * inv, a.w * inv);
            } else {
                *reinterpret_cast<float4*>(static_cast<float*>(p.out) + base) =
                    make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
            }
        }
    }
    if (tid == 0) p.tickets[b] = 0u;  // leave the workspace reusable
}

// ---------------------------------------------------------------------------
// host-side launch planning
// ---------------------------------------------------------------------------
struct Plan {
    int nt, split_mode, nwarps, maxhpw;
    int pages_per_split, num_splits, pages_per_stage, nstages;
    int64_t smem_bytes;
    int64_t ws_bytes;
};

int max_hpw(int hd, int nt) { return (hd == 64 && nt == 1) ? 4 : ((hd == 128 && nt == 2) ? 1 : 2); }

int pick_warps(int Hkv, int maxhpw) {
    // largest divisor of Hkv that is <= 8 and leaves <= maxhpw heads per warp
    for (int nw = 8; nw >= 1; --nw)
        if (Hkv % nw == 0 && Hkv / nw <= maxhpw) return nw;
    const int nw = (Hkv + maxhpw - 1) / maxhpw;
    return nw <= 8 ? nw : -1;
}

int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

mg_status make_plan(int kv4, int hd, int P, int Hkv, int Hq, int q_f16, int batch, int max_context, Plan* out) {
    MG_REQUIRE(hd == 64 || hd == 128, "attention supports head_dim 64 or 128, got %d", hd);
    MG_REQUIRE(Hkv >= 1 && Hq >= Hkv && Hq % Hkv == 0,
               "num_q_heads (%d) must be an exact multiple of num_kv_heads (%d)", Hq, Hkv);
    const int G = Hq / Hkv;
    Plan pl{};
    if (G <= 4 || !q_f16) {
        pl.split_mode = 1;
        pl.nt = (G + 3) / 4;
    } else {
        pl.split_mode = 0;
        pl.nt = (G + 7) / 8;
    }
    if (pl.nt > 2) return set_error(MG_ERR_UNSUPPORTED, "GQA group %d too large (fp32 q: <= 8, fp16 q: <= 16)", G);
    pl.maxhpw = max_hpw(hd, pl.nt);
    pl.nwarps = pick_warps(Hkv, pl.maxhpw);
    if (pl.nwarps < 1) return set_error(MG_ERR_UNSUPPORTED, "num_kv_heads %d too large for one CTA", Hkv);
    const int rowb = kv4 ? hd / 2 : hd;
    const int64_t page_bytes = static_cast<int64_t>(P) * Hkv * rowb;
    const int64_t pair = 2 * page_bytes;
    if (2 * pair > 200 * 1024)
        return set_error(MG_ERR_UNSUPPORTED, "page of %lld bytes too large to stage twice in shared memory",
                         (long long)page_bytes);
    const int max_pages = max_context / P;
    // pages per split: enough CTAs for ~2 per SM, and enough bytes per split
    // that the partial (Hq*(HD+2) floats) stays small against the pages read
    const int64_t partial = static_cast<int64_t>(Hq) * (hd + 2) * 4;
    int min_pps = static_cast<int>((4 * partial + pair - 1) / pair);
    if (min_pps < 1) min_pps = 1;
    const int target = 2 * sm_count();
    int pps;
    if (max_pages <= 0) {
        pps = 1;
    } else if (batch >= target) {
        pps = max_pages;
    } else {
        const int want = (target + batch - 1) / batch;
        pps = (max_pages + want - 1) / want;
        if (pps < min_pps) pps = min_pps;
        if (pps > max_pages) pps = max_pages;
    }
    pl.pages_per_split = pps;
    pl.num_splits = max_pages <= 0 ? 1 : (max_pages + pps - 1) / pps;
    // stage = whole pages, >= 16 KB when pages are small; ~96 KB of stages
    int ppst = static_cast<int>((16 * 1024 + pair - 1) / pair);
    if (ppst < 1) ppst = 1;
    if (ppst > kMaxPagesPerStage) ppst = kMaxPagesPerStage;
    if (ppst > pps) ppst = pps;
    pl.pages_per_stage = ppst;
    const int64_t stage = ppst * pair;
    int nst = static_cast<int>((96 * 1024) / stage);
    if (nst < 2) nst = 2;
    if (nst > kMaxStages) nst = kMaxStages;
    while (nst > 2 && nst * stage > 200 * 1024) --nst;
    pl.nstages = nst;
    pl.smem_bytes = nst * stage;
    const int64_t S = pl.num_splits;
    // [per-sequence tickets][acc][m][l]: the tickets sit at a fixed offset so
    // that calls with different split counts keep finding them at zero
    pl.ws_bytes = S > 1 ? align_up(static_cast<int64_t>(batch) * 4, 256) + static_cast<int64_t>(batch) * S * Hq * (hd + 2) * 4
                        : 0;
    *out = pl;
    return MG_OK;
}

template <bool KV4, int HD, int NT, bool SPLIT>
mg_status launch_t(const DecodeParams& p, const Plan& pl, int batch, cudaStream_t s) {
    auto k = paged_decode_kernel<KV4, HD, NT, SPLIT>;
    static int64_t attr_set[64] = {0};  // dynamic smem opt-in already granted, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (pl.smem_bytes > 48 * 1024 && (dev < 0 || dev >= 64 || attr_set[dev] < pl.smem_bytes)) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(pl.smem_bytes));
        if (e != cudaSuccess)
            return set_error(MG_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_set[dev] = pl.smem_bytes;
    }
    dim3 grid(pl.num_splits, batch);
    k<<<grid, pl.nwarps * 32, pl.smem_bytes, s>>>(p);
    return check_launch("paged_decode_kernel");
}

template <bool KV4, int HD>
mg_status launch_hd(const DecodeParams& p, const Plan& pl, int batch, cudaStream_t s) {
    if (pl.split_mode) {
        if (pl.nt == 1) return launch_t<KV4, HD, 1, true>(p, pl, batch, s);
        return launch_t<KV4, HD, 2, true>(p, pl, batch, s);
    }
    if (pl.nt == 1) return launch_t<KV4, HD, 1, false>(p, pl, batch, s);
    return launch_t<KV4, HD, 2, false>(p, pl, batch, s);
}

mg_status launch(int kv4, int hd, const DecodeParams& p, const Plan& pl, int batch, cudaStream_t s) {
    if (kv4) return hd == 64 ? launch_hd<true, 64>(p, pl, batch, s) : launch_hd<true, 128>(p, pl, batch, s);
    return hd == 64 ? launch_hd<false, 64>(p, pl, batch, s) : launch_hd<false, 128>(p, pl, batch, s);
}

void fill_common(DecodeParams& p, const Plan& pl, int P, int Hkv, int Hq, int hd, int kv4, double scale,
                 int64_t num_pages) {
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.G = Hq / Hkv;
    p.P = P;
    p.pdiv = FastDiv(static_cast<uint32_t>(P));
    p.page_bytes = P * Hkv * (kv4 ? hd / 2 : hd);
    p.pages_per_split = pl.pages_per_split;
    p.num_splits = pl.num_splits;
    p.pages_per_stage = pl.pages_per_stage;
    p.nstages = pl.nstages;
    p.nwarps = pl.nwarps;
    p.sm_scale_log2 = static_cast<float>(scale * 1.4426950408889634);
    p.num_pages = num_pages;
}

void set_workspace(DecodeParams& p, const Plan& pl, int batch, int Hq, int hd, void* ws) {
    if (pl.num_splits <= 1) {
        p.ws_acc = p.ws_m = p.ws_l = nullptr;
        p.tickets = nullptr;
        return;
    }
    const int64_t n = static_cast<int64_t>(batch) * pl.num_splits * Hq;
    p.tickets = static_cast<uint32_t*>(ws);
    float* f = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + align_up(static_cast<int64_t>(batch) * 4, 256));
    p.ws_acc = f;
    p.ws_m = f + n * hd;
    p.ws_l = p.ws_m + n;
}

}  // namespace
}  // namespace mg

using namespace mg;

extern "C" int64_t mg_paged_attention_committed_workspace_bytes(int64_t num_blocks, int64_t page_size,
                                                                int64_t num_q_heads, int64_t num_kv_heads,
                                                                int64_t head_dim) {
    Plan pl;
    if (make_plan(0, static_cast<int>(head_dim), static_cast<int>(page_size), static_cast<int>(num_kv_heads),
                  static_cast<int>(num_q_heads), 0, 1, static_cast<int>(num_blocks * page_size), &pl) != MG_OK)
        return 0;
    return pl.ws_bytes;
}

extern "C" mg_status mg_paged_attention_committed(const float* query, const int8_t* k_storage,
                                                  const int8_t* v_storage, const float* page_scales_k,
                                                  const float* page_scales_v, const int32_t* block_table,
                                                  int64_t num_blocks, int64_t max_pages, int64_t page_size,
                                                  int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                                  double scale, float* out_wv, float* out_sum, float* out_max,
                                                  void* workspace, int64_t workspace_bytes, int32_t* dev_status,
                                                  mg_stream_t stream) {
    MG_REQUIRE(scale > 0.0 && scale < 1.0 / 0.0 && scale == scale, "attention scale must be positive and finite, got %g",
               scale);
    MG_REQUIRE(page_size >= 1 && page_size <= 64, "page_size must be in [1, 64], got %lld", (long long)page_size);
    MG_REQUIRE(num_blocks >= 0 && num_blocks * page_size < (1ll << 30), "num_blocks out of range");
    MG_REQUIRE(max_pages >= 1, "max_pages must be positive");
    MG_REQUIRE(query && out_wv && out_sum && out_max, "null pointer");
    MG_REQUIRE(num_blocks == 0 || (k_storage && v_storage && page_scales_k && page_scales_v && block_table),
               "null pointer");
    Plan pl;
    mg_status st = make_plan(0, static_cast<int>(head_dim), static_cast<int>(page_size),
                             static_cast<int>(num_kv_heads), static_cast<int>(num_q_heads), 0, 1,
                             static_cast<int>(num_blocks * page_size), &pl);
    if (st != MG_OK) return st;
    MG_REQUIRE(workspace_bytes >= pl.ws_bytes && (pl.ws_bytes == 0 || workspace),
               "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)pl.ws_bytes);
    MG_REQUIRE((reinterpret_cast<uintptr_t>(k_storage) & 15) == 0 && (reinterpret_cast<uintptr_t>(v_storage) & 15) == 0,
               "k/v storage must be 16-byte aligned");
    DecodeParams p{};
    fill_common(p, pl, static_cast<int>(page_size), static_cast<int>(num_kv_heads), static_cast<int>(num_q_heads),
                static_cast<int>(head_dim), 0, scale, max_pages);
    p.q = query;
    p.q_f16 = 0;
    p.k_pool = reinterpret_cast<const uint8_t*>(k_storage);
    p.v_pool = reinterpret_cast<const uint8_t*>(v_storage);
    p.k_scales = page_scales_k;
    p.v_scales = page_scales_v;
    p.has_staging = 0;
    p.block_tables = block_table;
    p.max_blocks = static_cast<int32_t>(num_blocks > 0 ? num_blocks : 1);
    p.seq_lens = nullptr;
    p.uniform_len = static_cast<int32_t>(num_blocks * page_size);
    p.out = nullptr;
    p.out_wv = out_wv;
    p.out_l = out_sum;
    p.out_m = out_max;
    p.status = dev_status;
    set_workspace(p, pl, 1, static_cast<int>(num_q_heads), static_cast<int>(head_dim), workspace);
    return launch(0, static_cast<int>(head_dim), p, pl, 1, as_stream(stream));
}

extern "C" int64_t mg_paged_decode_workspace_bytes(const mg_cache_layout* L, int32_t batch, int32_t num_q_heads,
                                                   int32_t max_context) {
    if (!L) return 0;
    if (max_context <= 0) max_context = L->max_blocks * L->page_size + L->page_size - 1;
    Plan pl;
    if (make_plan(L->kv_dtype == MG_KV_INT4, L->head_dim, L->page_size, L->num_kv_heads, num_q_heads, 1, batch,
                  max_context, &pl) != MG_OK)
        return 0;
    // the fp32-q plan can need more splits' worth of partials than the fp16 one: size for the larger
    Plan pl32;
    if (make_plan(L->kv_dtype == MG_KV_INT4, L->head_dim, L->page_size, L->num_kv_heads, num_q_heads, 0, batch,
                  max_context, &pl32) == MG_OK && pl32.ws_bytes > pl.ws_bytes)
        return pl32.ws_bytes;
    return pl.ws_bytes;
}

namespace mg {
mg_status check_cache_layout(const mg_cache_layout* L);
}

extern "C" mg_status mg_paged_decode_attention(const mg_cache_layout* L, const mg_layer_ptrs* lp,
                                               const int32_t* block_tables, const int32_t* seq_lens, int32_t batch,
                                               const void* q, int32_t q_dtype, int32_t num_q_heads, float scale,
                                               void* out, int32_t out_dtype, int32_t max_context, void* workspace,
                                               int64_t workspace_bytes, int32_t* dev_status, mg_stream_t stream) {
    mg_status st = check_cache_layout(L);
    if (st != MG_OK) return st;
    MG_REQUIRE(lp && lp->k_pool && lp->v_pool && lp->k_scales && lp->v_scales, "null layer pointer");
    MG_REQUIRE(batch >= 0, "batch must be >= 0");
    if (batch == 0) return MG_OK;
    MG_REQUIRE(q && out && block_tables && seq_lens, "null pointer");
    MG_REQUIRE(q_dtype == MG_F32 || q_dtype == MG_F16, "q_dtype must be MG_F32 or MG_F16");
    MG_REQUIRE(out_dtype == MG_F32 || out_dtype == MG_F16, "out_dtype must be MG_F32 or MG_F16");
    MG_REQUIRE(scale > 0.0f && scale < 1.0f / 0.0f, "attention scale must be positive and finite");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(lp->k_pool) & 15) == 0 && (reinterpret_cast<uintptr_t>(lp->v_pool) & 15) == 0,
               "pools must be 16-byte aligned");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0, "out must be 16-byte aligned");
    if (max_context <= 0) max_context = L->max_blocks * L->page_size + L->page_size - 1;
    Plan pl;
    st = make_plan(L->kv_dtype == MG_KV_INT4, L->head_dim, L->page_size, L->num_kv_heads, num_q_heads,
                   q_dtype == MG_F16, batch, max_context, &pl);
    if (st != MG_OK) return st;
    MG_REQUIRE(pl.num_splits <= 1 || (workspace && workspace_bytes >= pl.ws_bytes),
               "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)pl.ws_bytes);
    MG_REQUIRE(pl.num_splits * pl.pages_per_split <= L->max_blocks + pl.pages_per_split,
               "max_context exceeds the block-table width");
    DecodeParams p{};
    fill_common(p, pl, L->page_size, L->num_kv_heads, num_q_heads, L->head_dim, L->kv_dtype == MG_KV_INT4, scale,
                L->num_pages);
    p.q = q;
    p.q_f16 = q_dtype == MG_F16;
    p.k_pool = static_cast<const uint8_t*>(lp->k_pool);
    p.v_pool = static_cast<const uint8_t*>(lp->v_pool);
    p.k_scales = lp->k_scales;
    p.v_scales = lp->v_scales;
    p.staging_k = lp->staging_k;
    p.staging_v = lp->staging_v;
    p.st_f16 = L->staging_dtype == MG_F16;
    p.has_staging = (lp->staging_k && lp->staging_v) ? 1 : 0;
    p.block_tables = block_tables;
    p.max_blocks = L->max_blocks;
    p.seq_lens = seq_lens;
    p.uniform_len = -1;
    p.out = out;
    p.out_f16 = out_dtype == MG_F16;
    p.out_wv = nullptr;
    p.status = dev_status;
    set_workspace(p, pl, batch, num_q_heads, L->head_dim, workspace);
    return launch(L->kv_dtype == MG_KV_INT4, L->head_dim, p, pl, batch, as_stream(stream));
}
