// Body of the fused paged decode-attention kernel (see mg_attention.cuh for
// the design).  Included by the per-format translation units.
#pragma once

#include "mg_attention.cuh"

namespace mg {

// One 16-token tile of one kv head, already in registers: S^T = K Q^T on the
// tensor cores, online softmax update, O^T += V^T P^T.
template <bool KV4, int HD, int NT, bool SPLIT>
__device__ __forceinline__ void attend_tile(HeadState<NT, HD / 16>& S, const TileRegs<KV4, HD>& T) {
    using C = Cfg<KV4, HD, NT>;
    constexpr int NCOLS = SPLIT ? 1 : 2;
    const bool live0 = (T.live & 1u) != 0, live1 = (T.live & 2u) != 0;

    // ---- scores: K rows g, g+8 against the q columns ------------------------------
    float sc[NT][4], sc2[NT][4];  // two accumulation chains (even / odd k-steps)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nt][i] = sc2[nt][i] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < C::KSTEPS; ++kk) {
        uint32_t a[4];
        k_frag_row<KV4>(T.k[0], kk, a[0], a[2]);
        k_frag_row<KV4>(T.k[1], kk, a[1], a[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            if (kk & 1) mma_16816(sc2[nt], a, S.qf[nt][kk][0], S.qf[nt][kk][1]);
            else mma_16816(sc[nt], a, S.qf[nt][kk][0], S.qf[nt][kk][1]);
        }
    }
    const float ks0 = T.ks[0], ks1 = T.ks[1];
    const float vs0 = T.vs[0], vs1 = T.vs[1];

    // ---- online softmax (log2 domain, lazy rescale) ---------------------------------
    float s[NT][NCOLS][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nt][i] += sc2[nt][i];
        if (SPLIT) {
            s[nt][0][0] = live0 ? (sc[nt][0] + sc[nt][1]) * ks0 : -INFINITY;
            s[nt][0][1] = live1 ? (sc[nt][2] + sc[nt][3]) * ks1 : -INFINITY;
        } else {
#pragma unroll
            for (int col = 0; col < NCOLS; ++col) {
                s[nt][col][0] = live0 ? sc[nt][col] * ks0 : -INFINITY;
                s[nt][col][1] = live1 ? sc[nt][2 + col] * ks1 : -INFINITY;
            }
        }
    }
    bool need = false;
    float mx[NT][NCOLS];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int col = 0; col < NCOLS; ++col) {
            float m = fmaxf(s[nt][col][0], s[nt][col][1]);
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
            mx[nt][col] = m;
            S.m_true[nt][col] = fmaxf(S.m_true[nt][col], m);
            need |= m > S.m_used[nt][col] + kRescaleThreshold;
        }
    if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int col = 0; col < NCOLS; ++col) {
                const float m_new = fmaxf(S.m_used[nt][col], mx[nt][col]);
                const float alpha = ex2(S.m_used[nt][col] - m_new);
                S.m_used[nt][col] = m_new;
                S.lpart[nt][col] *= alpha;
                if (SPLIT) {
#pragma unroll
                    for (int mt = 0; mt < C::MTILES; ++mt)
#pragma unroll
                        for (int i = 0; i < 4; ++i) S.acc[mt][nt][i] *= alpha;
                } else {
#pragma unroll
                    for (int mt = 0; mt < C::MTILES; ++mt) {
                        S.acc[mt][nt][col] *= alpha;
                        S.acc[mt][nt][col + 2] *= alpha;
                    }
                }
            }
    }
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        float pr[NCOLS][2];
#pragma unroll
        for (int col = 0; col < NCOLS; ++col)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                pr[col][r] = ex2(s[nt][col][r] - S.m_used[nt][col]);
                S.lpart[nt][col] += pr[col][r];
            }
        uint32_t hrow[2];
        if (SPLIT) {
            const float a0 = pr[0][0] * vs0, a1 = pr[0][1] * vs1;
            const float a0h = __half2float(__float2half_rn(a0));
            const float a1h = __half2float(__float2half_rn(a1));
            hrow[0] = pack_half2(a0h, a0 - a0h);
            hrow[1] = pack_half2(a1h, a1 - a1h);
        } else {
            hrow[0] = pack_half2(pr[0][0] * vs0, pr[NCOLS - 1][0] * vs0);
            hrow[1] = pack_half2(pr[0][1] * vs1, pr[NCOLS - 1][1] * vs1);
        }
        pb[nt][0] = movmatrix_trans(hrow[0]);
        pb[nt][1] = movmatrix_trans(hrow[1]);
    }

    // ---- V: tokens 2c, 2c+1, 2c+8, 2c+9 -------------------------------------------
    uint32_t r0a[C::MTILES], r1a[C::MTILES], r0b[C::MTILES], r1b[C::MTILES];
    v_pairs<KV4, HD>(T.v[0], T.v[1], r0a, r1a);
    v_pairs<KV4, HD>(T.v[2], T.v[3], r0b, r1b);
#pragma unroll
    for (int mt = 0; mt < C::MTILES; ++mt) {
        const uint32_t a[4] = {r0a[mt], r1a[mt], r0b[mt], r1b[mt]};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(S.acc[mt][nt], a, pb[nt][0], pb[nt][1]);
    }
}

template <bool KV4, int HD, int NT, bool SPLIT>
__device__ __forceinline__ void load_q(HeadState<NT, HD / 16>& S, const DecodeParams& p, int b, int h, int g,
                                       int c) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int gi = SPLIT ? nt * 4 + (g >> 1) : nt * 8 + g;  // B-fragment column g
        const bool live = gi < p.G;
        const int64_t qrow = (static_cast<int64_t>(b) * p.Hq + static_cast<int64_t>(h) * p.G + gi) * HD;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
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
            S.qf[nt][kk][0] = pack_half2(v[0], v[1]);
            S.qf[nt][kk][1] = pack_half2(v[2], v[3]);
        }
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            S.m_used[nt][col] = -INFINITY;
            S.m_true[nt][col] = -INFINITY;
            S.lpart[nt][col] = 0.0f;
        }
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) S.acc[mt][nt][i] = 0.0f;
    }
}

// VE consecutive staged values (fp16 or fp32) starting at element index i.
template <int VE>
__device__ __forceinline__ void load_row(const void* base, int64_t i, int f16, float (&v)[VE]) {
    if (f16) {
        const uint4* q = reinterpret_cast<const uint4*>(static_cast<const __half*>(base) + i);
#pragma unroll
        for (int k = 0; k < VE / 8; ++k) {
            const uint4 u = q[k];
            const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(h2[j]);
                v[8 * k + 2 * j] = f.x;
                v[8 * k + 2 * j + 1] = f.y;
            }
        }
    } else {
        const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
#pragma unroll
        for (int k = 0; k < VE / 4; ++k) {
            const float4 f = q[k];
            v[4 * k] = f.x;
            v[4 * k + 1] = f.y;
            v[4 * k + 2] = f.z;
            v[4 * k + 3] = f.w;
        }
    }
}

// The exact staged tail: rows t0, t0 + ts, ... < tail of K at kbase and of V
// at vbase (shared or global memory, layout [t][Hkv][D]), fp32 math on the
// CUDA cores.
template <bool KV4, int HD, int NT, bool SPLIT>
__device__ __forceinline__ void attend_tail(HeadState<NT, HD / 16>& S, const DecodeParams& p, const void* kbase,
                                            const void* vbase, int b, int h, int t0, int ts, int tail, int g,
                                            int c) {
    constexpr int VE = HD / 8;
    constexpr int NCOLS = SPLIT ? 1 : 2;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int col = 0; col < NCOLS; ++col) {
            const int gi = SPLIT ? nt * 4 + c : nt * 8 + 2 * c + col;
            const int gq = gi < p.G ? gi : 0;
            const int64_t qrow = (static_cast<int64_t>(b) * p.Hq + static_cast<int64_t>(h) * p.G + gq) * HD;
            float qv[VE];
#pragma unroll
            for (int e = 0; e < VE; ++e) qv[e] = load_f(p.q, qrow + VE * g + e, p.q_f16);
            for (int t = t0; t < tail; t += ts) {
                const int64_t rel = (static_cast<int64_t>(t) * p.Hkv + h) * HD + VE * g;
                float kv[VE], vv[VE];
                load_row<VE>(kbase, rel, p.st_f16, kv);
                load_row<VE>(vbase, rel, p.st_f16, vv);
                float part = 0.0f;
#pragma unroll
                for (int e = 0; e < VE; ++e) part += qv[e] * kv[e];
                part += __shfl_xor_sync(0xffffffffu, part, 4);
                part += __shfl_xor_sync(0xffffffffu, part, 8);
                part += __shfl_xor_sync(0xffffffffu, part, 16);
                const float sv = part * p.sm_scale_log2;
                S.m_true[nt][col] = fmaxf(S.m_true[nt][col], sv);
                const float m_new = fmaxf(S.m_used[nt][col], sv);
                const float alpha = ex2(S.m_used[nt][col] - m_new);
                const float pr = ex2(sv - m_new);
                S.m_used[nt][col] = m_new;
                S.lpart[nt][col] = S.lpart[nt][col] * alpha + (g == 0 ? pr : 0.0f);
#pragma unroll
                for (int mt = 0; mt < HD / 16; ++mt) {
                    if (SPLIT) {
                        S.acc[mt][nt][0] = S.acc[mt][nt][0] * alpha + pr * vv[2 * mt];
                        S.acc[mt][nt][1] *= alpha;
                        S.acc[mt][nt][2] = S.acc[mt][nt][2] * alpha + pr * vv[2 * mt + 1];
                        S.acc[mt][nt][3] *= alpha;
                    } else {
                        S.acc[mt][nt][col] = S.acc[mt][nt][col] * alpha + pr * vv[2 * mt];
                        S.acc[mt][nt][col + 2] = S.acc[mt][nt][col + 2] * alpha + pr * vv[2 * mt + 1];
                    }
                }
            }
        }
}

// Length of sequence b, or 0 (and BAD_ARGUMENT) when it is negative or its
// committed pages (len / P; the staged rows need no block-table entry) do not
// fit the block table.
__device__ __forceinline__ int valid_len(const DecodeParams& p, int b, bool report) {
    if (p.uniform_len >= 0) return p.uniform_len;
    const int len = p.seq_lens[b];
    if (len >= 0 && len / p.P <= p.max_blocks) return len;
    if (report) flag(p.status, MG_DEV_BAD_ARGUMENT);
    return 0;
}

// The part of sequence b inside the CTA's unit range [u0, u1).
struct Segment {
    int b;
    int lo;      // first committed page of the segment (sequence-relative)
    int npg;     // committed pages in the segment
    int tail;    // staged rows folded in here (0: none, or another CTA's)
    int ub, ue;  // the sequence's unit range
    bool complete;
};

__device__ __forceinline__ Segment make_segment(const DecodeParams& p, const int* prefix, int b, int64_t u0,
                                                int64_t u1) {
    Segment s;
    const int ub = prefix[b], ue = prefix[b + 1];
    const int lo = static_cast<int>((u0 > ub ? u0 : ub) - ub);
    const int hi = static_cast<int>((u1 < ue ? u1 : ue) - ub);
    const int len = valid_len(p, b, false);
    const int np_b = len / p.P;
    const int tail_b = p.has_staging ? len - np_b * p.P : 0;
    s.b = b;
    s.lo = lo;
    s.npg = (hi < np_b ? hi : np_b) - lo;
    if (s.npg < 0) s.npg = 0;
    s.tail = (tail_b > 0 && hi == ue - ub) ? tail_b : 0;
    s.ub = ub;
    s.ue = ue;
    s.complete = lo == 0 && hi == ue - ub;
    return s;
}

// Refill the warp's page-metadata cache from entry `base`.  P16: entry i is
// the warp's local tile base + i, i.e. segment page wsub + (base + i) * wph;
// otherwise entry i is segment page base + i.
template <bool P16>
__device__ __forceinline__ void meta_refill(MetaCache& mc, const DecodeParams& p, const Segment& sg, int base,
                                            int wsub, int wph, int lane) {
    const int sp = P16 ? wsub + (base + lane) * wph : base + lane;
    int32_t pid = 0;
    float ks = 0.0f, vs = 0.0f;
    if (sp < sg.npg) {
        pid = p.block_tables[static_cast<int64_t>(sg.b) * p.max_blocks + sg.lo + sp];
        if (pid < 0 || pid >= p.num_pages) {
            flag(p.status, MG_DEV_BAD_PAGE_ID);
            pid = 0;
        }
        ks = p.k_scales[pid] * p.sm_scale_log2;
        vs = p.v_scales[pid];
    }
    mc.base = base;
    mc.pid = pid;
    mc.ks = ks;
    mc.vs = vs;
}

// Issue the global loads of the warp's local tile jt (segment tile
// wsub + jt * wph) of kv head h into T.  Warp-uniform.
template <bool KV4, int HD, bool P16>
__device__ __forceinline__ void load_tile(TileRegs<KV4, HD>& T, MetaCache& mc, const DecodeParams& p,
                                          const Segment& sg, int jt, int h, int wsub, int wph, int g, int c,
                                          int lane) {
    using C = Cfg<KV4, HD, 1>;
    const int rs = p.Hkv * C::ROWB;  // bytes per token row of a page
    if (P16) {
        if (jt >= mc.base + kMetaLanes) meta_refill<true>(mc, p, sg, jt, wsub, wph, lane);
        const int i = jt - mc.base;
        const int32_t pid = __shfl_sync(0xffffffffu, mc.pid, i);
        const float ks = __shfl_sync(0xffffffffu, mc.ks, i);
        const float vs = __shfl_sync(0xffffffffu, mc.vs, i);
        T.ks[0] = T.ks[1] = ks;
        T.vs[0] = T.vs[1] = vs;
        T.live = 3u;
        const int64_t off = static_cast<int64_t>(pid) * p.page_bytes + h * C::ROWB;
        const uint8_t* kb = p.k_pool + off;
        const uint8_t* vb = p.v_pool + off;
        ldg_words<C::KCHB>(kb + g * rs + c * C::KCHB, T.k[0]);
        ldg_words<C::KCHB>(kb + (g + 8) * rs + c * C::KCHB, T.k[1]);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int row = 2 * c + (r & 1) + (r >> 1) * 8;
            ldg_words<C::VCHB>(vb + row * rs + g * C::VCHB, T.v[r]);
        }
    } else {
        const int P = p.P;
        const int x0 = 16 * (wsub + jt * wph);  // first token of the tile (segment-relative)
        const int pfirst = x0 / P;
        const int off0 = x0 - pfirst * P;
        const int ntok = sg.npg * P;
        int plast = pfirst + static_cast<int>(p.pdiv.div(static_cast<uint32_t>(off0 + 15)));
        if (plast > sg.npg - 1) plast = sg.npg - 1;
        if (pfirst < mc.base || plast >= mc.base + kMetaLanes) meta_refill<false>(mc, p, sg, pfirst, wsub, wph, lane);
        T.live = 0u;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            // rows past the end read token 0 of the tile's first page
            const int row = g + 8 * r;
            const bool live = x0 + row < ntok;
            const int rel = live ? off0 + row : 0;
            const int dp = static_cast<int>(p.pdiv.div(static_cast<uint32_t>(rel)));
            const int src = pfirst + dp - mc.base;
            const int tok = rel - dp * P;
            const int32_t pid = __shfl_sync(0xffffffffu, mc.pid, src);
            const float ks = __shfl_sync(0xffffffffu, mc.ks, src);
            const float vs = __shfl_sync(0xffffffffu, mc.vs, src);
            T.ks[r] = live ? ks : 0.0f;
            T.vs[r] = vs;
            T.live |= live ? (1u << r) : 0u;
            ldg_words<C::KCHB>(p.k_pool + static_cast<int64_t>(pid) * p.page_bytes + tok * rs + h * C::ROWB +
                                   c * C::KCHB,
                               T.k[r]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int row = 2 * c + (r & 1) + (r >> 1) * 8;
            const int rel = x0 + row < ntok ? off0 + row : 0;
            const int dp = static_cast<int>(p.pdiv.div(static_cast<uint32_t>(rel)));
            const int src = pfirst + dp - mc.base;
            const int tok = rel - dp * P;
            const int32_t pid = __shfl_sync(0xffffffffu, mc.pid, src);
            ldg_words<C::VCHB>(p.v_pool + static_cast<int64_t>(pid) * p.page_bytes + tok * rs + h * C::ROWB +
                                   g * C::VCHB,
                               T.v[r]);
        }
    }
}

template <bool KV4, int HD, int NT, bool SPLIT, bool P16, int HPW, int R, int NW>
__global__ void __launch_bounds__(NW * 32, 1) paged_decode_kernel(const DecodeParams p) {
    using C = Cfg<KV4, HD, NT>;
    constexpr int VE = C::VE;
    constexpr int NCOLS = SPLIT ? 1 : 2;
    constexpr float kLn2 = 0.6931471805599453f;
    static_assert(HPW == 1 || R == 2, "two heads per warp alternate between two tile buffers");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int sm_scan[33];
    __shared__ int sm_last;

    grid_dependency_wait();
    grid_launch_dependents();

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int P = p.P, B = p.batch, Hkv = p.Hkv, Hq = p.Hq;
    const int NCW = p.nconsumers, WPH = p.wph;
    int* prefix = reinterpret_cast<int*>(smem);
    float* mscratch = reinterpret_cast<float*>(smem + p.scratch_off);
    uint8_t* tailbuf = smem + p.tail_off;

    if (p.status && (*(volatile int32_t*)p.status & (MG_DEV_OUT_OF_PAGES | MG_DEV_BLOCK_TABLE_FULL))) return;

    // ---- units per sequence (committed pages + 1 if a staged tail) and prefix ----
    int base = 0;
    for (int start = 0; start < B; start += blockDim.x) {
        const int bb = start + tid;
        int u = 0;
        if (bb < B) {
            const int len = valid_len(p, bb, blockIdx.x == 0);
            const int np = len / P;
            u = np + ((p.has_staging && len - np * P > 0) ? 1 : 0);
        }
        int tot;
        const int ex = block_exclusive_scan(u, sm_scan, &tot);
        if (bb < B) prefix[bb] = base + ex;
        base += tot;
    }
    if (tid == 0) prefix[B] = base;
    __syncthreads();
    const int64_t W = base;
    const int cta = blockIdx.x;
    const int GR = static_cast<int>(W < gridDim.x ? W : gridDim.x);

    // empty sequences: zeros (normalised) or (0, 0, -inf) (unnormalised)
    for (int bb = cta; bb < B; bb += gridDim.x) {
        if (prefix[bb + 1] != prefix[bb]) continue;
        const int64_t r0 = static_cast<int64_t>(bb) * Hq;
        for (int i = tid; i < Hq * HD; i += blockDim.x) {
            if (p.out_wv) p.out_wv[r0 * HD + i] = 0.0f;
            else if (p.out_f16) static_cast<__half*>(p.out)[r0 * HD + i] = __float2half(0.0f);
            else static_cast<float*>(p.out)[r0 * HD + i] = 0.0f;
        }
        if (p.out_wv)
            for (int i = tid; i < Hq; i += blockDim.x) {
                p.out_l[r0 + i] = 0.0f;
                p.out_m[r0 + i] = -INFINITY;
            }
    }
    if (cta >= GR) return;
    const int64_t u0 = static_cast<int64_t>(cta) * W / GR, u1 = static_cast<int64_t>(cta + 1) * W / GR;
    int b = 0;
    {
        int lo = 0, hi = B - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (prefix[mid] <= u0) lo = mid;
            else hi = mid - 1;
        }
        b = lo;
    }

    const int wsub = WPH > 1 ? warp % WPH : 0;
    const int hbase = WPH > 1 ? warp / WPH : warp;
    HeadState<NT, HD / 16> st[HPW];
    MetaCache mc;

    for (;;) {
        const Segment sg = make_segment(p, prefix, b, u0, u1);

        // ---- the staged tail goes to shared memory while the pages stream ----------
        const int tail_bytes = sg.tail * p.st_row_bytes;
        const bool tail_smem = sg.tail > 0 && 2 * tail_bytes <= p.tail_cap;
        const int64_t tail_src = static_cast<int64_t>(sg.b) * P * p.st_row_bytes;
        if (tail_smem) {
            const uint8_t* sk = static_cast<const uint8_t*>(p.staging_k) + tail_src;
            const uint8_t* sv = static_cast<const uint8_t*>(p.staging_v) + tail_src;
            for (int i = tid * 16; i < tail_bytes; i += blockDim.x * 16) {
                cp_async16(tailbuf + i, sk + i);
                cp_async16(tailbuf + tail_bytes + i, sv + i);
            }
            cp_async_commit();
        }

#pragma unroll
        for (int hh = 0; hh < HPW; ++hh) {
            const int h = hbase + hh * NCW;
            if (h < Hkv) load_q<KV4, HD, NT, SPLIT>(st[hh], p, sg.b, h, g, c);
        }

        // ---- committed pages: this warp's tiles, R - 1 ahead of the math ------------
        const int ntiles = P16 ? sg.npg : (sg.npg * P + 15) >> 4;
        const int nloc = wsub < ntiles ? (ntiles - 1 - wsub) / WPH + 1 : 0;
        const int nitems = nloc * HPW;
        mc.base = -(1 << 30);
        TileRegs<KV4, HD> tb[R];
        auto issue = [&](int j, TileRegs<KV4, HD>& T) {
            const int h = hbase + (HPW == 2 ? (j & 1) : 0) * NCW;
            if (h < Hkv) load_tile<KV4, HD, P16>(T, mc, p, sg, HPW == 2 ? (j >> 1) : j, h, wsub, WPH, g, c, lane);
        };
#pragma unroll
        for (int r = 0; r < R - 1; ++r)
            if (r < nitems) issue(r, tb[r]);
        for (int j0 = 0; j0 < nitems; j0 += R) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int j = j0 + r;
                if (j < nitems) {
                    if (j + R - 1 < nitems) issue(j + R - 1, tb[(r + R - 1) % R]);
                    if (HPW == 2) {
                        if (hbase + (r & 1) * NCW < Hkv) attend_tile<KV4, HD, NT, SPLIT>(st[r & 1], tb[r]);
                    } else {
                        attend_tile<KV4, HD, NT, SPLIT>(st[0], tb[r]);
                    }
                }
            }
        }

        // ---- staged tail, split across the warps of a head -------------------------
        if (sg.tail > 0) {
            const void* kb;
            const void* vb;
            if (tail_smem) {
                cp_async_wait_all();
                __syncthreads();
                kb = tailbuf;
                vb = tailbuf + tail_bytes;
            } else {
                kb = static_cast<const uint8_t*>(p.staging_k) + tail_src;
                vb = static_cast<const uint8_t*>(p.staging_v) + tail_src;
            }
#pragma unroll
            for (int hh = 0; hh < HPW; ++hh) {
                const int h = hbase + hh * NCW;
                if (h < Hkv) attend_tail<KV4, HD, NT, SPLIT>(st[hh], p, kb, vb, sg.b, h, wsub, WPH, sg.tail, g, c);
            }
        }

        // ---- finalize: per (head, column) m / l / o[VE] on this thread ----------
        const int slot_ws = 2 * cta + (u0 >= sg.ub ? 0 : 1);
#pragma unroll
        for (int hh = 0; hh < HPW; ++hh) {
            const int h = hbase + hh * NCW;
            const bool hv = h < Hkv;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int col = 0; col < NCOLS; ++col) {
                    float l = st[hh].lpart[nt][col];
                    l += __shfl_xor_sync(0xffffffffu, l, 4);
                    l += __shfl_xor_sync(0xffffffffu, l, 8);
                    l += __shfl_xor_sync(0xffffffffu, l, 16);
                    const int gi = SPLIT ? nt * 4 + c : nt * 8 + 2 * c + col;
                    const float mt = st[hh].m_true[nt][col];
                    const float f = (mt == -INFINITY) ? 0.0f : ex2(st[hh].m_used[nt][col] - mt);
                    l *= f;
                    float o[VE];
#pragma unroll
                    for (int mi = 0; mi < HD / 16; ++mi) {
                        if (SPLIT) {
                            o[2 * mi] = (st[hh].acc[mi][nt][0] + st[hh].acc[mi][nt][1]) * f;
                            o[2 * mi + 1] = (st[hh].acc[mi][nt][2] + st[hh].acc[mi][nt][3]) * f;
                        } else {
                            o[2 * mi] = st[hh].acc[mi][nt][col] * f;
                            o[2 * mi + 1] = st[hh].acc[mi][nt][col + 2] * f;
                        }
                    }
                    float m = mt;
                    if (WPH > 1) {
                        // stage this warp's state; the head's first warp merges all WPH of them
                        float* ms = mscratch + (static_cast<int64_t>(warp) * 4 + c) * (HD + 2);
                        __syncthreads();  // the previous merge finished reading the scratch
                        if (hv && gi < p.G) {
#pragma unroll
                            for (int e = 0; e < VE; ++e) ms[VE * g + e] = o[e];
                            if (g == 0) {
                                ms[HD] = m;
                                ms[HD + 1] = l;
                            }
                        }
                        __syncthreads();
                        if (wsub == 0 && hv && gi < p.G) {
                            float M = -INFINITY;
                            for (int ww = 0; ww < WPH; ++ww)
                                M = fmaxf(M, mscratch[(static_cast<int64_t>(warp + ww) * 4 + c) * (HD + 2) + HD]);
                            float L = 0.0f;
                            float oo[VE];
#pragma unroll
                            for (int e = 0; e < VE; ++e) oo[e] = 0.0f;
                            for (int ww = 0; ww < WPH; ++ww) {
                                const float* mw = mscratch + (static_cast<int64_t>(warp + ww) * 4 + c) * (HD + 2);
                                const float fw = (mw[HD] == -INFINITY) ? 0.0f : ex2(mw[HD] - M);
                                L += mw[HD + 1] * fw;
#pragma unroll
                                for (int e = 0; e < VE; ++e) oo[e] += mw[VE * g + e] * fw;
                            }
                            m = M;
                            l = L;
#pragma unroll
                            for (int e = 0; e < VE; ++e) o[e] = oo[e];
                        }
                    }
                    if (!hv || gi >= p.G || wsub != 0) continue;
                    const int hq = h * p.G + gi;
                    const int64_t orow = static_cast<int64_t>(sg.b) * Hq + hq;
                    if (sg.complete) {
                        const int64_t base_o = orow * HD + VE * g;
                        if (p.out_wv) {
#pragma unroll
                            for (int e = 0; e < VE; ++e) p.out_wv[base_o + e] = o[e];
                            if (g == 0) {
                                p.out_l[orow] = l;
                                p.out_m[orow] = m * kLn2;
                            }
                        } else {
                            const float inv = 1.0f / l;
                            if (p.out_f16) {
                                __half* op = static_cast<__half*>(p.out) + base_o;
#pragma unroll
                                for (int e = 0; e < VE; e += 2)
                                    *reinterpret_cast<__half2*>(op + e) = __floats2half2_rn(o[e] * inv, o[e + 1] * inv);
                            } else {
                                float* op = static_cast<float*>(p.out) + base_o;
#pragma unroll
                                for (int e = 0; e < VE; e += 4)
                                    *reinterpret_cast<float4*>(op + e) =
                                        make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
                            }
                        }
                    } else {
                        const int64_t prow = static_cast<int64_t>(slot_ws) * Hq + hq;
                        float* wp = p.ws_acc + prow * HD + VE * g;
#pragma unroll
                        for (int e = 0; e < VE; e += 4)
                            __stcg(reinterpret_cast<float4*>(wp + e), make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]));
                        if (g == 0) {
                            __stcg(p.ws_m + prow, m);
                            __stcg(p.ws_l + prow, l);
                        }
                    }
                }
        }

        if (!sg.complete) {
            // ---- last covering CTA merges the partials of sequence b (one pass) ------
            __threadfence();
            __syncthreads();
            const int c_first = cta_of_unit(sg.ub, W, GR);
            const int c_last = cta_of_unit(sg.ue - 1, W, GR);
            if (tid == 0) {
                const uint32_t prev = atomicAdd(&p.tickets[sg.b], 1u);
                sm_last = (prev == static_cast<uint32_t>(c_last - c_first)) ? 1 : 0;
            }
            __syncthreads();
            if (sm_last) {
                __threadfence();
                const int ncov = c_last - c_first + 1;
                for (int it = tid; it < Hq * (HD / 4); it += blockDim.x) {
                    const int hq = it / (HD / 4), d4 = (it - hq * (HD / 4)) * 4;
                    float M = -INFINITY, L = 0.0f;
                    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int k0 = 0; k0 < ncov; k0 += 4) {
                        float mj[4], lj[4];
                        float4 vj[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            mj[u] = -INFINITY;
                            lj[u] = 0.0f;
                            vj[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (k0 + u < ncov) {
                                const int cc = c_first + k0 + u;
                                const int sl = 2 * cc + ((static_cast<int64_t>(cc) * W / GR) >= sg.ub ? 0 : 1);
                                const int64_t prow = static_cast<int64_t>(sl) * Hq + hq;
                                mj[u] = __ldcg(p.ws_m + prow);
                                lj[u] = __ldcg(p.ws_l + prow);
                                vj[u] = __ldcg(reinterpret_cast<const float4*>(p.ws_acc + prow * HD + d4));
                            }
                        }
                        float Mn = M;
#pragma unroll
                        for (int u = 0; u < 4; ++u) Mn = fmaxf(Mn, mj[u]);
                        const float fo = (M == -INFINITY) ? 0.0f : ex2(M - Mn);
                        L *= fo;
                        a.x *= fo;
                        a.y *= fo;
                        a.z *= fo;
                        a.w *= fo;
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const float fj = (mj[u] == -INFINITY) ? 0.0f : ex2(mj[u] - Mn);
                            L += lj[u] * fj;
                            a.x += vj[u].x * fj;
                            a.y += vj[u].y * fj;
                            a.z += vj[u].z * fj;
                            a.w += vj[u].w * fj;
                        }
                        M = Mn;
                    }
                    const int64_t orow = static_cast<int64_t>(sg.b) * Hq + hq;
                    const int64_t base_o = orow * HD + d4;
                    if (p.out_wv) {
                        *reinterpret_cast<float4*>(p.out_wv + base_o) = a;
                        if (d4 == 0) {
                            p.out_l[orow] = L;
                            p.out_m[orow] = M * kLn2;
                        }
                    } else {
                        const float inv = 1.0f / L;
                        if (p.out_f16) {
                            __half2* op = reinterpret_cast<__half2*>(static_cast<__half*>(p.out) + base_o);
                            op[0] = __floats2half2_rn(a.x * inv, a.y * inv);
                            op[1] = __floats2half2_rn(a.z * inv, a.w * inv);
                        } else {
                            *reinterpret_cast<float4*>(static_cast<float*>(p.out) + base_o) =
                                make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
                        }
                    }
                }
                if (tid == 0) p.tickets[sg.b] = 0u;  // leave the workspace reusable
            }
        }
        __syncthreads();  // tail buffer and merge scratch are free for the next segment

        // ---- next non-empty sequence inside [u0, u1) ------------------------------
        if (sg.ue >= u1) break;
        ++b;
        while (b < B && prefix[b + 1] == prefix[b]) ++b;
        if (b >= B) break;
    }
}

template <bool KV4, int HD, int NT, bool SPLIT, bool P16, int HPW, int R, int NW>
mg_status launch_one(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s) {
    auto k = paged_decode_kernel<KV4, HD, NT, SPLIT, P16, HPW, R, NW>;
    if (pl.nconsumers > NW) return set_error(MG_ERR_UNSUPPORTED, "decode plan wants %d warps > %d", pl.nconsumers, NW);
    static int64_t attr_set[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (pl.smem_bytes > 48 * 1024 && (dev < 0 || dev >= 64 || attr_set[dev] < pl.smem_bytes)) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(pl.smem_bytes));
        if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_set[dev] = pl.smem_bytes;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(32 * pl.nconsumers);
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem_bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k, p);
    if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "paged_decode_kernel launch: %s", cudaGetErrorString(e));
    return check_launch("paged_decode_kernel");
}

// Kernel shapes (the planner's choice, DecodePlan::nwarps / hpw):
//   head_dim 64, one n-tile:   16 warps, one kv head per warp (two tiles in
//                              flight for INT8, three for INT4) or two heads
//                              per warp (num_kv_heads 17..32);
//   otherwise, <= 8 kv heads:  8 warps with up to 255 registers, two tiles in flight;
//   otherwise, 9..16 kv heads: 16 warps, one tile at a time.
template <bool KV4, int HD, int NT, bool SPLIT, bool P16>
mg_status launch_h(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s) {
    if constexpr (HD == 64 && NT == 1) {
        if (pl.hpw == 2) return launch_one<KV4, HD, NT, SPLIT, P16, 2, 2, kWarps>(p, pl, s);
        return launch_one<KV4, HD, NT, SPLIT, P16, 1, (KV4 ? 3 : 2), kWarps>(p, pl, s);
    } else {
        if (pl.nwarps == kWarpsWide) return launch_one<KV4, HD, NT, SPLIT, P16, 1, 2, kWarpsWide>(p, pl, s);
        return launch_one<KV4, HD, NT, SPLIT, P16, 1, 1, kWarps>(p, pl, s);
    }
}

template <bool KV4, int HD, bool P16>
mg_status launch_p(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s) {
    if (pl.split_mode) {
        if (pl.nt == 1) return launch_h<KV4, HD, 1, true, P16>(p, pl, s);
        return launch_h<KV4, HD, 2, true, P16>(p, pl, s);
    }
    if (pl.nt == 1) return launch_h<KV4, HD, 1, false, P16>(p, pl, s);
    return launch_h<KV4, HD, 2, false, P16>(p, pl, s);
}

template <bool KV4>
mg_status launch_kv(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s, int hd) {
    const bool p16 = p.P == 16;
    if (hd == 64) return p16 ? launch_p<KV4, 64, true>(p, pl, s) : launch_p<KV4, 64, false>(p, pl, s);
    return p16 ? launch_p<KV4, 128, true>(p, pl, s) : launch_p<KV4, 128, false>(p, pl, s);
}

}  // namespace mg
