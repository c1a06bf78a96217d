// Body of the fused paged decode-attention kernel (see mg_attention.cuh for
// the design).  Included by the per-format translation units.
#pragma once

#include "mg_attention.cuh"

namespace mg {

// The math of one 16-token tile of one kv head: S^T = K Q^T on the tensor
// cores, online softmax update, O^T += V^T P^T.  The fp16 fragments come from
// kf(kk, a): K rows g, g+8 of k-step kk (a[0], a[2] row g; a[1], a[3] row g+8),
// and vf(r0a, r1a, r0b, r1b): V^T for tokens (2c, 2c+1) and (2c+8, 2c+9).
// ks0 / ks1: K scales of rows g / g+8 times the softmax scale (log2 domain),
// vs0 / vs1 their V scales; live0 / live1: the rows exist.
template <bool KV4, int HD, int NT, bool SPLIT, typename KF, typename VF>
__device__ __forceinline__ void attend_core(HeadState<NT, HD / 16>& S, KF&& kf, VF&& vf, float ks0, float ks1,
                                            float vs0, float vs1, bool live0, bool live1) {
    using C = Cfg<KV4, HD, NT>;
    constexpr int NCOLS = SPLIT ? 1 : 2;

    // ---- scores: K rows g, g+8 against the q columns ------------------------------
    float sc[NT][4], sc2[NT][4];  // two accumulation chains (even / odd k-steps)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nt][i] = sc2[nt][i] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < C::KSTEPS; ++kk) {
        uint32_t a[4];
        kf(kk, a);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            if (kk & 1) mma_16816(sc2[nt], a, S.qf[nt][kk][0], S.qf[nt][kk][1]);
            else mma_16816(sc[nt], a, S.qf[nt][kk][0], S.qf[nt][kk][1]);
        }
    }
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
    // The column max is reduced over the lanes (rows) only when some lane's
    // score passes the reference max by the threshold; m_true stays a per-lane
    // running max, reduced when the segment is finalized.
    bool need = false;
    float mx[NT][NCOLS];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int col = 0; col < NCOLS; ++col) {
            const float m = fmaxf(s[nt][col][0], s[nt][col][1]);
            mx[nt][col] = m;
            S.m_true[nt][col] = fmaxf(S.m_true[nt][col], m);
            need |= m > S.m_used[nt][col] + kRescaleThreshold;
        }
    if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int col = 0; col < NCOLS; ++col) {
                float m = mx[nt][col];
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
                const float m_new = fmaxf(S.m_used[nt][col], m);
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
    vf(r0a, r1a, r0b, r1b);
#pragma unroll
    for (int mt = 0; mt < C::MTILES; ++mt) {
        const uint32_t a[4] = {r0a[mt], r1a[mt], r0b[mt], r1b[mt]};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(S.acc[mt][nt], a, pb[nt][0], pb[nt][1]);
    }
}

// One 16-token tile of quantized pages, already in registers (TileRegs).
// sscale: softmax scale times log2(e).
template <bool KV4, int HD, int NT, bool SPLIT, bool P16>
__device__ __forceinline__ void attend_tile(HeadState<NT, HD / 16>& S, const TileRegs<KV4, HD>& T, float sscale) {
    // page size 16 (page scales): one page per tile, its scales live in slot 0 only
    const float ks0 = T.ks[0] * sscale, ks1 = T.ks[P16 ? 0 : 1] * sscale;
    const float vs0 = T.vs[0], vs1 = T.vs[P16 ? 0 : 1];
    attend_core<KV4, HD, NT, SPLIT>(
        S,
        [&](int kk, uint32_t (&a)[4]) {
            k_frag_row<KV4>(T.k[0], kk, a[0], a[2]);
            k_frag_row<KV4>(T.k[1], kk, a[1], a[3]);
        },
        [&](uint32_t (&r0a)[HD / 16], uint32_t (&r1a)[HD / 16], uint32_t (&r0b)[HD / 16], uint32_t (&r1b)[HD / 16]) {
            v_pairs<KV4, HD>(T.v[0], T.v[1], r0a, r1a);
            v_pairs<KV4, HD>(T.v[2], T.v[3], r0b, r1b);
        },
        ks0, ks1, vs0, vs1, (T.live & 1u) != 0, (T.live & 2u) != 0);
}

// One 16-row tile of the exact fp16 staged tail of kv head h of sequence b:
// staged rows r0 .. r0 + n - 1 (n <= 16), straight from global memory (the
// append kernel wrote them just before; an L1 prefetch went out when the item
// was issued).  The fp16 rows are the tensor-core operands as they are: K in
// the q columns' dimension order (k_slot_d), V^T paired by token, no scales.
template <bool KV4, int HD, int NT, bool SPLIT>
__device__ __forceinline__ void attend_tail_tile(HeadState<NT, HD / 16>& S, const DecodeParams& p, int b, int h,
                                                 int r0, int n, int g, int c, float sscale) {
    constexpr int KW = HD / 8;   // 32-bit words per lane of a K row: HD / 4 halves
    constexpr int VW = HD / 16;  // of a V row: HD / 8 halves
    const int64_t rs = static_cast<int64_t>(p.Hkv) * HD;  // halves per staged token row
    const __half* base = static_cast<const __half*>(p.staging_k) + ((static_cast<int64_t>(b) * p.P + r0) * p.Hkv + h) * HD;
    const __half* vbase = static_cast<const __half*>(p.staging_v) + (base - static_cast<const __half*>(p.staging_k));
    uint32_t kw[2][KW], vw[4][VW];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = g + 8 * r;
        const uint4* src = reinterpret_cast<const uint4*>(base + row * rs + (HD / 4) * c);
#pragma unroll
        for (int i = 0; i < KW / 4; ++i) {
            const uint4 u = row < n ? src[i] : make_uint4(0u, 0u, 0u, 0u);
            kw[r][4 * i] = u.x;
            kw[r][4 * i + 1] = u.y;
            kw[r][4 * i + 2] = u.z;
            kw[r][4 * i + 3] = u.w;
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int row = 2 * c + (r & 1) + (r >> 1) * 8;
        const uint4* src = reinterpret_cast<const uint4*>(vbase + row * rs + (HD / 8) * g);
#pragma unroll
        for (int i = 0; i < VW / 4; ++i) {
            const uint4 u = row < n ? src[i] : make_uint4(0u, 0u, 0u, 0u);
            vw[r][4 * i] = u.x;
            vw[r][4 * i + 1] = u.y;
            vw[r][4 * i + 2] = u.z;
            vw[r][4 * i + 3] = u.w;
        }
    }
    attend_core<KV4, HD, NT, SPLIT>(
        S,
        [&](int kk, uint32_t (&a)[4]) {
            // k_slot_d: a[0] = dims (d0, d0 + 2 or 4), a[2] = (d0 + 1, d0 + 3 or 5), d0 even
            const int i0 = KV4 ? 4 * (kk >> 1) + (kk & 1) : 2 * kk;
            const int i1 = KV4 ? i0 + 2 : i0 + 1;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                a[r] = __byte_perm(kw[r][i0], kw[r][i1], 0x5410);
                a[r + 2] = __byte_perm(kw[r][i0], kw[r][i1], 0x7632);
            }
        },
        [&](uint32_t (&r0a)[HD / 16], uint32_t (&r1a)[HD / 16], uint32_t (&r0b)[HD / 16], uint32_t (&r1b)[HD / 16]) {
            // m-tile mt: dims VE*g + 2mt (r0) and + 1 (r1), tokens paired
#pragma unroll
            for (int mt = 0; mt < HD / 16; ++mt) {
                r0a[mt] = __byte_perm(vw[0][mt], vw[1][mt], 0x5410);
                r1a[mt] = __byte_perm(vw[0][mt], vw[1][mt], 0x7632);
                r0b[mt] = __byte_perm(vw[2][mt], vw[3][mt], 0x5410);
                r1b[mt] = __byte_perm(vw[2][mt], vw[3][mt], 0x7632);
            }
        },
        sscale, sscale, 1.0f, 1.0f, g < n, g + 8 < n);
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

// One chunk of the exact staged tail for one kv head: n rows of K at
// kslot[i * HB] and of V at vslot[i * HB] (shared memory, HB = D * element
// size), fp32 math on the CUDA cores in two passes (max, then exponentials
// and the V accumulation) so the rows proceed independently.
template <bool KV4, int HD, int NT, bool SPLIT>
__device__ __forceinline__ void attend_tail_chunk(HeadState<NT, HD / 16>& S, const DecodeParams& p,
                                                  const uint8_t* kslot, const uint8_t* vslot, int n, int b, int h,
                                                  int g, int c) {
    constexpr int VE = HD / 8;
    constexpr int NCOLS = SPLIT ? 1 : 2;
    const int esz = p.st_f16 ? 2 : 4;
    const int hb = HD * esz;
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
            auto score = [&](int i) -> float {
                float kv[VE];
                load_row<VE>(kslot + i * hb, VE * g, p.st_f16, kv);
                float part = 0.0f;
#pragma unroll
                for (int e = 0; e < VE; ++e) part += qv[e] * kv[e];
                part += __shfl_xor_sync(0xffffffffu, part, 4);
                part += __shfl_xor_sync(0xffffffffu, part, 8);
                part += __shfl_xor_sync(0xffffffffu, part, 16);
                return part * p.sm_scale_log2;
            };
            float mloc = -INFINITY;
#pragma unroll 4
            for (int i = 0; i < n; ++i) mloc = fmaxf(mloc, score(i));
            const float m_new = fmaxf(S.m_used[nt][col], mloc);
            const float alpha = (S.m_used[nt][col] == -INFINITY) ? 0.0f : ex2(S.m_used[nt][col] - m_new);
            S.m_used[nt][col] = m_new;
            S.m_true[nt][col] = fmaxf(S.m_true[nt][col], mloc);
            S.lpart[nt][col] *= alpha;
#pragma unroll
            for (int mt = 0; mt < HD / 16; ++mt) {
                if (SPLIT) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) S.acc[mt][nt][i] *= alpha;
                } else {
                    S.acc[mt][nt][col] *= alpha;
                    S.acc[mt][nt][col + 2] *= alpha;
                }
            }
            float lsum = 0.0f;
#pragma unroll 4
            for (int i = 0; i < n; ++i) {
                const float pr = ex2(score(i) - m_new);
                lsum += pr;
                float vv[VE];
                load_row<VE>(vslot + i * hb, VE * g, p.st_f16, vv);
#pragma unroll
                for (int mt = 0; mt < HD / 16; ++mt) {
                    const int a0 = SPLIT ? 0 : col, a2 = SPLIT ? 2 : col + 2;
                    S.acc[mt][nt][a0] += pr * vv[2 * mt];
                    S.acc[mt][nt][a2] += pr * vv[2 * mt + 1];
                }
            }
            if (g == 0) S.lpart[nt][col] += lsum;
        }
}

// A piece of one sequence run by this CTA (one record of the decode plan),
// and this warp's work items in it: its tiles (segment tiles wsub,
// wsub + wph, ..., times the warp's heads) and its chunks of the staged tail,
// times the warp's heads.  An fp16 tail goes in 16-row tiles on the tensor
// cores: tail tile j to warp (j + ntiles) % wph, i.e. first to the warps that
// hold one page tile fewer.  An fp32 tail goes on the CUDA cores in chunks of
// up to tt rows (rows wsub, wsub + wph, ...).  The tail items come first: they
// then overlap the ramp of the page stream instead of trailing it.
struct Segment {
    int b;
    int lo;      // first committed page of the segment (sequence-relative)
    int npg;     // committed pages in the segment
    int tail;    // staged rows folded in here (0: none, or another CTA's)
    int pslot;   // partial slot, -1 when the segment is the whole sequence
    int pbase;   // first partial slot of the sequence's pieces
    int ncov;    // pieces of the sequence
    bool complete;
    int nh;      // the warp's heads (1, or 2 with two heads per warp)
    int ntile;   // the warp's tile items
    int ntt;     // the warp's tail rows (per head; fp32 tails)
    int tj0;     // its first 16-row tail tile (fp16 tails)
    int nchunk;  // its tail chunks or tail tiles (per head)
    int ntail;   // its tail items, nchunk * nh: items [0, ntail), its tiles after them
    int nitems;  // ntail + ntile
};

__device__ __forceinline__ Segment make_segment(const int4* rec, int P, int wsub, int wph, int nh, int tt, bool tc) {
    Segment s;
    const int4 r0 = rec[0], r1 = rec[1];
    s.b = r0.x;
    s.lo = r0.y;
    s.npg = r0.z;
    s.tail = r0.w;
    s.pslot = r1.x;
    s.pbase = r1.y;
    s.ncov = r1.z;
    s.complete = s.pslot < 0;
    s.nh = nh;
    const int ntiles = P == 16 ? s.npg : (s.npg * P + 15) >> 4;
    const int nloc = wsub < ntiles ? (ntiles - 1 - wsub) / wph + 1 : 0;
    s.ntile = nloc * nh;
    if (tc) {
        const int nT = (s.tail + 15) >> 4;
        s.tj0 = wsub - ntiles % wph;
        if (s.tj0 < 0) s.tj0 += wph;
        s.ntt = 0;
        s.nchunk = s.tj0 < nT ? (nT - 1 - s.tj0) / wph + 1 : 0;
    } else {
        s.tj0 = 0;
        s.ntt = wsub < s.tail ? (s.tail - 1 - wsub) / wph + 1 : 0;
        s.nchunk = (s.ntt + tt - 1) / tt;
    }
    s.ntail = s.nchunk * nh;
    s.nitems = s.ntail + s.ntile;
    return s;
}

// Page metadata of 32 upcoming tiles of the issuing walk, one entry per lane.
// P16: entry i is the warp's local tile base + i, i.e. segment page
// wsub + (base + i) * wph; otherwise entry i is segment page base + i.
template <bool P16>
__device__ __forceinline__ const int32_t* meta_row(const DecodeParams& p, const Segment& sg) {
    return p.block_tables + static_cast<int64_t>(sg.b) * p.max_blocks + sg.lo;
}

template <bool P16>
__device__ __forceinline__ void meta_refill(MetaCache& mc, const DecodeParams& p, const Segment& sg, int base,
                                            int wsub, int wph, int lane) {
    const int32_t* row = meta_row<P16>(p, sg);
    const int sp = P16 ? wsub + (base + lane) * wph : base + lane;
    int32_t pid = 0;
    if (sp < sg.npg) {
        pid = (mc.spids && sp < kPlanPids) ? mc.spids[sp] : row[sp];
        if (pid < 0 || pid >= p.num_pages) {
            flag(p.status, MG_DEV_BAD_PAGE_ID);
            pid = 0;
        }
    }
    mc.base = base;
    mc.pid = pid;
    // warm L1 with the next 32 entries (their lines) so the following refill does not wait on HBM
    const int spn = P16 ? wsub + (base + kMetaLanes + lane) * wph : base + kMetaLanes + lane;
    if (spn < sg.npg && (lane == 0 || P16)) prefetch_l1(row + spn);
}

// Warm L1 with a segment's first block-table entries and the q rows of the
// warp's heads (issued when the walk enters the segment, read much later).
template <bool P16>
__device__ __forceinline__ void warm_segment(const DecodeParams& p, const Segment& sg, int h0, int h1, int HD,
                                             int wsub, int wph, int lane) {
    if (sg.nitems == 0) return;
    const int32_t* row = meta_row<P16>(p, sg);
    const int sp = P16 ? wsub + lane * wph : lane;
    if (sp < sg.npg && (lane == 0 || P16)) prefetch_l1(row + sp);
    const int qbytes = p.G * HD * (p.q_f16 ? 2 : 4);
    const char* q0 = static_cast<const char*>(p.q) +
                     (static_cast<int64_t>(sg.b) * p.Hq + static_cast<int64_t>(h0) * p.G) * HD * (p.q_f16 ? 2 : 4);
    if (lane * 128 < qbytes) prefetch_l1(q0 + lane * 128);
    if (h1 >= 0) {
        const char* q1 = static_cast<const char*>(p.q) +
                         (static_cast<int64_t>(sg.b) * p.Hq + static_cast<int64_t>(h1) * p.G) * HD * (p.q_f16 ? 2 : 4);
        if (lane * 128 < qbytes) prefetch_l1(q1 + lane * 128);
    }
}

// Issue the global loads of the warp's local tile jt (segment tile
// wsub + jt * wph; the warp has nloc in the segment) of kv head h into T.
// Warp-uniform.
template <bool KV4, int HD, bool P16>
__device__ __forceinline__ void load_tile(TileRegs<KV4, HD>& T, MetaCache& mc, const DecodeParams& p,
                                          const Segment& sg, int jt, int nloc, int h, int wsub, int wph, int g,
                                          int c, int lane) {
    using C = Cfg<KV4, HD, 1>;
    const int rs = p.Hkv * C::ROWB;  // bytes per token row of a page
    if (P16) {
        if (jt >= mc.base + kMetaLanes) meta_refill<true>(mc, p, sg, jt, wsub, wph, lane);
        const int32_t pid = __shfl_sync(0xffffffffu, mc.pid, jt - mc.base);
        // scales straight into slot 0 (attend_tile reads slot 0 for both rows): a
        // copy of a load still in flight would stall the issuing warp
        T.ks[0] = __ldg(p.k_scales + pid);
        T.vs[0] = __ldg(p.v_scales + pid);
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
        // L2 prefetch of the warp's tile kPrefetchTiles ahead: lane l brings K row l
        // (l < 16) or V row l - 16, lanes 0 and 16 also the page's K / V scale, so
        // the register ring reads from L2.  Rows of neighbouring heads share
        // 128-byte lines: when the page rows are line-aligned, only a warp whose
        // head starts a line sends it.  The segment's first tiles also send the
        // tiles before that distance, two per tile (tiles 2jt + 1 and 2jt + 2).
        const bool pf_lead = (rs % 128 != 0) || ((h * C::ROWB) % 128 == 0);
        auto prefetch_tile = [&](int ja) {
            if (pf_lead && ja < nloc && ja < mc.base + kMetaLanes) {
                const int32_t pa = __shfl_sync(0xffffffffu, mc.pid, ja - mc.base);
                const uint8_t* pool = lane < 16 ? p.k_pool : p.v_pool;
                prefetch_l2(pool + static_cast<int64_t>(pa) * p.page_bytes + (lane & 15) * rs + h * C::ROWB);
                if ((lane & 15) == 0) prefetch_l2((lane < 16 ? p.k_scales : p.v_scales) + pa);
            }
        };
        if (2 * jt + 1 < kPrefetchTiles) {  // one test per tile once the opening is over
            prefetch_tile(2 * jt + 1);
            if (2 * jt + 2 < kPrefetchTiles) prefetch_tile(2 * jt + 2);
        }
        prefetch_tile(jt + kPrefetchTiles);
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
            const int tok = rel - dp * P;
            const int32_t pid = __shfl_sync(0xffffffffu, mc.pid, pfirst + dp - mc.base);
            const int64_t si = p.scale_th ? (static_cast<int64_t>(pid) * P + tok) * p.Hkv + h : pid;
            T.ks[r] = __ldg(p.k_scales + si);
            T.vs[r] = __ldg(p.v_scales + si);
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
            const int tok = rel - dp * P;
            const int32_t pid = __shfl_sync(0xffffffffu, mc.pid, pfirst + dp - mc.base);
            ldg_words<C::VCHB>(p.v_pool + static_cast<int64_t>(pid) * p.page_bytes + tok * rs + h * C::ROWB +
                                   g * C::VCHB,
                               T.v[r]);
        }
    }
}

// cp.async the warp's tail rows wsub + wph * (chunk * tt + i), i < n, of kv
// head h of sequence b into a shared slot: K rows [tt][HB], then V rows.
__device__ __forceinline__ void issue_tail_chunk(uint8_t* slot, const DecodeParams& p, int b, int h, int chunk,
                                                 int n, int tt, int hb, int wsub, int wph, int lane) {
    const int pieces = hb / 16;  // 16-byte pieces per row
    const int total = 2 * n * pieces;
    const uint8_t* sk = static_cast<const uint8_t*>(p.staging_k);
    const uint8_t* sv = static_cast<const uint8_t*>(p.staging_v);
    for (int q = lane; q < total; q += 32) {
        const int kv = q >= n * pieces;
        const int r = kv ? q - n * pieces : q;
        const int i = r / pieces, off = (r - i * pieces) * 16;
        const int t = wsub + wph * (chunk * tt + i);
        const int64_t src = ((static_cast<int64_t>(b) * p.P + t) * p.Hkv + h) * hb + off;
        cp_async16(slot + (kv ? tt * hb : 0) + i * hb + off, (kv ? sv : sk) + src);
    }
}

template <int N>
struct Slot {
    static constexpr int value = N;
};

// f(Slot<phase>{}) for a runtime phase in [K, R): the ring slot becomes a
// compile-time index, so the register ring never spills to local memory.
template <int R, int K = 0, typename F>
__device__ __forceinline__ void with_slot(int phase, F&& f) {
    if constexpr (K + 1 < R) {
        if (phase == K) f(Slot<K>{});
        else with_slot<R, K + 1>(phase, f);
    } else {
        f(Slot<K>{});
    }
}

__device__ __forceinline__ uint32_t ticket_add(uint32_t* t) {
    uint32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(t) : "memory");
    return prev;
}

// The last CTA to finish (sequence b, kv head h) merges the partials of all
// pieces of the sequence (slots pbase .. pbase + ncov - 1; log-sum-exp, one
// pass, four partials per load round) and writes the outputs of the head's
// G query heads; the wph warps of the head take alternate 32-column groups.
template <int HD>
__device__ __forceinline__ void merge_partials(const DecodeParams& p, int b, int h, int pbase, int ncov, int lane,
                                               int wsub, int wph) {
    constexpr float kLn2 = 0.6931471805599453f;
    const int Hq = p.Hq;
    for (int it = wsub * 32 + lane; it < p.G * (HD / 4); it += wph * 32) {
        const int gq = it / (HD / 4), d4 = (it - gq * (HD / 4)) * 4;
        const int hq = h * p.G + gq;
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
                    const int64_t prow = static_cast<int64_t>(pbase + k0 + u) * Hq + hq;
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
        const int64_t orow = static_cast<int64_t>(b) * Hq + hq;
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
    if (lane == 0) p.tickets[static_cast<int64_t>(b) * p.Hkv + h] = 0u;  // leave the workspace reusable
}

template <bool KV4, int HD, int NT, bool SPLIT, bool P16, int HPW, int R, int NW>
__global__ void __launch_bounds__(NW * 32, 1) paged_decode_kernel(const DecodeParams p) {
    using C = Cfg<KV4, HD, NT>;
    constexpr int VE = C::VE;
    constexpr int NCOLS = SPLIT ? 1 : 2;
    constexpr float kLn2 = 0.6931471805599453f;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int sm_hdr[3];
    __shared__ int sm_last[2 * 2 * kWarps];  // (cut segment, head of the warp, kv-head group): this CTA merges

    // With a settled plan the prologue (plan, status) and an L2 warm-up of the
    // first pages run before the wait on the previous launch, on SMs that launch
    // has already left; nothing is written to global memory before it.
    const bool settled = p.plan_settled != 0;
    if (!settled) {
        grid_dependency_wait();
        grid_launch_dependents();
    }

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int Hkv = p.Hkv, Hq = p.Hq;
    const int NCW = p.nconsumers, WPH = p.wph;
    const int cta = blockIdx.x;
    float* mscratch = reinterpret_cast<float*>(smem + p.scratch_off);
    uint8_t* tslots = smem + p.tail_off + static_cast<int64_t>(warp) * R * p.tail_slot;
    int4* recs = reinterpret_cast<int4*>(smem);  // this CTA's segment records (plan)
    int32_t* spids = reinterpret_cast<int32_t*>(smem + kRecCache * 32);  // first segment's page ids (plan)

    // ---- this CTA's segments from the step's plan: the first kPlanInline in one
    // round trip, more (stream-K over many short sequences) from the flat array.
    // The status word, the plan header and the CTA's counts are read in the same
    // round trip (all lie inside buffers the host sized); a step whose allocation
    // failed then runs no segment and writes nothing. ------------------------------
    const int4* prec = reinterpret_cast<const int4*>(p.plan + p.lay.off_recs) + static_cast<int64_t>(cta) * kPlanInline * 2;
    bool bad_plan = false;  // flagged after the wait (no global write before it)
    if (tid < 2 * kPlanInline) recs[tid] = __ldcg(prec + tid);
    const int4* ppid = reinterpret_cast<const int4*>(p.plan + p.lay.off_pids) + static_cast<int64_t>(cta) * (kPlanPids / 4);
    if (tid >= 32 && tid < 32 + kPlanPids / 4) reinterpret_cast<int4*>(spids)[tid - 32] = __ldcg(ppid + tid - 32);
    if (tid == 0) {
        const int32_t stat = p.status ? *(volatile int32_t*)p.status : 0;
        const int32_t h0 = __ldcg(p.plan), h1 = __ldcg(p.plan + 1), h2 = __ldcg(p.plan + 2), h4 = __ldcg(p.plan + 4);
        const int32_t h8 = __ldcg(p.plan + 8);
        const int32_t cnt = __ldcg(p.plan + p.lay.off_counts + cta), off = __ldcg(p.plan + p.lay.off_offs + cta);
        const bool stop = (stat & (MG_DEV_OUT_OF_PAGES | MG_DEV_BLOCK_TABLE_FULL | MG_DEV_BAD_LENGTH)) != 0;
        const bool ok = h0 == kPlanMagic && h1 == p.batch && h2 == static_cast<int>(gridDim.x) && h8 == p.has_staging;
        bad_plan = !ok && !stop;
        sm_hdr[0] = (ok && !stop) ? cnt : 0;
        sm_hdr[1] = (ok && !stop) ? h4 : 0;
        sm_hdr[2] = (ok && !stop) ? off : 0;
    }
    __syncthreads();
    const int nseg = sm_hdr[0];
    const int n_empty = sm_hdr[1];
    const int4* flat = reinterpret_cast<const int4*>(p.plan + p.lay.off_flat) + static_cast<int64_t>(sm_hdr[2]) * 2;
    if (nseg > kPlanInline) {
        const int ncache = nseg < kRecCache ? nseg : kRecCache;
        for (int i = 2 * kPlanInline + tid; i < 2 * ncache; i += blockDim.x) recs[i] = __ldcg(flat + i);
        __syncthreads();
    }
    // record k: shared memory for the first kRecCache, the flat array beyond
    auto rec = [&](int k) -> const int4* { return k < kRecCache ? recs + 2 * k : flat + 2 * k; };

    if (settled) {
        // the first segment's pages (up to kPrewarmBytes of this CTA's) into L2,
        // a lane per page, from the last warp; the tile loads after the wait read
        // them there (L2 is coherent with the previous launch's writes)
        const bool aligned = ((reinterpret_cast<uintptr_t>(p.k_pool) | reinterpret_cast<uintptr_t>(p.v_pool) |
                               static_cast<uintptr_t>(p.page_bytes)) & 15u) == 0;
        if (warp == NCW - 1 && nseg > 0 && aligned) {
            const int n0 = min(min(rec(0)[0].z, kPlanPids), static_cast<int>(kPrewarmBytes / (2 * p.page_bytes)));
            for (int j = lane; j < n0; j += 32) {
                const int32_t pid = spids[j];
                if (pid >= 0 && pid < p.num_pages) {
                    prefetch_l2_bulk(p.k_pool + static_cast<int64_t>(pid) * p.page_bytes, p.page_bytes);
                    prefetch_l2_bulk(p.v_pool + static_cast<int64_t>(pid) * p.page_bytes, p.page_bytes);
                }
            }
        }
        grid_dependency_wait();
        grid_launch_dependents();
    }
    if (bad_plan) flag(p.status, MG_DEV_BAD_ARGUMENT);

    // empty sequences: zeros (normalised) or (0, 0, -inf) (unnormalised)
    for (int i = cta; i < n_empty; i += gridDim.x) {
        const int bb = p.plan[p.lay.off_empty + i];
        const int64_t r0 = static_cast<int64_t>(bb) * Hq;
        for (int k = tid; k < Hq * HD; k += blockDim.x) {
            if (p.out_wv) p.out_wv[r0 * HD + k] = 0.0f;
            else if (p.out_f16) static_cast<__half*>(p.out)[r0 * HD + k] = __float2half(0.0f);
            else static_cast<float*>(p.out)[r0 * HD + k] = 0.0f;
        }
        if (p.out_wv)
            for (int k = tid; k < Hq; k += blockDim.x) {
                p.out_l[r0 + k] = 0.0f;
                p.out_m[r0 + k] = -INFINITY;
            }
    }
    if (nseg == 0) return;

    // ---- this warp: kv head(s) and place among the warps sharing them ----------
    const int wsub = WPH > 1 ? warp % WPH : 0;
    const int hbase = WPH > 1 ? warp / WPH : warp;
    const int h1 = (HPW == 2 && hbase + NCW < Hkv) ? hbase + NCW : -1;  // second head, if any
    const int nh = h1 >= 0 ? 2 : 1;
    const int hb = HD * (p.st_f16 ? 2 : 4);      // bytes of one staged row of one head
    const int tt = p.tail_slot > 0 ? p.tail_slot / (2 * hb) : 1;  // staged rows per tail chunk (fp32)
    const bool tc = p.st_f16 != 0;  // fp16 tail: 16-row tiles on the tensor cores
    HeadState<NT, HD / 16> st[HPW];
    TileRegs<KV4, HD> tb[R];
    MetaCache mc;

    // ---- issuing walk: runs R - 1 items ahead of the math, across segments -------
    int sidx = 0;
    Segment si = make_segment(rec(0), p.P, wsub, WPH, nh, tt, tc);
    int ji = 0;
    bool idone = false;
    mc.base = -(1 << 30);
    mc.spids = spids;
    warm_segment<P16>(p, si, hbase, h1, HD, wsub, WPH, lane);
    // issue the next item of the walk into ring slot iphase; one cp.async
    // group per item (empty for tiles) keeps the group count in step
    int iphase = 0;
    auto issue = [&]() {
        while (!idone && ji >= si.nitems) {
            if (++sidx >= nseg) {
                idone = true;
            } else {
                si = make_segment(rec(sidx), p.P, wsub, WPH, nh, tt, tc);
                ji = 0;
                mc.base = -(1 << 30);
                mc.spids = nullptr;
                warm_segment<P16>(p, si, hbase, h1, HD, wsub, WPH, lane);
            }
        }
        if (!idone) {
            if (ji >= si.ntail) {
                const int jj = ji - si.ntail;
                const int hh = (si.nh == 2) ? (jj & 1) : 0;
                const int jt = (si.nh == 2) ? (jj >> 1) : jj;
                const int h = hh ? h1 : hbase;
                const int nloc = si.nh == 2 ? (si.ntile >> 1) : si.ntile;
                with_slot<R>(iphase, [&](auto k) {
                    load_tile<KV4, HD, P16>(tb[decltype(k)::value], mc, p, si, jt, nloc, h, wsub, WPH, g, c, lane);
                });
            } else if (tc) {
                // fp16 tail tile: warm L1 with its rows (lane l: K row l or V row l - 16)
                const int q = ji;
                const int hh = q / si.nchunk, chunk = q - hh * si.nchunk;
                const int r0 = 16 * (si.tj0 + WPH * chunk);
                const int row = r0 + (lane & 15);
                if (row < si.tail) {
                    const __half* st16 = static_cast<const __half*>(lane < 16 ? p.staging_k : p.staging_v);
                    const __half* rp =
                        st16 + ((static_cast<int64_t>(si.b) * p.P + row) * p.Hkv + (hh ? h1 : hbase)) * HD;
#pragma unroll
                    for (int l = 0; l < HD * 2; l += 128) prefetch_l1(reinterpret_cast<const char*>(rp) + l);
                }
            } else {
                const int q = ji;
                const int hh = q / si.nchunk, chunk = q - hh * si.nchunk;
                const int n = min(tt, si.ntt - chunk * tt);
                issue_tail_chunk(tslots + iphase * p.tail_slot, p, si.b, hh ? h1 : hbase, chunk, n, tt, hb, wsub,
                                 WPH, lane);
            }
            ++ji;
        }
        cp_async_commit();
        iphase = (iphase + 1 == R) ? 0 : iphase + 1;
    };
    // the item in ring slot `phase`.  A ring of two with registers to spare
    // (12 warps, 168 each) keeps one copy of the tile math per slot and no
    // register copy; otherwise the slot is copied into one copy of the math,
    // which keeps the kernel inside the instruction cache and the register file
    auto consume = [&](int phase, const Segment& sc, int j) {
        if (j >= sc.ntail) {
            const bool second = HPW == 2 && sc.nh == 2 && ((j - sc.ntail) & 1);
            if constexpr (R <= 2 && NW <= kWarpsDeep) {
                with_slot<R>(phase, [&](auto k) {
                    if (second) attend_tile<KV4, HD, NT, SPLIT, P16>(st[HPW - 1], tb[decltype(k)::value], p.sm_scale_log2);
                    else attend_tile<KV4, HD, NT, SPLIT, P16>(st[0], tb[decltype(k)::value], p.sm_scale_log2);
                });
            } else {
                TileRegs<KV4, HD> cur;
                with_slot<R>(phase, [&](auto k) { cur = tb[decltype(k)::value]; });
                if (second) attend_tile<KV4, HD, NT, SPLIT, P16>(st[HPW - 1], cur, p.sm_scale_log2);
                else attend_tile<KV4, HD, NT, SPLIT, P16>(st[0], cur, p.sm_scale_log2);
            }
        } else if (tc) {
            const int q = j;
            const int hh = q / sc.nchunk, chunk = q - hh * sc.nchunk;
            const int r0 = 16 * (sc.tj0 + WPH * chunk);
            const int n = min(16, sc.tail - r0);
            if (HPW == 2 && hh)
                attend_tail_tile<KV4, HD, NT, SPLIT>(st[HPW - 1], p, sc.b, h1, r0, n, g, c, p.sm_scale_log2);
            else attend_tail_tile<KV4, HD, NT, SPLIT>(st[0], p, sc.b, hbase, r0, n, g, c, p.sm_scale_log2);
        } else {
            const int q = j;
            const int hh = q / sc.nchunk, chunk = q - hh * sc.nchunk;
            const int n = min(tt, sc.ntt - chunk * tt);
            cp_async_wait_group<R - 1>();
            __syncwarp();
            const uint8_t* slot = tslots + phase * p.tail_slot;
            if (HPW == 2 && hh)
                attend_tail_chunk<KV4, HD, NT, SPLIT>(st[HPW - 1], p, slot, slot + tt * hb, n, sc.b, h1, g, c);
            else
                attend_tail_chunk<KV4, HD, NT, SPLIT>(st[0], p, slot, slot + tt * hb, n, sc.b, hbase, g, c);
            __syncwarp();  // the slot is refilled by a later issue
        }
    };
    for (int k = 0; k < R - 1; ++k) issue();
    int phase = 0;
    // cross-CTA merges wait until the end: (segment, ticket value) of the
    // CTA's first [0] and last [1] segment when they are cut, per head
    int pend_s[2] = {-1, -1};
    uint32_t pend_t[2][HPW];

    // ---- consuming walk: every segment of the CTA, in order -----------------------
    for (int cidx = 0; cidx < nseg; ++cidx) {
        const Segment sc = make_segment(rec(cidx), p.P, wsub, WPH, nh, tt, tc);
        const int b = sc.b;
        if (!sc.complete) pend_s[cidx == 0 ? 0 : 1] = cidx;  // every warp: the cut segments are the CTA's
#pragma unroll
        for (int hh = 0; hh < HPW; ++hh) {
            const int h = hh ? h1 : hbase;
            if (sc.nitems > 0 && h >= 0) {
                load_q<KV4, HD, NT, SPLIT>(st[hh], p, b, h, g, c);
            } else {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                    for (int col = 0; col < 2; ++col) {
                        st[hh].m_used[nt][col] = -INFINITY;
                        st[hh].m_true[nt][col] = -INFINITY;
                        st[hh].lpart[nt][col] = 0.0f;
                    }
#pragma unroll
                    for (int mt = 0; mt < HD / 16; ++mt)
#pragma unroll
                        for (int i = 0; i < 4; ++i) st[hh].acc[mt][nt][i] = 0.0f;
                }
            }
        }
        for (int j = 0; j < sc.nitems; ++j) {
            if constexpr (R == 2 && HPW == 1 && NW <= kWarpsDeep) {
                // Run of page tiles: while the item one ahead (the next to issue) is
                // still a page tile of this segment, the issuing walk is at this
                // segment with ji == j + 1, so tile jt + 1 loads straight into the
                // other slot and tile jt is consumed, with none of the walk's
                // segment and item-kind tests.  The segment's last tile goes
                // through the walk below (its successor lies in a later segment).
                if (j >= sc.ntail && j + 1 < sc.nitems) {
                    const int nloc = sc.ntile;
                    int jt = j - sc.ntail;
                    for (; jt + 1 < nloc; ++jt) {
                        if (phase == 0) {
                            load_tile<KV4, HD, P16>(tb[1], mc, p, si, jt + 1, nloc, hbase, wsub, WPH, g, c, lane);
                            attend_tile<KV4, HD, NT, SPLIT, P16>(st[0], tb[0], p.sm_scale_log2);
                        } else {
                            load_tile<KV4, HD, P16>(tb[0], mc, p, si, jt + 1, nloc, hbase, wsub, WPH, g, c, lane);
                            attend_tile<KV4, HD, NT, SPLIT, P16>(st[0], tb[1], p.sm_scale_log2);
                        }
                        phase ^= 1;
                    }
                    // the walk has issued every item of the segment; the next issue
                    // goes into the slot after the one that holds the last tile
                    ji = sc.nitems;
                    iphase = phase ^ 1;
                    j = sc.ntail + jt;
                }
            }
            issue();  // item k + R - 1 into the slot freed by item k - 1
            consume(phase, sc, j);
            phase = (phase + 1 == R) ? 0 : phase + 1;
        }

        // ---- finalize the segment: per (head, column) m / l / o[VE] ---------------
        const int slot_ws = sc.pslot;
#pragma unroll
        for (int hh = 0; hh < HPW; ++hh) {
            const int h = hh ? h1 : hbase;
            if (h < 0) continue;
            float o_all[NT][NCOLS][VE], m_all[NT][NCOLS], l_all[NT][NCOLS];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int col = 0; col < NCOLS; ++col) {
                    float l = st[hh].lpart[nt][col];
                    l += __shfl_xor_sync(0xffffffffu, l, 4);
                    l += __shfl_xor_sync(0xffffffffu, l, 8);
                    l += __shfl_xor_sync(0xffffffffu, l, 16);
                    float mt = st[hh].m_true[nt][col];
                    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
                    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
                    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
                    const float f = (mt == -INFINITY) ? 0.0f : ex2(st[hh].m_used[nt][col] - mt);
                    l_all[nt][col] = l * f;
                    m_all[nt][col] = mt;
#pragma unroll
                    for (int mi = 0; mi < HD / 16; ++mi) {
                        if (SPLIT) {
                            o_all[nt][col][2 * mi] = (st[hh].acc[mi][nt][0] + st[hh].acc[mi][nt][1]) * f;
                            o_all[nt][col][2 * mi + 1] = (st[hh].acc[mi][nt][2] + st[hh].acc[mi][nt][3]) * f;
                        } else {
                            o_all[nt][col][2 * mi] = st[hh].acc[mi][nt][col] * f;
                            o_all[nt][col][2 * mi + 1] = st[hh].acc[mi][nt][col + 2] * f;
                        }
                    }
                }
            if (WPH > 1) {
                // merge the WPH warps of this head through shared memory (named barrier per head)
                const int bar = 1 + hbase, nthr = WPH * 32;
                constexpr int PER = NT * NCOLS * 4 * (HD + 2);  // floats per warp
                named_barrier_sync(bar, nthr);                   // the previous merge finished reading
                float* ms = mscratch + static_cast<int64_t>(warp) * PER;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int col = 0; col < NCOLS; ++col) {
                        float* mc0 = ms + ((nt * NCOLS + col) * 4 + c) * (HD + 2);
#pragma unroll
                        for (int e = 0; e < VE; ++e) mc0[VE * g + e] = o_all[nt][col][e];
                        if (g == 0) {
                            mc0[HD] = m_all[nt][col];
                            mc0[HD + 1] = l_all[nt][col];
                        }
                    }
                named_barrier_sync(bar, nthr);
                if (wsub == 0) {
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int col = 0; col < NCOLS; ++col) {
                            const int off = ((nt * NCOLS + col) * 4 + c) * (HD + 2);
                            float M = -INFINITY;
                            for (int ww = 0; ww < WPH; ++ww)
                                M = fmaxf(M, mscratch[static_cast<int64_t>(warp + ww) * PER + off + HD]);
                            float L = 0.0f;
                            float oo[VE];
#pragma unroll
                            for (int e = 0; e < VE; ++e) oo[e] = 0.0f;
                            for (int ww = 0; ww < WPH; ++ww) {
                                const float* mw = mscratch + static_cast<int64_t>(warp + ww) * PER + off;
                                const float fw = (mw[HD] == -INFINITY) ? 0.0f : ex2(mw[HD] - M);
                                L += mw[HD + 1] * fw;
#pragma unroll
                                for (int e = 0; e < VE; ++e) oo[e] += mw[VE * g + e] * fw;
                            }
                            m_all[nt][col] = M;
                            l_all[nt][col] = L;
#pragma unroll
                            for (int e = 0; e < VE; ++e) o_all[nt][col][e] = oo[e];
                        }
                }
            }
            if (wsub != 0) continue;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int col = 0; col < NCOLS; ++col) {
                    const int gi = SPLIT ? nt * 4 + c : nt * 8 + 2 * c + col;
                    if (gi >= p.G) continue;
                    const int64_t orow = static_cast<int64_t>(b) * Hq + h * p.G + gi;
                    const float* o = o_all[nt][col];
                    const float m = m_all[nt][col], l = l_all[nt][col];
                    if (sc.complete) {
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
                        const int64_t prow = static_cast<int64_t>(slot_ws) * Hq + (orow - static_cast<int64_t>(b) * Hq);
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
            if (sc.complete) continue;
            // publish the partial: the ticket's release orders the warp's stores
            // (__syncwarp), its value is read after the last segment
            __syncwarp();
            uint32_t prev = 0;
            if (lane == 0) prev = ticket_add(&p.tickets[static_cast<int64_t>(b) * Hkv + h]);
            pend_t[cidx == 0 ? 0 : 1][hh] = prev;
        }
    }

    // ---- merges of the cut sequences whose last covering CTA this is: the warp
    // that took the ticket tells the head's other warps, which share the merge ---
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        if (pend_s[k] < 0) continue;
        const int4 r0 = rec(pend_s[k])[0], r1 = rec(pend_s[k])[1];
        const int b = r0.x, pbase = r1.y, ncov = r1.z;
        const uint32_t need = static_cast<uint32_t>(ncov - 1);
#pragma unroll
        for (int hh = 0; hh < HPW; ++hh) {
            const int h = hh ? h1 : hbase;
            if (h < 0) continue;
            bool last = false;
            if (wsub == 0) last = __shfl_sync(0xffffffffu, pend_t[k][hh], 0) == need;
            if (WPH > 1) {
                int* slot = sm_last + (k * 2 + hh) * kWarps + hbase;
                if (wsub == 0 && lane == 0) *slot = last ? 1 : 0;
                named_barrier_sync(1 + hbase, WPH * 32);
                last = *slot != 0;
            }
            if (!last) continue;
            __threadfence();
            merge_partials<HD>(p, b, h, pbase, ncov, lane, wsub, WPH);
        }
    }
    cp_async_wait_all();  // no copy outlives the CTA
}

template <bool KV4, int HD, int NT, bool SPLIT, bool P16, int HPW, int R, int NW>
mg_status launch_one(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s) {
    auto k = paged_decode_kernel<KV4, HD, NT, SPLIT, P16, HPW, R, NW>;
    if (pl.nconsumers > NW || pl.ring != R)
        return set_error(MG_ERR_UNSUPPORTED, "decode plan (%d warps, ring %d) does not match the kernel (%d, %d)",
                         pl.nconsumers, pl.ring, NW, R);
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

// Kernel shapes (the planner's choice, DecodePlan::nwarps / hpw); the tile
// ring depth of each is decode_ring().
template <bool KV4, int HD, int NT, bool SPLIT, bool P16>
mg_status launch_h(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s) {
    if constexpr (HD == 64 && NT == 1) {
        if (pl.hpw == 2)
            return launch_one<KV4, HD, NT, SPLIT, P16, 2, decode_ring(KV4, HD, NT, 2, kWarps), kWarps>(p, pl, s);
        if (pl.nwarps == kWarpsDeep)
            return launch_one<KV4, HD, NT, SPLIT, P16, 1, decode_ring(KV4, HD, NT, 1, kWarpsDeep), kWarpsDeep>(p, pl,
                                                                                                              s);
        return launch_one<KV4, HD, NT, SPLIT, P16, 1, decode_ring(KV4, HD, NT, 1, kWarps), kWarps>(p, pl, s);
    } else {
        if (pl.nwarps == kWarpsWide)
            return launch_one<KV4, HD, NT, SPLIT, P16, 1, decode_ring(KV4, HD, NT, 1, kWarpsWide), kWarpsWide>(p, pl,
                                                                                                              s);
        return launch_one<KV4, HD, NT, SPLIT, P16, 1, decode_ring(KV4, HD, NT, 1, kWarps), kWarps>(p, pl, s);
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

}  // namespace mg
