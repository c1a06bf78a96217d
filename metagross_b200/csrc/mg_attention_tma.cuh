// Fused paged decode attention, bulk-copy variant: the pages reach shared
// memory through the Tensor Memory Accelerator, and the warps that do the math
// hold no page data in flight.
//
// Used for the layout every benchmark shape has: 16-token pages, one scale per
// physical page (K and V separately, metagross/cache.py:39), exact fp16 staged
// tails, head_dim 64 or 128, at most 16 kv heads.  Other layouts (token-head
// scales, other page sizes, fp32 tails, the legacy committed-page op) run the
// register-streaming kernel of mg_attention_kernel.cuh.  The reference
// semantics are those of csrc/paged_attention.cu:25-135 and
// metagross/attention.py:62-134; the work split is the step's decode plan
// (mg_plan.cu), shared with the other kernel.
//
//   producer  one warp per CTA walks the CTA's plan segments page by page.  Its
//             lanes read 32 block-table entries at a time (the next 32 are in
//             flight meanwhile) and the pages' two scales; lane 0 issues one
//             tiled TMA copy for the K page and one for the V page into a ring
//             of NS shared-memory stages.  The tensor map permutes the page's
//             [token][kv head][row] order to [kv head][token][row] and swizzles
//             16-byte chunks, so each head's 16-token tile is contiguous and
//             ldmatrix reads it without bank conflicts.  A stage's "full"
//             mbarrier completes when the copies have landed (transaction
//             bytes) and the lane that holds the page's scales has stored them
//             next to it; its "empty" mbarrier completes when every kv head's
//             consumer warp has read its tile.
//   consumers Hkv x WPH warps: warp (h, w) takes kv head h of pages k with
//             k % WPH == w.  It reads its tile's K and V fragments with four
//             (INT8) or two (INT4) ldmatrix.x4, releases the stage, and runs
//             the tile on the tensor cores (mma.sync m16n8k16, fp16 in, fp32
//             accumulate): S^T = K Q^T, online softmax in the log2 domain with
//             lazy rescaling, O^T += V^T P^T.
//   codes     an INT8 code b becomes the fp16 1152 + b with one LOP3 (bits of
//             1024 + (b ^ 0x80)); an INT4 nibble c in the low half of a byte
//             becomes 1032 + c, in the high half 1152 + 16 c.  INT8 K keeps
//             its offset: each tile's scores subtract q . offsets (one
//             constant per query column, computed with q), exact to fp32
//             rounding of one tile's sums.  Everywhere else the offsets are
//             subtracted per element (an exact fp16 HSUB2): the V
//             accumulators run over the whole context, so an offset x
//             sum-of-P term there grows with it (measured 3.6e-3 on
//             3587-token INT4 contexts), and INT4 page scales are large
//             enough that a folded K term showed too (2.03e-3 with outliers).
//             High nibbles come out as 16 c; q's B operand carries the 1/16
//             for those K dimensions, and those V rows are divided at the end.
//   tail      the < 16 exact fp16 staged rows of a sequence are one more tile,
//             read straight from global memory by the warp after its pages
//             (an L1 prefetch went out at the segment's start), with its own
//             unscaled copy of q and no offsets.
//   merges    as in the register kernel: the WPH warps of a head through shared
//             memory behind a named barrier of those warps, cut sequences
//             through per-(sequence, kv head) tickets and one log-sum-exp pass
//             by the last piece.
//   waits     every mbarrier wait is bounded (iterations and %globaltimer); a
//             wait that gives up sets MG_DEV_TIMEOUT, stops the warp's math but
//             not its barrier arrivals, and the producer waits (bounded) for
//             its copies in flight before the CTA exits.
#pragma once

#include <cuda.h>

#include "mg_attention.cuh"

namespace mg {

template <bool KV4, int HD>
struct TCfg;
// slots of a consumer warp's private ring in the self-copying mode (a power of two)
template <bool KV4, int HD>
constexpr int kSelfSlots = (KV4 ? HD : 2 * HD) * 16 <= 1024 ? 8 : 4;

template <bool KV4, int HD>
struct TCfg {
    static constexpr int ROWB = KV4 ? HD / 2 : HD;   // bytes of one (token, kv head) row
    static constexpr int TILE = 16 * ROWB;            // one head's 16-token tile in a stage
    static constexpr int CHUNKS = ROWB / 16;          // 16-byte chunks per row
    static constexpr int X4 = CHUNKS / 2;             // ldmatrix.x4 per tile per operand
    static constexpr int SWB = ROWB == 32 ? 1 : ROWB == 64 ? 2 : 3;  // TMA swizzle: Swizzle<SWB, 4, 3>
    static constexpr int MT = HD / 16;                // k-steps of K = m-tiles of V^T
    static constexpr int VE = HD / 8;                 // output values per lane per query column
};

// Offset of 16-byte chunk j of row t inside a tile written by a TMA copy with
// the tile's swizzle (address bits [4, 4 + SWB) XOR bits [7, 7 + SWB)); tiles
// start on a multiple of the swizzle period.
template <bool KV4, int HD>
__device__ __forceinline__ uint32_t tile_chunk_off(int t, int j) {
    using T = TCfg<KV4, HD>;
    const uint32_t o = static_cast<uint32_t>(t * T::ROWB + 16 * j);
    return o ^ (((o >> 7) & ((1u << T::SWB) - 1u)) << 4);
}

// Head dimension held by output value e (e = 2 m-tile + row half) of lane row g.
template <bool KV4>
__host__ __device__ __forceinline__ int tdim(int g, int e) {
    const int mt = e >> 1, r = e & 1;
    return KV4 ? 64 * (mt >> 2) + 32 * r + 4 * g + (mt & 3) : 32 * (mt >> 1) + 16 * r + 2 * g + (mt & 1);
}

// Head dimensions of q held in B-fragment slot s (0: k 2c, 1: 2c+1, 2: 2c+8,
// 3: 2c+9) of k-step kk, lane column c; must match the K fragments below.
template <bool KV4>
__device__ __forceinline__ int tq_dim(int kk, int c, int s) {
    if (!KV4) return 16 * kk + 4 * c + ((s == 0) ? 0 : (s == 1) ? 2 : (s == 2) ? 1 : 3);
    const int d0 = 32 * (kk >> 1) + 8 * c + 2 * (kk & 1);
    return d0 + ((s == 0) ? 0 : (s == 1) ? 4 : (s == 2) ? 1 : 5);
}

__device__ __forceinline__ uint32_t cvt8(uint32_t x) { return lop3_and_xor(x, 0x00FF00FFu, 0x64806480u); }  // 1152 + b
__device__ __forceinline__ uint32_t lo4(uint32_t x) { return lop3_and_or(x, 0x000F000Fu, 0x64006400u); }  // 1032 + c
__device__ __forceinline__ uint32_t hi4(uint32_t x) { return lop3_and_or(x, 0x00F000F0u, 0x64006400u); }  // 1152 + 16 c
// The same for two's-complement nibbles s (c = s mod 16), the sign flip folded
// into the one LOP3: (c ^ 8) = s + 8, so the low form is 1032 + s and the high
// form 1152 + 16 s (the bits XORed in and ORed in do not overlap).
__device__ __forceinline__ uint32_t lo4s(uint32_t x) { return lop3_and_xor(x, 0x000F000Fu, 0x64086408u); }
__device__ __forceinline__ uint32_t hi4s(uint32_t x) { return lop3_and_xor(x, 0x00F000F0u, 0x64806480u); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for the phase of `parity` to complete: at most 2^22 attempts and
// 200 ms; false when it gave up.
__device__ __forceinline__ bool mbar_wait_limited(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && global_ns() - t0 > 200000000ull) break;
    }
    return false;
}
// The compiler must have these registers' values (the loads that write them
// have completed) before anything after this point.
__device__ __forceinline__ void regs_ready(const uint32_t* r, int n) {
#pragma unroll
    for (int i = 0; i < n; ++i) asm volatile("" ::"r"(r[i]) : "memory");
}

// Tiled TMA copy of one whole page into a stage: the permuted 4-D map
// (row bytes, token, kv head, page) at (0, 0, 0, pid), or, when the driver
// declined that map, one 3-D copy (row bytes, kv head, token of the pool) per
// kv head issued by lanes 0 .. Hkv-1.  Every copy lands in this CTA's own shared memory.
__device__ __forceinline__ void tma_page(uint8_t* dst, const CUtensorMap* tm, int pid, uint64_t* bar, int per_head,
                                         int Hkv, int P, int tile, int lane) {
    if (!per_head) {
        if (lane == 0)
            asm volatile(
                "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
                "l"(reinterpret_cast<uint64_t>(tm)), "r"(0), "r"(0), "r"(0), "r"(pid), "r"(smem_u32(bar))
                : "memory");
    } else if (lane < Hkv) {
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst + lane * tile)),
            "l"(reinterpret_cast<uint64_t>(tm)), "r"(0), "r"(lane), "r"(pid * P), "r"(smem_u32(bar))
            : "memory");
    }
}

// Softmax state of one kv head's query columns; qb: q . (code offsets) of the
// columns this lane's score fragment holds (2c, 2c + 1).
template <int NT, int MT>
struct TmaHead {
    uint32_t qf[NT][MT][2];
    float acc[MT][NT][4];
    float m_used[NT][2];
    float m_true[NT][2];
    float lpart[NT][2];
    float qb[NT][2];
};

// q of kv head h of sequence b into the page B fragments (INT4: the slots of
// high-nibble dimensions divided by 16) and the per-column offsets.
template <bool KV4, int HD, int NT, bool SPLIT>
__device__ __forceinline__ void tma_load_q(TmaHead<NT, HD / 16>& S, const DecodeParams& p, int b, int h, int g,
                                           int c) {
    constexpr int MT = HD / 16;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int gi = SPLIT ? nt * 4 + (g >> 1) : nt * 8 + g;  // B-fragment column g
        const bool live = gi < p.G;
        const int64_t qrow = (static_cast<int64_t>(b) * p.Hq + static_cast<int64_t>(h) * p.G + gi) * HD;
        float qb = 0.0f;
#pragma unroll
        for (int kk = 0; kk < MT; ++kk) {
            float v[4];
#pragma unroll
            for (int s = 0; s < 4; ++s) v[s] = live ? load_f(p.q, qrow + tq_dim<KV4>(kk, c, s), p.q_f16) : 0.0f;
            if (SPLIT) {
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const float hi = __half2float(__float2half_rn(v[s]));
                    v[s] = (g & 1) ? (v[s] - hi) : hi;  // column pair (hi, lo)
                }
            }
            if (KV4) {
                v[2] *= 0.0625f;
                v[3] *= 0.0625f;
            }
            const __half2 b0 = __floats2half2_rn(v[0], v[1]), b1 = __floats2half2_rn(v[2], v[3]);
            S.qf[nt][kk][0] = *reinterpret_cast<const uint32_t*>(&b0);
            S.qf[nt][kk][1] = *reinterpret_cast<const uint32_t*>(&b1);
            if (!KV4) {  // INT8 K codes keep their +1152 offset: subtract q . offsets once per tile
                const float2 f0 = __half22float2(b0), f1 = __half22float2(b1);
                qb += 1152.0f * (f0.x + f0.y + f1.x + f1.y);
            }
        }
        qb += __shfl_xor_sync(0xffffffffu, qb, 1);
        qb += __shfl_xor_sync(0xffffffffu, qb, 2);
        // the score fragment of lane (g, c) holds columns 2c and 2c + 1
        S.qb[nt][0] = __shfl_sync(0xffffffffu, qb, 8 * c);
        S.qb[nt][1] = __shfl_sync(0xffffffffu, qb, 8 * c + 4);
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            S.m_used[nt][col] = -INFINITY;
            S.m_true[nt][col] = -INFINITY;
            S.lpart[nt][col] = 0.0f;
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) S.acc[mt][nt][i] = 0.0f;
    }
}

template <int NT, int MT>
__device__ __forceinline__ void tma_clear(TmaHead<NT, MT>& S) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            S.m_used[nt][col] = -INFINITY;
            S.m_true[nt][col] = -INFINITY;
            S.lpart[nt][col] = 0.0f;
            S.qb[nt][col] = 0.0f;
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) S.acc[mt][nt][i] = 0.0f;
    }
}

// Online-softmax update for NTL 16-token tiles taken together, whose raw
// scores (K Q^T, code offsets already removed) are sc[t][NT][4] (rows g, g + 8
// x columns 2c, 2c + 1 of tile t), then O^T += V^T P^T over the m-tiles
// vf(t, mt, a) supplies.  ks[t][r] / vs[t][r]: score scale (log2 domain) and V
// scale of row g + 8 r of tile t; live[t][r] masks dead rows.  is16(mt):
// multiply P by 16 for that m-tile (tail tiles of INT4 caches, whose V rows
// are not scaled by 16 as high-nibble codes are).  With two tiles the warp
// has two independent score chains in flight and pays one running-max check
// for 32 tokens.
template <int HD, int NT, bool SPLIT, int NTL, typename VF, typename H16>
__device__ __forceinline__ void tma_softmax_pv(TmaHead<NT, HD / 16>& S, float (&sc)[NTL][NT][4], VF&& vf,
                                               H16&& is16, const float (&ks)[NTL][2], const float (&vs)[NTL][2],
                                               const bool (&live)[NTL][2]) {
    constexpr int MT = HD / 16;
    constexpr int NCOLS = SPLIT ? 1 : 2;
    float s[NTL][NT][NCOLS][2];
#pragma unroll
    for (int t = 0; t < NTL; ++t)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            if (SPLIT) {
                s[t][nt][0][0] = live[t][0] ? (sc[t][nt][0] + sc[t][nt][1]) * ks[t][0] : -INFINITY;
                s[t][nt][0][1] = live[t][1] ? (sc[t][nt][2] + sc[t][nt][3]) * ks[t][1] : -INFINITY;
            } else {
#pragma unroll
                for (int col = 0; col < NCOLS; ++col) {
                    s[t][nt][col][0] = live[t][0] ? sc[t][nt][col] * ks[t][0] : -INFINITY;
                    s[t][nt][col][1] = live[t][1] ? sc[t][nt][2 + col] * ks[t][1] : -INFINITY;
                }
            }
        }
    bool need = false;
    float mx[NT][NCOLS];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int col = 0; col < NCOLS; ++col) {
            float m = fmaxf(s[0][nt][col][0], s[0][nt][col][1]);
#pragma unroll
            for (int t = 1; t < NTL; ++t) m = fmaxf(m, fmaxf(s[t][nt][col][0], s[t][nt][col][1]));
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
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    if (SPLIT) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) S.acc[mt][nt][i] *= alpha;
                    } else {
                        S.acc[mt][nt][col] *= alpha;
                        S.acc[mt][nt][col + 2] *= alpha;
                    }
                }
            }
    }
#pragma unroll
    for (int t = 0; t < NTL; ++t) {
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float pr[NCOLS][2];
#pragma unroll
            for (int col = 0; col < NCOLS; ++col)
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    pr[col][r] = ex2(s[t][nt][col][r] - S.m_used[nt][col]);
                    S.lpart[nt][col] += pr[col][r];
                }
            uint32_t hrow[2];
            if (SPLIT) {
                const float a0 = pr[0][0] * vs[t][0], a1 = pr[0][1] * vs[t][1];
                const float a0h = __half2float(__float2half_rn(a0));
                const float a1h = __half2float(__float2half_rn(a1));
                hrow[0] = pack_half2(a0h, a0 - a0h);
                hrow[1] = pack_half2(a1h, a1 - a1h);
            } else {
                hrow[0] = pack_half2(pr[0][0] * vs[t][0], pr[NCOLS - 1][0] * vs[t][0]);
                hrow[1] = pack_half2(pr[0][1] * vs[t][1], pr[NCOLS - 1][1] * vs[t][1]);
            }
            pb[nt][0] = movmatrix_trans(hrow[0]);
            pb[nt][1] = movmatrix_trans(hrow[1]);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            uint32_t a[4];
            vf(t, mt, a);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                if (is16(mt)) {
                    const uint32_t b0 = hfma2_u32(pb[nt][0], 0x4C004C00u, 0u);  // 0x4C00 = 16.0
                    const uint32_t b1 = hfma2_u32(pb[nt][1], 0x4C004C00u, 0u);
                    mma_16816(S.acc[mt][nt], a, b0, b1);
                } else {
                    mma_16816(S.acc[mt][nt], a, pb[nt][0], pb[nt][1]);
                }
            }
        }
    }
}

// Raw scores of one page tile in a stage (K fragments by ldmatrix at chunk
// offsets off[x] of this lane's matrix row); INT8 offsets removed here.  CH2:
// even and odd k-steps accumulate in two chains (shorter dependency, four more
// registers).
template <bool KV4, int HD, int NT, bool CH2>
__device__ __forceinline__ void tma_tile_scores(const TmaHead<NT, HD / 16>& S, uint32_t kbase,
                                                const uint32_t (&off)[TCfg<KV4, HD>::X4], float (&sc)[NT][4]) {
    using T = TCfg<KV4, HD>;
    constexpr int MT = T::MT;
    uint32_t kr[T::X4][4];
#pragma unroll
    for (int x = 0; x < T::X4; ++x) ldsm_x4(kr[x], kbase + off[x]);
    // kr[x] = {row g chunk 2x, row g+8 chunk 2x, row g chunk 2x+1, row g+8 chunk 2x+1}
    float sc2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sc[nt][i] = 0.0f;
            sc2[nt][i] = 0.0f;
        }
#pragma unroll
    for (int kk = 0; kk < MT; ++kk) {
        uint32_t a[4];
        if (!KV4) {
            const uint32_t w = kr[kk >> 1][(kk & 1) * 2], w8 = kr[kk >> 1][(kk & 1) * 2 + 1];
            a[0] = cvt8(w);
            a[1] = cvt8(w8);
            a[2] = cvt8(w >> 8);
            a[3] = cvt8(w8 >> 8);
        } else {
            const int j = kk >> 1;  // chunk
            uint32_t w = kr[j >> 1][(j & 1) * 2], w8 = kr[j >> 1][(j & 1) * 2 + 1];
            if (kk & 1) {
                w >>= 8;
                w8 >>= 8;
            }
            // INT4 scores subtract the offsets per element (exact), unlike INT8:
            // INT4 page scales are ~18x larger, and with 1 % outliers x8 the
            // rounding of a folded q . offsets term measurably reached the
            // output (2.03e-3 on the TinyLlama shape).  High nibbles stay 16 c
            // (q carries the 1/16).
            a[0] = hsub2_u32(lo4s(w), 0x64086408u);
            a[1] = hsub2_u32(lo4s(w8), 0x64086408u);
            a[2] = hsub2_u32(hi4s(w), 0x64806480u);
            a[3] = hsub2_u32(hi4s(w8), 0x64806480u);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            if (CH2 && (kk & 1)) mma_16816(sc2[nt], a, S.qf[nt][kk][0], S.qf[nt][kk][1]);
            else mma_16816(sc[nt], a, S.qf[nt][kk][0], S.qf[nt][kk][1]);
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sc[nt][i] = CH2 ? sc[nt][i] + sc2[nt][i] : sc[nt][i];
            if (!KV4) sc[nt][i] -= S.qb[nt][i & 1];  // INT4 K codes come without offsets
        }
}

// V^T A-fragment of m-tile mt from the ldmatrix.trans words vr of a page tile,
// codes without offsets (exact fp16 subtraction), so the accumulators never
// carry an offset x sum-of-P term across tiles.
template <bool KV4, int HD>
__device__ __forceinline__ void tma_vfrag(const uint32_t (&vr)[TCfg<KV4, HD>::X4][4], int mt, uint32_t (&a)[4]) {
    if (!KV4) {
        // vr[mt >> 1] = {tokens 0-7 chunk 2p, 8-15 chunk 2p, 0-7 chunk 2p+1, 8-15 chunk 2p+1}
        const uint32_t* r = vr[mt >> 1];
        const int sh = (mt & 1) * 8;
        a[0] = hsub2_u32(cvt8(r[0] >> sh), 0x64806480u);
        a[1] = hsub2_u32(cvt8(r[2] >> sh), 0x64806480u);
        a[2] = hsub2_u32(cvt8(r[1] >> sh), 0x64806480u);
        a[3] = hsub2_u32(cvt8(r[3] >> sh), 0x64806480u);
    } else {
        // high nibbles come out as 16 c (1152 + 16 c - 1152): that m-tile's
        // outputs are divided by 16 at the end
        const uint32_t* r = vr[mt >> 2];
        const int n = mt & 3;
        uint32_t x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = r[i] >> ((n >> 1) * 8);
        const bool hi = n & 1;
        const uint32_t o = hi ? 0x64806480u : 0x64086408u;
        a[0] = hsub2_u32(hi ? hi4s(x[0]) : lo4s(x[0]), o);
        a[1] = hsub2_u32(hi ? hi4s(x[2]) : lo4s(x[2]), o);
        a[2] = hsub2_u32(hi ? hi4s(x[1]) : lo4s(x[1]), o);
        a[3] = hsub2_u32(hi ? hi4s(x[3]) : lo4s(x[3]), o);
    }
}

// NTL (1 or 2) page tiles of kv head h from their stages: the scores of each,
// then the V fragments; each stage is released once its V words are in
// registers, then the softmax and O^T += V^T P^T for all of them.
template <bool KV4, int HD, int NT, bool SPLIT, int NTL, bool CH2>
__device__ __forceinline__ void tma_page_tiles(TmaHead<NT, HD / 16>& S, const uint32_t (&kbase)[NTL],
                                               const uint32_t (&off)[TCfg<KV4, HD>::X4], uint32_t vdelta,
                                               const float (&ksc)[NTL], const float (&vsc)[NTL],
                                               uint64_t* const (&empty)[NTL], int lane) {
    using T = TCfg<KV4, HD>;
    float sc[NTL][NT][4];
#pragma unroll
    for (int t = 0; t < NTL; ++t) tma_tile_scores<KV4, HD, NT, CH2>(S, kbase[t], off, sc[t]);
    uint32_t vr[NTL][T::X4][4];
#pragma unroll
    for (int t = 0; t < NTL; ++t)
#pragma unroll
        for (int x = 0; x < T::X4; ++x) ldsm_x4_t(vr[t][x], kbase[t] + vdelta + off[x]);
    regs_ready(&vr[0][0][0], 4 * T::X4 * NTL);
    __syncwarp();
    if (lane == 0) {
#pragma unroll
        for (int t = 0; t < NTL; ++t)
            if (empty[t]) mbar_arrive(empty[t]);  // (no barrier: the warp copied the tile itself)
    }
    float ks[NTL][2], vs[NTL][2];
    bool live[NTL][2];
#pragma unroll
    for (int t = 0; t < NTL; ++t) {
        ks[t][0] = ks[t][1] = ksc[t];
        vs[t][0] = vs[t][1] = vsc[t];
        live[t][0] = live[t][1] = true;
    }
    tma_softmax_pv<HD, NT, SPLIT, NTL>(
        S, sc, [&](int t, int mt, uint32_t (&a)[4]) { tma_vfrag<KV4, HD>(vr[t], mt, a); }, [](int) { return false; },
        ks, vs, live);
}

// The staged tail of kv head h of sequence b: rows 0 .. n - 1 (n < 16) of the
// exact fp16 staging, read from global memory (L1), with an unscaled q.
template <bool KV4, int HD, int NT, bool SPLIT>
__device__ __forceinline__ void tma_tail_tile(TmaHead<NT, HD / 16>& S, const DecodeParams& p, int b, int h, int n,
                                              int g, int c) {
    constexpr int MT = HD / 16;
    const int64_t rs = static_cast<int64_t>(p.Hkv) * HD;  // halves per staged token row
    const __half* kb = static_cast<const __half*>(p.staging_k) + (static_cast<int64_t>(b) * p.P * p.Hkv + h) * HD;
    const __half* vb = static_cast<const __half*>(p.staging_v) + (kb - static_cast<const __half*>(p.staging_k));
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nt][i] = 0.0f;
    // ---- scores: K rows g, g + 8 against an unscaled q ----
#pragma unroll
    for (int kk = 0; kk < MT; ++kk) {
        uint32_t a[4];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int row = g + 8 * r;
            const __half* src = kb + row * rs;
            if (!KV4) {
                uint2 u = make_uint2(0u, 0u);
                if (row < n) u = *reinterpret_cast<const uint2*>(src + 16 * kk + 4 * c);
                a[r] = __byte_perm(u.x, u.y, 0x5410);      // dims 4c, 4c + 2
                a[r + 2] = __byte_perm(u.x, u.y, 0x7632);  // dims 4c + 1, 4c + 3
            } else {
                uint4 u = make_uint4(0u, 0u, 0u, 0u);
                if (row < n) u = *reinterpret_cast<const uint4*>(src + 32 * (kk >> 1) + 8 * c);
                const uint32_t lo = (kk & 1) ? u.y : u.x, hi = (kk & 1) ? u.w : u.z;
                a[r] = __byte_perm(lo, hi, 0x5410);      // dims d0, d0 + 4
                a[r + 2] = __byte_perm(lo, hi, 0x7632);  // dims d0 + 1, d0 + 5
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int gi = SPLIT ? nt * 4 + (g >> 1) : nt * 8 + g;
            const bool live = gi < p.G;
            const int64_t qrow = (static_cast<int64_t>(b) * p.Hq + static_cast<int64_t>(h) * p.G + gi) * HD;
            float v[4];
#pragma unroll
            for (int s = 0; s < 4; ++s) v[s] = live ? load_f(p.q, qrow + tq_dim<KV4>(kk, c, s), p.q_f16) : 0.0f;
            if (SPLIT) {
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const float hi = __half2float(__float2half_rn(v[s]));
                    v[s] = (g & 1) ? (v[s] - hi) : hi;
                }
            }
            mma_16816(sc[nt], a, pack_half2(v[0], v[1]), pack_half2(v[2], v[3]));
        }
    }
    // ---- V rows of tokens 2c, 2c + 1, 2c + 8, 2c + 9 at this lane's output dims ----
    // INT8 map: dims 2g + {0, 1} + 16 q; INT4 map: dims 4g + {0..3} + 32 q
    constexpr int NQ = KV4 ? HD / 32 : HD / 16;
    uint32_t vw[4][KV4 ? 2 * NQ : NQ];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int row = 2 * c + (r & 1) + (r >> 1) * 8;
        const __half* src = vb + row * rs;
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            if (!KV4) {
                vw[r][q] = row < n ? *reinterpret_cast<const uint32_t*>(src + 16 * q + 2 * g) : 0u;
            } else {
                uint2 u = make_uint2(0u, 0u);
                if (row < n) u = *reinterpret_cast<const uint2*>(src + 32 * q + 4 * g);
                vw[r][2 * q] = u.x;
                vw[r][2 * q + 1] = u.y;
            }
        }
    }
    float sct[1][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sct[0][nt][i] = sc[nt][i];
    const float ks[1][2] = {{p.sm_scale_log2, p.sm_scale_log2}}, vs[1][2] = {{1.0f, 1.0f}};
    const bool live[1][2] = {{g < n, g + 8 < n}};
    tma_softmax_pv<HD, NT, SPLIT, 1>(
        S, sct,
        [&](int, int mt, uint32_t (&a)[4]) {
            // A row g: dim(mt, 0), row g + 8: dim(mt, 1); k: tokens (2c, 2c+1) | (2c+8, 2c+9)
            int w0, w1, sel;
            if (!KV4) {
                w0 = 2 * (mt >> 1);      // half2 word of dim(mt, 0)
                w1 = 2 * (mt >> 1) + 1;  // of dim(mt, 1)
                sel = mt & 1;
            } else {
                const int qq = 2 * (mt >> 2);
                w0 = 2 * qq + ((mt & 3) >> 1);
                w1 = 2 * (qq + 1) + ((mt & 3) >> 1);
                sel = mt & 1;
            }
            const uint32_t pm = sel ? 0x7632u : 0x5410u;
            a[0] = __byte_perm(vw[0][w0], vw[1][w0], pm);
            a[1] = __byte_perm(vw[0][w1], vw[1][w1], pm);
            a[2] = __byte_perm(vw[2][w0], vw[3][w0], pm);
            a[3] = __byte_perm(vw[2][w1], vw[3][w1], pm);
        },
        [](int mt) { return KV4 && (mt & 1); }, ks, vs, live);
}

template <bool KV4, int HD, int NT, bool SPLIT, int NW>
__global__ void __launch_bounds__((NW + 1) * 32, 1)
    paged_decode_tma_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const DecodeParams p);

mg_status tma_decode_plan(int kv4, int hd, int P, int Hkv, int Hq, int q_f16, int batch, int staging_esize,
                          int scale_th, int num_sm, DecodePlan* out);
template <bool KV4, int HD>
mg_status launch_tma(const DecodeParams& p, const DecodePlan& pl, const CUtensorMap& tk, const CUtensorMap& tv,
                     cudaStream_t s, bool self_copy);

}  // namespace mg
