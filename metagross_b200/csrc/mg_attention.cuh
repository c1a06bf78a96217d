// Fused paged decode attention: kernel template and host-side plan.
//
// Reference semantics: csrc/paged_attention.cu:25-135 (committed INT8 pages,
// one query per head, unnormalised (wv, sum, max) outputs) and
// metagross/attention.py:62-134 (exact staged tail merged with a log-sum-exp
// merge, then normalised).  Here one kernel does all of it for a batch:
//
//   work    the step's decode plan (mg_plan.cu): when the non-empty
//           sequences fit on the SMs, each is cut into near-equal chunks, one
//           per CTA; otherwise stream-K over the flattened list of "units" (one
//           committed page, or the staged tail, of one sequence): CTA c of G
//           processes units [c*W/G, (c+1)*W/G).  A sequence cut by a CTA boundary
//           gets a partial (m, l, acc) from each covering CTA; the last of
//           them to finish (atomic ticket, no waiting) merges and writes the
//           output.  Each CTA writes at most two partials (its first and its
//           last sequence), so the workspace is O(G), not O(batch); the
//           tickets are per (sequence, kv head).
//   data    no staging through shared memory for the pages: every warp loads
//           its own 16-token tiles (one kv head's rows of K and V) straight
//           from HBM into the registers in the tensor-core fragment layout,
//           one (INT8) or two (INT4) tiles ahead of the math, so 16 warps per
//           SM keep 32-64 KB of page data in flight.  The page ids and scales
//           of a warp's next 32 tiles sit one per lane and travel by shuffle.
//           A sequence's staged tail (< P exact fp16/fp32 rows) comes in
//           chunks through a small per-warp shared-memory ring (cp.async) as
//           further work items.  A warp walks all of its CTA's segments
//           (sequences) as one stream of items, so the loads of the next
//           segment are in flight while the current one is finalized.
//   warps   each warp owns one kv head (two when there are more kv heads than
//           warps); when the model has few kv heads, WPH warps share a head
//           and take alternate tiles and tail rows, merging their softmax
//           states in shared memory at the end of a sequence behind a named
//           barrier of that head's warps only.  A sequence cut by CTA
//           boundaries is merged per (sequence, kv head) by one warp of the
//           last covering CTA, so no CTA-wide barrier follows the prologue.
//   math    per 16-token tile, S^T = K Q^T and O^T += V^T P^T on the tensor
//           cores (mma.sync m16n8k16, fp16 in, fp32 accumulate).  INT8/INT4
//           codes are exact in fp16 and are converted in registers with the
//           0x6400 exponent trick (no I2F).  The K page scale multiplies the
//           fp32 scores; the V page scale is folded into P.  For fp32 queries
//           and small GQA groups (G <= 4) q and P travel as hi+lo fp16 pairs
//           in two mma columns (~22 mantissa bits).  Online softmax in the
//           log2 domain with lazy rescaling (the running reference max moves
//           only when a score exceeds it by 2^8).
//   tail    an fp16 staged tail (< P exact rows) is one more 16-row tile on
//           the tensor cores, its rows loaded straight into mma fragments; an
//           fp32 tail (not exact in fp16) goes through a per-warp shared-memory
//           ring and is folded in on the CUDA cores in fp32 (scores of a
//           chunk, then its exponentials and V sums).
#pragma once

#include "mg_common.cuh"

namespace mg {

constexpr int kWarps = 16;      // warps per CTA (one CTA per SM): <= 128 registers per thread
constexpr int kWarpsDeep = 12;  // head_dim 64, one n-tile: <= 168 registers (room for a copy of the tile math per ring slot)
constexpr int kWarpsWide = 8;   // head_dim 128 or two n-tiles with <= 8 kv heads: <= 255 registers
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8 in fp16
constexpr int kMetaLanes = 32;             // page ids cached per warp (one per lane)
constexpr int kPrefetchTiles = 8;          // L2 prefetch distance of a warp's tile stream (tiles)

// Work items (tiles or staged-tail items) in flight per warp (R - 1 of them
// are loading while one is computed), by register budget and measurement.  The
// L2 prefetch kPrefetchTiles ahead covers the DRAM latency, so the register
// ring only covers L2 hits; a deeper ring makes every warp issue more loads
// before its first tile, ~1 us of launch prologue per extra item:
//   head_dim 64, one n-tile, 12 warps (168 registers):      2
//   head_dim 64, one n-tile, 16 warps (128 registers):      4 INT4, 2 INT8,
//                                                            2 with two kv heads per warp
//   head_dim 128 or two n-tiles, 8 warps (255 registers):   2
//   head_dim 128 or two n-tiles, 16 warps:                   1
__host__ __device__ constexpr int decode_ring(bool kv4, int hd, int nt, int hpw, int nwarps) {
    return (hd == 64 && nt == 1) ? (hpw == 2 || nwarps == 12 ? 2 : (kv4 ? 4 : 2)) : (nwarps == 8 ? 2 : 1);
}

// Decode plan buffer (int32 words), written once per step by the plan
// kernel and read by every attention launch of the step:
//   [0, 16)              header: magic, batch, grid, 0, n_empty, mode,
//                        units, CTAs with work, has_staging
//   [off_counts, +grid)  segments of each CTA
//   [off_offs, +grid)    first record of each CTA in the flat array
//   [off_recs, ...)      per CTA, its first kPlanInline records (one load)
//   [off_pids, ...)      per CTA, the page ids of the first kPlanPids pages of its
//                        first segment (block-table entries, so an attention
//                        launch starts loading pages without that round trip)
//   [off_flat, ...)      all records in CTA order, batch + grid at most
//   [off_empty, +batch)  the sequences with nothing cached (outputs are zero)
// A record is 8 words: {b, first page, pages, tail rows, partial slot (-1:
// the whole sequence), first partial slot of b, pieces of b, 0}.
constexpr int32_t kPlanMagic = 0x6d67706c;
constexpr int kTailUnits = 2;     // work units the plan charges for a staged tail (a page is one)
constexpr int kPlanInline = 4;    // records per CTA in the inline area
constexpr int kPlanPids = 128;    // page ids per CTA in the plan
constexpr int kRecCache = 64;     // records an attention CTA keeps in shared memory
// page bytes a CTA warms in L2 before its wait (settled plan): the first copies
// only -- warming a whole 50 MB launch (384 KB a CTA) this way delayed them
constexpr int kPrewarmBytes = 48 * 1024;
struct PlanLayout {
    int off_counts, off_offs, off_recs, off_pids, off_flat, off_empty;
    int64_t words;
};
PlanLayout plan_layout(int batch, int grid);
constexpr int kMaxBatch = 8192;  // the plan kernel keeps six ints per sequence in shared memory
mg_status check_cache_layout(const mg_cache_layout* L);  // mg_cache.cu

struct AllocStep;
// the step's decode plan; with alloc, the step's allocation first, in the same launch
mg_status launch_decode_plan(const int32_t* block_tables, const int32_t* seq_lens, int32_t uniform_len, int batch,
                             int P, int max_blocks, int has_staging, int32_t* plan, int64_t plan_bytes,
                             int32_t* status, cudaStream_t s, const AllocStep* alloc = nullptr);

struct DecodeParams {
    const void* q;
    int q_f16;
    const uint8_t* k_pool;
    const uint8_t* v_pool;
    const float* k_scales;
    const float* v_scales;
    int scale_th;  // scales [N, P, Hkv] (one per token and kv head) instead of [N]
    const void* staging_k;
    const void* staging_v;
    int st_f16;
    int has_staging;
    const int32_t* block_tables;
    int32_t max_blocks;
    const int32_t* plan;  // the step's decode plan (see PlanLayout)
    PlanLayout lay;
    int batch;
    int Hq, Hkv, G, P;
    FastDiv pdiv;
    int page_bytes;
    int nconsumers;    // warps per CTA
    int wph;           // warps per kv head
    int st_row_bytes;  // bytes of one staged token row (Hkv * D * element size)
    int scratch_off;   // dynamic shared memory: softmax-state merge scratch (wph > 1)
    int tail_off;      // dynamic shared memory: per-warp rings of staged-tail slots
    int tail_slot;     // bytes of one slot
    float sm_scale_log2;
    int64_t num_pages;
    void* out;
    int out_f16;
    float* out_wv;  // unnormalised outputs (legacy op) when non-null
    float* out_l;
    float* out_m;
    float* ws_acc;  // [2*G, Hq, HD]
    float* ws_m;    // [2*G, Hq]
    float* ws_l;    // [2*G, Hq]
    uint32_t* tickets;  // [batch]
    int32_t* status;
    // the plan, the block tables and the allocation status were written before
    // the launch that immediately precedes this one (MG_ATTN_PLAN_SETTLED): the
    // kernel reads them, and warms L2 with its first pages, before it waits for
    // that launch to finish
    int plan_settled;
    // bulk-copy kernel (mg_attention_tma.cuh): dynamic shared memory layout,
    // offsets from the 1024-byte aligned base
    int tma_ns;           // stages in the ring
    FastDiv tma_nsdiv;    // division by tma_ns (exact for page counters below 2^26)
    int tma_stage_bytes;  // one stage: K page, then V page at half of it
    int tma_stage_off;
    int tma_bar_off;      // full[NS], empty[NS] mbarriers
    int tma_meta_off;     // per stage (K scale, V scale)
    int tma_per_head;     // the tensor maps are 3-D, one copy per kv head
};

struct DecodePlan {
    int nt, split_mode, hpw, wph, nconsumers, nwarps;
    int grid;
    int ring;  // work items in flight per warp
    int scratch_off, tail_off, tail_slot;
    int64_t partials_off, plan_off;  // workspace offsets
    int64_t smem_bytes;
    int64_t ws_bytes;
};

template <bool KV4, int HD, int NT>
struct Cfg {
    static constexpr int KSTEPS = HD / 16;
    static constexpr int MTILES = HD / 16;
    static constexpr int ROWB = KV4 ? HD / 2 : HD;  // bytes per (token, head) row
    static constexpr int KCHB = ROWB / 4;           // K bytes per lane per row
    static constexpr int VCHB = ROWB / 8;           // V bytes per lane per token
    static constexpr int VE = HD / 8;               // d values per lane
};

// BYTES (4, 8, 16 or 32, naturally aligned) of page data per lane into
// 32-bit words, cached in L2 only (ld.global.cg).  Not evict-first: the rows of
// neighbouring kv heads share 128-byte lines (one line prefetch serves them
// all), and a line marked evict-first after the first head's read could leave
// L2 before the other heads' warps, which drift apart over a long segment,
// read their sectors -- measured as 31 % more DRAM bytes than the pages hold.
template <int BYTES>
__device__ __forceinline__ void ldg_words(const uint8_t* p, uint32_t (&w)[BYTES / 4]) {
    if constexpr (BYTES == 4) {
        w[0] = __ldcg(reinterpret_cast<const unsigned int*>(p));
    } else if constexpr (BYTES == 8) {
        const uint2 v = __ldcg(reinterpret_cast<const uint2*>(p));
        w[0] = v.x;
        w[1] = v.y;
    } else if constexpr (BYTES == 16) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p));
        w[0] = v.x;
        w[1] = v.y;
        w[2] = v.z;
        w[3] = v.w;
    } else {
        static_assert(BYTES == 32, "row chunk");
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p));
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p + 16));
        w[0] = v.x;
        w[1] = v.y;
        w[2] = v.z;
        w[3] = v.w;
        w[4] = u.x;
        w[5] = u.y;
        w[6] = u.z;
        w[7] = u.w;
    }
}

// d (within the head) held by K-fragment slot s (0: k=2c, 1: 2c+1, 2: 2c+8,
// 3: 2c+9) of k-step kk for lane column c; must match k_frag_row().
template <bool KV4, int HD>
__device__ __forceinline__ int k_slot_d(int kk, int c, int s) {
    if (!KV4) {
        // word kk of the lane's chunk; a0 = bytes (0,2), a2 = bytes (1,3)
        const int off = (s == 0) ? 0 : (s == 1) ? 2 : (s == 2) ? 1 : 3;
        return (HD / 4) * c + 4 * kk + off;
    } else {
        // word kk>>1 (8 nibbles); h = kk&1 picks nibbles (2h,2h+4) and (2h+1,2h+5)
        const int off = (s == 0) ? 0 : (s == 1) ? 4 : (s == 2) ? 1 : 5;
        return (HD / 4) * c + 8 * (kk >> 1) + 2 * (kk & 1) + off;
    }
}

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

// V A-fragment pairs for one token pair (A at k-slot 2c[+8], B at 2c+1[+9]):
// for each m-tile mt, r0 = (A, B) codes at d = VE*g + 2mt, r1 at d + 1.
template <bool KV4, int HD>
__device__ __forceinline__ void v_pairs(const uint32_t* wa, const uint32_t* wb, uint32_t (&r0)[HD / 16],
                                        uint32_t (&r1)[HD / 16]) {
    if (!KV4) {
#pragma unroll
        for (int wi = 0; wi < HD / 32; ++wi) {
            const uint32_t X = __byte_perm(wa[wi], wb[wi], 0x5410);  // A0 A1 B0 B1
            const uint32_t Y = __byte_perm(wa[wi], wb[wi], 0x7632);  // A2 A3 B2 B3
            r0[2 * wi] = s8pair_to_half2(X);
            r1[2 * wi] = s8pair_to_half2(X >> 8);
            r0[2 * wi + 1] = s8pair_to_half2(Y);
            r1[2 * wi + 1] = s8pair_to_half2(Y >> 8);
        }
    } else {
#pragma unroll
        for (int wi = 0; wi < HD / 64; ++wi) {
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

// Largest CTA index c in [0, G) whose unit range starts at or before u.
__device__ __forceinline__ int cta_of_unit(int64_t u, int64_t W, int G) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if ((static_cast<int64_t>(mid) * W) / G <= u) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Per-warp softmax state of one kv head: NT n-tiles x (SPLIT ? 1 : 2) columns.
template <int NT, int MTILES>
struct HeadState {
    uint32_t qf[NT][MTILES][2];  // B fragments of q (MTILES == KSTEPS == HD/16)
    float acc[MTILES][NT][4];
    float m_used[NT][2];  // reference max used for the exponentials (log2 domain)
    float m_true[NT][2];  // running true max
    float lpart[NT][2];
};

// Register image of one 16-token tile of one kv head for lane (g, c): K rows
// g and g+8 (KCHB bytes each, the lane's slice of the head dimension), V rows
// 2c, 2c+1, 2c+8, 2c+9 (VCHB bytes each), and for rows g and g+8 the K scale
// (times the softmax scale, log2 domain; 0 for a row past the end) and the V
// scale of their pages.
template <bool KV4, int HD>
struct TileRegs {
    static constexpr int KW = Cfg<KV4, HD, 1>::KCHB / 4;
    static constexpr int VW = Cfg<KV4, HD, 1>::VCHB / 4;
    uint32_t k[2][KW];
    uint32_t v[4][VW];
    float ks[2];
    float vs[2];
    uint32_t live;  // bit r: row g + 8r exists
};

// Page ids of 32 upcoming pages of the warp's current segment, lane i
// holding entry base + i (one shuffle per tile to read them).  spids: the
// plan's copy of the first kPlanPids page ids of the CTA's first segment (in
// shared memory), null for later segments, which read the block table.
struct MetaCache {
    int base;
    int32_t pid;
    const int32_t* spids;
};

template <bool KV4, int HD, int NT, bool SPLIT, bool P16, int HPW, int R, int NW>
__global__ void __launch_bounds__(NW * 32, 1) paged_decode_kernel(const DecodeParams p);

mg_status make_decode_plan(int kv4, int hd, int P, int Hkv, int Hq, int q_f16, int batch, int staging_esize,
                           DecodePlan* out);
// One kernel shape family (page format, head_dim, page size 16 or other); each is
// instantiated in its own translation unit (mg_attn_<fmt>_d<hd>_<p16|pany>.cu).
template <bool KV4, int HD, bool P16>
mg_status launch_p(const DecodeParams& p, const DecodePlan& pl, cudaStream_t s);

}  // namespace mg
