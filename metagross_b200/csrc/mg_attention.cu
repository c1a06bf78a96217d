// Host side of the fused paged decode attention: launch planning and the C ABI
// entry points (mg_paged_attention_committed, mg_paged_decode_attention).
// The kernel and its design notes are in mg_attention.cuh /
// mg_attention_kernel.cuh.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "mg_attention.cuh"
#include "mg_attention_tma.cuh"

namespace mg {
namespace {

int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

constexpr int64_t kSmemBudget = 220 * 1024;  // prefix + merge scratch + tail slots, one CTA per SM

}  // namespace

mg_status make_decode_plan(int kv4, int hd, int P, int Hkv, int Hq, int q_f16, int batch, int staging_esize,
                           DecodePlan* out) {
    MG_REQUIRE(hd == 64 || hd == 128, "attention supports head_dim 64 or 128, got %d", hd);
    MG_REQUIRE(Hkv >= 1 && Hq >= Hkv && Hq % Hkv == 0,
               "num_q_heads (%d) must be an exact multiple of num_kv_heads (%d)", Hq, Hkv);
    MG_REQUIRE(P >= 1 && P <= 64, "page_size must be in [1, 64], got %d", P);
    MG_REQUIRE(batch >= 1 && batch <= kMaxBatch, "batch must be in [1, %d], got %d", kMaxBatch, batch);
    const int G = Hq / Hkv;
    DecodePlan pl{};
    // fp32 queries and small groups carry q and P as hi+lo fp16 pairs (two columns per head)
    if (G <= 4 || !q_f16) {
        pl.split_mode = 1;
        pl.nt = (G + 3) / 4;
    } else {
        pl.split_mode = 0;
        pl.nt = (G + 7) / 8;
    }
    if (pl.nt > 2) return set_error(MG_ERR_UNSUPPORTED, "GQA group %d too large (fp32 q: <= 8, fp16 q: <= 16)", G);
    // warps: one kv head each, several warps per head when there are few kv
    // heads, two heads per warp (head_dim 64, one n-tile) beyond that.  Head
    // dim 64 with one n-tile runs 12 warps at 168 registers unless 16 warps of
    // 128 registers put a third more warps on the kv heads (12 warps measured
    // 23.5 us per launch against 25.6 / 28.5 with 16 warps and a ring of 2 / 4
    // on the TinyLlama shape, 27.5 against 30.1 on the GPT-2 shape); the
    // register-heavy shapes (head_dim 128, two n-tiles) run 8 wide warps when
    // there are at most 8 kv heads.
    const bool light = hd == 64 && pl.nt == 1;
    if (light && Hkv <= kWarps) {
        auto used = [&](int nw) -> int { return Hkv <= nw ? Hkv * (nw / Hkv) : 0; };
        pl.nwarps = 4 * used(kWarpsDeep) >= 3 * used(kWarps) ? kWarpsDeep : kWarps;
    } else {
        pl.nwarps = (!light && Hkv <= kWarpsWide) ? kWarpsWide : kWarps;
    }
    if (Hkv <= pl.nwarps) {
        pl.hpw = 1;
        pl.wph = pl.nwarps / Hkv;
        pl.nconsumers = Hkv * pl.wph;
    } else if (light && Hkv <= 2 * kWarps) {
        pl.hpw = 2;
        pl.wph = 1;
        pl.nconsumers = (Hkv + 1) / 2;
    } else {
        return set_error(MG_ERR_UNSUPPORTED, "num_kv_heads %d with head_dim %d and group %d not supported", Hkv, hd,
                         G);
    }
    pl.ring = decode_ring(kv4 != 0, hd, pl.nt, pl.hpw, pl.nwarps);
    // dynamic shared memory: [the CTA's plan records, its first page ids][head merge scratch][tail slots: warps x ring]
    pl.grid = sm_count();
    const PlanLayout lay = plan_layout(batch, pl.grid);
    (void)lay;
    const int64_t prefix_bytes = align_up(static_cast<int64_t>(kRecCache) * 32 + kPlanPids * 4, 128);
    const int ncols = pl.split_mode ? 1 : 2;
    const int64_t scratch_bytes =
        pl.wph > 1 ? align_up(static_cast<int64_t>(pl.nconsumers) * pl.nt * ncols * 4 * (hd + 2) * 4, 128) : 0;
    int64_t slot = 0;
    if (staging_esize == 4) {  // fp32 tails go through shared memory (fp16 tails: straight to registers)
        const int64_t row = static_cast<int64_t>(hd) * staging_esize;  // one staged row of one head
        slot = 2 * row > 2048 ? 2 * row : 2048;
        // shrink to one row pair per slot when the batch needs the room
        if (prefix_bytes + scratch_bytes + slot * pl.ring * pl.nconsumers > kSmemBudget) slot = 2 * row;
    }
    const int64_t tail_bytes = slot * pl.ring * pl.nconsumers;
    MG_REQUIRE(prefix_bytes + scratch_bytes + tail_bytes <= kSmemBudget,
               "batch %d too large for the shared-memory plan", batch);
    pl.scratch_off = static_cast<int>(prefix_bytes);
    pl.tail_off = static_cast<int>(prefix_bytes + scratch_bytes);
    pl.tail_slot = static_cast<int>(slot);
    pl.smem_bytes = prefix_bytes + scratch_bytes + tail_bytes;
    // workspace: [tickets][partials: 2G slots][plan (used by the unplanned entry point)]
    pl.partials_off = align_up(static_cast<int64_t>(batch) * Hkv * 4, 256);
    pl.plan_off = align_up(pl.partials_off + 2LL * pl.grid * Hq * (hd + 2) * 4, 256);
    pl.ws_bytes = pl.plan_off + lay.words * 4;
    *out = pl;
    return MG_OK;
}

namespace {

// ---------------------------------------------------------------------------
// bulk-copy kernel: which calls it serves, its shape, and its tensor maps
// ---------------------------------------------------------------------------
constexpr int64_t kTmaSmemLimit = 232448 - 1024;  // 227 KB per CTA, less the static arrays and slack

// The layout the bulk-copy kernel serves (mg_attention_tma.cuh).  INT8 pages
// stream through its producer's bulk copies.  INT4 pages of the TinyLlama
// attention shape are 2 KB per K or V copy, and streams of 2 KB copies
// measured 0.9-1.7 TB/s (a per-SM rate of copies, not of bytes) against 5-6
// TB/s for 12 KB pages, so INT4 pools run the kernel's self-copying mode, whose
// consumer warps cp.async their own tiles: on the 1024-sequence log-normal INT4
// launch 371 us against 395 us on the register-streaming kernel and 520-606 us
// with bulk copies (16.8 against 16.3 us on the short TinyLlama-shape launch).
// The environment variable METAGROSS_B200_ATTENTION=registers selects the
// register kernel for every call, =bulk the bulk copies for INT4 pools too.
// 0: the register kernel; 1: the bulk-copy kernel; 2: its self-copying mode
// (INT4 pools).
int tma_mode(const mg_cache_layout* L, bool staged) {
    const char* sel = std::getenv("METAGROSS_B200_ATTENTION");
    if (sel && std::strcmp(sel, "registers") == 0) return 0;
    const bool layout_ok = L->page_size == 16 && L->scale_layout == MG_SCALE_PAGE &&
                           (!staged || L->staging_dtype == MG_F16) && (L->head_dim == 64 || L->head_dim == 128) &&
                           L->num_kv_heads >= 1 && L->num_kv_heads <= 15;
    if (!layout_ok) return 0;
    if (L->kv_dtype == MG_KV_INT8) return 1;
    if (sel && std::strcmp(sel, "bulk") == 0) return 1;
    return 2;
}

// Shape of the bulk-copy kernel for a plan `base` of the register kernel (same
// work split, workspace and query-column layout).  False when the pages do not
// fit two stages.
bool make_tma_plan(const DecodePlan& base, int kv4, int hd, int Hkv, bool self_copy, DecodePlan* out,
                   DecodeParams* p) {
    if (hd == 128 && base.nt > 1) return false;  // two n-tiles of head_dim 128 exceed 128 registers
    DecodePlan pl = base;
    const int wph = Hkv > 12 ? 1 : 12 / Hkv;  // consumer warps: 12, or one per kv head for 13-15
    pl.hpw = 1;
    pl.wph = wph;
    pl.nconsumers = Hkv * wph;
    pl.nwarps = pl.nconsumers + (self_copy ? 0 : 1);
    const int64_t rowb = kv4 ? hd / 2 : hd;
    const int64_t page = 16 * Hkv * rowb;
    const int64_t half = align_up(page, 1024);
    const int ncols = pl.split_mode ? 1 : 2;
    const int64_t prefix = align_up(static_cast<int64_t>(kRecCache) * 32 + kPlanPids * 4, 128);
    const int64_t scratch = wph > 1 ? align_up(static_cast<int64_t>(pl.nconsumers) * pl.nt * ncols * 4 * (hd + 2) * 4, 128) : 0;
    if (self_copy) {
        // per consumer warp: RS slots of one head's K and V tiles, then RS (K, V) scale pairs
        const int rs = (kv4 ? hd : 2 * hd) * 16 <= 1024 ? 8 : 4;  // kSelfSlots
        const int64_t slot = 2 * 16 * rowb;
        const int64_t stage_off = align_up(prefix + scratch, 1024);
        const int64_t meta_off = stage_off + static_cast<int64_t>(pl.nconsumers) * rs * slot;
        const int64_t total = 1024 + meta_off + static_cast<int64_t>(pl.nconsumers) * rs * 8;
        if (total > kTmaSmemLimit) return false;
        pl.scratch_off = static_cast<int>(prefix);
        pl.tail_off = 0;
        pl.tail_slot = 0;
        pl.smem_bytes = total;
        p->nconsumers = pl.nconsumers;
        p->wph = pl.wph;
        p->scratch_off = pl.scratch_off;
        p->tma_ns = rs;
        p->tma_nsdiv = FastDiv(static_cast<uint32_t>(rs));
        p->tma_stage_bytes = static_cast<int>(slot);
        p->tma_stage_off = static_cast<int>(stage_off);
        p->tma_bar_off = static_cast<int>(meta_off);
        p->tma_meta_off = static_cast<int>(meta_off);
        *out = pl;
        return true;
    }
    // the deepest ring (up to 64 stages) that fits; a consumer warp holds two of
    // its pages (WPH apart) at once, so the ring must be deeper than that span
    int ns = 64;
    int64_t bar_off = 0, meta_off = 0, stage_off = 0;
    for (; ns > 2 * wph; --ns) {
        bar_off = prefix + scratch;
        meta_off = bar_off + 2 * ns * 8;
        stage_off = align_up(meta_off + ns * 8, 1024);
        if (1024 + stage_off + ns * 2 * half <= kTmaSmemLimit) break;
    }
    if (ns <= 2 * wph) return false;
    pl.scratch_off = static_cast<int>(prefix);
    pl.tail_off = 0;
    pl.tail_slot = 0;
    pl.smem_bytes = 1024 + stage_off + static_cast<int64_t>(ns) * 2 * half;
    p->nconsumers = pl.nconsumers;
    p->wph = pl.wph;
    p->scratch_off = pl.scratch_off;
    p->tma_ns = ns;
    p->tma_nsdiv = FastDiv(static_cast<uint32_t>(ns));
    p->tma_stage_bytes = static_cast<int>(2 * half);
    p->tma_stage_off = static_cast<int>(stage_off);
    p->tma_bar_off = static_cast<int>(bar_off);
    p->tma_meta_off = static_cast<int>(meta_off);
    *out = pl;
    return true;
}

// Tensor maps of page pools, encoded once per (pool, shape, device).  A pool
// [N, 16, Hkv, rowb] is described as the 4-D tensor (rowb, token, kv head,
// page) with strides (Hkv*rowb, rowb, page bytes) -- the box (rowb, 16, Hkv, 1)
// lands one page as [kv head][token][rowb] -- or, where the driver declines
// those strides, as the 3-D tensor (rowb, kv head, token of the pool) copied one
// kv head at a time.  16-byte chunks are swizzled within 32/64/128-byte rows.
struct PageMapKey {
    const void* pool;
    int64_t n;
    int hkv, rowb, dev;
    bool operator==(const PageMapKey& o) const {
        return pool == o.pool && n == o.n && hkv == o.hkv && rowb == o.rowb && dev == o.dev;
    }
};
struct PageMapEntry {
    PageMapKey key;
    CUtensorMap map;
    int per_head;
    bool used;
};

mg_status page_tensor_map(const void* pool, int64_t n, int hkv, int rowb, CUtensorMap* out, int* per_head) {
    static PageMapEntry cache[128];
    static int next = 0;
    static std::mutex mu;
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    const PageMapKey key{pool, n, hkv, rowb, dev};
    std::lock_guard<std::mutex> lock(mu);
    for (auto& e : cache)
        if (e.used && e.key == key) {
            *out = e.map;
            *per_head = e.per_head;
            return MG_OK;
        }
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
            return set_error(MG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable: %s", cudaGetErrorString(e));
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const CUtensorMapSwizzle sw = rowb == 32   ? CU_TENSOR_MAP_SWIZZLE_32B
                                  : rowb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                               : CU_TENSOR_MAP_SWIZZLE_128B;
    const cuuint64_t page = 16ull * hkv * rowb;
    CUtensorMap m;
    int ph = 0;
    {
        const cuuint64_t dims[4] = {static_cast<cuuint64_t>(rowb), 16, static_cast<cuuint64_t>(hkv),
                                    static_cast<cuuint64_t>(n)};
        const cuuint64_t strides[3] = {static_cast<cuuint64_t>(hkv) * rowb, static_cast<cuuint64_t>(rowb), page};
        const cuuint32_t box[4] = {static_cast<cuuint32_t>(rowb), 16, static_cast<cuuint32_t>(hkv), 1};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(pool), dims, strides, box,
                                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) ph = 1;
    }
    if (ph) {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(rowb), static_cast<cuuint64_t>(hkv),
                                    static_cast<cuuint64_t>(n) * 16};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(rowb), static_cast<cuuint64_t>(hkv) * rowb};
        const cuuint32_t box[3] = {static_cast<cuuint32_t>(rowb), 1, 16};
        const cuuint32_t es[3] = {1, 1, 1};
        const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(pool), dims, strides, box,
                                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_error(MG_ERR_CUDA, "cuTensorMapEncodeTiled(page pool) failed: %d", (int)r);
    }
    PageMapEntry& e = cache[next];
    next = (next + 1) % 128;
    e.key = key;
    e.map = m;
    e.per_head = ph;
    e.used = true;
    *out = m;
    *per_head = ph;
    return MG_OK;
}

// A batched call's kernel: the bulk-copy one when `use`.
struct TmaLaunch {
    bool use = false;
    bool self_copy = false;  // the consumer warps copy their own tiles (no tensor maps)
    DecodePlan pl;
    CUtensorMap tk, tv;
};

void fill_common(DecodeParams& p, const DecodePlan& pl, int P, int Hkv, int Hq, int hd, int kv4, double scale,
                 int64_t num_pages, int batch) {
    p.batch = batch;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.G = Hq / Hkv;
    p.P = P;
    p.pdiv = FastDiv(static_cast<uint32_t>(P));
    p.page_bytes = P * Hkv * (kv4 ? hd / 2 : hd);
    p.nconsumers = pl.nconsumers;
    p.wph = pl.wph;
    p.scratch_off = pl.scratch_off;
    p.tail_off = pl.tail_off;
    p.tail_slot = pl.tail_slot;
    p.st_row_bytes = Hkv * hd * 4;  // replaced with the staging dtype's size where there is staging
    p.lay = plan_layout(batch, pl.grid);
    p.sm_scale_log2 = static_cast<float>(scale * 1.4426950408889634);
    p.num_pages = num_pages;
}

// workspace: [tickets: batch x Hkv u32][acc: 2G x Hq x HD][m: 2G x Hq][l: 2G x Hq][plan]
void set_workspace(DecodeParams& p, const DecodePlan& pl, int Hq, int hd, void* ws) {
    p.tickets = static_cast<uint32_t*>(ws);
    float* f = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + pl.partials_off);
    const int64_t n = 2LL * pl.grid * Hq;
    p.ws_acc = f;
    p.ws_m = f + n * hd;
    p.ws_l = p.ws_m + n;
}

mg_status launch(int kv4, int hd, const DecodeParams& p, const DecodePlan& pl, cudaStream_t s) {
    // the 16-token-page kernels read one scale per tile; per-token scales take
    // the general path, which looks up each row's page and scale
    const bool p16 = p.P == 16 && !p.scale_th;
    if (kv4) {
        if (hd == 64) return p16 ? launch_p<true, 64, true>(p, pl, s) : launch_p<true, 64, false>(p, pl, s);
        return p16 ? launch_p<true, 128, true>(p, pl, s) : launch_p<true, 128, false>(p, pl, s);
    }
    if (hd == 64) return p16 ? launch_p<false, 64, true>(p, pl, s) : launch_p<false, 64, false>(p, pl, s);
    return p16 ? launch_p<false, 128, true>(p, pl, s) : launch_p<false, 128, false>(p, pl, s);
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace

}  // namespace mg

using namespace mg;

extern "C" int64_t mg_paged_attention_committed_workspace_bytes(int64_t num_blocks, int64_t page_size,
                                                                int64_t num_q_heads, int64_t num_kv_heads,
                                                                int64_t head_dim) {
    DecodePlan pl;
    if (make_decode_plan(0, static_cast<int>(head_dim), static_cast<int>(page_size), static_cast<int>(num_kv_heads),
                         static_cast<int>(num_q_heads), 0, 1, 0, &pl) != MG_OK)
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
    MG_REQUIRE(aligned16(k_storage) && aligned16(v_storage), "k/v storage must be 16-byte aligned");
    DecodePlan pl;
    mg_status st = make_decode_plan(0, static_cast<int>(head_dim), static_cast<int>(page_size),
                                    static_cast<int>(num_kv_heads), static_cast<int>(num_q_heads), 0, 1, 0, &pl);
    if (st != MG_OK) return st;
    MG_REQUIRE(workspace && workspace_bytes >= pl.ws_bytes, "workspace too small: %lld < %lld bytes",
               (long long)workspace_bytes, (long long)pl.ws_bytes);
    DecodeParams p{};
    fill_common(p, pl, static_cast<int>(page_size), static_cast<int>(num_kv_heads), static_cast<int>(num_q_heads),
                static_cast<int>(head_dim), 0, scale, max_pages, 1);
    p.q = query;
    p.q_f16 = 0;
    p.k_pool = reinterpret_cast<const uint8_t*>(k_storage);
    p.v_pool = reinterpret_cast<const uint8_t*>(v_storage);
    p.k_scales = page_scales_k;
    p.v_scales = page_scales_v;
    p.has_staging = 0;
    p.block_tables = block_table;
    p.max_blocks = static_cast<int32_t>(num_blocks > 0 ? num_blocks : 1);
    p.out = nullptr;
    p.out_wv = out_wv;
    p.out_l = out_sum;
    p.out_m = out_max;
    p.status = dev_status;
    set_workspace(p, pl, static_cast<int>(num_q_heads), static_cast<int>(head_dim), workspace);
    // one sequence of num_blocks committed pages: plan it, then attend
    int32_t* plan = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + pl.plan_off);
    st = launch_decode_plan(block_table, nullptr, static_cast<int32_t>(num_blocks * page_size), 1,
                            static_cast<int>(page_size),
                            p.max_blocks, 0, plan, pl.ws_bytes - pl.plan_off, dev_status, as_stream(stream));
    if (st != MG_OK) return st;
    p.plan = plan;
    return launch(0, static_cast<int>(head_dim), p, pl, as_stream(stream));
}

extern "C" int64_t mg_paged_decode_workspace_bytes(const mg_cache_layout* L, int32_t batch, int32_t num_q_heads,
                                                   int32_t max_context) {
    if (!L) return 0;
    DecodePlan pl;
    (void)max_context;
    // The size does not depend on the query dtype, but the set of supported
    // shapes does (GQA groups of 9-16 run with fp16 queries only): size from
    // whichever plan exists, fp32 queries first.
    const int kv4 = L->kv_dtype == MG_KV_INT4, esz = L->staging_dtype == MG_F16 ? 2 : 4;
    if (make_decode_plan(kv4, L->head_dim, L->page_size, L->num_kv_heads, num_q_heads, 0, batch, esz, &pl) != MG_OK &&
        make_decode_plan(kv4, L->head_dim, L->page_size, L->num_kv_heads, num_q_heads, 1, batch, esz, &pl) != MG_OK)
        return 0;
    return pl.ws_bytes;  // independent of the query dtype and of max_context
}

namespace {

// Checks and kernel parameters shared by the planned and unplanned batched entry points.
mg_status prepare_batched(const mg_cache_layout* L, const mg_layer_ptrs* lp, const int32_t* block_tables, int32_t batch,
                          const void* q, int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                          int32_t out_dtype, void* workspace, int64_t workspace_bytes, int32_t* dev_status,
                          DecodeParams* pp, DecodePlan* plp, TmaLaunch* tl) {
    mg_status st = check_cache_layout(L);
    if (st != MG_OK) return st;
    MG_REQUIRE(lp && lp->k_pool && lp->v_pool && lp->k_scales && lp->v_scales, "null layer pointer");
    MG_REQUIRE(q && out && block_tables, "null pointer");
    MG_REQUIRE(q_dtype == MG_F32 || q_dtype == MG_F16, "q_dtype must be MG_F32 or MG_F16");
    MG_REQUIRE(out_dtype == MG_F32 || out_dtype == MG_F16, "out_dtype must be MG_F32 or MG_F16");
    MG_REQUIRE(scale > 0.0f && scale < 1.0f / 0.0f, "attention scale must be positive and finite");
    MG_REQUIRE(aligned16(lp->k_pool) && aligned16(lp->v_pool), "pools must be 16-byte aligned");
    MG_REQUIRE(!(lp->staging_k && lp->staging_v) || (aligned16(lp->staging_k) && aligned16(lp->staging_v)),
               "staging buffers must be 16-byte aligned");
    MG_REQUIRE(aligned16(out), "out must be 16-byte aligned");
    const bool staged = lp->staging_k && lp->staging_v;
    DecodePlan pl;
    st = make_decode_plan(L->kv_dtype == MG_KV_INT4, L->head_dim, L->page_size, L->num_kv_heads, num_q_heads,
                          q_dtype == MG_F16, batch, staged ? (L->staging_dtype == MG_F16 ? 2 : 4) : 0, &pl);
    if (st != MG_OK) return st;
    MG_REQUIRE(workspace && workspace_bytes >= pl.plan_off, "workspace too small: %lld < %lld bytes",
               (long long)workspace_bytes, (long long)pl.plan_off);
    DecodeParams p{};
    fill_common(p, pl, L->page_size, L->num_kv_heads, num_q_heads, L->head_dim, L->kv_dtype == MG_KV_INT4, scale,
                L->num_pages, batch);
    p.q = q;
    p.q_f16 = q_dtype == MG_F16;
    p.k_pool = static_cast<const uint8_t*>(lp->k_pool);
    p.v_pool = static_cast<const uint8_t*>(lp->v_pool);
    p.k_scales = lp->k_scales;
    p.v_scales = lp->v_scales;
    p.scale_th = L->scale_layout == MG_SCALE_TOKEN_HEAD;
    p.staging_k = lp->staging_k;
    p.staging_v = lp->staging_v;
    p.st_f16 = L->staging_dtype == MG_F16;
    p.has_staging = staged ? 1 : 0;
    p.st_row_bytes = L->num_kv_heads * L->head_dim * (p.st_f16 ? 2 : 4);
    MG_REQUIRE(!p.has_staging || (aligned16(lp->staging_k) && aligned16(lp->staging_v)),
               "staging buffers must be 16-byte aligned");
    p.block_tables = block_tables;
    p.max_blocks = L->max_blocks;
    p.out = out;
    p.out_f16 = out_dtype == MG_F16;
    p.out_wv = nullptr;
    p.status = dev_status;
    set_workspace(p, pl, num_q_heads, L->head_dim, workspace);
    tl->use = false;
    tl->self_copy = false;
    const int mode = tma_mode(L, staged);
    if (mode == 2 &&
        make_tma_plan(pl, L->kv_dtype == MG_KV_INT4, L->head_dim, L->num_kv_heads, true, &tl->pl, &p)) {
        std::memset(&tl->tk, 0, sizeof(tl->tk));
        std::memset(&tl->tv, 0, sizeof(tl->tv));
        tl->use = true;
        tl->self_copy = true;
    } else if (mode == 1 &&
               make_tma_plan(pl, L->kv_dtype == MG_KV_INT4, L->head_dim, L->num_kv_heads, false, &tl->pl, &p)) {
        const int rowb = L->kv_dtype == MG_KV_INT4 ? L->head_dim / 2 : L->head_dim;
        int ph_k = 0, ph_v = 0;
        st = page_tensor_map(lp->k_pool, L->num_pages, L->num_kv_heads, rowb, &tl->tk, &ph_k);
        if (st != MG_OK) return st;
        st = page_tensor_map(lp->v_pool, L->num_pages, L->num_kv_heads, rowb, &tl->tv, &ph_v);
        if (st != MG_OK) return st;
        MG_REQUIRE(ph_k == ph_v, "K and V pools got different tensor-map forms");
        p.tma_per_head = ph_k;
        tl->use = true;
    }
    *pp = p;
    *plp = pl;
    return MG_OK;
}

mg_status launch_any(int kv4, int hd, const DecodeParams& p, const DecodePlan& pl, const TmaLaunch& tl,
                     cudaStream_t s) {
    if (!tl.use) return launch(kv4, hd, p, pl, s);
    const bool sc = tl.self_copy;
    if (kv4)
        return hd == 64 ? launch_tma<true, 64>(p, tl.pl, tl.tk, tl.tv, s, sc)
                        : launch_tma<true, 128>(p, tl.pl, tl.tk, tl.tv, s, sc);
    return hd == 64 ? launch_tma<false, 64>(p, tl.pl, tl.tk, tl.tv, s, sc)
                    : launch_tma<false, 128>(p, tl.pl, tl.tk, tl.tv, s, sc);
}

}  // namespace

extern "C" int64_t mg_paged_decode_plan_bytes(int32_t batch) {
    if (batch < 1 || batch > kMaxBatch) return 0;
    return plan_layout(batch, sm_count()).words * 4;
}

extern "C" mg_status mg_paged_decode_plan(const mg_cache_layout* L, const int32_t* block_tables,
                                          const int32_t* seq_lens, int32_t batch, int32_t with_staging, void* plan,
                                          int64_t plan_bytes, int32_t* dev_status, mg_stream_t stream) {
    mg_status st = check_cache_layout(L);
    if (st != MG_OK) return st;
    MG_REQUIRE(batch >= 1 && batch <= kMaxBatch, "batch must be in [1, %d], got %d", kMaxBatch, batch);
    MG_REQUIRE(seq_lens && block_tables, "null pointer");
    return launch_decode_plan(block_tables, seq_lens, -1, batch, L->page_size, L->max_blocks, with_staging ? 1 : 0,
                              static_cast<int32_t*>(plan), plan_bytes, dev_status, as_stream(stream));
}

extern "C" mg_status mg_paged_decode_attention_planned_flags(const mg_cache_layout* L, const mg_layer_ptrs* lp,
                                                             const int32_t* block_tables, const void* plan,
                                                             int64_t plan_bytes, int32_t batch, const void* q,
                                                             int32_t q_dtype, int32_t num_q_heads, float scale,
                                                             void* out, int32_t out_dtype, void* workspace,
                                                             int64_t workspace_bytes, uint32_t flags,
                                                             int32_t* dev_status, mg_stream_t stream) {
    MG_REQUIRE(batch >= 0, "batch must be >= 0");
    MG_REQUIRE((flags & ~MG_ATTN_PLAN_SETTLED) == 0, "unknown attention flags 0x%x", flags);
    if (batch == 0) return MG_OK;
    DecodeParams p;
    DecodePlan pl;
    TmaLaunch tl;
    mg_status st = prepare_batched(L, lp, block_tables, batch, q, q_dtype, num_q_heads, scale, out, out_dtype,
                                   workspace, workspace_bytes, dev_status, &p, &pl, &tl);
    if (st != MG_OK) return st;
    MG_REQUIRE(plan && aligned16(plan) && plan_bytes >= p.lay.words * 4, "decode plan missing, unaligned or too small");
    p.plan = static_cast<const int32_t*>(plan);
    p.plan_settled = (flags & MG_ATTN_PLAN_SETTLED) ? 1 : 0;
    return launch_any(L->kv_dtype == MG_KV_INT4, L->head_dim, p, pl, tl, as_stream(stream));
}

extern "C" mg_status mg_paged_decode_attention_planned(const mg_cache_layout* L, const mg_layer_ptrs* lp,
                                                       const int32_t* block_tables, const void* plan,
                                                       int64_t plan_bytes, int32_t batch, const void* q,
                                                       int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                                                       int32_t out_dtype, void* workspace, int64_t workspace_bytes,
                                                       int32_t* dev_status, mg_stream_t stream) {
    return mg_paged_decode_attention_planned_flags(L, lp, block_tables, plan, plan_bytes, batch, q, q_dtype,
                                                   num_q_heads, scale, out, out_dtype, workspace, workspace_bytes, 0u,
                                                   dev_status, stream);
}

extern "C" mg_status mg_paged_decode_attention(const mg_cache_layout* L, const mg_layer_ptrs* lp,
                                               const int32_t* block_tables, const int32_t* seq_lens, int32_t batch,
                                               const void* q, int32_t q_dtype, int32_t num_q_heads, float scale,
                                               void* out, int32_t out_dtype, int32_t max_context, void* workspace,
                                               int64_t workspace_bytes, int32_t* dev_status, mg_stream_t stream) {
    (void)max_context;
    MG_REQUIRE(batch >= 0, "batch must be >= 0");
    if (batch == 0) return MG_OK;
    MG_REQUIRE(seq_lens, "null pointer");
    DecodeParams p;
    DecodePlan pl;
    TmaLaunch tl;
    mg_status st = prepare_batched(L, lp, block_tables, batch, q, q_dtype, num_q_heads, scale, out, out_dtype,
                                   workspace, workspace_bytes, dev_status, &p, &pl, &tl);
    if (st != MG_OK) return st;
    MG_REQUIRE(workspace_bytes >= pl.ws_bytes, "workspace too small: %lld < %lld bytes", (long long)workspace_bytes,
               (long long)pl.ws_bytes);
    int32_t* plan = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + pl.plan_off);
    st = launch_decode_plan(block_tables, seq_lens, -1, batch, L->page_size, L->max_blocks, p.has_staging, plan,
                            pl.ws_bytes - pl.plan_off, dev_status, as_stream(stream));
    if (st != MG_OK) return st;
    p.plan = plan;
    return launch_any(L->kv_dtype == MG_KV_INT4, L->head_dim, p, pl, tl, as_stream(stream));
}
