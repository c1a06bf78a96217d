// Per-step decode plan: how the batch's work is split over the CTAs of the
// paged decode-attention kernel.  It depends only on the sequence lengths
// (and the page size), which every layer of a decode step shares, so one
// plan serves all the step's attention launches.
//
// Work is counted in "units": one committed page is one unit, the staged
// tail (< P exact rows, folded in on the CUDA cores) of a sequence is
// kTailUnits units, about what it costs next to a page.  A piece of the
// tail's weight that falls into another CTA's range is an empty piece (no
// pages, no tail; it merges as a zero partial).  Two partitions:
//   chunk     when the non-empty sequences fit on the SMs and the split stays
//             even: each sequence gets k_b = ceil(U_b / S) near-equal chunks
//             with S the smallest chunk size for which sum_b k_b <= #CTAs (so
//             the longest chunk is as short as possible), and every CTA runs
//             exactly one chunk of one sequence -- no CTA pays for a second
//             sequence.  Taken only while S <= max(5/4 of, or 16 units above,
//             the even share W / min(W, #CTAs));
//   stream-K  otherwise: CTA c takes units [c*W/G, (c+1)*W/G) of the
//             flattened list, i.e. a few whole short sequences plus the cut
//             ends of at most two others.
// A sequence cut into several pieces gets one partial (m, l, acc) slot per
// piece, contiguous from pbase; the last piece to finish merges them.
#include "mg_alloc_step.cuh"
#include "mg_attention.cuh"

namespace mg {

namespace {

constexpr int kPlanThreads = 1024;
// chunk mode while its longest chunk is within 5/4 of the even share, or within
// kSegmentUnits units of it (measured on one B200: a 64-sequence batch of
// 128..2048 tokens took 16.5 us per launch in chunks of at most 41 units and
// 25.6 us in stream-K shares of 33; 128 log-normal contexts took 123 us in
// chunks of at most 442 units and 74 us in stream-K shares of 193)
constexpr int kChunkSlackNum = 5, kChunkSlackDen = 4;
constexpr int kSegmentUnits = 16;

struct PlanParams {
    const int32_t* block_tables;  // [batch, max_blocks]
    const int32_t* seq_lens;
    int32_t uniform_len;  // >= 0: every sequence has this many committed tokens
    int batch, P, max_blocks, has_staging;
    int grid;
    PlanLayout lay;
    int32_t* plan;
    int32_t* status;
    const int32_t* n_new;  // the step's token counts (step plan), or null: no page is known to predate the step
};

__device__ __forceinline__ int block_sum(int v, int* scratch) {
    int tot;
    block_exclusive_scan(v, scratch, &tot);
    return tot;
}

__device__ __forceinline__ int block_max_int(int v, int* scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    int r = lane < static_cast<int>(blockDim.x >> 5) ? scratch[lane] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r = max(r, __shfl_xor_sync(0xffffffffu, r, o));
    return r;
}

// Exclusive scan of vals[0..n) into out[0..n] (out[n] = total), block-wide.
__device__ __forceinline__ int block_scan_array(const int* vals, int* out, int n, int* scratch) {
    int base = 0;
    for (int start = 0; start < n; start += blockDim.x) {
        const int i = start + threadIdx.x;
        const int v = i < n ? vals[i] : 0;
        int tot;
        const int ex = block_exclusive_scan(v, scratch, &tot);
        if (i < n) out[i] = base + ex;
        base += tot;
    }
    if (threadIdx.x == 0) out[n] = base;
    __syncthreads();
    return base;
}

// Record k of CTA cta, whose records start at flat index off: into the flat
// array, and into the CTA's inline area when k < kPlanInline.
// r1.w: how many of the segment's pages (from lo) were committed before the
// step (the step plan knows each sequence's n_new; 0 otherwise) -- pages no
// append of the step writes, which a settled attention launch may copy before
// its wait on the previous launch.
__device__ __forceinline__ void write_rec(const PlanParams& pp, int cta, int off, int k, int b, int lo, int npg,
                                          int tail, int pslot, int pbase, int ncov, int len_b) {
    int old_pages = 0;
    if (pp.n_new != nullptr) {
        const int add = pp.n_new[b];
        old_pages = add >= 0 && add <= len_b ? (len_b - add) / pp.P - lo : 0;
        old_pages = old_pages < 0 ? 0 : (old_pages > npg ? npg : old_pages);
    }
    const int4 r0 = make_int4(b, lo, npg, tail), r1 = make_int4(pslot, pbase, ncov, old_pages);
    int4* f = reinterpret_cast<int4*>(pp.plan + pp.lay.off_flat + static_cast<int64_t>(off + k) * 8);
    f[0] = r0;
    f[1] = r1;
    if (k < kPlanInline) {
        int4* r = reinterpret_cast<int4*>(pp.plan + pp.lay.off_recs + (static_cast<int64_t>(cta) * kPlanInline + k) * 8);
        r[0] = r0;
        r[1] = r1;
    }
}

__device__ __forceinline__ void decode_plan_body(const PlanParams& pp) {
    extern __shared__ __align__(16) int psm[];
    __shared__ int scratch[33];
    const int B = pp.batch, P = pp.P, G = pp.grid;
    int* len = psm;             // [B]
    int* units = len + B;       // [B]
    int* pre = units + B;       // [B + 1] unit prefix
    int* aux = pre + B + 1;     // [B + 1] chunks per sequence / pieces per sequence, then their prefix
    int* aux2 = aux + B + 1;    // [B + 1] partial-slot prefix
    int* tmp = aux2 + B + 1;    // [max(B, 2 * grid + 1)]
    int* first = tmp + (B > 2 * G + 1 ? B : 2 * G + 1);  // [3 * grid]: (b, lo, npg) of each CTA's first segment

    // ---- lengths and units --------------------------------------------------------
    int nonempty = 0, maxu = 0;
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        int l;
        if (pp.uniform_len >= 0) {
            l = pp.uniform_len;
        } else {
            l = pp.seq_lens[b];
            if (l < 0 || l / P > pp.max_blocks) {
                flag(pp.status, MG_DEV_BAD_ARGUMENT);
                l = 0;
            }
        }
        const int np = l / P;
        const int u = np + ((pp.has_staging && l - np * P > 0) ? kTailUnits : 0);
        len[b] = l;
        units[b] = u;
        nonempty += u > 0;
        maxu = max(maxu, u);
    }
    __syncthreads();
    nonempty = block_sum(nonempty, scratch);
    maxu = block_max_int(maxu, scratch);
    const int W = block_scan_array(units, pre, B, scratch);

    // ---- empty sequences (written as zeros by the attention CTAs) ------------------
    for (int b = threadIdx.x; b < B; b += blockDim.x) tmp[b] = units[b] == 0 ? 1 : 0;
    __syncthreads();
    const int n_empty = block_scan_array(tmp, aux2, B, scratch);
    for (int b = threadIdx.x; b < B; b += blockDim.x)
        if (units[b] == 0) pp.plan[pp.lay.off_empty + aux2[b]] = b;

    bool chunk = W > 0 && nonempty <= G;
    int S = 0;
    if (chunk) {
        // ---- smallest chunk size S with sum_b ceil(U_b / S) <= G -----------------
        int lo = (W + G - 1) / G, hi = maxu > lo ? maxu : lo;
        while (lo < hi) {
            const int mid = lo + (hi - lo) / 2;
            int need = 0;
            for (int b = threadIdx.x; b < B; b += blockDim.x) need += (units[b] + mid - 1) / mid;
            need = block_sum(need, scratch);
            if (need <= G) hi = mid;
            else lo = mid + 1;
        }
        S = lo;
        // The longest chunk sets the launch's length: with few long sequences
        // among many short ones (at most one chunk per CTA) it can be several
        // times the even share W / min(W, G) that stream-K gives every CTA.  But
        // a stream-K CTA pays for each further sequence it starts (its q, its
        // page-id window, its partial and merge), about kSegmentUnits units.
        const int64_t GR = min(W, G);
        chunk = static_cast<int64_t>(S) * GR * kChunkSlackDen <= static_cast<int64_t>(W) * kChunkSlackNum ||
                static_cast<int64_t>(S - kSegmentUnits) * GR <= static_cast<int64_t>(W);
    }
    int used = 0;
    if (chunk) {
        for (int b = threadIdx.x; b < B; b += blockDim.x) tmp[b] = (units[b] + S - 1) / S;
        __syncthreads();
        used = block_scan_array(tmp, aux, B, scratch);  // aux[b]: first CTA of sequence b
        for (int b = threadIdx.x; b < B; b += blockDim.x) tmp[b] = tmp[b] > 1 ? tmp[b] : 0;
        __syncthreads();
        block_scan_array(tmp, aux2, B, scratch);  // aux2[b]: first partial slot of sequence b
        for (int b = threadIdx.x; b < B; b += blockDim.x) {
            const int u = units[b];
            const int k = aux[b + 1] - aux[b];
            const int np = len[b] / P;
            const int tb = pp.has_staging ? len[b] - np * P : 0;
            for (int j = 0; j < k; ++j) {
                const int ulo = static_cast<int>(static_cast<int64_t>(j) * u / k);
                const int uhi = static_cast<int>(static_cast<int64_t>(j + 1) * u / k);
                const int npg = max(0, min(uhi, np) - ulo);
                const int tail = (uhi == u && tb > 0) ? tb : 0;
                const int cta = aux[b] + j;
                write_rec(pp, cta, cta, 0, b, ulo, npg, tail, k > 1 ? aux2[b] + j : -1, aux2[b], k, len[b]);
                first[3 * cta] = b;
                first[3 * cta + 1] = ulo;
                first[3 * cta + 2] = npg;
                pp.plan[pp.lay.off_counts + cta] = 1;
                pp.plan[pp.lay.off_offs + cta] = cta;
            }
        }
    } else if (W > 0) {
        // ---- stream-K: even unit ranges ------------------------------------------
        const int GR = W < G ? W : G;
        used = GR;
        auto cta_of_unit = [&](int64_t u) {
            int l = 0, h = GR - 1;
            while (l < h) {
                const int mid = (l + h + 1) >> 1;
                if ((static_cast<int64_t>(mid) * W) / GR <= u) l = mid;
                else h = mid - 1;
            }
            return l;
        };
        for (int b = threadIdx.x; b < B; b += blockDim.x) {
            int pieces = 0;
            if (units[b] > 0) pieces = cta_of_unit(pre[b + 1] - 1) - cta_of_unit(pre[b]) + 1;
            aux[b] = pieces;
            tmp[b] = pieces > 1 ? pieces : 0;
        }
        __syncthreads();
        block_scan_array(tmp, aux2, B, scratch);  // aux2[b]: first partial slot of sequence b
        // segments per CTA, their prefix (flat offsets), then the records
        auto first_seq = [&](int64_t u0) {
            int l = 0, h = B - 1;
            while (l < h) {
                const int mid = (l + h + 1) >> 1;
                if (pre[mid] <= u0) l = mid;
                else h = mid - 1;
            }
            return l;
        };
        for (int c = threadIdx.x; c < G; c += blockDim.x) {
            int k = 0;
            if (c < GR) {
                const int64_t u0 = static_cast<int64_t>(c) * W / GR, u1 = static_cast<int64_t>(c + 1) * W / GR;
                for (int b = first_seq(u0); b < B && pre[b] < u1; ++b) k += pre[b + 1] > pre[b];
            }
            tmp[c] = k;
        }
        __syncthreads();
        block_scan_array(tmp, tmp + G, G, scratch);  // tmp[G..2G]: flat offsets
        const int* offs = tmp + G;
        int* firstseg = first;
        for (int c = threadIdx.x; c < GR; c += blockDim.x) {
            const int64_t u0 = static_cast<int64_t>(c) * W / GR, u1 = static_cast<int64_t>(c + 1) * W / GR;
            int k = 0;
            for (int b = first_seq(u0); b < B && pre[b] < u1; ++b) {
                const int ub = pre[b], ue = pre[b + 1];
                if (ue == ub) continue;
                const int lo = static_cast<int>((u0 > ub ? u0 : ub) - ub);
                const int hi = static_cast<int>((u1 < ue ? u1 : ue) - ub);
                const int np = len[b] / P;
                const int tb = pp.has_staging ? len[b] - np * P : 0;
                const int npg = max(0, min(hi, np) - lo);
                const int tail = (hi == ue - ub && tb > 0) ? tb : 0;
                const bool whole = lo == 0 && hi == ue - ub;
                const int first = cta_of_unit(ub);
                write_rec(pp, c, offs[c], k, b, lo, npg, tail, whole ? -1 : aux2[b] + (c - first), aux2[b], aux[b],
                          len[b]);
                if (k == 0) {
                    firstseg[3 * c] = b;
                    firstseg[3 * c + 1] = lo;
                    firstseg[3 * c + 2] = npg;
                }
                ++k;
            }
            pp.plan[pp.lay.off_counts + c] = k;
            pp.plan[pp.lay.off_offs + c] = offs[c];
        }
    }
    for (int c = used + threadIdx.x; c < G; c += blockDim.x) {
        pp.plan[pp.lay.off_counts + c] = 0;
        first[3 * c + 2] = 0;
    }
    __syncthreads();
    // ---- page ids of each CTA's first kPlanPids pages (its first segment), so an
    // attention launch starts loading pages without a block-table round trip ------
    // (kBatch independent block-table loads in flight per thread before the stores)
    constexpr int kBatch = 8;
    for (int base = 0; base < G * kPlanPids; base += kBatch * blockDim.x) {
        int32_t pid[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = base + u * blockDim.x + threadIdx.x;
            pid[u] = 0;
            if (i < G * kPlanPids) {
                const int c = i / kPlanPids, k = i - c * kPlanPids;
                if (k < first[3 * c + 2])
                    pid[u] = pp.block_tables[static_cast<int64_t>(first[3 * c]) * pp.max_blocks + first[3 * c + 1] + k];
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = base + u * blockDim.x + threadIdx.x;
            if (i < G * kPlanPids) pp.plan[pp.lay.off_pids + i] = pid[u];
        }
    }
    if (threadIdx.x == 0) {
        int32_t* h = pp.plan;
        h[0] = kPlanMagic;
        h[1] = B;
        h[2] = G;
        h[3] = 0;
        h[4] = n_empty;
        h[5] = chunk ? 1 : 2;
        h[6] = W;
        h[7] = used;
        h[8] = pp.has_staging;
    }
}

__global__ void __launch_bounds__(kPlanThreads, 1) decode_plan_kernel(const PlanParams pp) {
    grid_dependency_wait();
    grid_launch_dependents();
    decode_plan_body(pp);
}

// A decode step's allocation, then its plan from the grown lengths, in one CTA
// (mg_plan_step): the plan reads the lengths and block-table rows the
// allocation wrote, after a CTA barrier.
__global__ void __launch_bounds__(kPlanThreads, 1) step_plan_kernel(const AllocStep a, const PlanParams pp) {
    grid_dependency_wait();
    grid_launch_dependents();
    alloc_step(a);
    __syncthreads();
    decode_plan_body(pp);
}

}  // namespace

PlanLayout plan_layout(int batch, int grid) {
    PlanLayout L{};
    L.off_counts = 16;
    L.off_offs = L.off_counts + grid;
    L.off_recs = ((L.off_offs + grid) + 7) / 8 * 8;
    L.off_pids = L.off_recs + grid * kPlanInline * 8;
    L.off_flat = L.off_pids + grid * kPlanPids;
    L.off_empty = L.off_flat + (batch + grid) * 8;
    L.words = L.off_empty + batch;
    return L;
}

mg_status launch_decode_plan(const int32_t* block_tables, const int32_t* seq_lens, int32_t uniform_len, int batch,
                             int P, int max_blocks, int has_staging, int32_t* plan, int64_t plan_bytes,
                             int32_t* status, cudaStream_t s, const AllocStep* alloc) {
    const int G = sm_count();
    const PlanLayout lay = plan_layout(batch, G);
    MG_REQUIRE(plan && plan_bytes >= static_cast<int64_t>(lay.words) * 4, "decode plan buffer too small: %lld < %lld",
               (long long)plan_bytes, (long long)lay.words * 4);
    MG_REQUIRE((reinterpret_cast<uintptr_t>(plan) & 15u) == 0, "decode plan buffer must be 16-byte aligned");
    PlanParams pp{};
    pp.block_tables = block_tables;
    pp.seq_lens = seq_lens;
    pp.uniform_len = uniform_len;
    pp.batch = batch;
    pp.P = P;
    pp.max_blocks = max_blocks;
    pp.has_staging = has_staging;
    pp.grid = G;
    pp.lay = lay;
    pp.plan = plan;
    pp.status = status;
    pp.n_new = alloc ? alloc->n_new : nullptr;
    const size_t tmp_ints = static_cast<size_t>(batch > 2 * G + 1 ? batch : 2 * G + 1);
    const size_t smem = (static_cast<size_t>(5) * batch + 3 + tmp_ints + 3 * static_cast<size_t>(G)) * sizeof(int);
    // the dynamic shared-memory opt-in, per kernel and device (raised as batches grow)
    static int64_t attr_set[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int ki = alloc ? 1 : 0;
    if (smem > 48 * 1024 && (dev < 0 || dev >= 64 || attr_set[ki][dev] < static_cast<int64_t>(smem))) {
        const cudaError_t e =
            alloc ? cudaFuncSetAttribute(step_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem))
                  : cudaFuncSetAttribute(decode_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
        if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_set[ki][dev] = static_cast<int64_t>(smem);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kPlanThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (alloc) {
        const cudaError_t e = cudaLaunchKernelEx(&cfg, step_plan_kernel, *alloc, pp);
        if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "step_plan_kernel launch: %s", cudaGetErrorString(e));
        return check_launch("step_plan_kernel");
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_plan_kernel, pp);
    if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "decode_plan_kernel launch: %s", cudaGetErrorString(e));
    return check_launch("decode_plan_kernel");
}

}  // namespace mg

using namespace mg;

extern "C" mg_status mg_plan_step(const mg_allocator* a, const mg_cache_layout* L, int32_t* block_tables,
                                  int32_t* seq_lens, const int32_t* n_new, int32_t batch, int32_t with_staging,
                                  void* plan, int64_t plan_bytes, int32_t* dev_status, mg_stream_t stream) {
    MG_REQUIRE(a && a->free_stack && a->n_free && a->in_use, "null allocator pointer");
    mg_status st = check_cache_layout(L);
    if (st != MG_OK) return st;
    MG_REQUIRE(batch >= 1 && batch <= kMaxBatch, "batch must be in [1, %d], got %d", kMaxBatch, batch);
    MG_REQUIRE(block_tables && seq_lens && n_new, "null pointer");
    const AllocStep as{a->free_stack, a->n_free, a->in_use, block_tables, L->max_blocks, seq_lens, n_new, batch,
                       L->page_size, dev_status};
    return launch_decode_plan(block_tables, seq_lens, -1, batch, L->page_size, L->max_blocks, with_staging ? 1 : 0,
                              static_cast<int32_t*>(plan), plan_bytes, dev_status, as_stream(stream), &as);
}
