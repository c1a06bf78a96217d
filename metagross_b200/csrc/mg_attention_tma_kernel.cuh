// Body of the bulk-copy decode-attention kernel (design: mg_attention_tma.cuh).
// Included by the per-format translation units mg_attn_tma_<fmt>_d<hd>.cu.
#pragma once

#include "mg_attention_kernel.cuh"
#include "mg_attention_tma.cuh"

namespace mg {

// SELF: no producer warp; each consumer warp copies its own kv head's rows of
// its pages (cp.async, 16 bytes a lane) into a private ring of p.tma_ns slots
// laid out as the bulk copies lay out a head's tile, and waits on its own copy
// groups -- for pools whose pages are too small for one bulk copy each to keep
// up (a 16-token INT4 page of 4 kv heads is 2 KB).
template <bool KV4, int HD, int NT, bool SPLIT, int NW, bool SELF>
__global__ void __launch_bounds__((NW + (SELF ? 0 : 1)) * 32, 1)
    paged_decode_tma_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const DecodeParams p) {
    using T = TCfg<KV4, HD>;
    constexpr int MT = T::MT;
    constexpr int VE = T::VE;
    constexpr int NCOLS = SPLIT ? 1 : 2;
    // two pages per consumer step (a single page at a segment's odd end).  24
    // consumer warps of one page per step (72 registers) measured slower on the
    // GPT-2 shape (21.3 against 19.6 us): the launch is bound by page arrival,
    // not by the consumers' issue rate
    constexpr bool PAIRS = true;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ int sm_hdr[3];
    __shared__ int sm_last[2 * kWarps];
    // stages must start on a 1024-byte boundary (the swizzle follows address bits)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

    // the first copy must not wait on a cold descriptor fetch (SELF: no maps)
    if (!SELF && threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_k)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_v)) : "memory");
    }
    // With a settled plan the prologue (plan, status, barriers) and an L2 warm-up
    // of the first pages run before the wait on the previous launch, on SMs that
    // launch has already left; nothing is written to global memory before it.
    const bool settled = p.plan_settled != 0;
    if (!settled) {
        grid_dependency_wait();
        grid_launch_dependents();
    }

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int Hkv = p.Hkv, Hq = p.Hq;
    const int NCW = p.nconsumers, WPH = p.wph;
    const int NS = p.tma_ns;
    const FastDiv nsd = p.tma_nsdiv;
    // ring stage and phase parity of page counter k
    auto stage_of = [&](int k) { return k - static_cast<int>(nsd.div(static_cast<uint32_t>(k))) * NS; };
    auto round_of = [&](int k) { return static_cast<int>(nsd.div(static_cast<uint32_t>(k))); };
    const int cta = blockIdx.x;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.tma_bar_off);
    uint64_t* empty = full + NS;
    float2* meta = reinterpret_cast<float2*>(smem + p.tma_meta_off);
    uint8_t* stages = smem + p.tma_stage_off;
    const int sbytes = p.tma_stage_bytes;  // K page at 0, V page at sbytes / 2
    float* mscratch = reinterpret_cast<float*>(smem + p.scratch_off);
    int4* recs = reinterpret_cast<int4*>(smem);
    int32_t* spids = reinterpret_cast<int32_t*>(smem + kRecCache * 32);

    // ---- plan: this CTA's segment records and first page ids (one round trip) --
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
        if (!SELF) {
            for (int s = 0; s < NS; ++s) {
                mbar_init(&full[s], 2);  // the copies' arrive.expect_tx + the scales' arrive
                mbar_init(&empty[s], static_cast<uint32_t>(Hkv));  // one consumer warp per kv head
            }
            fence_mbar_init();
        }
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
    auto rec = [&](int k) -> const int4* { return k < kRecCache ? recs + 2 * k : flat + 2 * k; };

    // pages (producer) or tiles (SELF: each consumer warp's own) of the first
    // segment copied before the wait
    int pre = 0;
    if (settled) {
        // The producer copies the first segment's pages that predate the step
        // (the step plan's count, r1.w: no launch of this step writes them)
        // before the wait, with their scales, into the first stages.
        if (!SELF && warp == NCW && nseg > 0 && rec(0)[0].z > 0) {
            const int G = p.tma_per_head ? 1 : 2;
            int m = min(min(rec(0)[1].w, rec(0)[0].z), min(NS, 32));
            if (G == 2) m &= ~1;
            const int32_t pid = lane < m ? spids[lane] : 0;
            if (m > 0 && !__any_sync(0xffffffffu, lane < m && (pid < 0 || pid >= p.num_pages))) {
                const float ks = lane < m ? __ldg(p.k_scales + pid) : 0.0f;
                const float vs = lane < m ? __ldg(p.v_scales + pid) : 0.0f;
                const uint32_t tx = static_cast<uint32_t>(2 * p.page_bytes);
                for (int i = 0; i < m; i += G) {
                    if (G == 1) {  // stage i < NS: fresh, nothing to wait for
                        const int32_t pi = __shfl_sync(0xffffffffu, pid, i);
                        uint8_t* dk = stages + static_cast<int64_t>(i) * sbytes;
                        if (lane == 0) mbar_arrive_expect_tx(&full[i], tx);
                        __syncwarp();
                        tma_page(dk, &tm_k, pi, &full[i], 1, Hkv, p.P, T::TILE, lane);
                        tma_page(dk + sbytes / 2, &tm_v, pi, &full[i], 1, Hkv, p.P, T::TILE, lane);
                    } else {
                        const int j = lane >> 1;
                        const int32_t pj = __shfl_sync(0xffffffffu, pid, min(i + j, 31));
                        uint8_t* dst = stages + static_cast<int64_t>(i + j) * sbytes + ((lane & 1) ? sbytes / 2 : 0);
                        if (j < 2 && (lane & 1) == 0) mbar_arrive_expect_tx(&full[i + j], tx);
                        __syncwarp();
                        if (j < 2) tma_page(dst, (lane & 1) ? &tm_v : &tm_k, pj, &full[i + j], 0, Hkv, p.P, T::TILE, 0);
                    }
                }
                if (lane < m) {
                    meta[lane] = make_float2(ks, vs);
                    mbar_arrive(&full[lane]);
                }
                pre = m;
            }
        }
        // SELF: each consumer warp copies its own first tiles of the first
        // segment's pages that predate the step into its ring's first slots
        if (SELF && warp < NCW && nseg > 0) {
            constexpr int RS0 = kSelfSlots<KV4, HD>;
            const int wsub0 = WPH > 1 ? warp % WPH : 0, h0 = WPH > 1 ? warp / WPH : warp;
            const int lim = min(rec(0)[1].w, rec(0)[0].z);  // pages [0, lim) of segment 0 predate the step
            int n = lim > wsub0 ? (lim - 1 - wsub0) / WPH + 1 : 0;  // tile i: page wsub0 + i * WPH
            n = min(n, RS0);
            const int32_t pid = lane < n ? spids[wsub0 + lane * WPH] : 0;
            if (n > 0 && !__any_sync(0xffffffffu, lane < n && (pid < 0 || pid >= p.num_pages))) {
                uint8_t* ring0p = stages + static_cast<int64_t>(warp) * RS0 * sbytes;
                float2* wmeta0 = meta + warp * RS0;
                const int rs = Hkv * T::ROWB;
                for (int i = 0; i < n; ++i) {
                    const int32_t pi = __shfl_sync(0xffffffffu, pid, i);
                    uint8_t* dk = ring0p + static_cast<int64_t>(i) * sbytes;
                    const int64_t go = static_cast<int64_t>(pi) * p.page_bytes + h0 * T::ROWB;
#pragma unroll
                    for (int q = lane; q < 16 * T::CHUNKS; q += 32) {
                        const int t = q / T::CHUNKS, j = q - t * T::CHUNKS;
                        const uint32_t o = tile_chunk_off<KV4, HD>(t, j);
                        cp_async16(dk + o, p.k_pool + go + t * rs + 16 * j);
                        cp_async16(dk + T::TILE + o, p.v_pool + go + t * rs + 16 * j);
                    }
                    if (lane == 0) cp_async4(&wmeta0[i].x, p.k_scales + pi);
                    if (lane == 1) cp_async4(&wmeta0[i].y, p.v_scales + pi);
                    cp_async_commit();
                }
                pre = n;
            }
        }
        // otherwise the first segment's pages (up to kPrewarmBytes of this CTA's)
        // into L2; the copies after the wait read them there (L2 is coherent with
        // the previous launch's writes, so a page it commits is read as written)
        if (pre == 0 && warp == (SELF ? 0 : NCW) && nseg > 0) {
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

    // empty sequences: zero outputs
    for (int i = cta; i < n_empty; i += gridDim.x) {
        const int bb = p.plan[p.lay.off_empty + i];
        const int64_t r0 = static_cast<int64_t>(bb) * Hq;
        for (int k = tid; k < Hq * HD; k += blockDim.x) {
            if (p.out_f16) static_cast<__half*>(p.out)[r0 * HD + k] = __float2half(0.0f);
            else static_cast<float*>(p.out)[r0 * HD + k] = 0.0f;
        }
    }
    if (nseg == 0) return;

    // ======================= producer warp ========================================
    if (!SELF && warp == NCW) {
        const int32_t* bt = p.block_tables;
        auto npg_of = [&](int s) { return rec(s)[0].z; };
        auto advance = [&](int& s, int& j) {
            j += 32;
            if (j >= npg_of(s)) {
                j = 0;
                ++s;
                while (s < nseg && npg_of(s) == 0) ++s;
            }
        };
        // page j + lane of segment s (block-table entry; validated when used)
        auto raw_pid = [&](int s, int j) -> int32_t {
            if (s >= nseg) return 0;
            const int4 r0 = rec(s)[0];
            const int jj = j + lane;
            if (jj >= r0.z) return 0;
            if (s == 0 && jj < kPlanPids) return spids[jj];
            return __ldg(bt + static_cast<int64_t>(r0.x) * p.max_blocks + r0.y + jj);
        };
        int cs = 0, cj = 0;
        while (cs < nseg && npg_of(cs) == 0) ++cs;
        int ns = cs, nj = 0;
        if (ns < nseg) advance(ns, nj);
        int32_t pid = raw_pid(cs, cj);
        int32_t pid_next = raw_pid(ns, nj);  // the next chunk's entries are in flight meanwhile
        int k = 0, issued = pre;  // pages [0, pre) of segment 0 went out before the wait
        bool dead = false;
        const uint32_t tx = static_cast<uint32_t>(2 * p.page_bytes);
        while (cs < nseg) {
            const int n = min(32, npg_of(cs) - cj);
            if (lane < n && (pid < 0 || pid >= p.num_pages)) {
                flag(p.status, MG_DEV_BAD_PAGE_ID);
                pid = 0;
            }
            const float ks = lane < n ? __ldg(p.k_scales + pid) : 0.0f;
            const float vs = lane < n ? __ldg(p.v_scales + pid) : 0.0f;
            // Pages go out in pairs: the pair's stage waits first, then lanes 2j /
            // 2j + 1 issue the K / V copy of page j in one instruction (several
            // issuing lanes: one lane measured 4.2 against 6.2 TB/s with four on
            // streams of 12 KB pages; groups of 4 pages held issues back until four
            // stages were free).  Before any wait, the scales of every page issued
            // so far are published (their consumers may be what frees the stage).
            // With per-head copies, one page at a time.
            const int G = p.tma_per_head ? 1 : 2;
            const int i0 = k == 0 ? pre : 0;  // (the pages copied before the wait are published too)
            int pub = i0;  // pages [pub, issued - k) of the chunk are issued, scales not yet published
            for (int i = i0; i < n; i += G) {
                const int gi = min(G, n - i);
                if (k + i + gi > NS) {
                    if (lane >= pub && k + lane < issued) {
                        const int sl = stage_of(k + lane);
                        meta[sl] = make_float2(ks, vs);
                        mbar_arrive(&full[sl]);
                    }
                    pub = max(pub, issued - k);
                    for (int j = 0; j < gi; ++j) {
                        const int kk = k + i + j;
                        if (kk >= NS && !dead &&
                            !__all_sync(0xffffffffu, mbar_wait_limited(&empty[stage_of(kk)], (round_of(kk) - 1) & 1))) {
                            dead = true;
                            if (lane == 0) flag(p.status, MG_DEV_TIMEOUT);
                        }
                    }
                }
                if (dead) continue;
                if (p.tma_per_head) {
                    const int kk = k + i;
                    const int st = stage_of(kk);
                    const int32_t pi = __shfl_sync(0xffffffffu, pid, i);
                    uint8_t* dk = stages + static_cast<int64_t>(st) * sbytes;
                    if (lane == 0) mbar_arrive_expect_tx(&full[st], tx);
                    __syncwarp();
                    tma_page(dk, &tm_k, pi, &full[st], 1, Hkv, p.P, T::TILE, lane);
                    tma_page(dk + sbytes / 2, &tm_v, pi, &full[st], 1, Hkv, p.P, T::TILE, lane);
                } else {
                    const int j = lane >> 1;
                    const int32_t pj = __shfl_sync(0xffffffffu, pid, min(i + j, 31));
                    const int st = stage_of(k + i + j);
                    uint8_t* dst = stages + static_cast<int64_t>(st) * sbytes + ((lane & 1) ? sbytes / 2 : 0);
                    if (j < gi && (lane & 1) == 0) mbar_arrive_expect_tx(&full[st], tx);
                    __syncwarp();
                    if (j < gi) tma_page(dst, (lane & 1) ? &tm_v : &tm_k, pj, &full[st], 0, Hkv, p.P, T::TILE, 0);
                }
                issued = k + i + gi;
            }
            if (lane >= pub && lane < n && k + lane < issued) {  // (after a give-up, only issued pages)
                const int sl = stage_of(k + lane);
                meta[sl] = make_float2(ks, vs);
                mbar_arrive(&full[sl]);
            }
            k += n;
            cs = ns;
            cj = nj;
            pid = pid_next;
            if (ns < nseg) {
                advance(ns, nj);
                pid_next = raw_pid(ns, nj);
            }
        }
        // no copy may outlive the CTA: wait (bounded) for the last phase of every stage used
        for (int st = lane; st < NS && st < issued; st += 32)
            if (!mbar_wait_limited(&full[st], round_of(issued - 1 - st) & 1)) flag(p.status, MG_DEV_TIMEOUT);
        return;
    }

    // ======================= consumer warps =======================================
    const int wsub = WPH > 1 ? warp % WPH : 0;
    const int h = WPH > 1 ? warp / WPH : warp;
    // this lane's ldmatrix row: matrix m = lane / 8 (rows 0-7 / 8-15 of chunk 2x / 2x + 1)
    uint32_t off[T::X4];
#pragma unroll
    for (int x = 0; x < T::X4; ++x)
        off[x] = static_cast<uint32_t>((SELF ? 0 : h) * T::TILE) +
                 tile_chunk_off<KV4, HD>((lane & 7) + 8 * ((lane >> 3) & 1), 2 * x + (lane >> 4));
    const uint32_t st0 = smem_u32(stages);
    TmaHead<NT, MT> S;
    // SELF: this warp's ring of RS slots ([K tile | V tile], sbytes each, and the
    // page's two scales) and its page-id window (lane l: local tile mbase + l)
    constexpr int RS = kSelfSlots<KV4, HD>;
    uint8_t* ring = stages + static_cast<int64_t>(warp) * RS * sbytes;
    float2* wmeta = meta + warp * RS;
    const uint32_t ring0 = smem_u32(ring);
    int mbase = 0;
    int32_t mpid = 0;
    int kbase = 0;
    bool dead = false;
    int pend_s[2] = {-1, -1};
    uint32_t pend_t[2] = {0u, 0u};

    for (int cidx = 0; cidx < nseg; ++cidx) {
        const int4 r0 = rec(cidx)[0], r1 = rec(cidx)[1];
        const int b = r0.x, npg = r0.z, tail = r0.w, pslot = r1.x;
        const bool complete = pslot < 0;
        if (!complete) pend_s[cidx == 0 ? 0 : 1] = cidx;
        const int first = (wsub - kbase % WPH + WPH) % WPH;
        const int ntile = first < npg ? (npg - 1 - first) / WPH + 1 : 0;
        const bool has_tail = tail > 0 && wsub == (kbase + npg) % WPH;
        // SELF: local tile i (segment page first + i * WPH) into slot i % RS, one
        // copy group per call (empty past the warp's last tile)
        auto refill = [&](int i0) {
            const int i = i0 + lane;
            int32_t v = 0;
            if (i < ntile) {
                const int pi = first + i * WPH;
                v = (cidx == 0 && pi < kPlanPids)
                        ? spids[pi]
                        : __ldg(p.block_tables + static_cast<int64_t>(b) * p.max_blocks + r0.y + pi);
                if (v < 0 || v >= p.num_pages) {
                    flag(p.status, MG_DEV_BAD_PAGE_ID);
                    v = 0;
                }
            }
            mbase = i0;
            mpid = v;
        };
        auto issue = [&](int i) {
            if (i < ntile) {
                if (i >= mbase + 32) refill(i);
                const int32_t pid = __shfl_sync(0xffffffffu, mpid, i - mbase);
                const int sl = i & (RS - 1);
                uint8_t* dk = ring + static_cast<int64_t>(sl) * sbytes;
                const int64_t go = static_cast<int64_t>(pid) * p.page_bytes + h * T::ROWB;
                const int rs = Hkv * T::ROWB;
#pragma unroll
                for (int q = lane; q < 16 * T::CHUNKS; q += 32) {
                    const int t = q / T::CHUNKS, j = q - t * T::CHUNKS;
                    const uint32_t o = tile_chunk_off<KV4, HD>(t, j);
                    cp_async16(dk + o, p.k_pool + go + t * rs + 16 * j);
                    cp_async16(dk + T::TILE + o, p.v_pool + go + t * rs + 16 * j);
                }
                if (lane == 0) cp_async4(&wmeta[sl].x, p.k_scales + pid);
                if (lane == 1) cp_async4(&wmeta[sl].y, p.v_scales + pid);
            }
            cp_async_commit();
        };
        if constexpr (SELF) {
            mbase = -(1 << 30);
            for (int i = cidx == 0 ? pre : 0; i < RS; ++i) issue(i);
        }
        // the tail rows' L1 prefetch goes out before q's loads, which the warp waits for
        if (has_tail && (lane & 15) < tail) {
            const __half* st16 = static_cast<const __half*>(lane < 16 ? p.staging_k : p.staging_v);
            const __half* rp = st16 + ((static_cast<int64_t>(b) * p.P + (lane & 15)) * Hkv + h) * HD;
#pragma unroll
            for (int l = 0; l < HD * 2; l += 128) prefetch_l1(reinterpret_cast<const char*>(rp) + l);
        }
        if (ntile > 0 || has_tail) tma_load_q<KV4, HD, NT, SPLIT>(S, p, b, h, g, c);
        else tma_clear(S);
        // the warp's pages two at a time (one 32-token step), an odd last one alone
        auto wait_full = [&](int k) {
            if (!dead && !__all_sync(0xffffffffu, mbar_wait_limited(&full[stage_of(k)], round_of(k) & 1))) {
                dead = true;
                if (lane == 0) flag(p.status, MG_DEV_TIMEOUT);
            }
        };
        const uint32_t vdelta = static_cast<uint32_t>(sbytes / 2);
        int i = 0;
        if constexpr (SELF) {
            // two tiles a step: wait for their copy groups, run them, refill their slots
            for (; i < ntile; i += 2) {
                cp_async_wait_group<RS - 2>();
                __syncwarp();
                const int s0 = i & (RS - 1), s1 = (i + 1) & (RS - 1);
                if (i + 1 < ntile) {
                    const float2 m0 = wmeta[s0], m1 = wmeta[s1];
                    const uint32_t kb[2] = {ring0 + static_cast<uint32_t>(s0 * sbytes),
                                            ring0 + static_cast<uint32_t>(s1 * sbytes)};
                    const float ksc[2] = {m0.x * p.sm_scale_log2, m1.x * p.sm_scale_log2}, vsc[2] = {m0.y, m1.y};
                    uint64_t* const em[2] = {nullptr, nullptr};
                    tma_page_tiles<KV4, HD, NT, SPLIT, 2, true>(S, kb, off, T::TILE, ksc, vsc, em, lane);
                } else {
                    const float2 m0 = wmeta[s0];
                    const uint32_t kb[1] = {ring0 + static_cast<uint32_t>(s0 * sbytes)};
                    const float ksc[1] = {m0.x * p.sm_scale_log2}, vsc[1] = {m0.y};
                    uint64_t* const em[1] = {nullptr};
                    tma_page_tiles<KV4, HD, NT, SPLIT, 1, PAIRS>(S, kb, off, T::TILE, ksc, vsc, em, lane);
                }
                issue(i + RS);
                issue(i + RS + 1);
            }
        }
        for (; !SELF && PAIRS && i + 1 < ntile; i += 2) {
            const int k0 = kbase + first + i * WPH, k1 = k0 + WPH;
            const int s0 = stage_of(k0), s1 = stage_of(k1);
            wait_full(k0);
            wait_full(k1);
            const float2 m0 = meta[s0], m1 = meta[s1];
            const uint32_t kb[2] = {st0 + static_cast<uint32_t>(s0 * sbytes), st0 + static_cast<uint32_t>(s1 * sbytes)};
            const float ksc[2] = {m0.x * p.sm_scale_log2, m1.x * p.sm_scale_log2}, vsc[2] = {m0.y, m1.y};
            uint64_t* const em[2] = {&empty[s0], &empty[s1]};
            tma_page_tiles<KV4, HD, NT, SPLIT, 2, true>(S, kb, off, vdelta, ksc, vsc, em, lane);
        }
        for (; !SELF && i < ntile; ++i) {
            const int k0 = kbase + first + i * WPH;
            const int s0 = stage_of(k0);
            wait_full(k0);
            const float2 m0 = meta[s0];
            const uint32_t kb[1] = {st0 + static_cast<uint32_t>(s0 * sbytes)};
            const float ksc[1] = {m0.x * p.sm_scale_log2}, vsc[1] = {m0.y};
            uint64_t* const em[1] = {&empty[s0]};
            tma_page_tiles<KV4, HD, NT, SPLIT, 1, PAIRS>(S, kb, off, vdelta, ksc, vsc, em, lane);
        }
        if (has_tail) tma_tail_tile<KV4, HD, NT, SPLIT>(S, p, b, h, tail, g, c);
        kbase += npg;

        // ---- finalize: per (column) m / l / o[VE] ---------------------------------------
        float o_all[NT][NCOLS][VE], m_all[NT][NCOLS], l_all[NT][NCOLS];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int col = 0; col < NCOLS; ++col) {
                float l = S.lpart[nt][col];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                float mtr = S.m_true[nt][col];
                mtr = fmaxf(mtr, __shfl_xor_sync(0xffffffffu, mtr, 4));
                mtr = fmaxf(mtr, __shfl_xor_sync(0xffffffffu, mtr, 8));
                mtr = fmaxf(mtr, __shfl_xor_sync(0xffffffffu, mtr, 16));
                const float f = (mtr == -INFINITY) ? 0.0f : ex2(S.m_used[nt][col] - mtr);
                l_all[nt][col] = l * f;
                m_all[nt][col] = mtr;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const float fs = (KV4 && (mt & 1)) ? f * 0.0625f : f;  // high-nibble rows carry 16 c
                    if (SPLIT) {
                        o_all[nt][col][2 * mt] = (S.acc[mt][nt][0] + S.acc[mt][nt][1]) * fs;
                        o_all[nt][col][2 * mt + 1] = (S.acc[mt][nt][2] + S.acc[mt][nt][3]) * fs;
                    } else {
                        o_all[nt][col][2 * mt] = S.acc[mt][nt][col] * fs;
                        o_all[nt][col][2 * mt + 1] = S.acc[mt][nt][col + 2] * fs;
                    }
                }
            }
        if (WPH > 1) {
            const int bar = 1 + h, nthr = WPH * 32;
            constexpr int PER = NT * NCOLS * 4 * (HD + 2);
            named_barrier_sync(bar, nthr);
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
                        const int o0 = ((nt * NCOLS + col) * 4 + c) * (HD + 2);
                        float M = -INFINITY;
                        for (int ww = 0; ww < WPH; ++ww)
                            M = fmaxf(M, mscratch[static_cast<int64_t>(warp + ww) * PER + o0 + HD]);
                        float L = 0.0f;
                        float oo[VE];
#pragma unroll
                        for (int e = 0; e < VE; ++e) oo[e] = 0.0f;
                        for (int ww = 0; ww < WPH; ++ww) {
                            const float* mw = mscratch + static_cast<int64_t>(warp + ww) * PER + o0;
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
                if (complete) {
                    const float inv = 1.0f / l;
                    if (p.out_f16) {
                        __half* op = static_cast<__half*>(p.out) + orow * HD;
#pragma unroll
                        for (int e = 0; e < VE; ++e) op[tdim<KV4>(g, e)] = __float2half_rn(o[e] * inv);
                    } else {
                        float* op = static_cast<float*>(p.out) + orow * HD;
#pragma unroll
                        for (int e = 0; e < VE; ++e) op[tdim<KV4>(g, e)] = o[e] * inv;
                    }
                } else {
                    const int64_t prow = static_cast<int64_t>(pslot) * Hq + (orow - static_cast<int64_t>(b) * Hq);
                    float* wp = p.ws_acc + prow * HD;
#pragma unroll
                    for (int e = 0; e < VE; ++e) __stcg(wp + tdim<KV4>(g, e), o[e]);
                    if (g == 0) {
                        __stcg(p.ws_m + prow, m);
                        __stcg(p.ws_l + prow, l);
                    }
                }
            }
        if (complete) continue;
        // publish the partial: the ticket's release orders the warp's stores
        __syncwarp();
        uint32_t prev = 0;
        if (lane == 0) prev = ticket_add(&p.tickets[static_cast<int64_t>(b) * Hkv + h]);
        pend_t[cidx == 0 ? 0 : 1] = prev;
    }

    // ---- merges of the cut sequences whose last covering CTA this is -------------
#pragma unroll
    for (int kx = 0; kx < 2; ++kx) {
        if (pend_s[kx] < 0) continue;
        const int4 q0 = rec(pend_s[kx])[0], q1 = rec(pend_s[kx])[1];
        const int b = q0.x, pbase = q1.y, ncov = q1.z;
        const uint32_t need = static_cast<uint32_t>(ncov - 1);
        bool last = false;
        if (wsub == 0) last = __shfl_sync(0xffffffffu, pend_t[kx], 0) == need;
        if (WPH > 1) {
            int* slot = sm_last + kx * kWarps + h;
            if (wsub == 0 && lane == 0) *slot = last ? 1 : 0;
            named_barrier_sync(1 + h, WPH * 32);
            last = *slot != 0;
        }
        if (!last) continue;
        __threadfence();
        merge_partials<HD>(p, b, h, pbase, ncov, lane, wsub, WPH);
    }
    if (SELF) cp_async_wait_all();  // (only empty groups are left) no copy outlives the CTA
}

template <bool KV4, int HD, int NT, bool SPLIT, int NW, bool SELF>
mg_status launch_tma_one(const DecodeParams& p, const DecodePlan& pl, const CUtensorMap& tk, const CUtensorMap& tv,
                         cudaStream_t s) {
    auto k = paged_decode_tma_kernel<KV4, HD, NT, SPLIT, NW, SELF>;
    if (SELF && p.tma_ns != kSelfSlots<KV4, HD>)
        return set_error(MG_ERR_UNSUPPORTED, "self-copying decode kernel: %d ring slots planned, %d compiled", p.tma_ns,
                         kSelfSlots<KV4, HD>);
    if (pl.nconsumers > NW)
        return set_error(MG_ERR_UNSUPPORTED, "decode plan (%d consumer warps) does not fit the kernel (%d)",
                         pl.nconsumers, NW);
    static int64_t attr_set[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || attr_set[dev] < pl.smem_bytes) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(pl.smem_bytes));
        if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_set[dev] = pl.smem_bytes;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(32 * (pl.nconsumers + (SELF ? 0 : 1)));
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem_bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k, tk, tv, p);
    if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "paged_decode_tma_kernel launch: %s", cudaGetErrorString(e));
    return check_launch("paged_decode_tma_kernel");
}

template <bool KV4, int HD, bool SELF>
mg_status launch_tma_mode(const DecodeParams& p, const DecodePlan& pl, const CUtensorMap& tk, const CUtensorMap& tv,
                          cudaStream_t s) {
    // 12 consumer warps + the producer (13 warps, budgeted as 16: 128 registers), or
    // 15 + 1 for 13-15 kv heads; 17 warps would be budgeted as 20 (96 registers)
    // (head_dim 128 with two n-tiles does not fit 128 registers: the register
    // kernel serves it)
    const bool w15 = pl.nconsumers > 12;
    if (pl.nt == 1) {
        if (pl.split_mode)
            return w15 ? launch_tma_one<KV4, HD, 1, true, 15, SELF>(p, pl, tk, tv, s)
                       : launch_tma_one<KV4, HD, 1, true, 12, SELF>(p, pl, tk, tv, s);
        return w15 ? launch_tma_one<KV4, HD, 1, false, 15, SELF>(p, pl, tk, tv, s)
                   : launch_tma_one<KV4, HD, 1, false, 12, SELF>(p, pl, tk, tv, s);
    }
    if constexpr (HD == 64) {
        if (pl.split_mode)
            return w15 ? launch_tma_one<KV4, HD, 2, true, 15, SELF>(p, pl, tk, tv, s)
                       : launch_tma_one<KV4, HD, 2, true, 12, SELF>(p, pl, tk, tv, s);
        return w15 ? launch_tma_one<KV4, HD, 2, false, 15, SELF>(p, pl, tk, tv, s)
                   : launch_tma_one<KV4, HD, 2, false, 12, SELF>(p, pl, tk, tv, s);
    }
    return set_error(MG_ERR_UNSUPPORTED, "bulk-copy decode kernel: head_dim 128 with a group over 4 (8) q heads");
}

// self_copy: the consumer warps copy their own tiles (INT4 pools only)
template <bool KV4, int HD>
mg_status launch_tma(const DecodeParams& p, const DecodePlan& pl, const CUtensorMap& tk, const CUtensorMap& tv,
                     cudaStream_t s, bool self_copy) {
    if constexpr (KV4) {
        if (self_copy) return launch_tma_mode<KV4, HD, true>(p, pl, tk, tv, s);
    }
    if (self_copy) return set_error(MG_ERR_UNSUPPORTED, "self-copying decode kernel: INT4 pools only");
    return launch_tma_mode<KV4, HD, false>(p, pl, tk, tv, s);
}

}  // namespace mg
