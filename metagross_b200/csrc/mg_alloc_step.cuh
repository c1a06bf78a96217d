// One decode step's page allocation, shared by plan_append_kernel (mg_cache.cu)
// and the fused allocation + plan kernel (mg_plan.cu).
#pragma once

#include "mg_common.cuh"

namespace mg {

// status bits after which a step's later launches do nothing
constexpr int32_t kStopBits = MG_DEV_OUT_OF_PAGES | MG_DEV_BLOCK_TABLE_FULL | MG_DEV_BAD_LENGTH;

struct AllocStep {
    int32_t* free_stack;
    int32_t* n_free;
    int32_t* in_use;
    int32_t* block_tables;  // [batch, max_blocks]
    int32_t max_blocks;
    int32_t* seq_lens;
    const int32_t* n_new;
    int32_t batch;
    int32_t P;
    int32_t* status;
};

// Grow every sequence b by n_new[b] tokens and pop the pages that fill from the
// LIFO free stack into its block-table row (metagross/cache.py:45-72 batched:
// a page is allocated when the token count crosses a page boundary), for the
// whole batch or not at all: pass 1 validates the step, pass 2 applies it.
// Called by every thread of one CTA (every return is CTA-uniform); after a
// __syncthreads() that follows the call, the step's seq_lens and block tables
// are visible to the whole CTA.
__device__ __forceinline__ void alloc_step(const AllocStep& a) {
    __shared__ int scratch[33];
    __shared__ int s_flags;
    __shared__ int s_stop;
    if (threadIdx.x == 0) {
        s_flags = 0;
        s_stop = (a.status && (*(volatile int32_t*)a.status & kStopBits)) ? 1 : 0;
        if (s_stop) flag(a.status, MG_DEV_SKIPPED);
    }
    __syncthreads();
    if (s_stop) return;
    int local = 0;
    int bad = 0;  // bit 0: a row would overflow; bit 1: a negative length or count
    for (int b = threadIdx.x; b < a.batch; b += blockDim.x) {
        const int old = a.seq_lens[b], add = a.n_new[b];
        if (add < 0 || old < 0) {
            bad |= 2;
            continue;
        }
        const int nw = old + add;
        if (nw / a.P > a.max_blocks) bad |= 1;
        local += nw / a.P - old / a.P;
    }
    int total;
    if (bad) atomicOr(&s_flags, bad);
    (void)block_exclusive_scan(local, scratch, &total);
    __syncthreads();
    const int n_free = *a.n_free;
    if (s_flags) {
        if (threadIdx.x == 0)
            flag(a.status, ((s_flags & 1) ? MG_DEV_BLOCK_TABLE_FULL : 0) | ((s_flags & 2) ? MG_DEV_BAD_LENGTH : 0));
        return;
    }
    if (total > n_free) {
        if (threadIdx.x == 0) flag(a.status, MG_DEV_OUT_OF_PAGES);
        return;
    }
    int base = 0;
    for (int start = 0; start < a.batch; start += blockDim.x) {
        const int b = start + threadIdx.x;
        int old = 0, nw = 0, c = 0;
        if (b < a.batch) {
            old = a.seq_lens[b];
            nw = old + a.n_new[b];
            c = nw / a.P - old / a.P;
        }
        int chunk_total;
        const int excl = block_exclusive_scan(c, scratch, &chunk_total) + base;
        if (b < a.batch) {
            int32_t* row = a.block_tables + static_cast<int64_t>(b) * a.max_blocks;
            for (int j = 0; j < c; ++j) {
                const int32_t page = a.free_stack[n_free - 1 - (excl + j)];
                row[old / a.P + j] = page;
                a.in_use[page] = 1;
            }
            a.seq_lens[b] = nw;
        }
        base += chunk_total;
    }
    __syncthreads();
    if (threadIdx.x == 0) *a.n_free = n_free - total;
}

}  // namespace mg
