/*
 * metagross_b200.h -- C ABI of the B200-native paged quantized KV-cache and
 * decode-attention path.
 *
 * Every entry point takes plain device pointers, 64-bit sizes and a CUDA
 * stream (as an opaque pointer; NULL is the legacy default stream) and
 * returns an mg_status.  No C++ exception, torch type or host allocation
 * crosses this boundary.  Kernels are enqueued on the given stream and the
 * calls never synchronise the device, except where a comment says so.
 *
 * The first group replaces, one for one, the seven ops the reference binds in
 * csrc/bindings.cpp:3-19 (declared in csrc/metagross_ops.h:6-32).  The
 * second group is the batched, device-resident path that replaces the
 * per-token Python loops of metagross/cache.py and the per-sequence calls of
 * metagross/attention.py.
 *
 * Layouts (identical to the reference's storage, metagross/cache.py:36-38 and
 * csrc/quantize_int4.cu:74):
 *   INT8 pool   int8  [num_pages, page_size, num_kv_heads, head_dim]
 *   INT4 pool   uint8 [num_pages, page_size, num_kv_heads, head_dim/2],
 *               element 2j in the low nibble of byte j, two's complement
 *   page scales float [num_pages], one per physical page, K and V separate
 *               (metagross/cache.py:39)
 */
#ifndef METAGROSS_B200_H
#define METAGROSS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MG_API __attribute__((visibility("default")))
#else
#define MG_API
#endif

typedef void* mg_stream_t; /* a cudaStream_t */

typedef enum mg_status {
    MG_OK = 0,
    MG_ERR_INVALID_ARGUMENT = 1, /* shape, offset, scale, dtype or pointer rejected before launch */
    MG_ERR_OUT_OF_PAGES = 2,     /* host-side allocation request larger than the free pool */
    MG_ERR_CUDA = 3,             /* a CUDA runtime call failed (launch, attribute, copy) */
    MG_ERR_UNSUPPORTED = 4       /* valid request outside what the kernels implement */
} mg_status;

/* Bits a kernel ORs into the caller's device status word (int32).  The
 * batched calls never synchronise; the host reads the word when it chooses. */
#define MG_DEV_OUT_OF_PAGES 0x1      /* mg_plan_append: commits exceed the free pages; nothing changed */
#define MG_DEV_BAD_PAGE_ID 0x2       /* a block-table id outside [0, num_pages); page 0 read instead */
#define MG_DEV_DOUBLE_FREE 0x4       /* mg_free_*: page already free; skipped */
#define MG_DEV_TIMEOUT 0x8           /* a bounded wait on a bulk copy gave up; output invalid */
#define MG_DEV_BLOCK_TABLE_FULL 0x10 /* mg_plan_append: a sequence would outgrow its block-table row */
#define MG_DEV_SKIPPED 0x20          /* a kernel skipped its work because an earlier bit was set */
#define MG_DEV_CONTEXT_OVERFLOW 0x40 /* reserved (no current kernel sets it) */
#define MG_DEV_BAD_ARGUMENT 0x80     /* a per-sequence argument (n_new > max_new, seq id, cu_seqlens) was inconsistent; that sequence was skipped */
#define MG_DEV_BAD_LENGTH 0x100      /* mg_plan_append: a negative n_new or seq_lens entry; the step changed nothing */

typedef enum mg_kv_dtype { MG_KV_INT8 = 0, MG_KV_INT4 = 1 } mg_kv_dtype;
/* Scale granularity of a batched pool.  MG_SCALE_PAGE is the reference's only
 * layout (metagross/cache.py:39,69-70: one fp32 per physical page, K and V
 * separately).  MG_SCALE_TOKEN_HEAD has no counterpart in the reference: one
 * fp32 absmax scale per (page, token, kv head), each D-vector quantized as the
 * reference's quantize_new_scale quantizes a [1, 1, D] slice. */
typedef enum mg_scale_layout { MG_SCALE_PAGE = 0, MG_SCALE_TOKEN_HEAD = 1 } mg_scale_layout;
typedef enum mg_float_dtype { MG_F32 = 0, MG_F16 = 1 } mg_float_dtype;

MG_API const char* mg_version(void);
/* Text of the last non-OK status returned on the calling host thread. */
MG_API const char* mg_last_error(void);

/* ------------------------------------------------------------------------
 * Reference op equivalents (csrc/bindings.cpp:4-18)
 * ---------------------------------------------------------------------- */

/* add (csrc/sanity_add.cu:11-38): out = a + b, n fp32 elements. */
MG_API mg_status mg_add_f32(const float* a, const float* b, float* out, int64_t n, mg_stream_t stream);

/* quantize_new_scale (csrc/quantize.cu:65-120).  input fp32 [num_tokens, row]
 * (row = num_heads*head_dim, contiguous); page int8 [page_tokens, row].
 * One kernel: absmax over the input, scale = absmax/127 in double (1e-8 when
 * the absmax is not finite or <= 1e-12), codes written to
 * page[(token_offset + t)*row + i].  The scale (double) is written to the
 * device word *scale_out.  num_tokens == 0 writes 1e-8 and leaves the page. */
MG_API mg_status mg_quantize_int8_new_scale(const float* input, int64_t num_tokens, int64_t row,
                                     int8_t* page, int64_t page_tokens, int64_t token_offset,
                                     double* scale_out, mg_stream_t stream);

/* quantize_fixed_scale (csrc/quantize.cu:122-167): same with a caller scale
 * (finite and > 0). */
MG_API mg_status mg_quantize_int8_fixed_scale(const float* input, int64_t num_tokens, int64_t row,
                                       int8_t* page, int64_t page_tokens, int64_t token_offset,
                                       double scale, mg_stream_t stream);

/* dequantize_page (csrc/dequantize.cu:30-71): out fp32 [num_tokens, row] =
 * page[token_offset + t] * (float)scale. */
MG_API mg_status mg_dequantize_int8_page(const int8_t* page, int64_t page_tokens, int64_t row,
                                  int64_t token_offset, int64_t num_tokens, double scale,
                                  float* out, mg_stream_t stream);

/* quantize_int4_new_scale (csrc/quantize_int4.cu:69-125).  input fp32
 * [num_tokens, num_heads, head_dim], head_dim even; packed uint8
 * [page_tokens, num_heads, head_dim/2].  Scale = absmax/7 in double. */
MG_API mg_status mg_quantize_int4_new_scale(const float* input, int64_t num_tokens, int64_t num_heads,
                                     int64_t head_dim, uint8_t* packed, int64_t page_tokens,
                                     int64_t token_offset, double* scale_out, mg_stream_t stream);

/* dequantize_int4_page (csrc/dequantize_int4.cu:41-82): out fp32
 * [num_tokens, half_row*2] from packed[token_offset + t]. */
MG_API mg_status mg_dequantize_int4_page(const uint8_t* packed, int64_t page_tokens, int64_t half_row,
                                  int64_t token_offset, int64_t num_tokens, double scale,
                                  float* out, mg_stream_t stream);

/* paged_attention_committed (csrc/paged_attention.cu:139-255).  One sequence,
 * one decode query per head, committed INT8 pages only.  query fp32
 * [num_q_heads, head_dim]; k/v storage int8 [max_pages, page_size,
 * num_kv_heads, head_dim]; page_scales_k/v fp32 [max_pages]; block_table
 * int32 [num_blocks] (device).  Outputs (unnormalised, as the reference):
 * out_wv fp32 [num_q_heads, head_dim] = sum_t e^(s_t - m) v_t,
 * out_sum [num_q_heads] = sum_t e^(s_t - m), out_max [num_q_heads] = m, with
 * s_t = scale * q.k_t.  No pages: (0, 0, -inf).  head_dim 64 or 128,
 * num_q_heads a multiple of num_kv_heads.  The kernel checks every block-table
 * id; a bad id sets MG_DEV_BAD_PAGE_ID in *dev_status (nullable).
 * workspace: mg_paged_attention_committed_workspace_bytes() bytes, zeroed by
 * the caller before its first use (the kernels leave it reusable). */
MG_API mg_status mg_paged_attention_committed(const float* query, const int8_t* k_storage,
                                       const int8_t* v_storage, const float* page_scales_k,
                                       const float* page_scales_v, const int32_t* block_table,
                                       int64_t num_blocks, int64_t max_pages, int64_t page_size,
                                       int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                       double scale, float* out_wv, float* out_sum, float* out_max,
                                       void* workspace, int64_t workspace_bytes,
                                       int32_t* dev_status, mg_stream_t stream);
MG_API int64_t mg_paged_attention_committed_workspace_bytes(int64_t num_blocks, int64_t page_size,
                                                     int64_t num_q_heads, int64_t num_kv_heads,
                                                     int64_t head_dim);

/* ------------------------------------------------------------------------
 * Batched device-resident cache (replaces metagross/cache.py:45-85 and the
 * per-sequence loop of metagross/attention.py:62-134 for a batch)
 * ---------------------------------------------------------------------- */

/* Pool geometry shared by every layer of one cache. */
typedef struct mg_cache_layout {
    int32_t kv_dtype;      /* mg_kv_dtype */
    int32_t staging_dtype; /* mg_float_dtype of the exact staged tail */
    int32_t page_size;     /* P, tokens per page, 1..64 */
    int32_t num_kv_heads;  /* Hkv */
    int32_t head_dim;      /* D: 64 or 128 for attention; the quantize/dequantize kernels take any even D with D*bits/8 % 16 == 0 */
    int32_t max_blocks;    /* width of a block-table row */
    int64_t num_pages;     /* pool capacity N */
    int32_t scale_layout;  /* mg_scale_layout; MG_SCALE_TOKEN_HEAD needs head_dim a power of two <= 256 */
    int32_t reserved;      /* 0 */
} mg_cache_layout;

/* Device pointers of one layer. */
typedef struct mg_layer_ptrs {
    void* k_pool;    /* [N, P, Hkv, D] int8 or [N, P, Hkv, D/2] uint8 */
    void* v_pool;
    float* k_scales; /* [N] (MG_SCALE_PAGE) or [N, P, Hkv] (MG_SCALE_TOKEN_HEAD) */
    float* v_scales; /* same shape as k_scales */
    void* staging_k; /* [B, P, Hkv, D] staging_dtype: tokens of the page being filled */
    void* staging_v;
} mg_layer_ptrs;

/* Device page allocator: LIFO stack with the reference's order
 * (metagross/allocator.py:1-33): a fresh pool hands out N-1, N-2, ...; a
 * freed id is handed out next. */
typedef struct mg_allocator {
    int32_t* free_stack; /* [N] */
    int32_t* n_free;     /* [1] */
    int32_t* in_use;     /* [N] 1 while allocated */
    int64_t num_pages;
} mg_allocator;

/* Reset the allocator to the fresh state (all pages free, stack 0..N-1). */
MG_API mg_status mg_alloc_init(const mg_allocator* alloc, mg_stream_t stream);

/* Step planner, once per decode/prefill step for all layers: for every
 * sequence b, seq_lens[b] grows by n_new[b] tokens; every page that becomes
 * full gets a physical id popped from the allocator, sequences in index
 * order and pages in logical order (so the ids equal a reference
 * BlockAllocator replaying the same commits) and written to
 * block_tables[b, j].  All-or-nothing: when the commits exceed the free pages
 * (MG_DEV_OUT_OF_PAGES) or a row (MG_DEV_BLOCK_TABLE_FULL), or a length or
 * count is negative (MG_DEV_BAD_LENGTH), nothing changes and the
 * append/attention calls that take the same dev_status skip their work. */
MG_API mg_status mg_plan_append(const mg_allocator* alloc, int32_t* block_tables, int32_t max_blocks,
                         int32_t* seq_lens, const int32_t* n_new, int32_t batch, int32_t page_size,
                         int32_t* dev_status, mg_stream_t stream);

/* mg_plan_append (with layout's max_blocks and page_size) followed by
 * mg_paged_decode_plan from the grown lengths, in one launch: a decode step's
 * allocation and its attention plan.  Same results as the two calls in that
 * order; batch in [1, 8192].  Issued before the step's first append, it
 * leaves every attention launch of the step free to take MG_ATTN_PLAN_SETTLED. */
MG_API mg_status mg_plan_step(const mg_allocator* alloc, const mg_cache_layout* layout, int32_t* block_tables,
                       int32_t* seq_lens, const int32_t* n_new, int32_t batch, int32_t with_staging, void* plan,
                       int64_t plan_bytes, int32_t* dev_status, mg_stream_t stream);

/* Per layer, after mg_plan_append: write the step's new tokens.  k_new/v_new
 * [batch, max_new, Hkv, D] in new_dtype (f16 or f32); seq_lens are the lengths
 * AFTER the step, n_new the tokens added.  A page that fills is quantized with
 * one fresh absmax scale over the whole page (K and V separately) exactly as
 * metagross/cache.py:63-72 + csrc/quantize.cu; with MG_SCALE_TOKEN_HEAD every
 * (token, head) D-vector of the page gets its own fresh absmax scale.  The
 * partial page's tokens go to staging unquantized.  One call writes at most
 * 65534 pages per sequence (max_new <= 65534 * page_size); a longer prefill
 * is split over several steps. */
MG_API mg_status mg_kv_append(const mg_cache_layout* layout, const mg_layer_ptrs* layer,
                       const int32_t* block_tables, const int32_t* seq_lens, const int32_t* n_new,
                       int32_t batch, const void* k_new, const void* v_new, int32_t new_dtype,
                       int32_t max_new, int32_t* dev_status, mg_stream_t stream);

/* mg_kv_append with launch flags (the plain form passes 0).
 * MG_APPEND_EARLY_LAUNCH: a programmatic dependent launch, whose blocks start
 * as the previous kernel's leave the SMs and wait for it on the device, and
 * which releases the next launch (an attention launch) at its start.  It pays
 * between this library's own kernels: the 12-layer GPT-2-shape decode step
 * measured 0.271 against 0.290 ms.  In the TinyLlama model step (GEMMs between
 * the library's launches) the early release measured slower, 1.35 against
 * 1.22 ms a step, so that step does not set it.  An unknown flag is
 * MG_ERR_INVALID_ARGUMENT. */
#define MG_APPEND_EARLY_LAUNCH 0x1u
MG_API mg_status mg_kv_append_flags(const mg_cache_layout* layout, const mg_layer_ptrs* layer,
                             const int32_t* block_tables, const int32_t* seq_lens, const int32_t* n_new,
                             int32_t batch, const void* k_new, const void* v_new, int32_t new_dtype,
                             int32_t max_new, uint32_t flags, int32_t* dev_status, mg_stream_t stream);

/* mg_kv_append for a Llama-style decode or prefill step whose new tokens come
 * straight from the fused q|k|v projection: qkv fp16 [batch, max_new,
 * (num_q_heads + 2 Hkv) * D] (q heads, then k heads, then v heads, as
 * mg_rope_qkv_f16 takes them).  K is rotated (rotate-half rotary embedding at
 * position seq_len_before + t, tables cos/sin [table_rows, D / 2] fp32,
 * products rounded separately, the result rounded to fp16) on its way into
 * staging or a committed page, V is appended as it is, and the rotated q of
 * every new token is written to q_out [batch, max_new, num_q_heads, D] fp16 --
 * one launch where mg_rope_qkv_f16 + mg_kv_append take two, with identical
 * results.  fp16 staging only; a position beyond the table sets
 * MG_DEV_BAD_ARGUMENT.  Replaces the rotary embedding + per-layer append of
 * metagross/generate_llama.py:20-37,104-107 for a batch. */
MG_API mg_status mg_kv_append_rope(const mg_cache_layout* layout, const mg_layer_ptrs* layer,
                            const int32_t* block_tables, const int32_t* seq_lens, const int32_t* n_new,
                            int32_t batch, const void* qkv, int32_t num_q_heads, const float* cos_table,
                            const float* sin_table, int32_t table_rows, void* q_out, int32_t max_new,
                            int32_t* dev_status, mg_stream_t stream);

/* Fused paged decode attention for a batch: committed quantized pages through
 * the block table plus the exact staged tail, one online softmax, split over
 * the context with an in-kernel merge.  q [batch, num_q_heads, D] (q_dtype),
 * out [batch, num_q_heads, D] (out_dtype) = softmax(scale * q K^T) V.
 * The work is split over the GPU by pages (see mg_paged_decode_plan, which
 * this call runs first), so no length bound is needed: max_context is
 * accepted for compatibility and ignored.
 * workspace: mg_paged_decode_workspace_bytes() bytes.  Its first
 * 256*ceil(4*batch*num_kv_heads/256) bytes are per-(sequence, kv head) merge
 * counters that must be zero before the first call; every call leaves them
 * zero, so one zeroed buffer can serve calls of any max_context and q-head
 * count.  Calls that share a workspace must not overlap on the device. */
MG_API mg_status mg_paged_decode_attention(const mg_cache_layout* layout, const mg_layer_ptrs* layer,
                                    const int32_t* block_tables, const int32_t* seq_lens,
                                    int32_t batch, const void* q, int32_t q_dtype,
                                    int32_t num_q_heads, float scale, void* out, int32_t out_dtype,
                                    int32_t max_context, void* workspace, int64_t workspace_bytes,
                                    int32_t* dev_status, mg_stream_t stream);
MG_API int64_t mg_paged_decode_workspace_bytes(const mg_cache_layout* layout, int32_t batch,
                                        int32_t num_q_heads, int32_t max_context);

/* Decode plan: how one decode step's attention work is split over the GPU's
 * SMs.  It depends only on seq_lens (and the page size), which every layer
 * of a step shares, so a caller that runs attention for many layers builds
 * it once per step (after the step's lengths change) and passes it to
 * mg_paged_decode_attention_planned; mg_paged_decode_attention builds one
 * inside its workspace on every call.  No counterpart in the reference (its
 * paged_attention op handles one sequence per call, csrc/bindings.cpp:82-106).
 * plan: mg_paged_decode_plan_bytes(batch) bytes, 16-byte aligned, device
 * memory; with_staging says whether the attention calls will fold the staged
 * tails in (it must match their staging pointers).  The plan also keeps a
 * copy of each CTA's first block-table entries, so it is rebuilt whenever the
 * block tables or seq_lens change.  Invalid lengths set MG_DEV_BAD_ARGUMENT
 * and are planned as empty. */
MG_API int64_t mg_paged_decode_plan_bytes(int32_t batch);
MG_API mg_status mg_paged_decode_plan(const mg_cache_layout* layout, const int32_t* block_tables,
                               const int32_t* seq_lens, int32_t batch, int32_t with_staging, void* plan,
                               int64_t plan_bytes, int32_t* dev_status, mg_stream_t stream);
/* mg_paged_decode_attention for callers that cannot call cudaMalloc (a
 * serving runtime whose pool allocator owns all device memory, or a decode
 * loop that must not pay cudaMalloc's device synchronisation): no workspace
 * argument; the workspace lives in a 4 MiB static device array inside
 * libmgb200.so, held by every GPU that loads the library until exit.  The
 * first call on each device looks its address up (make that call before any
 * stream capture begins).  Calls whose workspace
 * (mg_paged_decode_workspace_bytes) exceeds 4 MiB are rejected with
 * MG_ERR_INVALID_ARGUMENT.  Each call zeroes the merge counters on `stream`
 * first.  Calls that overlap on the GPU share the array and race.  No
 * counterpart in the reference. */
MG_API mg_status mg_paged_decode_attention_noalloc(const mg_cache_layout* layout, const mg_layer_ptrs* layer,
                                            const int32_t* block_tables, const int32_t* seq_lens,
                                            int32_t batch, const void* q, int32_t q_dtype,
                                            int32_t num_q_heads, float scale, void* out, int32_t out_dtype,
                                            int32_t max_context, int32_t* dev_status, mg_stream_t stream);

/* mg_paged_decode_attention with a plan from mg_paged_decode_plan for the
 * same batch and lengths; workspace as for mg_paged_decode_attention. */
MG_API mg_status mg_paged_decode_attention_planned(const mg_cache_layout* layout, const mg_layer_ptrs* layer,
                                            const int32_t* block_tables, const void* plan, int64_t plan_bytes,
                                            int32_t batch, const void* q, int32_t q_dtype, int32_t num_q_heads,
                                            float scale, void* out, int32_t out_dtype, void* workspace,
                                            int64_t workspace_bytes, int32_t* dev_status, mg_stream_t stream);

/* mg_paged_decode_attention_planned with launch flags (the plain form passes 0).
 * MG_ATTN_PLAN_SETTLED: the plan, the block tables and the allocation status
 * (mg_plan_append) were written by launches that precede the launch right
 * before this one on the stream, and that launch either is not a programmatic
 * dependent launch or waits for its own prerequisites before it releases its
 * dependents (every kernel of this library does; a plain launch does).  The
 * kernel then reads the plan and warms L2 with its first pages before it waits
 * for that launch to finish, on the SMs it has already left; with a plan from
 * mg_plan_step, which records how many of each segment's pages were committed
 * before the step, the bulk-copy kernel starts copying those pages (no launch
 * of the step writes them) before the wait.  Never set it on the launch right
 * after mg_paged_decode_plan or mg_plan_step.  An unknown flag is
 * MG_ERR_INVALID_ARGUMENT. */
#define MG_ATTN_PLAN_SETTLED 0x1u
MG_API mg_status mg_paged_decode_attention_planned_flags(const mg_cache_layout* layout, const mg_layer_ptrs* layer,
                                                  const int32_t* block_tables, const void* plan,
                                                  int64_t plan_bytes, int32_t batch, const void* q,
                                                  int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                                                  int32_t out_dtype, void* workspace, int64_t workspace_bytes,
                                                  uint32_t flags, int32_t* dev_status, mg_stream_t stream);

/* Standalone block gather + dequantize (the batched read_fp32 of
 * metagross/cache.py:74-85): for each sequence b, its committed pages in
 * block-table order, then (include_staging != 0) the exact staged tail, are
 * written to out_k/out_v [total_tokens, Hkv, D] (out_dtype) starting at row
 * cu_seqlens[b].  cu_seqlens[b+1] - cu_seqlens[b] must equal the tokens
 * written for b. */
MG_API mg_status mg_gather_dequant(const mg_cache_layout* layout, const mg_layer_ptrs* layer,
                            const int32_t* block_tables, const int32_t* seq_lens,
                            const int32_t* cu_seqlens, int32_t batch, int32_t max_context,
                            int32_t include_staging, void* out_k, void* out_v, int32_t out_dtype,
                            int32_t* dev_status, mg_stream_t stream);

/* Free every page of the listed sequences back to the allocator (pages in
 * block-table order, sequences in list order -- the order in which the
 * reference's BlockAllocator.free would be called) and set their seq_lens to
 * 0.  A page already free sets MG_DEV_DOUBLE_FREE and is skipped. */
MG_API mg_status mg_free_sequences(const mg_allocator* alloc, const int32_t* block_tables,
                                   int32_t max_blocks, int32_t* seq_lens, int32_t batch,
                                   const int32_t* seq_ids, int32_t num_seqs, int32_t page_size,
                                   int32_t* dev_status, mg_stream_t stream);

/* Truncate the listed sequences to new_lens (in list order): pages at
 * logical index >= new_len/page_size go back to the allocator in block-table
 * order.  A new length must not cut a committed page in two (new_len %
 * page_size == 0, or new_len >= the sequence's committed tokens); such a
 * request sets MG_DEV_BAD_ARGUMENT and leaves that sequence unchanged.
 * mg_free_sequences is truncation to 0. */
MG_API mg_status mg_truncate_sequences(const mg_allocator* alloc, const int32_t* block_tables,
                                       int32_t max_blocks, int32_t* seq_lens, int32_t batch,
                                       const int32_t* seq_ids, const int32_t* new_lens,
                                       int32_t num_seqs, int32_t page_size, int32_t* dev_status,
                                       mg_stream_t stream);

/* ------------------------------------------------------------------------
 * Dense-side helpers of a Llama decode step (fp16 storage, fp32 math).  No
 * counterpart among the reference's ops: they stand for the reference model's
 * Hugging Face modules (LlamaRMSNorm, the rotate-half rotary embedding of
 * metagross/generate_llama.py:20-37, the SiLU-gated MLP) in the batched decode
 * loop, one launch each instead of chains of small torch kernels.
 * ---------------------------------------------------------------------- */

/* y[r, :] = fp16(x[r, :] * rsqrt(mean(x[r, :]^2) + eps)) * w, rows x cols. */
MG_API mg_status mg_rmsnorm_f16(const void* x, const void* w, void* y, int64_t rows, int64_t cols, float eps,
                                mg_stream_t stream);

/* qkv [batch, (Hq + 2 Hkv) * D] (q | k | v heads) -> q [batch, Hq, D] and
 * k [batch, Hkv, D] rotated at position pos[b] by the tables cos / sin
 * [positions, D / 2] (pairs d, d + D/2), v [batch, Hkv, D] copied. */
MG_API mg_status mg_rope_qkv_f16(const void* qkv, const int64_t* pos, const float* cos_table,
                                 const float* sin_table, void* q, void* k, void* v, int32_t batch,
                                 int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, mg_stream_t stream);

/* h[r, j] = fp16(silu(gu[r, j])) * gu[r, ffn + j], gu [rows, 2 ffn]. */
MG_API mg_status mg_silu_mul_f16(const void* gu, void* h, int64_t rows, int64_t ffn, mg_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* METAGROSS_B200_H */
