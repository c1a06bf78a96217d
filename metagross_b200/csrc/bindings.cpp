// metagross_b200._C -- the reference's op surface (csrc/bindings.cpp:3-19:
// add, quantize_new_scale, quantize_fixed_scale, dequantize_page,
// paged_attention_committed, quantize_int4_new_scale, dequantize_int4_page)
// with the same names, argument meaning and RuntimeError behaviour
// (TORCH_CHECK), plus the batched device-resident ops.  This file only
// validates and unpacks tensors; all device work goes through the C ABI of
// libmgb200.so (include/metagross_b200.h) on the current CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <limits>
#include <tuple>

#include "metagross_b200.h"

namespace {

mg_stream_t cur_stream() { return reinterpret_cast<mg_stream_t>(at::cuda::getCurrentCUDAStream().stream()); }

void check_status(mg_status s, const char* what) {
    TORCH_CHECK(s == MG_OK, what, ": ", mg_last_error());
}

int32_t* status_ptr(const c10::optional<torch::Tensor>& st) {
    if (!st.has_value() || !st->defined()) return nullptr;
    TORCH_CHECK(st->is_cuda() && st->scalar_type() == torch::kInt32 && st->numel() >= 1,
                "status must be a CUDA int32 tensor with at least one element");
    return st->data_ptr<int32_t>();
}

// ---------------------------------------------------------------------------
// reference op surface
// ---------------------------------------------------------------------------

torch::Tensor add(torch::Tensor a, torch::Tensor b) {
    TORCH_CHECK(a.is_cuda(), "a must be a CUDA tensor");
    TORCH_CHECK(b.is_cuda(), "b must be a CUDA tensor");
    TORCH_CHECK(a.sizes() == b.sizes(), "a and b must have the same shape");
    TORCH_CHECK(a.scalar_type() == torch::kFloat32, "a must be float32");
    TORCH_CHECK(b.scalar_type() == torch::kFloat32, "b must be float32");
    const c10::cuda::CUDAGuard guard(a.device());
    auto ac = a.contiguous(), bc = b.contiguous();
    auto out = torch::empty_like(ac);
    check_status(mg_add_f32(ac.data_ptr<float>(), bc.data_ptr<float>(), out.data_ptr<float>(), ac.numel(),
                            cur_stream()),
                 "add");
    return out;
}

void check_quant_common(const torch::Tensor& in, const torch::Tensor& page, int64_t off, bool int4) {
    TORCH_CHECK(in.is_cuda() && page.is_cuda(), "inputs must be CUDA tensors");
    TORCH_CHECK(in.scalar_type() == torch::kFloat32, "input must be float32");
    if (int4) {
        TORCH_CHECK(page.scalar_type() == torch::kUInt8, "packed_storage must be uint8");
    } else {
        TORCH_CHECK(page.scalar_type() == torch::kInt8, "page_storage must be int8");
    }
    TORCH_CHECK(in.dim() == 3, "input must be [num_tokens, num_heads, head_dim], got ", in.dim(), "-D");
    TORCH_CHECK(page.dim() == 3, int4 ? "packed_storage must be [page_size, num_heads, head_dim/2], got "
                                      : "page_storage must be [page_size, num_heads, head_dim], got ",
                page.dim(), "-D");
    TORCH_CHECK(page.is_contiguous(), int4 ? "packed_storage must be contiguous" : "page_storage must be contiguous");
    TORCH_CHECK(off >= 0, "token_offset_in_page must be >= 0, got ", off);
}

double quantize_new_scale(torch::Tensor input, torch::Tensor page, int64_t off) {
    check_quant_common(input, page, off, false);
    const c10::cuda::CUDAGuard guard(page.device());
    auto x = input.contiguous();
    TORCH_CHECK(x.size(1) == page.size(1), "input and page_storage must have the same num_heads, got ", x.size(1),
                " and ", page.size(1));
    TORCH_CHECK(x.size(2) == page.size(2), "input and page_storage must have the same head_dim, got ", x.size(2),
                " and ", page.size(2));
    TORCH_CHECK(off + x.size(0) <= page.size(0), "quantize_new_scale: write would overflow the page (offset=", off,
                ", num_tokens=", x.size(0), ", page_size=", page.size(0), ")");
    if (x.numel() == 0) return 1e-8;
    auto scale = torch::empty({1}, x.options().dtype(torch::kFloat64));
    check_status(mg_quantize_int8_new_scale(x.data_ptr<float>(), x.size(0), x.size(1) * x.size(2),
                                            page.data_ptr<int8_t>(), page.size(0), off, scale.data_ptr<double>(),
                                            cur_stream()),
                 "quantize_new_scale");
    return scale.item<double>();  // the reference returns the scale to Python too (a device->host copy)
}

void quantize_fixed_scale(torch::Tensor input, torch::Tensor page, int64_t off, double scale) {
    check_quant_common(input, page, off, false);
    TORCH_CHECK(std::isfinite(scale) && scale > 0.0, "scale must be a positive finite number, got ", scale);
    const c10::cuda::CUDAGuard guard(page.device());
    auto x = input.contiguous();
    TORCH_CHECK(x.size(1) == page.size(1), "input and page_storage must have the same num_heads, got ", x.size(1),
                " and ", page.size(1));
    TORCH_CHECK(x.size(2) == page.size(2), "input and page_storage must have the same head_dim, got ", x.size(2),
                " and ", page.size(2));
    TORCH_CHECK(off + x.size(0) <= page.size(0), "quantize_fixed_scale: write would overflow the page (offset=", off,
                ", num_tokens=", x.size(0), ", page_size=", page.size(0), ")");
    if (x.numel() == 0) return;
    check_status(mg_quantize_int8_fixed_scale(x.data_ptr<float>(), x.size(0), x.size(1) * x.size(2),
                                              page.data_ptr<int8_t>(), page.size(0), off, scale, cur_stream()),
                 "quantize_fixed_scale");
}

void check_deq_common(const torch::Tensor& page, int64_t off, int64_t n, double scale, bool int4) {
    TORCH_CHECK(page.is_cuda(), int4 ? "packed_storage must be a CUDA tensor" : "page_storage must be a CUDA tensor");
    if (int4) {
        TORCH_CHECK(page.scalar_type() == torch::kUInt8, "packed_storage must be uint8");
    } else {
        TORCH_CHECK(page.scalar_type() == torch::kInt8, "page_storage must be int8");
    }
    TORCH_CHECK(page.dim() == 3, int4 ? "packed_storage must be [page_size, num_heads, head_dim/2], got "
                                      : "page_storage must be [page_size, num_heads, head_dim], got ",
                page.dim(), "-D");
    TORCH_CHECK(page.is_contiguous(), int4 ? "packed_storage must be contiguous" : "page_storage must be contiguous");
    TORCH_CHECK(off >= 0, "token_offset_in_page must be >= 0, got ", off);
    TORCH_CHECK(n >= 0, "num_tokens must be >= 0, got ", n);
    TORCH_CHECK(std::isfinite(scale) && scale > 0.0, "scale must be a positive finite number, got ", scale);
    TORCH_CHECK(off + n <= page.size(0), "dequantize: read would overflow the page (offset=", off,
                ", num_tokens=", n, ", page_size=", page.size(0), ")");
}

torch::Tensor dequantize_page(torch::Tensor page, int64_t off, int64_t n, double scale) {
    check_deq_common(page, off, n, scale, false);
    const c10::cuda::CUDAGuard guard(page.device());
    auto out = torch::empty({n, page.size(1), page.size(2)}, page.options().dtype(torch::kFloat32));
    if (out.numel() == 0) return out;
    check_status(mg_dequantize_int8_page(page.data_ptr<int8_t>(), page.size(0), page.size(1) * page.size(2), off, n,
                                         scale, out.data_ptr<float>(), cur_stream()),
                 "dequantize_page");
    return out;
}

double quantize_int4_new_scale(torch::Tensor input, torch::Tensor packed, int64_t off) {
    check_quant_common(input, packed, off, true);
    TORCH_CHECK(input.size(2) > 0, "head_dim must be positive, got ", input.size(2));
    TORCH_CHECK(input.size(2) % 2 == 0, "head_dim must be even for INT4 packing, got ", input.size(2));
    const c10::cuda::CUDAGuard guard(packed.device());
    auto x = input.contiguous();
    TORCH_CHECK(x.size(1) == packed.size(1), "input and packed_storage must have the same num_heads, got ",
                x.size(1), " and ", packed.size(1));
    TORCH_CHECK(packed.size(2) == x.size(2) / 2,
                "packed_storage's packed head_dim must be input's head_dim / 2, got ", packed.size(2),
                " for head_dim=", x.size(2));
    TORCH_CHECK(off + x.size(0) <= packed.size(0), "quantize_int4_new_scale: write would overflow the page (offset=",
                off, ", num_tokens=", x.size(0), ", page_size=", packed.size(0), ")");
    if (x.numel() == 0) return 1e-8;
    auto scale = torch::empty({1}, x.options().dtype(torch::kFloat64));
    check_status(mg_quantize_int4_new_scale(x.data_ptr<float>(), x.size(0), x.size(1), x.size(2),
                                            packed.data_ptr<uint8_t>(), packed.size(0), off, scale.data_ptr<double>(),
                                            cur_stream()),
                 "quantize_int4_new_scale");
    return scale.item<double>();
}

torch::Tensor dequantize_int4_page(torch::Tensor packed, int64_t off, int64_t n, double scale) {
    check_deq_common(packed, off, n, scale, true);
    const c10::cuda::CUDAGuard guard(packed.device());
    auto out = torch::empty({n, packed.size(1), packed.size(2) * 2}, packed.options().dtype(torch::kFloat32));
    if (out.numel() == 0) return out;
    check_status(mg_dequantize_int4_page(packed.data_ptr<uint8_t>(), packed.size(0), packed.size(1) * packed.size(2),
                                         off, n, scale, out.data_ptr<float>(), cur_stream()),
                 "dequantize_int4_page");
    return out;
}

// Limits the reference's committed-page kernel rejects (csrc/paged_attention.cu:11-16);
// kept on this entry point so that callers see the same errors.  The
// reference's 4096-token cap is lifted: the split kernel has no length limit.
constexpr int64_t kRefHeadDim = 64;
constexpr int64_t kRefMaxPageSize = 64;

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> paged_attention_committed(
    torch::Tensor query, torch::Tensor k_storage, torch::Tensor v_storage, torch::Tensor page_scales_k,
    torch::Tensor page_scales_v, torch::Tensor block_table, double scale) {
    TORCH_CHECK(query.is_cuda() && k_storage.is_cuda() && v_storage.is_cuda(), "all inputs must be CUDA tensors");
    TORCH_CHECK(page_scales_k.is_cuda() && page_scales_v.is_cuda() && block_table.is_cuda(),
                "page_scales_k/v and block_table must be CUDA tensors");
    TORCH_CHECK(query.scalar_type() == torch::kFloat32, "query must be float32");
    TORCH_CHECK(k_storage.scalar_type() == torch::kInt8 && v_storage.scalar_type() == torch::kInt8,
                "k_storage/v_storage must be int8");
    TORCH_CHECK(page_scales_k.scalar_type() == torch::kFloat32 && page_scales_v.scalar_type() == torch::kFloat32,
                "page_scales_k/v must be float32");
    TORCH_CHECK(block_table.scalar_type() == torch::kInt32, "block_table must be int32");
    TORCH_CHECK(query.dim() == 2, "query must be 2-D [num_q_heads, head_dim], got ", query.dim(), "-D");
    TORCH_CHECK(k_storage.dim() == 4, "k_storage must be 4-D [max_pages, page_size, num_kv_heads, head_dim], got ",
                k_storage.dim(), "-D");
    TORCH_CHECK(v_storage.dim() == 4, "v_storage must be 4-D [max_pages, page_size, num_kv_heads, head_dim], got ",
                v_storage.dim(), "-D");
    TORCH_CHECK(block_table.dim() == 1, "block_table must be 1-D [num_committed_pages], got ", block_table.dim(), "-D");
    TORCH_CHECK(page_scales_k.dim() == 1 && page_scales_v.dim() == 1, "page_scales_k/v must be 1-D [max_pages]");
    TORCH_CHECK(k_storage.is_contiguous(), "k_storage must be contiguous");
    TORCH_CHECK(v_storage.is_contiguous(), "v_storage must be contiguous");
    const c10::cuda::CUDAGuard guard(query.device());
    auto q = query.contiguous();
    auto bt = block_table.contiguous();
    auto sk = page_scales_k.contiguous();
    auto sv = page_scales_v.contiguous();
    const int64_t max_pages = k_storage.size(0);
    TORCH_CHECK(v_storage.size(0) == max_pages,
                "k_storage and v_storage must have the same number of physical pages, got ", max_pages, " and ",
                v_storage.size(0));
    TORCH_CHECK(sk.size(0) == max_pages && sv.size(0) == max_pages, "page_scales_k/v must have length max_pages=",
                max_pages, ", got ", sk.size(0), " and ", sv.size(0));
    const int64_t P = k_storage.size(1);
    TORCH_CHECK(P > 0, "page_size must be positive, got ", P);
    TORCH_CHECK(v_storage.size(1) == P, "k_storage and v_storage must have the same page_size, got ", P, " and ",
                v_storage.size(1));
    TORCH_CHECK(P <= kRefMaxPageSize, "page_size (", P, ") exceeds the maximum supported page_size (",
                kRefMaxPageSize, ")");
    TORCH_CHECK(q.size(1) == kRefHeadDim, "this op supports head_dim=", kRefHeadDim, ", got ", q.size(1));
    TORCH_CHECK(k_storage.size(3) == kRefHeadDim && v_storage.size(3) == kRefHeadDim,
                "k_storage/v_storage head_dim must also be ", kRefHeadDim);
    TORCH_CHECK(k_storage.size(2) == v_storage.size(2), "k_storage and v_storage must have the same num_kv_heads");
    const int64_t Hq = q.size(0), Hkv = k_storage.size(2), D = q.size(1), nb = bt.size(0);
    TORCH_CHECK(Hkv > 0 && Hq % Hkv == 0, "num_q_heads (", Hq, ") must be an exact multiple of num_kv_heads (", Hkv,
                ") for grouped-query attention -- got a non-integer group size");
    TORCH_CHECK(std::isfinite(scale), "attention scale must be finite, got ", scale);
    TORCH_CHECK(scale > 0.0, "attention scale must be positive, got ", scale);
    if (nb > 0) {
        // same host-side range check as the reference (a device->host copy)
        auto host = bt.to(torch::kCPU);
        auto acc = host.accessor<int32_t, 1>();
        for (int64_t i = 0; i < nb; ++i) {
            const int32_t p = acc[i];
            TORCH_CHECK(p >= 0 && p < max_pages, "block_table[", i, "] = ", p, " is out of range for max_pages=",
                        max_pages);
        }
    }
    auto wv = torch::empty({Hq, D}, q.options());
    auto l = torch::empty({Hq}, q.options());
    auto m = torch::empty({Hq}, q.options());
    const int64_t wsb = mg_paged_attention_committed_workspace_bytes(nb, P, Hq, Hkv, D);
    torch::Tensor ws;
    if (wsb > 0) ws = torch::zeros({wsb}, q.options().dtype(torch::kUInt8));
    check_status(mg_paged_attention_committed(q.data_ptr<float>(), k_storage.data_ptr<int8_t>(),
                                              v_storage.data_ptr<int8_t>(), sk.data_ptr<float>(), sv.data_ptr<float>(),
                                              bt.data_ptr<int32_t>(), nb, max_pages, P, Hq, Hkv, D, scale,
                                              wv.data_ptr<float>(), l.data_ptr<float>(), m.data_ptr<float>(),
                                              wsb > 0 ? ws.data_ptr() : nullptr, wsb, nullptr, cur_stream()),
                 "paged_attention_committed");
    return {wv, l, m};
}

// ---------------------------------------------------------------------------
// batched device-resident ops
// ---------------------------------------------------------------------------

int32_t float_code(const torch::Tensor& t, const char* what) {
    if (t.scalar_type() == torch::kFloat16) return MG_F16;
    TORCH_CHECK(t.scalar_type() == torch::kFloat32, what, " must be float16 or float32");
    return MG_F32;
}

struct Pools {
    mg_cache_layout L;
    mg_layer_ptrs ptrs;
};

// k_pool/v_pool [N, P, Hkv, D] int8 or [N, P, Hkv, D/2] uint8; scales [N]
// fp32; staging [B, P, Hkv, D] (optional: undefined tensors = no staging).
Pools make_pools(const torch::Tensor& k_pool, const torch::Tensor& v_pool, const torch::Tensor& k_scales,
                 const torch::Tensor& v_scales, const c10::optional<torch::Tensor>& staging_k,
                 const c10::optional<torch::Tensor>& staging_v, const torch::Tensor& block_tables) {
    TORCH_CHECK(k_pool.is_cuda() && v_pool.is_cuda() && k_scales.is_cuda() && v_scales.is_cuda(),
                "pools and scales must be CUDA tensors");
    TORCH_CHECK(k_pool.dim() == 4 && v_pool.sizes() == k_pool.sizes(), "k_pool/v_pool must be 4-D and equal-shaped");
    TORCH_CHECK(k_pool.is_contiguous() && v_pool.is_contiguous(), "pools must be contiguous");
    const bool i4 = k_pool.scalar_type() == torch::kUInt8;
    TORCH_CHECK(i4 || k_pool.scalar_type() == torch::kInt8, "pools must be int8 (INT8) or uint8 (packed INT4)");
    TORCH_CHECK(v_pool.scalar_type() == k_pool.scalar_type(), "k_pool and v_pool dtypes differ");
    // scales [N]: one per page (the reference's layout); [N, P, Hkv]: one per token and kv head
    const bool th = k_scales.dim() == 3;
    TORCH_CHECK(k_scales.scalar_type() == torch::kFloat32 && v_scales.scalar_type() == torch::kFloat32 &&
                    k_scales.is_contiguous() && v_scales.is_contiguous() && v_scales.sizes() == k_scales.sizes() &&
                    (th ? (k_scales.size(0) == k_pool.size(0) && k_scales.size(1) == k_pool.size(1) &&
                           k_scales.size(2) == k_pool.size(2))
                        : (k_scales.dim() == 1 && k_scales.size(0) == k_pool.size(0))),
                "k_scales/v_scales must be contiguous float32 [num_pages] or [num_pages, page_size, num_kv_heads]");
    TORCH_CHECK(block_tables.is_cuda() && block_tables.scalar_type() == torch::kInt32 && block_tables.dim() == 2 &&
                    block_tables.is_contiguous(),
                "block_tables must be a contiguous CUDA int32 [batch, max_blocks] tensor");
    Pools p{};
    p.L.kv_dtype = i4 ? MG_KV_INT4 : MG_KV_INT8;
    p.L.page_size = static_cast<int32_t>(k_pool.size(1));
    p.L.num_kv_heads = static_cast<int32_t>(k_pool.size(2));
    p.L.head_dim = static_cast<int32_t>(i4 ? k_pool.size(3) * 2 : k_pool.size(3));
    p.L.max_blocks = static_cast<int32_t>(block_tables.size(1));
    p.L.num_pages = k_pool.size(0);
    p.L.scale_layout = th ? MG_SCALE_TOKEN_HEAD : MG_SCALE_PAGE;
    p.L.staging_dtype = MG_F32;
    p.ptrs.k_pool = k_pool.data_ptr();
    p.ptrs.v_pool = v_pool.data_ptr();
    p.ptrs.k_scales = k_scales.data_ptr<float>();
    p.ptrs.v_scales = v_scales.data_ptr<float>();
    const bool has_st = staging_k.has_value() && staging_k->defined();
    if (has_st) {
        TORCH_CHECK(staging_v.has_value() && staging_v->defined(), "staging_k and staging_v go together");
        const auto& sk = *staging_k;
        const auto& sv = *staging_v;
        TORCH_CHECK(sk.is_cuda() && sk.is_contiguous() && sv.is_contiguous() && sk.sizes() == sv.sizes() &&
                        sk.scalar_type() == sv.scalar_type(),
                    "staging_k/staging_v must be equal contiguous CUDA tensors");
        TORCH_CHECK(sk.dim() == 4 && sk.size(1) == p.L.page_size && sk.size(2) == p.L.num_kv_heads &&
                        sk.size(3) == p.L.head_dim && sk.size(0) >= block_tables.size(0),
                    "staging must be [batch, page_size, num_kv_heads, head_dim]");
        p.L.staging_dtype = float_code(sk, "staging");
        p.ptrs.staging_k = sk.data_ptr();
        p.ptrs.staging_v = sv.data_ptr();
    }
    return p;
}

void check_i32_vec(const torch::Tensor& t, int64_t n, const char* what) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kInt32 && t.is_contiguous() && t.numel() >= n, what,
                " must be a contiguous CUDA int32 tensor with >= ", n, " elements");
}

mg_allocator make_alloc(torch::Tensor free_stack, torch::Tensor n_free, torch::Tensor in_use) {
    check_i32_vec(free_stack, 1, "free_stack");
    check_i32_vec(n_free, 1, "n_free");
    check_i32_vec(in_use, free_stack.numel(), "in_use");
    mg_allocator a;
    a.free_stack = free_stack.data_ptr<int32_t>();
    a.n_free = n_free.data_ptr<int32_t>();
    a.in_use = in_use.data_ptr<int32_t>();
    a.num_pages = free_stack.numel();
    return a;
}

void alloc_init(torch::Tensor free_stack, torch::Tensor n_free, torch::Tensor in_use) {
    const c10::cuda::CUDAGuard guard(free_stack.device());
    auto a = make_alloc(free_stack, n_free, in_use);
    check_status(mg_alloc_init(&a, cur_stream()), "alloc_init");
}

void plan_append(torch::Tensor free_stack, torch::Tensor n_free, torch::Tensor in_use, torch::Tensor block_tables,
                 torch::Tensor seq_lens, torch::Tensor n_new, int64_t page_size,
                 c10::optional<torch::Tensor> status) {
    const c10::cuda::CUDAGuard guard(free_stack.device());
    auto a = make_alloc(free_stack, n_free, in_use);
    TORCH_CHECK(block_tables.dim() == 2, "block_tables must be [batch, max_blocks]");
    const int64_t B = block_tables.size(0);
    check_i32_vec(block_tables, 1, "block_tables");
    check_i32_vec(seq_lens, B, "seq_lens");
    check_i32_vec(n_new, B, "n_new");
    check_status(mg_plan_append(&a, block_tables.data_ptr<int32_t>(), static_cast<int32_t>(block_tables.size(1)),
                                seq_lens.data_ptr<int32_t>(), n_new.data_ptr<int32_t>(), static_cast<int32_t>(B),
                                static_cast<int32_t>(page_size), status_ptr(status), cur_stream()),
                 "plan_append");
}

void free_sequences(torch::Tensor free_stack, torch::Tensor n_free, torch::Tensor in_use, torch::Tensor block_tables,
                    torch::Tensor seq_lens, torch::Tensor seq_ids, int64_t page_size,
                    c10::optional<torch::Tensor> status) {
    const c10::cuda::CUDAGuard guard(free_stack.device());
    auto a = make_alloc(free_stack, n_free, in_use);
    check_i32_vec(block_tables, 1, "block_tables");
    check_i32_vec(seq_lens, block_tables.size(0), "seq_lens");
    check_i32_vec(seq_ids, 0, "seq_ids");
    check_status(mg_free_sequences(&a, block_tables.data_ptr<int32_t>(), static_cast<int32_t>(block_tables.size(1)),
                                   seq_lens.data_ptr<int32_t>(), static_cast<int32_t>(block_tables.size(0)),
                                   seq_ids.data_ptr<int32_t>(),
                                   static_cast<int32_t>(seq_ids.numel()), static_cast<int32_t>(page_size),
                                   status_ptr(status), cur_stream()),
                 "free_sequences");
}

void kv_append(torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor k_scales, torch::Tensor v_scales,
               torch::Tensor staging_k, torch::Tensor staging_v, torch::Tensor block_tables, torch::Tensor seq_lens,
               torch::Tensor n_new, torch::Tensor k_new, torch::Tensor v_new, c10::optional<torch::Tensor> status,
               bool early_launch) {
    const c10::cuda::CUDAGuard guard(k_pool.device());
    auto p = make_pools(k_pool, v_pool, k_scales, v_scales, staging_k, staging_v, block_tables);
    const int64_t B = block_tables.size(0);
    check_i32_vec(seq_lens, B, "seq_lens");
    check_i32_vec(n_new, B, "n_new");
    TORCH_CHECK(k_new.is_cuda() && k_new.dim() == 4 && k_new.sizes() == v_new.sizes() &&
                    k_new.scalar_type() == v_new.scalar_type(),
                "k_new/v_new must be equal CUDA tensors [batch, max_new, num_kv_heads, head_dim]");
    TORCH_CHECK(k_new.size(0) == B && k_new.size(2) == p.L.num_kv_heads && k_new.size(3) == p.L.head_dim,
                "k_new shape does not match the cache");
    auto kn = k_new.contiguous(), vn = v_new.contiguous();
    check_status(mg_kv_append_flags(&p.L, &p.ptrs, block_tables.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                                    n_new.data_ptr<int32_t>(), static_cast<int32_t>(B), kn.data_ptr(), vn.data_ptr(),
                                    float_code(kn, "k_new"), static_cast<int32_t>(kn.size(1)),
                                    early_launch ? MG_APPEND_EARLY_LAUNCH : 0u, status_ptr(status), cur_stream()),
                 "kv_append");
}

void kv_append_rope(torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor k_scales, torch::Tensor v_scales,
                    torch::Tensor staging_k, torch::Tensor staging_v, torch::Tensor block_tables,
                    torch::Tensor seq_lens, torch::Tensor n_new, torch::Tensor qkv, int64_t num_q_heads,
                    torch::Tensor cos_table, torch::Tensor sin_table, torch::Tensor q_out,
                    c10::optional<torch::Tensor> status) {
    const c10::cuda::CUDAGuard guard(k_pool.device());
    auto p = make_pools(k_pool, v_pool, k_scales, v_scales, staging_k, staging_v, block_tables);
    const int64_t B = block_tables.size(0);
    check_i32_vec(seq_lens, B, "seq_lens");
    check_i32_vec(n_new, B, "n_new");
    const int64_t D = p.L.head_dim, hkv = p.L.num_kv_heads;
    TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == torch::kHalf && qkv.dim() == 3 && qkv.size(0) == B &&
                    qkv.size(2) == (num_q_heads + 2 * hkv) * D && qkv.is_contiguous(),
                "qkv must be a contiguous fp16 CUDA tensor [batch, max_new, (num_q_heads + 2 num_kv_heads) * head_dim]");
    TORCH_CHECK(cos_table.is_cuda() && sin_table.is_cuda() && cos_table.scalar_type() == torch::kFloat32 &&
                    sin_table.scalar_type() == torch::kFloat32 && cos_table.dim() == 2 &&
                    cos_table.sizes() == sin_table.sizes() && cos_table.size(1) == D / 2 &&
                    cos_table.is_contiguous() && sin_table.is_contiguous(),
                "cos/sin tables must be contiguous fp32 CUDA tensors [positions, head_dim / 2]");
    TORCH_CHECK(q_out.is_cuda() && q_out.scalar_type() == torch::kHalf && q_out.is_contiguous() &&
                    q_out.numel() == B * qkv.size(1) * num_q_heads * D,
                "q_out must be a contiguous fp16 CUDA tensor of batch x max_new x num_q_heads x head_dim elements");
    check_status(mg_kv_append_rope(&p.L, &p.ptrs, block_tables.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                                   n_new.data_ptr<int32_t>(), static_cast<int32_t>(B), qkv.data_ptr(),
                                   static_cast<int32_t>(num_q_heads), cos_table.data_ptr<float>(),
                                   sin_table.data_ptr<float>(), static_cast<int32_t>(cos_table.size(0)),
                                   q_out.data_ptr(), static_cast<int32_t>(qkv.size(1)), status_ptr(status),
                                   cur_stream()),
                 "kv_append_rope");
}

void truncate_sequences(torch::Tensor free_stack, torch::Tensor n_free, torch::Tensor in_use,
                        torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor seq_ids,
                        torch::Tensor new_lens, int64_t page_size, c10::optional<torch::Tensor> status) {
    const c10::cuda::CUDAGuard guard(free_stack.device());
    auto a = make_alloc(free_stack, n_free, in_use);
    check_i32_vec(block_tables, 1, "block_tables");
    check_i32_vec(seq_lens, block_tables.size(0), "seq_lens");
    check_i32_vec(seq_ids, 0, "seq_ids");
    check_i32_vec(new_lens, seq_ids.numel(), "new_lens");
    check_status(mg_truncate_sequences(&a, block_tables.data_ptr<int32_t>(),
                                       static_cast<int32_t>(block_tables.size(1)), seq_lens.data_ptr<int32_t>(),
                                       static_cast<int32_t>(block_tables.size(0)), seq_ids.data_ptr<int32_t>(),
                                       new_lens.data_ptr<int32_t>(), static_cast<int32_t>(seq_ids.numel()),
                                       static_cast<int32_t>(page_size), status_ptr(status), cur_stream()),
                 "truncate_sequences");
}

int64_t decode_workspace_bytes(torch::Tensor k_pool, torch::Tensor block_tables, int64_t num_q_heads,
                               int64_t max_context) {
    mg_cache_layout L{};
    const bool i4 = k_pool.scalar_type() == torch::kUInt8;
    L.kv_dtype = i4 ? MG_KV_INT4 : MG_KV_INT8;
    L.staging_dtype = MG_F16;
    L.page_size = static_cast<int32_t>(k_pool.size(1));
    L.num_kv_heads = static_cast<int32_t>(k_pool.size(2));
    L.head_dim = static_cast<int32_t>(i4 ? k_pool.size(3) * 2 : k_pool.size(3));
    L.max_blocks = static_cast<int32_t>(block_tables.size(1));
    L.num_pages = k_pool.size(0);
    return mg_paged_decode_workspace_bytes(&L, static_cast<int32_t>(block_tables.size(0)),
                                           static_cast<int32_t>(num_q_heads), static_cast<int32_t>(max_context));
}

void paged_decode_attention(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor k_scales,
                            torch::Tensor v_scales, c10::optional<torch::Tensor> staging_k,
                            c10::optional<torch::Tensor> staging_v, torch::Tensor block_tables, torch::Tensor seq_lens,
                            double scale, int64_t max_context, torch::Tensor workspace, torch::Tensor out,
                            c10::optional<torch::Tensor> status) {
    const c10::cuda::CUDAGuard guard(q.device());
    auto p = make_pools(k_pool, v_pool, k_scales, v_scales, staging_k, staging_v, block_tables);
    const int64_t B = block_tables.size(0);
    check_i32_vec(seq_lens, B, "seq_lens");
    TORCH_CHECK(q.is_cuda() && q.dim() == 3 && q.size(0) == B && q.size(2) == p.L.head_dim && q.is_contiguous(),
                "q must be a contiguous CUDA tensor [batch, num_q_heads, head_dim]");
    TORCH_CHECK(out.is_cuda() && out.sizes() == q.sizes() && out.is_contiguous(),
                "out must be a contiguous CUDA tensor shaped like q");
    TORCH_CHECK(std::isfinite(scale) && scale > 0.0, "attention scale must be positive and finite, got ", scale);
    TORCH_CHECK(workspace.is_cuda() && workspace.is_contiguous(), "workspace must be a contiguous CUDA tensor");
    check_status(mg_paged_decode_attention(&p.L, &p.ptrs, block_tables.data_ptr<int32_t>(),
                                           seq_lens.data_ptr<int32_t>(), static_cast<int32_t>(B), q.data_ptr(),
                                           float_code(q, "q"), static_cast<int32_t>(q.size(1)),
                                           static_cast<float>(scale), out.data_ptr(), float_code(out, "out"),
                                           static_cast<int32_t>(max_context),
                                           workspace.numel() > 0 ? workspace.data_ptr() : nullptr,
                                           workspace.numel() * workspace.element_size(), status_ptr(status),
                                           cur_stream()),
                 "paged_decode_attention");
}

int64_t decode_plan_bytes(int64_t batch) { return mg_paged_decode_plan_bytes(static_cast<int32_t>(batch)); }

// Build the step's decode plan from seq_lens into `plan` (uint8 CUDA tensor of
// decode_plan_bytes(batch) bytes).  k_pool / block_tables give the layout.
void decode_plan(torch::Tensor k_pool, torch::Tensor block_tables, torch::Tensor seq_lens, bool with_staging,
                 torch::Tensor plan, c10::optional<torch::Tensor> status) {
    const c10::cuda::CUDAGuard guard(seq_lens.device());
    TORCH_CHECK(k_pool.is_cuda() && k_pool.dim() == 4, "k_pool must be a 4-D CUDA tensor");
    check_i32_vec(block_tables, 1, "block_tables");
    TORCH_CHECK(block_tables.dim() == 2, "block_tables must be [batch, max_blocks]");
    const int64_t B = block_tables.size(0);
    check_i32_vec(seq_lens, B, "seq_lens");
    TORCH_CHECK(plan.is_cuda() && plan.is_contiguous() && plan.scalar_type() == torch::kUInt8,
                "plan must be a contiguous CUDA uint8 tensor");
    mg_cache_layout L{};
    const bool i4 = k_pool.scalar_type() == torch::kUInt8;
    L.kv_dtype = i4 ? MG_KV_INT4 : MG_KV_INT8;
    L.staging_dtype = MG_F16;
    L.page_size = static_cast<int32_t>(k_pool.size(1));
    L.num_kv_heads = static_cast<int32_t>(k_pool.size(2));
    L.head_dim = static_cast<int32_t>(i4 ? k_pool.size(3) * 2 : k_pool.size(3));
    L.max_blocks = static_cast<int32_t>(block_tables.size(1));
    L.num_pages = k_pool.size(0);
    check_status(mg_paged_decode_plan(&L, block_tables.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                                      static_cast<int32_t>(B), with_staging ? 1 : 0,
                                      plan.data_ptr(), plan.numel(), status_ptr(status), cur_stream()),
                 "decode_plan");
}

void plan_step(torch::Tensor free_stack, torch::Tensor n_free, torch::Tensor in_use, torch::Tensor k_pool,
               torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor n_new, bool with_staging,
               torch::Tensor plan, c10::optional<torch::Tensor> status) {
    const c10::cuda::CUDAGuard guard(free_stack.device());
    auto a = make_alloc(free_stack, n_free, in_use);
    TORCH_CHECK(k_pool.is_cuda() && k_pool.dim() == 4, "k_pool must be a 4-D CUDA tensor");
    check_i32_vec(block_tables, 1, "block_tables");
    TORCH_CHECK(block_tables.dim() == 2, "block_tables must be [batch, max_blocks]");
    const int64_t B = block_tables.size(0);
    check_i32_vec(seq_lens, B, "seq_lens");
    check_i32_vec(n_new, B, "n_new");
    TORCH_CHECK(plan.is_cuda() && plan.is_contiguous() && plan.scalar_type() == torch::kUInt8,
                "plan must be a contiguous CUDA uint8 tensor");
    mg_cache_layout L{};
    const bool i4 = k_pool.scalar_type() == torch::kUInt8;
    L.kv_dtype = i4 ? MG_KV_INT4 : MG_KV_INT8;
    L.staging_dtype = MG_F16;
    L.page_size = static_cast<int32_t>(k_pool.size(1));
    L.num_kv_heads = static_cast<int32_t>(k_pool.size(2));
    L.head_dim = static_cast<int32_t>(i4 ? k_pool.size(3) * 2 : k_pool.size(3));
    L.max_blocks = static_cast<int32_t>(block_tables.size(1));
    L.num_pages = k_pool.size(0);
    check_status(mg_plan_step(&a, &L, block_tables.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                              n_new.data_ptr<int32_t>(), static_cast<int32_t>(B), with_staging ? 1 : 0,
                              plan.data_ptr(), plan.numel(), status_ptr(status), cur_stream()),
                 "plan_step");
}

void paged_decode_attention_planned(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool,
                                    torch::Tensor k_scales, torch::Tensor v_scales,
                                    c10::optional<torch::Tensor> staging_k, c10::optional<torch::Tensor> staging_v,
                                    torch::Tensor block_tables, torch::Tensor plan, double scale,
                                    torch::Tensor workspace, torch::Tensor out, c10::optional<torch::Tensor> status,
                                    bool settled) {
    const c10::cuda::CUDAGuard guard(q.device());
    auto p = make_pools(k_pool, v_pool, k_scales, v_scales, staging_k, staging_v, block_tables);
    const int64_t B = block_tables.size(0);
    TORCH_CHECK(q.is_cuda() && q.dim() == 3 && q.size(0) == B && q.size(2) == p.L.head_dim && q.is_contiguous(),
                "q must be a contiguous CUDA tensor [batch, num_q_heads, head_dim]");
    TORCH_CHECK(out.is_cuda() && out.sizes() == q.sizes() && out.is_contiguous(),
                "out must be a contiguous CUDA tensor shaped like q");
    TORCH_CHECK(std::isfinite(scale) && scale > 0.0, "attention scale must be positive and finite, got ", scale);
    TORCH_CHECK(workspace.is_cuda() && workspace.is_contiguous(), "workspace must be a contiguous CUDA tensor");
    TORCH_CHECK(plan.is_cuda() && plan.is_contiguous() && plan.scalar_type() == torch::kUInt8,
                "plan must be a contiguous CUDA uint8 tensor");
    check_status(mg_paged_decode_attention_planned_flags(
                     &p.L, &p.ptrs, block_tables.data_ptr<int32_t>(), plan.data_ptr(), plan.numel(),
                     static_cast<int32_t>(B), q.data_ptr(), float_code(q, "q"), static_cast<int32_t>(q.size(1)),
                     static_cast<float>(scale), out.data_ptr(), float_code(out, "out"),
                     workspace.numel() > 0 ? workspace.data_ptr() : nullptr,
                     workspace.numel() * workspace.element_size(), settled ? MG_ATTN_PLAN_SETTLED : 0u,
                     status_ptr(status), cur_stream()),
                 "paged_decode_attention_planned");
}

void gather_dequant(torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor k_scales, torch::Tensor v_scales,
                    c10::optional<torch::Tensor> staging_k, c10::optional<torch::Tensor> staging_v,
                    torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor cu_seqlens, int64_t max_context,
                    torch::Tensor out_k, torch::Tensor out_v, c10::optional<torch::Tensor> status) {
    const c10::cuda::CUDAGuard guard(k_pool.device());
    auto p = make_pools(k_pool, v_pool, k_scales, v_scales, staging_k, staging_v, block_tables);
    const int64_t B = block_tables.size(0);
    check_i32_vec(seq_lens, B, "seq_lens");
    check_i32_vec(cu_seqlens, B + 1, "cu_seqlens");
    TORCH_CHECK(out_k.is_cuda() && out_k.is_contiguous() && out_v.is_contiguous() && out_k.sizes() == out_v.sizes() &&
                    out_k.scalar_type() == out_v.scalar_type() && out_k.dim() == 3 &&
                    out_k.size(1) == p.L.num_kv_heads && out_k.size(2) == p.L.head_dim,
                "out_k/out_v must be equal contiguous CUDA tensors [total_tokens, num_kv_heads, head_dim]");
    const bool with_st = staging_k.has_value() && staging_k->defined();
    check_status(mg_gather_dequant(&p.L, &p.ptrs, block_tables.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                                   cu_seqlens.data_ptr<int32_t>(), static_cast<int32_t>(B),
                                   static_cast<int32_t>(max_context), with_st ? 1 : 0, out_k.data_ptr(),
                                   out_v.data_ptr(), float_code(out_k, "out"), status_ptr(status), cur_stream()),
                 "gather_dequant");
}

}  // namespace

// ---------------------------------------------------------------------------
// dense-side helpers of a Llama decode step (fp16)
// ---------------------------------------------------------------------------

void check_f16_cuda(const torch::Tensor& t, const char* what) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat16 && t.is_contiguous(), what,
                " must be a contiguous CUDA float16 tensor");
}

torch::Tensor rmsnorm(torch::Tensor x, torch::Tensor w, double eps) {
    const c10::cuda::CUDAGuard guard(x.device());
    check_f16_cuda(x, "x");
    check_f16_cuda(w, "w");
    TORCH_CHECK(w.dim() == 1 && x.size(-1) == w.size(0), "w must be [x.shape[-1]]");
    auto y = torch::empty_like(x);
    const int64_t cols = x.size(-1);
    check_status(mg_rmsnorm_f16(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.numel() / cols, cols,
                                static_cast<float>(eps), cur_stream()),
                 "rmsnorm");
    return y;
}

void rope_qkv(torch::Tensor qkv, torch::Tensor pos, torch::Tensor cos_table, torch::Tensor sin_table,
              torch::Tensor q, torch::Tensor k, torch::Tensor v) {
    const c10::cuda::CUDAGuard guard(qkv.device());
    check_f16_cuda(qkv, "qkv");
    check_f16_cuda(q, "q");
    check_f16_cuda(k, "k");
    check_f16_cuda(v, "v");
    TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.sizes() == k.sizes(), "q [B, Hq, D], k / v [B, Hkv, D]");
    const int64_t B = q.size(0), Hq = q.size(1), D = q.size(2), Hkv = k.size(1);
    TORCH_CHECK(qkv.dim() == 2 && qkv.size(0) == B && qkv.size(1) == (Hq + 2 * Hkv) * D, "qkv must be [B, (Hq + 2 Hkv) D]");
    TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == torch::kInt64 && pos.numel() == B && pos.is_contiguous(),
                "pos must be a contiguous CUDA int64 [B] tensor");
    TORCH_CHECK(cos_table.is_cuda() && cos_table.scalar_type() == torch::kFloat32 && cos_table.is_contiguous() &&
                    cos_table.dim() == 2 && cos_table.size(1) == D / 2 && sin_table.sizes() == cos_table.sizes() &&
                    sin_table.is_contiguous() && sin_table.scalar_type() == torch::kFloat32,
                "cos / sin tables must be contiguous CUDA float32 [positions, D / 2]");
    check_status(mg_rope_qkv_f16(qkv.data_ptr(), pos.data_ptr<int64_t>(), cos_table.data_ptr<float>(),
                                 sin_table.data_ptr<float>(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                 static_cast<int32_t>(B), static_cast<int32_t>(Hq), static_cast<int32_t>(Hkv),
                                 static_cast<int32_t>(D), cur_stream()),
                 "rope_qkv");
}

torch::Tensor silu_mul(torch::Tensor gu) {
    const c10::cuda::CUDAGuard guard(gu.device());
    check_f16_cuda(gu, "gu");
    TORCH_CHECK(gu.size(-1) % 2 == 0, "gu's last dimension must be even (gate | up)");
    const int64_t F = gu.size(-1) / 2;
    auto shape = gu.sizes().vec();
    shape.back() = F;
    auto h = torch::empty(shape, gu.options());
    check_status(mg_silu_mul_f16(gu.data_ptr(), h.data_ptr(), gu.numel() / (2 * F), F, cur_stream()), "silu_mul");
    return h;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "B200-native paged quantized KV-cache ops (C ABI: libmgb200.so)";
    m.def("add", &add, "Elementwise add of two CUDA float32 tensors (build sanity check)");
    m.def("quantize_new_scale", &quantize_new_scale,
          "INT8-quantize into a page with a fresh absmax scale (one kernel); returns the scale");
    m.def("quantize_fixed_scale", &quantize_fixed_scale, "INT8-quantize into a page with a known scale");
    m.def("dequantize_page", &dequantize_page, "Dequantize one page's INT8 tokens to FP32");
    m.def("paged_attention_committed", &paged_attention_committed,
          "Attention over committed INT8 pages; returns UNNORMALIZED (weighted_v, weight_sum, max)");
    m.def("quantize_int4_new_scale", &quantize_int4_new_scale,
          "Packed INT4 quantize (2 values/byte, low nibble first) with a fresh absmax scale");
    m.def("dequantize_int4_page", &dequantize_int4_page, "Inverse of quantize_int4_new_scale");
    // batched device-resident path
    m.def("alloc_init", &alloc_init, "Reset a device page allocator");
    m.def("plan_append", &plan_append, "Allocate the step's committing pages and grow seq_lens (all-or-nothing)",
          pybind11::arg("free_stack"), pybind11::arg("n_free"), pybind11::arg("in_use"), pybind11::arg("block_tables"),
          pybind11::arg("seq_lens"), pybind11::arg("n_new"), pybind11::arg("page_size"),
          pybind11::arg("status") = pybind11::none());
    m.def("free_sequences", &free_sequences, "Free all pages of the listed sequences", pybind11::arg("free_stack"),
          pybind11::arg("n_free"), pybind11::arg("in_use"), pybind11::arg("block_tables"), pybind11::arg("seq_lens"),
          pybind11::arg("seq_ids"), pybind11::arg("page_size"), pybind11::arg("status") = pybind11::none());
    m.def("truncate_sequences", &truncate_sequences, "Truncate sequences, freeing whole trailing pages",
          pybind11::arg("free_stack"), pybind11::arg("n_free"), pybind11::arg("in_use"),
          pybind11::arg("block_tables"), pybind11::arg("seq_lens"), pybind11::arg("seq_ids"),
          pybind11::arg("new_lens"), pybind11::arg("page_size"), pybind11::arg("status") = pybind11::none());
    m.def("kv_append", &kv_append, "Write a step's K/V tokens: commit filled pages, stage the rest",
          pybind11::arg("k_pool"), pybind11::arg("v_pool"), pybind11::arg("k_scales"), pybind11::arg("v_scales"),
          pybind11::arg("staging_k"), pybind11::arg("staging_v"), pybind11::arg("block_tables"),
          pybind11::arg("seq_lens"), pybind11::arg("n_new"), pybind11::arg("k_new"), pybind11::arg("v_new"),
          pybind11::arg("status") = pybind11::none(), pybind11::arg("early_launch") = false);
    m.def("decode_workspace_bytes", &decode_workspace_bytes, "Workspace bytes for paged_decode_attention");
    m.def("paged_decode_attention", &paged_decode_attention, "Fused batched paged decode attention",
          pybind11::arg("q"), pybind11::arg("k_pool"), pybind11::arg("v_pool"), pybind11::arg("k_scales"),
          pybind11::arg("v_scales"), pybind11::arg("staging_k"), pybind11::arg("staging_v"),
          pybind11::arg("block_tables"), pybind11::arg("seq_lens"), pybind11::arg("scale"),
          pybind11::arg("max_context"), pybind11::arg("workspace"), pybind11::arg("out"),
          pybind11::arg("status") = pybind11::none());
    m.def("decode_plan_bytes", &decode_plan_bytes, "Bytes of a decode plan for a batch");
    m.def("decode_plan", &decode_plan, "Build the step's decode plan (work split over the SMs) from seq_lens",
          pybind11::arg("k_pool"), pybind11::arg("block_tables"), pybind11::arg("seq_lens"),
          pybind11::arg("with_staging"), pybind11::arg("plan"), pybind11::arg("status") = pybind11::none());
    m.def("plan_step", &plan_step,
          "plan_append then decode_plan in one launch: the step's allocation and its attention plan",
          pybind11::arg("free_stack"), pybind11::arg("n_free"), pybind11::arg("in_use"), pybind11::arg("k_pool"),
          pybind11::arg("block_tables"), pybind11::arg("seq_lens"), pybind11::arg("n_new"),
          pybind11::arg("with_staging"), pybind11::arg("plan"), pybind11::arg("status") = pybind11::none());
    m.def("paged_decode_attention_planned", &paged_decode_attention_planned,
          "Fused batched paged decode attention with a prebuilt decode plan (settled: MG_ATTN_PLAN_SETTLED)",
          pybind11::arg("q"), pybind11::arg("k_pool"), pybind11::arg("v_pool"), pybind11::arg("k_scales"),
          pybind11::arg("v_scales"), pybind11::arg("staging_k"), pybind11::arg("staging_v"),
          pybind11::arg("block_tables"), pybind11::arg("plan"), pybind11::arg("scale"), pybind11::arg("workspace"),
          pybind11::arg("out"), pybind11::arg("status") = pybind11::none(), pybind11::arg("settled") = false);
    m.def("gather_dequant", &gather_dequant, "Block-table gather + dequantize of whole sequences",
          pybind11::arg("k_pool"), pybind11::arg("v_pool"), pybind11::arg("k_scales"), pybind11::arg("v_scales"),
          pybind11::arg("staging_k"), pybind11::arg("staging_v"), pybind11::arg("block_tables"),
          pybind11::arg("seq_lens"), pybind11::arg("cu_seqlens"), pybind11::arg("max_context"),
          pybind11::arg("out_k"), pybind11::arg("out_v"), pybind11::arg("status") = pybind11::none());
    m.def("rmsnorm", &rmsnorm, "RMSNorm over the last dimension (fp16, fp32 math)", pybind11::arg("x"),
          pybind11::arg("w"), pybind11::arg("eps"));
    m.def("kv_append_rope", &kv_append_rope,
          "kv_append with the rotary embedding of K fused in, reading K / V from a q|k|v projection and writing "
          "the rotated q",
          pybind11::arg("k_pool"), pybind11::arg("v_pool"), pybind11::arg("k_scales"), pybind11::arg("v_scales"),
          pybind11::arg("staging_k"), pybind11::arg("staging_v"), pybind11::arg("block_tables"),
          pybind11::arg("seq_lens"), pybind11::arg("n_new"), pybind11::arg("qkv"), pybind11::arg("num_q_heads"),
          pybind11::arg("cos_table"), pybind11::arg("sin_table"), pybind11::arg("q_out"),
          pybind11::arg("status") = pybind11::none());
    m.def("rope_qkv", &rope_qkv, "Split q | k | v, rotary embedding of q and k at per-row positions",
          pybind11::arg("qkv"), pybind11::arg("pos"), pybind11::arg("cos_table"), pybind11::arg("sin_table"),
          pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"));
    m.def("silu_mul", &silu_mul, "silu(gate) * up of a [.., 2F] gate | up tensor", pybind11::arg("gu"));
    m.def("version", []() { return std::string(mg_version()); });
}
