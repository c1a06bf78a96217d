// mg_paged_decode_attention_noalloc: the batched decode attention with its
// workspace (merge counters, partial slots, decode plan) in a fixed static
// device array instead of caller memory.  It is for callers that cannot call
// cudaMalloc: serving runtimes whose own pool allocator has reserved all
// device memory up front (a raw cudaMalloc there fails or fragments the
// pool), and latency-critical decode loops where cudaMalloc / cudaFree would
// synchronize the device and stall the other streams.
//
// The scratch is one file-scope __device__ array of kNoAllocScratchBytes;
// every GPU that loads the library holds it until the process exits.  In
// host code its name is only a host-side stand-in, so the device address is
// looked up with cudaGetSymbolAddress, once per device with that device
// current, on the first call there (make that first call before any stream
// capture begins), and that address is what the kernels get.  Every call
// zeroes the merge counters at its start (a memset on the call's stream; the
// array keeps whatever the previous call left) and then runs
// mg_paged_decode_attention on the array.  Calls that overlap on the GPU
// share the array and race: run one at a time per device.
#include <cstdio>
#include <mutex>

#include "mg_common.cuh"

namespace mg {
namespace {

constexpr int64_t kNoAllocScratchBytes = 4ll << 20;  // 4 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

mg_status scratch_address(void** out) {
    static void* addr[kMaxDevices] = {};
    static std::mutex mu;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return set_error(MG_ERR_UNSUPPORTED, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(MG_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return MG_OK;
}

}  // namespace
}  // namespace mg

using namespace mg;

extern "C" mg_status mg_paged_decode_attention_noalloc(const mg_cache_layout* L, const mg_layer_ptrs* lp,
                                                       const int32_t* block_tables, const int32_t* seq_lens,
                                                       int32_t batch, const void* q, int32_t q_dtype,
                                                       int32_t num_q_heads, float scale, void* out,
                                                       int32_t out_dtype, int32_t max_context,
                                                       int32_t* dev_status, mg_stream_t stream) {
    MG_REQUIRE(L, "null layout");
    MG_REQUIRE(batch >= 0, "batch must be >= 0");
    if (batch == 0) return MG_OK;
    const int64_t need = mg_paged_decode_workspace_bytes(L, batch, num_q_heads, max_context);
    if (need <= 0) {
        // the sizing call left its reason in the thread's error text: copy it
        // out before formatting into that same buffer
        char why[512];
        snprintf(why, sizeof(why), "%s", mg_last_error());
        return set_error(MG_ERR_INVALID_ARGUMENT, "no-alloc decode attention: %s", why);
    }
    MG_REQUIRE(need <= kNoAllocScratchBytes,
               "no-alloc decode attention needs %lld bytes of workspace, more than its %lld-byte static scratch "
               "(smaller batch or fewer heads, or use mg_paged_decode_attention with a caller workspace)",
               (long long)need, (long long)kNoAllocScratchBytes);
    void* scratch = nullptr;
    mg_status st = scratch_address(&scratch);
    if (st != MG_OK) return st;
    // the per-(sequence, kv head) merge counters must start at zero
    const int64_t counters = (static_cast<int64_t>(batch) * L->num_kv_heads * 4 + 255) / 256 * 256;
    const cudaError_t e = cudaMemsetAsync(scratch, 0, static_cast<size_t>(counters), as_stream(stream));
    if (e != cudaSuccess) return set_error(MG_ERR_CUDA, "cudaMemsetAsync(no-alloc counters): %s", cudaGetErrorString(e));
    return mg_paged_decode_attention(L, lp, block_tables, seq_lens, batch, q, q_dtype, num_q_heads, scale, out,
                                     out_dtype, max_context, scratch, kNoAllocScratchBytes, dev_status, stream);
}
