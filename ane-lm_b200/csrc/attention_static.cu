// attention_static.cu -- decode attention whose scratch is a fixed array in
// device memory, so the call allocates nothing.
//
// Who needs it: a caller that must not change its device-memory footprint
// once it is running -- a serving process that has handed every remaining
// byte of HBM to its KV cache, or a memory-budgeted job whose allocator is
// capped -- and a caller that cannot afford the device-wide synchronisation
// of cudaMalloc / cudaFree in the middle of its decode loop.  The regular
// entry point either takes the caller's workspace or grows a buffer of its
// own with cudaMalloc; this one uses kStaticScratchBytes of storage that
// is part of the library's device image instead, and rejects problems whose
// split partials do not fit in it.
//
// The storage is one per device and shared by every call: two calls whose
// executions overlap (different streams, or host threads without ordering)
// race on it and give wrong results.  Order such calls on one stream.
#include <mutex>

#include "attention.cuh"

namespace ane {

// per-split (m, l, o) for at most this many bytes: enough for one sequence
// of 32K keys with 32 q heads of 128 (Qwen3-8B decode), or 64 sequences of
// 1K keys.
constexpr int64_t kStaticScratchBytes = (int64_t)16 << 20;

static __device__ __align__(256) unsigned char g_attn_scratch[kStaticScratchBytes];

// defined in attention.cu
int attention_args(int dtype, void* out, int64_t out_stride, const void* q, int64_t q_stride,
                   int q_head_stride, const void* k_cache, const void* v_cache,
                   int64_t cache_stride, const int32_t* cache_start, const int32_t* cache_len,
                   int cache_capacity, int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                   int max_len, AttnArgs* a);
int64_t attention_workspace_bytes(int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                                  int max_len);
void attention_bind_workspace(AttnArgs* a, void* ws, int64_t batch, int head_dim);
int attention_launch(int dtype, const AttnArgs& a, int64_t batch, int head_dim, cudaStream_t s);

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices];

// The array's device address on the current device, looked up by the first
// call made with that device current and kept once the lookup succeeds (a
// failed lookup is tried again by the next call).  The lookup is a runtime
// call of its own, so that first call belongs before any stream capture on
// the device: a call that would look the address up while `s` is capturing
// is refused instead.
int static_scratch(cudaStream_t s, void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return fail(ANE_CUDA_ERR_CUDA, "decode_attention_static: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "decode_attention_static: device %d", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing(s, &cs);
        if (e != cudaSuccess)
            return fail(ANE_CUDA_ERR_CUDA, "decode_attention_static: %s", cudaGetErrorString(e));
        if (cs != cudaStreamCaptureStatusNone)
            return fail(ANE_CUDA_ERR_INVALID_ARG,
                        "decode_attention_static: first call on device %d during a stream "
                        "capture; make one call on the device before capturing", dev);
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p)
            return fail(ANE_CUDA_ERR_CUDA, "decode_attention_static: scratch address: %s",
                        cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return ANE_CUDA_OK;
}

}  // namespace
}  // namespace ane

extern "C" {

int64_t ane_cuda_decode_attention_static_capacity(void) { return ane::kStaticScratchBytes; }

int ane_cuda_decode_attention_static(int dtype, void* out, int64_t out_stride, const void* q,
                                     int64_t q_stride, int q_head_stride, const void* k_cache,
                                     const void* v_cache, int64_t cache_stride,
                                     const int32_t* cache_start, const int32_t* cache_len,
                                     int cache_capacity, int64_t batch, int n_heads,
                                     int n_kv_heads, int head_dim, int max_len, void* stream) {
    using namespace ane;
    AttnArgs a;
    int st = attention_args(dtype, out, out_stride, q, q_stride, q_head_stride, k_cache, v_cache,
                            cache_stride, cache_start, cache_len, cache_capacity, batch, n_heads,
                            n_kv_heads, head_dim, max_len, &a);
    if (st) return st;
    if (batch == 0) return ANE_CUDA_OK;
    const int64_t need = attention_workspace_bytes(batch, n_heads, n_kv_heads, head_dim, max_len);
    if (need > kStaticScratchBytes)
        return fail(ANE_CUDA_ERR_INVALID_ARG,
                    "decode_attention_static: %lld bytes of split scratch needed, %lld available "
                    "(fewer sequences or a smaller max_len)",
                    (long long)need, (long long)kStaticScratchBytes);
    const cudaStream_t s = as_stream(stream);
    if (need > 0) {
        void* scratch = nullptr;
        st = static_scratch(s, &scratch);
        if (st) return st;
        attention_bind_workspace(&a, scratch, batch, head_dim);
    }
    return attention_launch(dtype, a, batch, head_dim, s);
}

}  // extern "C"
