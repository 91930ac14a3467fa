// attention.cu -- C ABI of the decode attention (core/cpu_ops.cpp:173-240):
// argument checks, the workspace layout, and the library-held workspace
// used when the caller passes none.
#include <mutex>
#include <unordered_map>
#include <vector>

#include "attention.cuh"

namespace ane {
// compiled in attention_{f32,f16,bf16}.cu
extern template int launch_decode_attention<F32>(const AttnArgs&, int, int, int64_t, cudaStream_t);
extern template int launch_decode_attention<F16>(const AttnArgs&, int, int, int64_t, cudaStream_t);
extern template int launch_decode_attention<BF16>(const AttnArgs&, int, int, int64_t, cudaStream_t);
}  // namespace ane

namespace ane {
namespace {

int64_t round256(int64_t v) { return (v + 255) & ~(int64_t)255; }

struct WsLayout {
    int64_t ml = 0, o = 0, total = 0;  // byte offsets, total size
};

// [m, l: batch x n_heads x splits x 2 f32][o: batch x n_heads x splits x
// head_dim f32]; nothing with one split.  Only the partials of the call in
// flight live here: nothing needs to be zero, and nothing is kept between
// calls.
WsLayout ws_layout(int64_t batch, int n_heads, int /*n_kv*/, int head_dim, int max_splits) {
    WsLayout w;
    if (max_splits <= 1) return w;
    w.ml = 0;
    w.o = round256(batch * n_heads * (int64_t)max_splits * 2 * 4);
    w.total = w.o + round256(batch * n_heads * (int64_t)max_splits * head_dim * 4);
    return w;
}

int splits_of(int max_len) { return max_len <= 0 ? 1 : (max_len + kAttnKeys - 1) / kAttnKeys; }

// Library-held workspace, one per (device, stream), kept until the process
// exits.  A buffer is never freed once handed to a kernel: a CUDA graph
// captured with it may be replayed at any time, so when a larger call needs
// more, a new buffer is allocated and the old one is kept (retired) too.
// Allocating is refused while the stream is capturing (a cudaMalloc
// during a capture can invalidate it, depending on the capture mode):
// graphs take a caller workspace, or an eager call of the largest shape on
// the stream comes first.
struct HeldWs {
    void* ptr = nullptr;
    int64_t bytes = 0;
};
std::mutex g_ws_mu;
std::unordered_map<uint64_t, HeldWs>* g_ws = nullptr;
std::vector<void*>* g_ws_retired = nullptr;

int held_workspace(cudaStream_t s, int64_t need, void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(ANE_CUDA_ERR_CUDA, "decode_attention: %s", cudaGetErrorString(e));
    const uint64_t key = ((uint64_t)(uintptr_t)s << 8) ^ (uint64_t)dev;
    std::lock_guard<std::mutex> lock(g_ws_mu);
    if (!g_ws) g_ws = new std::unordered_map<uint64_t, HeldWs>();
    if (!g_ws_retired) g_ws_retired = new std::vector<void*>();
    HeldWs& h = (*g_ws)[key];
    if (h.bytes < need) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing(s, &cs);
        if (e != cudaSuccess)
            return fail(ANE_CUDA_ERR_CUDA, "decode_attention: %s", cudaGetErrorString(e));
        if (cs != cudaStreamCaptureStatusNone)
            return fail(ANE_CUDA_ERR_INVALID_ARG,
                        "decode_attention: the library-held workspace of this stream must grow to "
                        "%lld bytes during a stream capture; pass a workspace, or make one eager "
                        "call of the largest shape on the stream before capturing",
                        (long long)need);
        const int64_t bytes = need < ((int64_t)1 << 20) ? ((int64_t)1 << 20) : need;
        void* p = nullptr;
        e = cudaMalloc(&p, (size_t)bytes);
        if (e != cudaSuccess)
            return fail(ANE_CUDA_ERR_CUDA, "decode_attention: workspace of %lld bytes: %s",
                        (long long)bytes, cudaGetErrorString(e));
        if (h.ptr) g_ws_retired->push_back(h.ptr);  // a captured graph may still use it
        h.ptr = p;
        h.bytes = bytes;
    }
    *out = h.ptr;
    return ANE_CUDA_OK;
}

}  // namespace

// Checks shared by the decode-attention entry points; fills `a` except the
// workspace pointers.
int attention_args(int dtype, void* out, int64_t out_stride, const void* q, int64_t q_stride,
                   int q_head_stride, const void* k_cache, const void* v_cache,
                   int64_t cache_stride, const int32_t* cache_start, const int32_t* cache_len,
                   int cache_capacity, int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                   int max_len, AttnArgs* a) {
    const char* fn = "decode_attention";
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: bad dtype %d", fn, dtype);
    if (batch < 0 || batch > 65535 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 ||
        cache_capacity <= 0 || max_len < 0 || n_heads % n_kv_heads != 0)
        return fail(ANE_CUDA_ERR_INVALID_ARG,
                    "%s: batch=%lld n_heads=%d n_kv_heads=%d head_dim=%d capacity=%d max_len=%d", fn,
                    (long long)batch, n_heads, n_kv_heads, head_dim, cache_capacity, max_len);
    if (head_dim != 64 && head_dim != 128 && head_dim != 256)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "%s: head_dim %d (64, 128 or 256)", fn, head_dim);
    if (n_heads / n_kv_heads > kAttnMaxGroup)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "%s: %d q heads per kv head (at most %d)", fn,
                    n_heads / n_kv_heads, kAttnMaxGroup);
    if (cache_capacity > (1 << 30))
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "%s: capacity %d > 2^30", fn, cache_capacity);
    if (n_kv_heads > 65535)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "%s: n_kv_heads %d", fn, n_kv_heads);
    if (!out || !q || !k_cache || !v_cache || !cache_start || !cache_len)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: null pointer", fn);
    const int es = elem_size(dtype);
    if (out_stride < (int64_t)n_heads * head_dim || q_head_stride < head_dim ||
        q_stride < (int64_t)(n_heads - 1) * q_head_stride + head_dim ||
        cache_stride < (int64_t)cache_capacity * n_kv_heads * head_dim)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: strides out=%lld q=%lld q_head=%d cache=%lld", fn,
                    (long long)out_stride, (long long)q_stride, q_head_stride, (long long)cache_stride);
    // rows are moved by 16-byte bulk copies and vector loads
    if (!is_aligned(q, 16) || !is_aligned(k_cache, 16) || !is_aligned(v_cache, 16) ||
        (q_stride * es) % 16 || ((int64_t)q_head_stride * es) % 16 || (cache_stride * es) % 16)
        return fail(ANE_CUDA_ERR_UNSUPPORTED,
                    "%s: q and the caches need 16-byte aligned bases and strides", fn);
    a->out = out;
    a->out_stride = out_stride;
    a->q = q;
    a->q_stride = q_stride;
    a->q_head_stride = q_head_stride;
    a->k_cache = k_cache;
    a->v_cache = v_cache;
    a->cache_stride = cache_stride;
    a->start = cache_start;
    a->len = cache_len;
    a->capacity = cache_capacity;
    a->n_heads = n_heads;
    a->n_kv = n_kv_heads;
    a->max_len = max_len;
    a->max_splits = splits_of(max_len);
    a->chunks = 1;  // set per launch
    a->stages = 0;
    a->scale = 1.0f / sqrtf((float)head_dim);  // core/cpu_ops.cpp:182
    a->part_ml = nullptr;
    a->part_o = nullptr;
    a->flags = status_flags_device();
    return ANE_CUDA_OK;
}

int64_t attention_workspace_bytes(int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                                  int max_len) {
    return ws_layout(batch, n_heads, n_kv_heads, head_dim, splits_of(max_len)).total;
}

void attention_bind_workspace(AttnArgs* a, void* ws, int64_t batch, int head_dim) {
    const WsLayout w = ws_layout(batch, a->n_heads, a->n_kv, head_dim, a->max_splits);
    if (w.total == 0) return;
    unsigned char* base = static_cast<unsigned char*>(ws);
    a->part_ml = reinterpret_cast<float*>(base + w.ml);
    a->part_o = reinterpret_cast<float*>(base + w.o);
}

int attention_launch(int dtype, const AttnArgs& a, int64_t batch, int head_dim, cudaStream_t s) {
    const int group = a.n_heads / a.n_kv;
    if (dtype == ANE_CUDA_F32) return launch_decode_attention<F32>(a, head_dim, group, batch, s);
    if (dtype == ANE_CUDA_F16) return launch_decode_attention<F16>(a, head_dim, group, batch, s);
    return launch_decode_attention<BF16>(a, head_dim, group, batch, s);
}

}  // namespace ane

extern "C" {

int64_t ane_cuda_decode_attention_workspace_size(int64_t batch, int n_heads, int n_kv_heads,
                                                 int head_dim, int max_len) {
    if (batch < 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || max_len < 0) return -1;
    return ane::attention_workspace_bytes(batch, n_heads, n_kv_heads, head_dim, max_len);
}

int ane_cuda_decode_attention(int dtype, void* out, int64_t out_stride, const void* q,
                              int64_t q_stride, int q_head_stride, const void* k_cache,
                              const void* v_cache, int64_t cache_stride,
                              const int32_t* cache_start, const int32_t* cache_len,
                              int cache_capacity, int64_t batch, int n_heads, int n_kv_heads,
                              int head_dim, int max_len, void* workspace,
                              int64_t workspace_bytes, void* stream) {
    using namespace ane;
    AttnArgs a;
    int st = attention_args(dtype, out, out_stride, q, q_stride, q_head_stride, k_cache, v_cache,
                            cache_stride, cache_start, cache_len, cache_capacity, batch, n_heads,
                            n_kv_heads, head_dim, max_len, &a);
    if (st) return st;
    if (batch == 0) return ANE_CUDA_OK;
    const cudaStream_t s = as_stream(stream);
    const int64_t need = attention_workspace_bytes(batch, n_heads, n_kv_heads, head_dim, max_len);
    if (need > 0) {
        if (workspace) {
            if (workspace_bytes < need || !is_aligned(workspace, 256))
                return fail(ANE_CUDA_ERR_INVALID_ARG,
                            "decode_attention: workspace of %lld bytes at %p (need %lld, 256-byte aligned)",
                            (long long)workspace_bytes, workspace, (long long)need);
        } else {
            st = held_workspace(s, need, &workspace);
            if (st) return st;
        }
        attention_bind_workspace(&a, workspace, batch, head_dim);
    }
    return attention_launch(dtype, a, batch, head_dim, s);
}

}  // extern "C"
