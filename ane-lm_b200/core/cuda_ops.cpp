// cuda_ops.cpp -- the reference-signature layer over the C ABI.
#include "cuda_ops.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace ane_lm {
namespace cuda {

namespace {

thread_local void* t_stream = nullptr;
thread_local int t_status = ANE_CUDA_OK;

int note(const char* fn, int st) {
    t_status = st;
    if (st != ANE_CUDA_OK) fprintf(stderr, "ane_lm::cuda::%s: %s\n", fn, ane_cuda_last_error());
    return st;
}

// Per-thread device staging for sample_token, one fixed-size block per
// device: [0] the result, [4] the uniform, [8] the window length, [16..]
// the window of at most kStageWindow ids.  Only the last
// repetition_context_size ids of the history are read by the reference
// (core/sampling.cpp:17-27) and the kernel takes windows up to
// kStageWindow, so the block never grows: allocated by the thread's first
// call on a device, freed when the thread exits.
constexpr int kStageWindow = 4096;
constexpr int kStageHeader = 4;  // int32 slots before the window
constexpr int kMaxDevices = 64;
struct SampleStage {
    int32_t* dev[kMaxDevices] = {};
    std::vector<int32_t> host;  // the same layout, staged for one copy
    ~SampleStage() {
        for (int d = 0; d < kMaxDevices; d++)
            if (dev[d]) cudaFree(dev[d]);
    }
};
thread_local SampleStage t_stage;

}  // namespace

void set_stream(void* s) { t_stream = s; }
void* stream() { return t_stream; }
int last_status() { return t_status; }
const char* last_error() { return ane_cuda_last_error(); }

void silu_vec_inplace(float* x, int n, float*) {
    note("silu_vec_inplace", ane_cuda_silu_inplace(ANE_CUDA_F32, x, n, t_stream));
}

void mul_sigmoid_inplace(float* y, const float* z, int n, float*) {
    note("mul_sigmoid_inplace", ane_cuda_mul_sigmoid_inplace(ANE_CUDA_F32, y, z, n, t_stream));
}

void rmsnorm(float* out, const float* x, const float* weight, int dim, float eps) {
    note("rmsnorm", ane_cuda_residual_rmsnorm(ANE_CUDA_F32, const_cast<float*>(x), dim, nullptr, 0,
                                              out, dim, weight, 1, dim, eps, t_stream));
}

void apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads, int head_dim,
                       int q_head_stride, int k_head_stride, int rot_dim, int pos, float theta,
                       const float* cos_row, const float* sin_row) {
    note("apply_rope_cached",
         ane_cuda_apply_rope_cached(q, k, n_q_heads, n_kv_heads, head_dim, q_head_stride,
                                    k_head_stride, rot_dim, pos, theta, cos_row, sin_row, t_stream));
}

void softmax(float* x, int n) { note("softmax", ane_cuda_softmax_rows(x, 1, n, n, t_stream)); }

void rmsnorm_gated(float* out, const float* x, const float* z, const float* weight, int dim) {
    note("rmsnorm_gated", ane_cuda_rmsnorm_gated(ANE_CUDA_F32, out, dim, x, dim, z, dim, weight, 1,
                                                 dim, 1e-6f, t_stream));
}

void l2_normalize(float* x, int dim) {
    note("l2_normalize", ane_cuda_l2_normalize(ANE_CUDA_F32, x, dim, 1, dim, 1.0f, t_stream));
}

int kv_ring_advance(int* start, int* len, int capacity) {
    int slot;
    if (*len < capacity) {
        slot = *start + *len;
        if (slot >= capacity) slot -= capacity;
        (*len)++;
    } else {
        slot = *start;
        if (++*start >= capacity) *start = 0;
    }
    return slot;
}

void gqa_attention(float* out, const float* q, const float* k_cache, const float* v_cache,
                   int n_heads, int n_kv_heads, int head_dim, int q_head_stride,
                   int cache_start, int cache_len, int cache_capacity) {
    // The ring position goes to a per-thread device slot with the call: a
    // copy from pageable memory is staged before cudaMemcpyAsync returns, and
    // stream order keeps the slot until the kernel has read it.
    thread_local int32_t* d_pos = nullptr;
    thread_local int pos_dev = -1;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        note("gqa_attention", ANE_CUDA_ERR_CUDA);
        return;
    }
    if (pos_dev != dev) {
        if (d_pos) cudaFree(d_pos);
        d_pos = nullptr;
        pos_dev = -1;
        if (cudaMalloc((void**)&d_pos, 2 * sizeof(int32_t)) != cudaSuccess) {
            d_pos = nullptr;
            note("gqa_attention", ANE_CUDA_ERR_CUDA);
            return;
        }
        pos_dev = dev;
    }
    const int32_t pos[2] = {cache_start, cache_len};
    cudaStream_t s = static_cast<cudaStream_t>(t_stream);
    if (cudaMemcpyAsync(d_pos, pos, sizeof(pos), cudaMemcpyHostToDevice, s) != cudaSuccess) {
        note("gqa_attention", ANE_CUDA_ERR_CUDA);
        return;
    }
    const int max_len = cache_len > 0 ? cache_len : 0;
    note("gqa_attention",
         ane_cuda_decode_attention(ANE_CUDA_F32, out, (int64_t)n_heads * head_dim, q,
                                   (int64_t)n_heads * q_head_stride, q_head_stride, k_cache, v_cache,
                                   (int64_t)cache_capacity * n_kv_heads * head_dim, d_pos, d_pos + 1,
                                   cache_capacity, 1, n_heads, n_kv_heads, head_dim, max_len,
                                   nullptr, 0, t_stream));
}

int sample_token(const float* logits, int vocab_size, const SamplingParams& params,
                 const std::vector<int>& recent_tokens) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        note("sample_token", ANE_CUDA_ERR_CUDA);
        return -1;
    }
    // the window the reference counts: ids [max(0, n - ctx), n)
    const int64_t n = (int64_t)recent_tokens.size();
    const int64_t ctx = params.repetition_context_size > 0 ? params.repetition_context_size : 0;
    const int64_t w0 = n - ctx > 0 ? n - ctx : 0;
    const int64_t wn = n - w0;
    if (wn > kStageWindow) {
        fprintf(stderr, "ane_lm::cuda::sample_token: repetition window %lld > %d\n", (long long)wn,
                kStageWindow);
        t_status = ANE_CUDA_ERR_UNSUPPORTED;
        return -1;
    }
    int32_t*& d_stage = t_stage.dev[dev];
    if (!d_stage) {
        const size_t bytes = (size_t)(kStageHeader + kStageWindow) * sizeof(int32_t);
        if (cudaMalloc(&d_stage, bytes) != cudaSuccess) {
            fprintf(stderr, "ane_lm::cuda::sample_token: cudaMalloc of %zu bytes failed\n", bytes);
            d_stage = nullptr;
            t_status = ANE_CUDA_ERR_CUDA;
            return -1;
        }
    }
    // the reference draws only when it samples (core/sampling.cpp:45-58)
    const float r = params.temperature > 0.0f ? (float)drand48() : 0.0f;
    std::vector<int32_t>& h = t_stage.host;
    h.resize((size_t)(kStageHeader + wn));
    h[0] = -1;
    memcpy(&h[1], &r, sizeof(r));
    h[2] = (int32_t)wn;
    h[3] = 0;
    for (int64_t j = 0; j < wn; j++) h[(size_t)(kStageHeader + j)] = recent_tokens[(size_t)(w0 + j)];
    cudaStream_t s = static_cast<cudaStream_t>(t_stream);
    cudaError_t e = cudaMemcpyAsync(d_stage, h.data(), h.size() * sizeof(int32_t),
                                    cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
        fprintf(stderr, "ane_lm::cuda::sample_token: %s\n", cudaGetErrorString(e));
        t_status = ANE_CUDA_ERR_CUDA;
        return -1;
    }
    int32_t* d_out = d_stage;
    const float* d_u = reinterpret_cast<const float*>(d_stage + 1);
    const int32_t* d_len = d_stage + 2;
    const int32_t* d_hist = d_stage + kStageHeader;
    int st = ane_cuda_sample_rows(logits, 1, vocab_size, vocab_size, wn ? d_hist : nullptr,
                                  wn ? d_len : nullptr, wn, d_u, params.temperature,
                                  params.repetition_penalty, (int)(wn ? wn : 0),
                                  params.frequency_penalty, d_out, s);
    if (note("sample_token", st) != ANE_CUDA_OK) return -1;
    int32_t tok = -1;
    e = cudaMemcpyAsync(&tok, d_out, sizeof(tok), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        fprintf(stderr, "ane_lm::cuda::sample_token: %s\n", cudaGetErrorString(e));
        t_status = ANE_CUDA_ERR_CUDA;
        return -1;
    }
    return tok;
}

void bf16_to_f16_vec(uint16_t* out, const uint16_t* in, int n) {
    note("bf16_to_f16_vec", ane_cuda_bf16_to_f16(out, in, n, t_stream));
}

void residual_rmsnorm(ane_cuda_dtype dtype, void* x, const void* d, void* out, const float* weight,
                      int64_t rows, int dim, float eps) {
    note("residual_rmsnorm", ane_cuda_residual_rmsnorm(dtype, x, dim, d, dim, out, dim, weight,
                                                       rows, dim, eps, t_stream));
}

void qk_norm_rope(ane_cuda_dtype dtype, void* qkv, const float* q_weight, const float* k_weight,
                  const int32_t* positions, int64_t rows, int n_q_heads, int n_kv_heads,
                  int head_dim, float theta, float eps) {
    const int64_t width = (int64_t)(n_q_heads + 2 * n_kv_heads) * head_dim;
    const size_t es = dtype == ANE_CUDA_F32 ? 4 : 2;
    void* k = static_cast<unsigned char*>(qkv) + (size_t)n_q_heads * head_dim * es;
    note("qk_norm_rope", ane_cuda_qk_norm_rope(dtype, qkv, k, width, width, head_dim, head_dim,
                                               n_q_heads, n_kv_heads, head_dim, head_dim, q_weight,
                                               k_weight, positions, rows, theta, eps, t_stream));
}

void silu_mul(ane_cuda_dtype dtype, void* out, const void* gate, const void* up, int64_t rows,
              int n) {
    note("silu_mul", ane_cuda_silu_mul(dtype, out, n, gate, n, up, n, rows, n, t_stream));
}

void embedding_gather(void* out, ane_cuda_dtype out_dtype, const void* table,
                      ane_cuda_dtype table_dtype, const int32_t* ids, int64_t rows, int vocab,
                      int hidden) {
    note("embedding_gather", ane_cuda_embedding_gather(out, out_dtype, table, table_dtype, ids,
                                                       rows, vocab, hidden, t_stream));
}

void embedding_rmsnorm(void* x, void* out, ane_cuda_dtype out_dtype, const void* table,
                       ane_cuda_dtype table_dtype, const int32_t* ids, int64_t rows, int vocab,
                       int hidden, bool accumulate, const float* weight, float eps) {
    note("embedding_rmsnorm",
         ane_cuda_embedding_rmsnorm(out_dtype, x, hidden, out, hidden, table, table_dtype, ids, rows,
                                    vocab, hidden, accumulate ? 1 : 0, weight, eps, t_stream));
}

void sample_rows(const float* logits, int64_t rows, int vocab, const int32_t* history,
                 const int32_t* history_len, int64_t history_stride, const float* uniforms,
                 const SamplingParams& p, int32_t* out_tokens) {
    note("sample_rows", ane_cuda_sample_rows(logits, rows, vocab, vocab, history, history_len,
                                             history_stride, uniforms, p.temperature,
                                             p.repetition_penalty, p.repetition_context_size,
                                             p.frequency_penalty, out_tokens, t_stream));
}

}  // namespace cuda
}  // namespace ane_lm
