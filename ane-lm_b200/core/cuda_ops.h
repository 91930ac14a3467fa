// cuda_ops.h -- drop-in CUDA (B200, sm_100a) backend for ANE-LM's core/cpu_ops
// layer ops, core/sampling's sample_token and common.h's bf16_to_f16_vec.
//
// Same names, argument order and meaning as the reference
// (core/cpu_ops.h:12-32, core/sampling.h:7-16, include/ane_lm/common.h:81-83),
// in namespace ane_lm::cuda, operating on DEVICE pointers of the current
// CUDA device.  Calls are asynchronous on the calling thread's stream
// (set_stream; default: the legacy default stream) except sample_token,
// which returns the token and therefore waits for it.
//
// Like the reference routines these return nothing; a failure (bad
// argument, CUDA error) prints one line to stderr and is readable with
// last_status() / last_error().  There is no CPU fallback: every call runs
// the sm_100a kernels of libane_cuda.so.
//
// The batched forms below the reference signatures take a row count and
// per-row positions / uniforms; they map 1:1 onto include/ane_cuda.h.
#pragma once

#include <cstdint>
#include <vector>

#include "ane_cuda.h"

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

namespace ane_lm {
namespace cuda {

// ---- per-thread call context -------------------------------------------
void set_stream(void* stream);  // cudaStream_t
void* stream();
int last_status();               // ane_cuda_status of the last call on this thread
const char* last_error();

// ---- core/cpu_ops.h ------------------------------------------------------
// silu_vec_inplace / mul_sigmoid_inplace: `tmp` is accepted for signature
// compatibility and not used (the kernels keep their temporaries in registers).
void silu_vec_inplace(float* x, int n, float* tmp);
void mul_sigmoid_inplace(float* y, const float* z, int n, float* tmp);
void rmsnorm(float* out, const float* x, const float* weight, int dim, float eps = 1e-6f);
void apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads,
                       int head_dim, int q_head_stride, int k_head_stride,
                       int rot_dim, int pos, float theta,
                       const float* cos_row, const float* sin_row);
void softmax(float* x, int n);
void rmsnorm_gated(float* out, const float* x, const float* z, const float* weight, int dim);
void l2_normalize(float* x, int dim);
// gqa_attention (core/cpu_ops.h:55-58): q, k_cache, v_cache and out on the
// device; the ring position is passed by value as in the reference.  Uses
// the library-held workspace of the calling thread's stream.
void gqa_attention(float* out, const float* q, const float* k_cache, const float* v_cache,
                   int n_heads, int n_kv_heads, int head_dim, int q_head_stride,
                   int cache_start, int cache_len, int cache_capacity);

// The KV ring bookkeeping of the decode step (models/llm/qwen3.cpp:475-484):
// the slot the new token's k / v rows go to (qk_norm_rope_kv's slots[r]);
// start and len advance as in the reference (fill, then overwrite the
// oldest slot).  Host only.
int kv_ring_advance(int* start, int* len, int capacity);

// ---- core/sampling.h -----------------------------------------------------
struct SamplingParams {
    float temperature = 0.6f;
    float repetition_penalty = 1.2f;
    int repetition_context_size = 256;
    float frequency_penalty = 0.1f;
};

// `logits` is a device pointer; `recent_tokens` is host memory, as in the
// reference.  The uniform draw is (float)drand48(), taken only when
// temperature > 0, as at core/sampling.cpp:58, so srand48 seeds the same
// sequence.  Returns -1 on failure.
int sample_token(const float* logits, int vocab_size, const SamplingParams& params,
                 const std::vector<int>& recent_tokens = {});

// ---- include/ane_lm/common.h ----------------------------------------------
void bf16_to_f16_vec(uint16_t* out, const uint16_t* in, int n);

// ---- batched forms -----------------------------------------------------------
void residual_rmsnorm(ane_cuda_dtype dtype, void* x, const void* d, void* out,
                      const float* weight, int64_t rows, int dim, float eps = 1e-6f);
void qk_norm_rope(ane_cuda_dtype dtype, void* qkv, const float* q_weight, const float* k_weight,
                  const int32_t* positions, int64_t rows, int n_q_heads, int n_kv_heads,
                  int head_dim, float theta, float eps = 1e-6f);
void silu_mul(ane_cuda_dtype dtype, void* out, const void* gate, const void* up, int64_t rows,
              int n);
void embedding_gather(void* out, ane_cuda_dtype out_dtype, const void* table,
                      ane_cuda_dtype table_dtype, const int32_t* ids, int64_t rows, int vocab,
                      int hidden);
// x = table[ids] (accumulate: x += table[ids]), out = rmsnorm(x) * weight, in
// one launch (models/llm/qwen3.cpp:498 then :503); ane_cuda_embedding_rmsnorm.
void embedding_rmsnorm(void* x, void* out, ane_cuda_dtype out_dtype, const void* table,
                       ane_cuda_dtype table_dtype, const int32_t* ids, int64_t rows, int vocab,
                       int hidden, bool accumulate, const float* weight, float eps = 1e-6f);
void sample_rows(const float* logits, int64_t rows, int vocab, const int32_t* history,
                 const int32_t* history_len, int64_t history_stride, const float* uniforms,
                 const SamplingParams& params, int32_t* out_tokens);

}  // namespace cuda
}  // namespace ane_lm

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
