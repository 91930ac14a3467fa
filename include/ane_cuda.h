/*
 * ane_cuda.h -- C ABI of the B200 (sm_100a) backend for ANE-LM's non-matmul
 * hot path: the layer ops of core/cpu_ops, the sampler of core/sampling and
 * the BF16 -> FP16 weight conversion behind `ane-lm convert`.
 *
 * Conventions (all entry points):
 *   - Every pointer argument is a DEVICE pointer of the calling thread's
 *     current CUDA device unless stated otherwise; the caller owns every
 *     buffer.  In-place use is allowed where the reference allows it.
 *   - Strides are in elements.  `stream` is a cudaStream_t (NULL = the
 *     legacy default stream).  Calls are asynchronous on `stream`.
 *   - The return value is an ane_cuda_status; ane_cuda_last_error() gives a
 *     one-line description of the calling thread's last failure.
 *   - Re-entrant: no call keeps state between calls except the per-device
 *     status word read by ane_cuda_read_status_flags() and, for decode
 *     attention, the library-held workspaces and the shape last used with
 *     each workspace.
 *
 * Reference citations are file:line in the ANE-LM source tree.
 */
#ifndef ANE_CUDA_H
#define ANE_CUDA_H

#include <stdint.h>

#if defined(__GNUC__)
#define ANE_CUDA_API __attribute__((visibility("default")))
#else
#define ANE_CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    ANE_CUDA_OK = 0,
    ANE_CUDA_ERR_INVALID_ARG = 1, /* null pointer, bad size or stride        */
    ANE_CUDA_ERR_UNSUPPORTED = 2, /* valid request this build does not cover */
    ANE_CUDA_ERR_CUDA = 3         /* a CUDA runtime call or launch failed    */
} ane_cuda_status;

/* element types of activation rows and tables */
typedef enum { ANE_CUDA_F32 = 0, ANE_CUDA_F16 = 1, ANE_CUDA_BF16 = 2 } ane_cuda_dtype;

/* fp32 -> fp16 rounding at the ANE boundary */
typedef enum {
    ANE_CUDA_ROUND_NEAREST = 0,  /* native __fp16 store on arm64 (round to nearest even) */
    ANE_CUDA_ROUND_TRUNCATE = 1  /* f32_to_f16 of include/ane_lm/common.h:58-71 (x86) */
} ane_cuda_round;

/* bits of the per-device status word */
#define ANE_CUDA_FLAG_BAD_TOKEN_ID 0x1u /* a gather id was outside [0, vocab) */
#define ANE_CUDA_FLAG_BAD_CACHE    0x2u /* a KV ring start / len outside the cache */
#define ANE_CUDA_FLAG_WAIT_TIMEOUT 0x4u /* a kernel gave up waiting on its own copies */

ANE_CUDA_API int ane_cuda_abi_version(void);
ANE_CUDA_API const char* ane_cuda_status_string(int status);
ANE_CUDA_API const char* ane_cuda_last_error(void);

/* Reads (and, when clear != 0, resets) the status word of the current device.
 * Synchronises the device. */
ANE_CUDA_API int ane_cuda_read_status_flags(uint32_t* flags, int clear);

/* ---- BF16 -> FP16 conversion ------------------------------------------
 * Replaces bf16_to_f16_vec (include/ane_lm/common.h:81-83), i.e.
 * bf16_to_f16 (:73-75) = f32_to_f16 (:58-71) of bf16_to_f32 (:21-26):
 * TRUNCATING, exponent >= 31 (Inf and NaN included) -> signed Inf,
 * below 2^-25 -> signed zero.  Bit-exact.  Call sites: write_ane_blob
 * (core/safetensors.cpp:335) and build_weight_blob (core/ane_runtime.cpp:207). */
ANE_CUDA_API int ane_cuda_bf16_to_f16(uint16_t* out, const uint16_t* in, int64_t n, void* stream);

/* ---- `ane-lm convert` ----------------------------------------------------
 * HOST paths, not device pointers.  The conversion runs on the calling
 * thread's current device, on up to 4 threads (the caller's and 3 more),
 * each with its own stream and staging (128 MiB pinned, 128 MiB device,
 * allocated per call); work already queued on `stream` completes first.
 * Output files are byte-identical to the reference's.
 *
 * ane_cuda_write_ane_blobs replaces SafeTensors::write_ane_blobs
 * (core/safetensors.cpp:345-383, blob format :316-343): every BF16 tensor of
 * one .safetensors file becomes output_dir/<name with '.' -> '/'>.bin, a
 * 128-byte header followed by the FP16 data; other dtypes are skipped.
 * *written receives the number of blobs.
 *
 * ane_cuda_convert_model replaces ModelWeights::open + write_ane_blobs
 * (core/model_loader.cpp:14-118, :163-171) as used by cmd_convert
 * (main.cpp:169-192): shards from model.safetensors.index.json's weight_map
 * (unique, sorted), else every *.safetensors below model_dir (sorted). */
ANE_CUDA_API int ane_cuda_write_ane_blobs(const char* safetensors_path, const char* output_dir,
                                          int64_t* written, void* stream);
ANE_CUDA_API int ane_cuda_convert_model(const char* model_dir, const char* output_dir,
                                        int64_t* written, void* stream);

/* ---- embedding gather --------------------------------------------------
 * Replaces the row memcpy of Qwen3Model::forward (models/llm/qwen3.cpp:498),
 * batched: out[r, :] = table[ids[r], :].  out_dtype equals table_dtype (a
 * byte copy) or is F32 with an F16/BF16 table (exact widening).  An id
 * outside [0, vocab) writes a zero row and sets ANE_CUDA_FLAG_BAD_TOKEN_ID. */
ANE_CUDA_API int ane_cuda_embedding_gather(void* out, int out_dtype, const void* table, int table_dtype,
                              const int32_t* ids, int64_t rows, int vocab, int hidden,
                              void* stream);

/* ---- residual add + RMSNorm -------------------------------------------
 * Replaces rmsnorm (core/cpu_ops.cpp:25-31) fused with the residual add
 * vDSP_vadd(x, d, x) that precedes it (models/llm/qwen3.cpp:516-518, :527,
 * :503).  Per row: if d != NULL, x += d is stored back into x (in x's
 * dtype); then out = (x * inv) * weight with inv = 1/sqrtf(sum(x^2)/dim +
 * eps).  Without d this is rmsnorm(out, x, weight, dim, eps); out may alias x.
 * dtype: F32, F16 or BF16 for x, d and out; weight is fp32 [dim]. */
ANE_CUDA_API int ane_cuda_residual_rmsnorm(int dtype, void* x, int64_t x_stride, const void* d,
                              int64_t d_stride, void* out, int64_t out_stride,
                              const float* weight, int64_t rows, int dim, float eps,
                              void* stream);

/* The decode step's first two ops in one launch: the embedding gather
 * (models/llm/qwen3.cpp:498) and the RMSNorm that reads it (:503; with
 * accumulate, the residual add before it, :516-518).  Per row r: e =
 * table[ids[r]] widened to out_dtype (exact), x[r] = e (accumulate = 0) or
 * x[r] + e (accumulate = 1), stored; out[r] = (x[r] * inv) * weight as in
 * ane_cuda_residual_rmsnorm.  The same bits as ane_cuda_embedding_gather
 * followed by ane_cuda_residual_rmsnorm.  out_dtype equals table_dtype, or
 * is F32 with an F16 / BF16 table; hidden a multiple of 16 bytes of
 * out_dtype, at most 4096 fp16 / 2048 fp32 elements; x, out and weight
 * 16-byte aligned.  An id outside [0, vocab) reads as a zero row and sets
 * ANE_CUDA_FLAG_BAD_TOKEN_ID. */
ANE_CUDA_API int ane_cuda_embedding_rmsnorm(int out_dtype, void* x, int64_t x_stride, void* out,
                                            int64_t out_stride, const void* table, int table_dtype,
                                            const int32_t* ids, int64_t rows, int vocab, int hidden,
                                            int accumulate, const float* weight, float eps,
                                            void* stream);

/* ---- per-head QK-norm + RoPE ------------------------------------------
 * Replaces the per-head rmsnorm of q and k (models/llm/qwen3.cpp:444-461)
 * followed by apply_rope_cached (core/cpu_ops.cpp:56-80, half-split fast
 * path :43-54; models/llm/qwen3.cpp:17-52, :463-473), in place, for a batch
 * of rows each with its own position.  Head h of row r sits at
 * q + r*q_row_stride + h*q_head_stride (k likewise).  cos/sin are computed
 * in registers from inv_freq[j] = 1/powf(theta, 2j/rot_dim) (the table of
 * models/llm/qwen3.cpp:200-219, without its 16384-position cap).
 * q_weight / k_weight (fp32 [head_dim]) may both be NULL: RoPE only. */
ANE_CUDA_API int ane_cuda_qk_norm_rope(int dtype, void* q, void* k, int64_t q_row_stride,
                          int64_t k_row_stride, int q_head_stride, int k_head_stride,
                          int n_q_heads, int n_kv_heads, int head_dim, int rot_dim,
                          const float* q_weight, const float* k_weight,
                          const int32_t* positions, int64_t rows, float theta, float eps,
                          void* stream);

/* Per-head QK-norm + RoPE with the KV-cache write of the decode step
 * (models/llm/qwen3.cpp:440-488): as ane_cuda_qk_norm_rope (rot_dim =
 * head_dim), and in the same pass row r's k heads after RoPE and its v
 * heads (v + r*v_row_stride + j*v_head_stride, unchanged) are written to
 * ring slot slots[r] of the caches [slot][n_kv_heads][head_dim] at
 * k_cache / v_cache + r*cache_row_stride (0 when all rows are tokens of one
 * sequence; a per-sequence cache stride for a batch of decode rows);
 * slots[r] < 0 writes no cache row; slots[r] >= cache_capacity writes none
 * and sets ANE_CUDA_FLAG_BAD_CACHE.  The slot follows the reference's ring
 * bookkeeping (:475-484), done by the caller.  Needs the row kernel's
 * shapes: head_dim / (16 / element size) a power of two <= 32, 16-byte
 * aligned rows, heads and caches (ANE_CUDA_ERR_UNSUPPORTED otherwise). */
ANE_CUDA_API int ane_cuda_qk_norm_rope_kv(int dtype, void* q, void* k, const void* v,
                                          int64_t q_row_stride, int64_t k_row_stride,
                                          int64_t v_row_stride, int q_head_stride,
                                          int k_head_stride, int v_head_stride, int n_q_heads,
                                          int n_kv_heads, int head_dim, const float* q_weight,
                                          const float* k_weight, const int32_t* positions,
                                          void* k_cache, void* v_cache, int64_t cache_row_stride,
                                          const int32_t* slots, int cache_capacity, int64_t rows,
                                          float theta, float eps, void* stream);

/* The single-position form, apply_rope_cached (core/cpu_ops.h:25-28,
 * core/cpu_ops.cpp:56-80) on fp32 device data.  With both cos_row and
 * sin_row: the half-split fast path on those tables (:43-54).  When either
 * is NULL: the reference's on-the-fly fallback (:66-77), which rotates
 * interleaved pairs (v[2j], v[2j+1]) by angle pos / theta^(2j/rot_dim),
 * cos/sin computed in registers (within 2 ulp of libm's cosf / sinf at
 * unit scale).  rot_dim must be even. */
ANE_CUDA_API int ane_cuda_apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads,
                               int head_dim, int q_head_stride, int k_head_stride,
                               int rot_dim, int pos, float theta, const float* cos_row,
                               const float* sin_row, void* stream);

/* ---- SiLU-gated activation ---------------------------------------------
 * out = silu(gate) * up with silu(x) = x / (1 + exp(-x)): silu_vec_inplace
 * (core/cpu_ops.cpp:7-14) times up, the gate*sigmoid(gate)*up of the fused
 * FFN (core/ane_runtime.cpp:393-395) in fp32 arithmetic.  out may alias
 * gate or up. */
ANE_CUDA_API int ane_cuda_silu_mul(int dtype, void* out, int64_t out_stride, const void* gate,
                      int64_t gate_stride, const void* up, int64_t up_stride, int64_t rows,
                      int n, void* stream);

/* silu_vec_inplace (core/cpu_ops.cpp:7-14): x = x / (1 + exp(-x)). */
ANE_CUDA_API int ane_cuda_silu_inplace(int dtype, void* x, int64_t n, void* stream);

/* mul_sigmoid_inplace (core/cpu_ops.cpp:16-23): y = y / (1 + exp(-z)). */
ANE_CUDA_API int ane_cuda_mul_sigmoid_inplace(int dtype, void* y, const void* z, int64_t n, void* stream);

/* ---- softmax ------------------------------------------------------------
 * softmax (core/cpu_ops.cpp:83-99), in place on fp32 rows: max, subtract,
 * exp, sum, multiply by 1/sum. */
ANE_CUDA_API int ane_cuda_softmax_rows(float* x, int64_t rows, int n, int64_t stride, void* stream);

/* ---- sampler -------------------------------------------------------------
 * sample_token (core/sampling.cpp:10-66) for a batch of rows.  For row r:
 * the last `repetition_context` ids of history[r, 0:history_len[r]] (ids
 * outside [0, vocab) ignored) give a count per distinct id; each such id's
 * logit gets the repetition penalty (x > 0 ? x / p : x * p, when p > 1) and
 * then x -= frequency_penalty * count (when > 0).  temperature <= 0: argmax
 * (first maximum).  Otherwise x *= 1/temperature, softmax, and the result
 * is the first i whose running fp32 sum of probabilities is >= uniforms[r]
 * (vocab - 1 if none).  uniforms[r] plays the part of (float)drand48()
 * (:58).  history / history_len may be NULL (no penalties).  Token ids are
 * bit-exact given the same logits and uniforms. */
ANE_CUDA_API int ane_cuda_sample_rows(const float* logits, int64_t rows, int vocab, int64_t logits_stride,
                         const int32_t* history, const int32_t* history_len,
                         int64_t history_stride, const float* uniforms, float temperature,
                         float repetition_penalty, int repetition_context,
                         float frequency_penalty, int32_t* out_tokens, void* stream);

/* ---- row ops of the hybrid (linear-attention) layers ------------------------
 * ane_cuda_rmsnorm_gated replaces rmsnorm_gated (core/cpu_ops.cpp:33-39,
 * call site models/llm/qwen3_5.cpp:545-550) over rows:
 *   out = ((rmsnorm(x) * w) / (1 + exp(-z))) * z      (eps 1e-6 there).
 * ane_cuda_l2_normalize replaces l2_normalize (core/cpu_ops.cpp:106-111), in
 * place over rows: x = (x * (1 / sqrtf(sum(x^2) + 1e-12))) * scale, scale
 * being the q scaling that follows it (models/llm/qwen3_5.cpp:528-531; 1.0f
 * leaves x as l2_normalize does).  fp32 math, the pinned sum order and exp;
 * bit-exact against the reference in fp32. */
ANE_CUDA_API int ane_cuda_rmsnorm_gated(int dtype, void* out, int64_t out_stride, const void* x,
                                        int64_t x_stride, const void* z, int64_t z_stride,
                                        const float* weight, int64_t rows, int dim, float eps,
                                        void* stream);
ANE_CUDA_API int ane_cuda_l2_normalize(int dtype, void* x, int64_t x_stride, int64_t rows, int dim,
                                       float scale, void* stream);

/* ---- norm-weight loading ----------------------------------------------------
 * Replaces load_bf16_to_f32 (core/safetensors.cpp:264-279; add_one = 0) and
 * the (1 + w) load_norm_weight of the hybrid model (:300-306; add_one = 1):
 * out[i] = bf16_to_f32(in[i]) (+ 1.0f).  Bit-exact. */
ANE_CUDA_API int ane_cuda_bf16_to_f32(float* out, const uint16_t* in, int64_t n, int add_one,
                                      void* stream);

/* ---- fp32 <-> fp16 packing at the ANE boundary ---------------------------
 * Replaces the element loops of ane_matvec (core/ane_runtime.cpp:611-653):
 * input channel c of a token goes to element c * spatial of the fp16
 * surface [channels][spatial] (ANE_SPATIAL = 32, core/ane_runtime.h:10), and
 * output channel c is read back from element c * spatial.  Batched: token t
 * of in[tokens][in_stride] uses surface t / spatial and spatial slot
 * t % spatial of surface [ceil(tokens / spatial)][channels][spatial];
 * elements of slots without a token are not written.  round_mode picks the
 * arm64 conversion (round to nearest even; NaN -> quiet NaN 0x7E00 with the
 * sign) or the x86 one (truncating f32_to_f16: Inf and NaN -> signed Inf).
 * Unpacking widens exactly (NaN payloads kept).  Bit-exact.  spatial 32 with
 * a 16-byte aligned surface takes the tiled path; other sizes are accepted. */
ANE_CUDA_API int ane_cuda_ane_pack(int round_mode, uint16_t* surface, const float* in,
                                   int64_t in_stride, int64_t tokens, int channels, int spatial,
                                   void* stream);
ANE_CUDA_API int ane_cuda_ane_unpack(float* out, int64_t out_stride, const uint16_t* surface,
                                     int64_t tokens, int channels, int spatial, void* stream);

/* ---- decode attention over a ring KV cache ----------------------------
 * Replaces gqa_attention (core/cpu_ops.cpp:173-240, declared at
 * core/cpu_ops.h:55-58) for `batch` sequences of one query token each.
 * Sequence b: q heads at q + b*q_stride + h*q_head_stride; its cache rows
 * [capacity][n_kv_heads][head_dim] at k_cache / v_cache + b*cache_stride;
 * the cache_len[b] keys start at slot cache_start[b] and wrap at
 * cache_capacity (models/llm/qwen3.cpp:475-488).  q head h reads kv head
 * h / (n_heads / n_kv_heads).  out + b*out_stride + h*head_dim receives
 * softmax(q.k / sqrtf(head_dim)) . v, zeros when cache_len[b] <= 0.
 * A (start, len) outside the cache, or len > max_len, writes zeros and
 * sets ANE_CUDA_FLAG_BAD_CACHE.  max_len bounds every cache_len[b] and
 * sizes the launch.  fp32 arithmetic; the reference's softmax-weighted sum
 * with its sums taken in a fixed parallel order (within 1e-6 x max|v| of
 * the reference in fp32).  fp16 / bf16 caches: the two products on the
 * tensor cores with fp32 accumulation and an online softmax; outputs within
 * one unit of the output type (plus 1e-5 x max|v| near zero) of the
 * fixed-order fp32 result.
 * head_dim 64, 128 or 256; at most 8 q heads per kv head; q and the caches
 * 16-byte aligned with strides that keep rows 16-byte aligned.
 * Workspace: ane_cuda_decode_attention_workspace_size() bytes (0 when
 * max_len <= 64), 256-byte aligned, any contents: it holds only the split
 * partials of the call in flight (a second kernel, launched behind the
 * first, merges them), so nothing is kept between calls and nothing needs
 * clearing; calls that share one must be ordered on one stream.
 * workspace == NULL uses a buffer the library allocates per device and
 * stream and keeps until exit; when a larger call needs more it allocates
 * another and keeps the old one too (a captured graph may still use it).
 * That buffer is never allocated during a stream capture: such a call
 * returns ANE_CUDA_ERR_INVALID_ARG -- capture with a caller workspace, or
 * after one eager call of the largest shape on the stream. */
ANE_CUDA_API int64_t ane_cuda_decode_attention_workspace_size(int64_t batch, int n_heads,
                                                              int n_kv_heads, int head_dim,
                                                              int max_len);
ANE_CUDA_API int ane_cuda_decode_attention(int dtype, void* out, int64_t out_stride, const void* q,
                                           int64_t q_stride, int q_head_stride,
                                           const void* k_cache, const void* v_cache,
                                           int64_t cache_stride, const int32_t* cache_start,
                                           const int32_t* cache_len, int cache_capacity,
                                           int64_t batch, int n_heads, int n_kv_heads,
                                           int head_dim, int max_len, void* workspace,
                                           int64_t workspace_bytes, void* stream);

/* ---- decode attention without allocation ----------------------------------
 * No counterpart in the reference (its gqa_attention mallocs a score buffer
 * per call, core/cpu_ops.cpp:191).  The same computation and results as
 * ane_cuda_decode_attention, with the split scratch taken from a fixed
 * array in the library's device image (ane_cuda_decode_attention_static_capacity()
 * bytes per device) instead of a workspace: the call allocates no memory.
 * For callers whose device-memory footprint must not change once running,
 * or that cannot take cudaMalloc's synchronisation in a decode loop.
 * Problems needing more scratch than the capacity are rejected
 * (ANE_CUDA_ERR_INVALID_ARG).  The array is shared by all calls on a
 * device: calls whose executions overlap race on it -- order them on one
 * stream.  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress, with that device current); make that first
 * call before any stream capture on the device (a first call made during a
 * capture returns ANE_CUDA_ERR_INVALID_ARG and leaves the capture intact). */
ANE_CUDA_API int64_t ane_cuda_decode_attention_static_capacity(void);
ANE_CUDA_API int ane_cuda_decode_attention_static(int dtype, void* out, int64_t out_stride,
                                                  const void* q, int64_t q_stride,
                                                  int q_head_stride, const void* k_cache,
                                                  const void* v_cache, int64_t cache_stride,
                                                  const int32_t* cache_start,
                                                  const int32_t* cache_len, int cache_capacity,
                                                  int64_t batch, int n_heads, int n_kv_heads,
                                                  int head_dim, int max_len, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ANE_CUDA_H */
