/*
 * oracle.h -- CPU restatement of ANE-LM's layer-op / sampler / convert path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * kernels: only tests, the smoke check and the benchmark's CPU-baseline
 * leg load it.  Nothing in the product links or calls it.
 *
 * Every function restates one routine of the reference (paths are relative
 * to the ANE-LM source tree) in plain C, and pins the parts the reference
 * leaves to Apple Accelerate (reduction orders, vvexpf) to one explicit
 * definition that the CUDA kernels reproduce bit for bit:
 *
 *   - sum of squares (vDSP_svesq in rmsnorm, core/cpu_ops.cpp:27):
 *     32 "lanes"; the row is cut into chunks of VEC elements (VEC = 16 bytes
 *     / element size); chunk c belongs to lane c % 32; each lane accumulates
 *     acc = fmaf(x, x, acc) over its chunks in increasing order; the 32 lane
 *     sums are combined by an xor butterfly with offsets 16, 8, 4, 2, 1.
 *   - softmax sum (vDSP_sve, core/cpu_ops.cpp:92): 1024 "threads" in 32
 *     groups of 32; groups of 4 consecutive elements go round robin to the
 *     threads; each thread adds its elements in order; an xor butterfly
 *     (16..1) inside each group of 32, then an xor butterfly (16..1) over
 *     the 32 group sums.
 *   - exp (vvexpf, core/cpu_ops.cpp:11,90): ane_expf below, Cody-Waite
 *     reduction by ln 2 and the degree-7 Taylor polynomial, all in fmaf.
 *   - RoPE cos/sin (cosf/sinf of the table in models/llm/qwen3.cpp:200-219):
 *     ane_sincosf below, reduction by pi/2 in double, Taylor polynomials in
 *     float.  inv_freq[j] = 1 / (float)pow(theta, (float)(2j)/rot_dim),
 *     i.e. powf evaluated as the correctly rounded float of the double pow.
 *
 * Parity against Accelerate itself is unpinned (Accelerate is closed and
 * absent on this platform): the definitions above are the contract.  The
 * conversion (common.h), the sampler control flow (core/sampling.cpp) and
 * the gather are integer / control-flow restatements and are checked bit for
 * bit against the reference sources compiled with the shim under shim/.
 */
#ifndef ANE_ORACLE_H
#define ANE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types of activation rows */
enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2 };

/* ---- conversions ---- */
uint16_t or_bf16_to_f16(uint16_t bf);
void     or_bf16_to_f16_vec(uint16_t* out, const uint16_t* in, int64_t n);
uint16_t or_f32_to_f16_rne(float f);
uint16_t or_f32_to_f16_trunc(float f);
uint16_t or_f32_to_bf16_rne(float f);
float    or_f16_to_f32(uint16_t h);
float    or_bf16_to_f32(uint16_t h);

/* ---- pinned math ---- */
float or_expf(float x);
void  or_sincosf(float x, float* s, float* c);
void  or_rope_inv_freq(float* inv_freq, int rot_dim, float theta);
float or_sumsq(const float* x, int dim, int vec);
float or_softmax_sum(const float* e, int n);

/* ---- row ops ---- */
void or_residual_rmsnorm(int dtype, void* x, int64_t x_stride,
                         const void* d, int64_t d_stride,
                         void* out, int64_t out_stride,
                         const float* weight, int64_t rows, int dim, float eps);

void or_rmsnorm_gated(int dtype, void* out, int64_t out_stride, const void* x, int64_t x_stride,
                      const void* z, int64_t z_stride, const float* weight, int64_t rows, int dim,
                      float eps);

void or_l2_normalize(int dtype, void* x, int64_t x_stride, int64_t rows, int dim, float scale);

void or_bf16_to_f32_weights(float* out, const uint16_t* in, int64_t n, int add_one);

void or_qk_norm_rope(int dtype, void* q, void* k,
                     int64_t q_row_stride, int64_t k_row_stride,
                     int q_head_stride, int k_head_stride,
                     int n_q_heads, int n_kv_heads, int head_dim, int rot_dim,
                     const float* q_weight, const float* k_weight,
                     const int32_t* positions, int64_t rows,
                     float theta, float eps);

void or_apply_rope_interleaved(float* q, float* k, int n_q_heads, int n_kv_heads,
                               int q_head_stride, int k_head_stride, int rot_dim, int pos,
                               float theta);

void or_qk_norm_rope_kv(int dtype, void* q, void* k, const void* v, int64_t q_row_stride,
                        int64_t k_row_stride, int64_t v_row_stride, int q_head_stride,
                        int k_head_stride, int v_head_stride, int n_q_heads, int n_kv_heads,
                        int head_dim, const float* q_weight, const float* k_weight,
                        const int32_t* positions, void* k_cache, void* v_cache,
                        int64_t cache_row_stride, const int32_t* slots, int64_t rows,
                        float theta, float eps);

void or_silu_mul(int dtype, void* out, int64_t out_stride,
                 const void* gate, int64_t gate_stride,
                 const void* up, int64_t up_stride,
                 int64_t rows, int n);

int64_t or_embedding_gather(void* out, int out_dtype, const void* table,
                            int table_dtype, const int32_t* ids,
                            int64_t rows, int vocab, int hidden);

void or_softmax_rows(float* x, int64_t rows, int n, int64_t stride);

/* ---- fp32 <-> fp16 at the ANE boundary (core/ane_runtime.cpp:611-653) ---- */
void or_ane_pack(int round_mode, uint16_t* surface, const float* in, int64_t in_stride,
                 int64_t tokens, int channels, int spatial);
void or_ane_unpack(float* out, int64_t out_stride, const uint16_t* surface, int64_t tokens,
                   int channels, int spatial);

/* ---- decode attention (core/cpu_ops.cpp:173-240) ---- */
void or_decode_attention(int dtype, void* out, int64_t out_stride,
                         const void* q, int64_t q_stride, int q_head_stride,
                         const void* k_cache, const void* v_cache, int64_t cache_stride,
                         const int32_t* cache_start, const int32_t* cache_len, int capacity,
                         int64_t batch, int n_heads, int n_kv_heads, int head_dim);

/* KV ring bookkeeping of models/llm/qwen3.cpp:475-484: the slot the new
 * token goes to; start / len updated in place. */
int or_kv_ring_advance(int32_t* start, int32_t* len, int capacity);

/* ---- sampler ---- */
void or_sample_rows(const float* logits, int64_t rows, int vocab,
                    int64_t logits_stride,
                    const int32_t* history, const int32_t* history_len,
                    int64_t history_stride, const float* uniforms,
                    float temperature, float repetition_penalty,
                    int repetition_context, float frequency_penalty,
                    int32_t* out_tokens);

#ifdef __cplusplus
}
#endif
#endif
