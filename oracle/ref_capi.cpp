/*
 * ref_capi.cpp -- extern "C" entry points into the REFERENCE's own sources
 * (core/cpu_ops.cpp, core/sampling.cpp, core/safetensors.cpp,
 * include/ane_lm/common.h), compiled against the stand-in headers in shim/.
 *
 * TEST INFRASTRUCTURE ONLY: it lets the tests check the C restatement in
 * oracle.c against the reference code itself, and lets the benchmark time
 * the reference's CPU path.  The reference sources are compiled where they
 * lie; nothing of them is copied into this repository.  Built by
 * oracle/Makefile into oracle/_ref/.
 */
#include <ane_lm/common.h>
#include "cpu_ops.h"
#include "sampling.h"
#include "safetensors.h"

#include <cstdlib>
#include <cstring>
#include <vector>

extern "C" {

void ref_bf16_to_f16_vec(uint16_t* out, const uint16_t* in, int64_t n) {
    while (n > 0) {
        int chunk = n > (1 << 30) ? (1 << 30) : (int)n;
        ane_lm::bf16_to_f16_vec(out, in, chunk);
        out += chunk; in += chunk; n -= chunk;
    }
}

uint16_t ref_f32_to_f16(float f) { return ane_lm::f32_to_f16(f); }
float ref_f16_to_f32(uint16_t h) { return ane_lm::f16_to_f32(h); }

/* The element conversions of ane_matvec's x86 branch
 * (core/ane_runtime.cpp:625-627 and :646-648), over arrays. */
void ref_f32_to_f16_vec(uint16_t* out, const float* in, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = ane_lm::f32_to_f16(in[i]);
}
void ref_f16_to_f32_vec(float* out, const uint16_t* in, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = ane_lm::f16_to_f32(in[i]);
}

void ref_rmsnorm(float* out, const float* x, const float* w, int dim, float eps) {
    ane_lm::rmsnorm(out, x, w, dim, eps);
}

void ref_apply_rope_cached(float* q, float* k, int nq, int nkv, int hd, int qhs, int khs,
                           int rot, int pos, float theta, const float* cos_row, const float* sin_row) {
    ane_lm::apply_rope_cached(q, k, nq, nkv, hd, qhs, khs, rot, pos, theta, cos_row, sin_row);
}

/* The RoPE table exactly as the model builds it (models/llm/qwen3.cpp:205-216)
 * with the platform libm powf / cosf / sinf. */
void ref_rope_row(float* cos_row, float* sin_row, int pos, int rot_dim, float theta) {
    int half = rot_dim / 2;
    std::vector<float> inv_freq((size_t)half);
    for (int j2 = 0, i = 0; i < rot_dim; i += 2, j2++)
        inv_freq[(size_t)j2] = 1.0f / powf(theta, (float)i / (float)rot_dim);
    for (int j2 = 0; j2 < half; j2++) {
        float angle = pos * inv_freq[(size_t)j2];
        cos_row[j2] = cosf(angle);
        sin_row[j2] = sinf(angle);
    }
}

void ref_silu_vec_inplace(float* x, int n) {
    std::vector<float> tmp((size_t)n);
    ane_lm::silu_vec_inplace(x, n, tmp.data());
}

void ref_softmax(float* x, int n) { ane_lm::softmax(x, n); }

/* sample_token with its drand48 draw fixed by `seed`; the draw it used is
 * returned in *u_out as (float)drand48(), the value the reference compares
 * against (core/sampling.cpp:58). */
int ref_sample_token(const float* logits, int vocab, float temperature, float rep, int ctx,
                     float freq, const int32_t* hist, int hist_len, long seed, float* u_out) {
    ane_lm::SamplingParams p;
    p.temperature = temperature;
    p.repetition_penalty = rep;
    p.repetition_context_size = ctx;
    p.frequency_penalty = freq;
    std::vector<int> h(hist, hist + (hist_len > 0 ? hist_len : 0));
    srand48(seed);
    double u = drand48();
    srand48(seed);
    int tok = ane_lm::sample_token(logits, vocab, p, h);
    if (u_out) *u_out = (float)u;
    return tok;
}

/* The decode loop's use of sample_token (generate.cpp:80, :129; the
 * generated tokens are the history, :87):
 * srand48(seed) once, then `steps` calls, each appending the token it
 * returns to the history; step i reads logits row i % nrows. */
void ref_sample_token_loop(const float* logits, int nrows, int vocab, float temperature,
                           float rep, int ctx, float freq, const int32_t* hist0, int hist0_len,
                           long seed, int steps, int32_t* tokens_out) {
    ane_lm::SamplingParams p;
    p.temperature = temperature;
    p.repetition_penalty = rep;
    p.repetition_context_size = ctx;
    p.frequency_penalty = freq;
    std::vector<int> recent(hist0, hist0 + (hist0_len > 0 ? hist0_len : 0));
    srand48(seed);
    for (int i = 0; i < steps; i++) {
        int tok = ane_lm::sample_token(logits + (size_t)(i % nrows) * vocab, vocab, p, recent);
        tokens_out[i] = tok;
        recent.push_back(tok);
    }
}

/* rmsnorm_gated (core/cpu_ops.cpp:33-39) and l2_normalize (:106-111). */
void ref_rmsnorm_gated(float* out, const float* x, const float* z, const float* w, int dim) {
    ane_lm::rmsnorm_gated(out, x, z, w, dim);
}
void ref_l2_normalize(float* x, int dim) { ane_lm::l2_normalize(x, dim); }

/* SafeTensors::load_norm_weight (core/safetensors.cpp:300-306) and
 * load_bf16_to_f32 (:264-279) of one tensor; 0 on success. */
int ref_load_weight(const char* path, const char* name, int64_t n, int norm, float* out) {
    ane_lm::SafeTensors* sf = ane_lm::SafeTensors::open(path);
    if (!sf) return -1;
    float* w = norm ? sf->load_norm_weight(name, n) : sf->load_bf16_to_f32(name, n);
    delete sf;
    if (!w) return -2;
    memcpy(out, w, (size_t)n * sizeof(float));
    free(w);
    return 0;
}

/* gqa_attention (core/cpu_ops.cpp:173-240) for one query token. */
void ref_gqa_attention(float* out, const float* q, const float* k_cache, const float* v_cache,
                       int n_heads, int n_kv_heads, int head_dim, int q_head_stride,
                       int cache_start, int cache_len, int cache_capacity) {
    ane_lm::gqa_attention(out, q, k_cache, v_cache, n_heads, n_kv_heads, head_dim, q_head_stride,
                          cache_start, cache_len, cache_capacity);
}

/* `ane-lm convert` for one safetensors file: SafeTensors::open followed by
 * SafeTensors::write_ane_blobs (core/safetensors.cpp:203-245, :345-383). */
int ref_write_ane_blobs(const char* safetensors_path, const char* out_dir) {
    ane_lm::SafeTensors* sf = ane_lm::SafeTensors::open(safetensors_path);
    if (!sf) return -1;
    int n = ane_lm::SafeTensors::write_ane_blobs(*sf, out_dir);
    delete sf;
    return n;
}

static inline uint16_t rne_f16(float f) { return or_f32_to_f16_rne(f); }

/* One Qwen3 layer's CPU op chain over rows [r0, r1) of a batched-prefill
 * buffer set with fp16 storage, built from the reference routines:
 *   x += d; y = rmsnorm(x)                    (qwen3.cpp:516-518)
 *   per-head rmsnorm of q and k, then RoPE    (qwen3.cpp:444-473)
 *   h = silu(gate) * up                       (cpu_ops.cpp:7-14)
 * fp16 rows are widened to fp32 for the reference calls and rounded back
 * to nearest-even on store, as the ANE boundary does on arm64. */
void ref_layer_chain_f16(uint16_t* x, const uint16_t* d, uint16_t* y, const float* norm_w,
                         uint16_t* qkv, const float* qw, const float* kw, const int32_t* pos,
                         const uint16_t* gate, const uint16_t* up, uint16_t* hout,
                         int64_t r0, int64_t r1, int hidden, int nq, int nkv, int hd,
                         int inter, float theta, float eps) {
    std::vector<float> xf((size_t)hidden), yf((size_t)hidden);
    int qkv_w = (nq + 2 * nkv) * hd;
    std::vector<float> qf((size_t)(nq + nkv) * hd);
    std::vector<float> cs((size_t)hd / 2), sn((size_t)hd / 2);
    std::vector<float> gf((size_t)inter), tmp((size_t)inter);
    for (int64_t r = r0; r < r1; r++) {
        uint16_t* xr = x + r * hidden;
        const uint16_t* dr = d + r * hidden;
        for (int i = 0; i < hidden; i++) {
            float s = ane_lm::f16_to_f32(xr[i]) + ane_lm::f16_to_f32(dr[i]);
            xr[i] = rne_f16(s);
            xf[(size_t)i] = ane_lm::f16_to_f32(xr[i]);
        }
        ane_lm::rmsnorm(yf.data(), xf.data(), norm_w, hidden, eps);
        for (int i = 0; i < hidden; i++) y[r * hidden + i] = rne_f16(yf[(size_t)i]);

        uint16_t* qr = qkv + r * qkv_w;
        for (int i = 0; i < (nq + nkv) * hd; i++) qf[(size_t)i] = ane_lm::f16_to_f32(qr[i]);
        for (int h = 0; h < nq + nkv; h++) {
            float* vh = qf.data() + (size_t)h * hd;
            ane_lm::rmsnorm(vh, vh, h < nq ? qw : kw, hd, eps);
        }
        ref_rope_row(cs.data(), sn.data(), pos[r], hd, theta);
        ane_lm::apply_rope_cached(qf.data(), qf.data() + (size_t)nq * hd, nq, nkv, hd, hd, hd, hd,
                                  pos[r], theta, cs.data(), sn.data());
        for (int i = 0; i < (nq + nkv) * hd; i++) qr[i] = rne_f16(qf[(size_t)i]);

        const uint16_t* gr = gate + r * inter;
        const uint16_t* ur = up + r * inter;
        for (int i = 0; i < inter; i++) gf[(size_t)i] = ane_lm::f16_to_f32(gr[i]);
        ane_lm::silu_vec_inplace(gf.data(), inter, tmp.data());
        for (int i = 0; i < inter; i++)
            hout[r * inter + i] = rne_f16(gf[(size_t)i] * ane_lm::f16_to_f32(ur[i]));
    }
}

}  // extern "C"
