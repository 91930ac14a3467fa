/*
 * oracle.c -- CPU restatement of ANE-LM's layer-op / sampler / convert path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or
 * shipped).  See oracle.h for the pinned definitions of what the reference
 * leaves to Apple Accelerate.  Compile with -ffp-contract=off so that every
 * multiply and add rounds on its own, exactly like the reference's vDSP
 * element-wise calls and like the CUDA kernels' explicit __f*_rn intrinsics.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* bit helpers                                                         */
/* ------------------------------------------------------------------ */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------ */
/* Conversions                                                         */
/* ------------------------------------------------------------------ */

/* BF16 -> FP16 through FP32 with the reference's TRUNCATING f32_to_f16:
 * include/ane_lm/common.h:21-26 (bf16_to_f32), :58-71 (f32_to_f16),
 * :73-75 (bf16_to_f16).  Exponent re-bias by -112; exponent >= 31 (this
 * includes Inf and NaN) saturates to signed Inf; exponent <= 0 shifts the
 * mantissa (with its hidden bit) right and drops the low bits; below
 * 2^-25 the result is a signed zero. */
uint16_t or_bf16_to_f16(uint16_t bf) {
    uint32_t bits = (uint32_t)bf << 16;
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t e = (int32_t)((bits >> 23) & 0xFFu) - 112;
    uint32_t frac = bits & 0x7FFFFFu;
    if (e <= 0) {
        if (e < -10) return sign;
        return (uint16_t)(sign | (uint16_t)((((frac | 0x800000u) >> (1 - e)) >> 13)));
    }
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | (uint16_t)(e << 10) | (uint16_t)(frac >> 13));
}

/* include/ane_lm/common.h:81-83 */
void or_bf16_to_f16_vec(uint16_t* out, const uint16_t* in, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = or_bf16_to_f16(in[i]);
}

/* Round-to-nearest-even FP32 -> FP16, the rounding of a native __fp16 store
 * on arm64 (core/ane_runtime.cpp:604-609, :624), used for activations. */
uint16_t or_f32_to_f16_rne(float f) {
    uint32_t u = f2u(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);      /* NaN */
    if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);     /* >= 65520 */
    if (a < 0x38800000u) {                                        /* < 2^-14 */
        if (a < 0x33000000u) return sign;                         /* <= 2^-25 */
        uint32_t e = a >> 23;
        uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        uint32_t sh = 126u - e;                                   /* 14..24 */
        uint32_t q = m >> sh;
        uint32_t rem = m & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e16 = (a >> 23) - 112u;
    uint32_t q = (e16 << 10) | ((a & 0x7FFFFFu) >> 13);
    uint32_t rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

uint16_t or_f32_to_bf16_rne(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

/* The reference's truncating f32_to_f16 (include/ane_lm/common.h:58-71),
 * used by the x86 branch of the ANE input packing (core/ane_runtime.cpp:
 * 625-627): exponent re-bias by -112; >= 31 (Inf and NaN too) -> signed Inf;
 * <= 0 -> the mantissa with its hidden bit shifted right, low bits dropped;
 * below 2^-25 -> signed zero. */
uint16_t or_f32_to_f16_trunc(float f) {
    uint32_t u = f2u(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    int32_t e = (int32_t)((u >> 23) & 0xFFu) - 112;
    uint32_t frac = u & 0x7FFFFFu;
    if (e <= 0) {
        if (e < -10) return sign;
        return (uint16_t)(sign | (uint16_t)(((frac | 0x800000u) >> (1 - e)) >> 13));
    }
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | (uint16_t)(e << 10) | (uint16_t)(frac >> 13));
}

/* include/ane_lm/common.h:35-56 (exact widening) */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    if (e == 0) {
        float v = (float)m * (1.0f / 16777216.0f);                /* m * 2^-24, exact */
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

float or_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* ------------------------------------------------------------------ */
/* Pinned math                                                         */
/* ------------------------------------------------------------------ */

/* exp for vvexpf (core/cpu_ops.cpp:11,20,90).  Method: Cody & Waite (1980)
 * argument reduction x = k ln2 + r with k = rint(x log2 e) and ln 2 split
 * into a float head and tail, then the Taylor series of e^r to degree 7 by
 * Horner's rule, then scaling by 2^k with at most two exact-or-once-rounded
 * multiplies.  Constants are ln 2 and 1/n! rounded to float. */
#define EXP_LOG2E  1.44269502162933349609375f       /* 0x3fb8aa3b */
#define EXP_LN2_HI 0.693147182464599609375f         /* 0x3f317218 */
#define EXP_LN2_LO (-1.904654212125933608e-09f)     /* 0xb102e308 */
#define INV_FACT3  0.16666667163372039794921875f
#define INV_FACT4  0.041666667908430099487304688f
#define INV_FACT5  0.0083333337679505348205566406f
#define INV_FACT6  0.0013888889225199818611145020f
#define INV_FACT7  0.00019841270113829523324966431f

static inline float pow2i(int k) { return u2f((uint32_t)(k + 127) << 23); } /* k in [-126,127] */

float or_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return u2f(0x7F800000u);
    if (x < -104.0f) return 0.0f;
    float k = rintf(x * EXP_LOG2E);
    float r = fmaf(-k, EXP_LN2_HI, x);
    r = fmaf(-k, EXP_LN2_LO, r);
    float p = fmaf(INV_FACT7, r, INV_FACT6);
    p = fmaf(p, r, INV_FACT5);
    p = fmaf(p, r, INV_FACT4);
    p = fmaf(p, r, INV_FACT3);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ki = (int)k;
    if (ki > 127) return (p * 2.0f) * pow2i(127);
    if (ki < -126) return (p * pow2i(ki + 64)) * pow2i(-64);
    return p * pow2i(ki);
}

/* sin/cos for the RoPE table (cosf/sinf at models/llm/qwen3.cpp:214-215).
 * Method: Cody-Waite reduction by pi/2 carried out in double (pi/2 as a
 * double head plus tail, two fma), the reduced argument rounded to float,
 * Taylor polynomials of sin (degree 9) and cos (degree 10) in float by
 * Horner's rule with fmaf, then the quadrant rotation. */
#define SC_TWO_OVER_PI 0x1.45f306dc9c883p-1
#define SC_PIO2_HI     0x1.921fb54442d18p+0
#define SC_PIO2_LO     0x1.1a62633145c07p-54
#define SIN_C1 (-0.16666667163372039794921875f)
#define SIN_C2   0.0083333337679505348205566406f
#define SIN_C3 (-0.00019841270113829523324966431f)
#define SIN_C4   2.7557318844628753e-06f
#define COS_C1 (-0.5f)
#define COS_C2   0.041666667908430099487304688f
#define COS_C3 (-0.0013888889225199818611145020f)
#define COS_C4   2.4801587642286904e-05f
#define COS_C5 (-2.755731998149713e-07f)

void or_sincosf(float x, float* s, float* c) {
    double xd = (double)x;
    double kd = rint(xd * SC_TWO_OVER_PI);
    double rd = fma(-kd, SC_PIO2_HI, xd);
    rd = fma(-kd, SC_PIO2_LO, rd);
    float r = (float)rd;
    int q = (int)(kd - 4.0 * floor(kd * 0.25));
    float r2 = r * r;
    float t = fmaf(SIN_C4, r2, SIN_C3);
    t = fmaf(t, r2, SIN_C2);
    t = fmaf(t, r2, SIN_C1);
    t = t * r2;
    float sp = fmaf(t, r, r);
    float u = fmaf(COS_C5, r2, COS_C4);
    u = fmaf(u, r2, COS_C3);
    u = fmaf(u, r2, COS_C2);
    u = fmaf(u, r2, COS_C1);
    float cp = fmaf(u, r2, 1.0f);
    switch (q) {
        case 0:  *s = sp;  *c = cp;  break;
        case 1:  *s = cp;  *c = -sp; break;
        case 2:  *s = -sp; *c = -cp; break;
        default: *s = -cp; *c = sp;  break;
    }
}

/* inv_freq table of models/llm/qwen3.cpp:205-208:
 * inv_freq[j] = 1.0f / powf(theta, (float)(2j) / (float)rot_dim),
 * with powf taken as the float rounding of the double pow. */
void or_rope_inv_freq(float* inv_freq, int rot_dim, float theta) {
    for (int j = 0; 2 * j < rot_dim; j++) {
        float e = (float)(2 * j) / (float)rot_dim;
        float p = (float)pow((double)theta, (double)e);
        inv_freq[j] = 1.0f / p;
    }
}

/* vDSP_svesq of core/cpu_ops.cpp:27 with the pinned 32-lane order. */
float or_sumsq(const float* x, int dim, int vec) {
    float acc[32];
    for (int l = 0; l < 32; l++) acc[l] = 0.0f;
    int nchunk = (dim + vec - 1) / vec;
    for (int ch = 0; ch < nchunk; ch++) {
        int l = ch & 31;
        int end = (ch + 1) * vec < dim ? (ch + 1) * vec : dim;
        for (int e = ch * vec; e < end; e++) acc[l] = fmaf(x[e], x[e], acc[l]);
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float nx[32];
        for (int l = 0; l < 32; l++) nx[l] = acc[l] + acc[l ^ off];
        memcpy(acc, nx, sizeof(acc));
    }
    return acc[0];
}

/* vDSP_sve of core/cpu_ops.cpp:92 with the pinned 1024-thread order. */
float or_softmax_sum(const float* e, int n) {
    static const int T = 1024;
    float acc[1024];
    for (int t = 0; t < T; t++) acc[t] = 0.0f;
    for (int i = 0; i < n; i++) {
        int t = (i >> 2) & (T - 1);
        acc[t] = acc[t] + e[i];
    }
    float w[32];
    for (int g = 0; g < 32; g++) {
        float* a = acc + 32 * g;
        for (int off = 16; off >= 1; off >>= 1) {
            float nx[32];
            for (int l = 0; l < 32; l++) nx[l] = a[l] + a[l ^ off];
            memcpy(a, nx, sizeof(nx));
        }
        w[g] = a[0];
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float nx[32];
        for (int l = 0; l < 32; l++) nx[l] = w[l] + w[l ^ off];
        memcpy(w, nx, sizeof(nx));
    }
    return w[0];
}

/* ------------------------------------------------------------------ */
/* element access by dtype                                             */
/* ------------------------------------------------------------------ */
static inline float ld(const void* p, int dt, int64_t i) {
    if (dt == OR_F32) return ((const float*)p)[i];
    if (dt == OR_F16) return or_f16_to_f32(((const uint16_t*)p)[i]);
    return or_bf16_to_f32(((const uint16_t*)p)[i]);
}
static inline void st(void* p, int dt, int64_t i, float v) {
    if (dt == OR_F32) ((float*)p)[i] = v;
    else if (dt == OR_F16) ((uint16_t*)p)[i] = or_f32_to_f16_rne(v);
    else ((uint16_t*)p)[i] = or_f32_to_bf16_rne(v);
}
static inline int vec_of(int dt) { return dt == OR_F32 ? 4 : 8; }

/* rmsnorm, core/cpu_ops.cpp:25-31:
 *   inv = 1 / sqrtf(sumsq / dim + eps); out = (x * inv) * w   (two roundings)
 * preceded, when d is given, by the residual add of models/llm/qwen3.cpp:516
 * and :527 (x += d).  The sum is stored back into x in x's dtype and the
 * norm reads the stored value, as an unfused add-then-norm would. */
void or_residual_rmsnorm(int dt, void* x, int64_t xs, const void* d, int64_t ds,
                         void* out, int64_t os, const float* w,
                         int64_t rows, int dim, float eps) {
    float* v = (float*)malloc((size_t)dim * sizeof(float));
    for (int64_t r = 0; r < rows; r++) {
        for (int i = 0; i < dim; i++) {
            float xv = ld(x, dt, r * xs + i);
            if (d) {
                float s = xv + ld(d, dt, r * ds + i);
                st(x, dt, r * xs + i, s);
                xv = ld(x, dt, r * xs + i);
            }
            v[i] = xv;
        }
        float ss = or_sumsq(v, dim, vec_of(dt));
        float inv = 1.0f / sqrtf(ss / (float)dim + eps);
        for (int i = 0; i < dim; i++) {
            float y = v[i] * inv;
            y = y * w[i];
            st(out, dt, r * os + i, y);
        }
    }
    free(v);
}

/* rmsnorm_gated, core/cpu_ops.cpp:33-39, over rows:
 *   y = rmsnorm(x) * w                 (:25-31, eps as given; 1e-6 there)
 *   y = y / (1 + exp(-z))              (mul_sigmoid_inplace, :16-23)
 *   y = y * z                          (vDSP_vmul, :38)
 * in fp32, rounded once to the row type at the end. */
void or_rmsnorm_gated(int dt, void* out, int64_t os, const void* x, int64_t xs,
                      const void* z, int64_t zs, const float* w, int64_t rows, int dim, float eps) {
    float* v = (float*)malloc((size_t)dim * sizeof(float));
    for (int64_t r = 0; r < rows; r++) {
        for (int i = 0; i < dim; i++) v[i] = ld(x, dt, r * xs + i);
        float ss = or_sumsq(v, dim, vec_of(dt));
        float inv = 1.0f / sqrtf(ss / (float)dim + eps);
        for (int i = 0; i < dim; i++) {
            float zv = ld(z, dt, r * zs + i);
            float y = v[i] * inv;
            y = y * w[i];
            float den = 1.0f + or_expf(-zv);
            y = y / den;
            y = y * zv;
            st(out, dt, r * os + i, y);
        }
    }
    free(v);
}

/* l2_normalize, core/cpu_ops.cpp:106-111, in place over rows:
 * inv = 1 / sqrtf(sum(x^2) + 1e-12); x = x * inv; then x = x * scale (the
 * q scaling of models/llm/qwen3_5.cpp:530-531; 1 leaves x unchanged). */
void or_l2_normalize(int dt, void* x, int64_t xs, int64_t rows, int dim, float scale) {
    float* v = (float*)malloc((size_t)dim * sizeof(float));
    for (int64_t r = 0; r < rows; r++) {
        for (int i = 0; i < dim; i++) v[i] = ld(x, dt, r * xs + i);
        float inv = 1.0f / sqrtf(or_sumsq(v, dim, vec_of(dt)) + 1e-12f);
        for (int i = 0; i < dim; i++) {
            float y = v[i] * inv;
            y = y * scale;
            st(x, dt, r * xs + i, y);
        }
    }
    free(v);
}

/* Norm-weight loading: load_bf16_to_f32 (core/safetensors.cpp:264-279,
 * bf16_to_f32_vec) and, with add_one, the (1 + w) form of load_norm_weight
 * (:300-306): w = bf16_to_f32(b) + 1.0f. */
void or_bf16_to_f32_weights(float* out, const uint16_t* in, int64_t n, int add_one) {
    for (int64_t i = 0; i < n; i++) {
        float w = or_bf16_to_f32(in[i]);
        out[i] = add_one ? w + 1.0f : w;
    }
}

/* Per-head QK-norm (models/llm/qwen3.cpp:444-461, rmsnorm of each head with
 * q_norm / k_norm) followed by half-split RoPE (core/cpu_ops.cpp:43-54,
 * :56-66; models/llm/qwen3.cpp:17-52):
 *   v[j]      = v[j] * cos - v[j+half] * sin
 *   v[j+half] = v[j+half] * cos + v[j] * sin        (unfused, as vmmsb/vmma)
 * with half = rot_dim / 2; elements past rot_dim are only normalised. */
void or_qk_norm_rope(int dt, void* q, void* k, int64_t qrs, int64_t krs,
                     int qhs, int khs, int nq, int nkv, int hd, int rot,
                     const float* qw, const float* kw, const int32_t* pos,
                     int64_t rows, float theta, float eps) {
    int half = rot / 2;
    float* inv_freq = (float*)malloc((size_t)(half > 0 ? half : 1) * sizeof(float));
    float* cs = (float*)malloc((size_t)(half > 0 ? half : 1) * sizeof(float));
    float* sn = (float*)malloc((size_t)(half > 0 ? half : 1) * sizeof(float));
    float* v = (float*)malloc((size_t)hd * sizeof(float));
    or_rope_inv_freq(inv_freq, rot, theta);
    for (int64_t r = 0; r < rows; r++) {
        float fp = (float)pos[r];
        for (int j = 0; j < half; j++) or_sincosf(fp * inv_freq[j], &sn[j], &cs[j]);
        for (int h = 0; h < nq + nkv; h++) {
            void* base = h < nq ? q : k;
            int64_t off = h < nq ? r * qrs + (int64_t)h * qhs
                                 : r * krs + (int64_t)(h - nq) * khs;
            const float* w = h < nq ? qw : kw;
            for (int i = 0; i < hd; i++) v[i] = ld(base, dt, off + i);
            float ss = or_sumsq(v, hd, vec_of(dt));
            float inv = 1.0f / sqrtf(ss / (float)hd + eps);
            for (int i = 0; i < hd; i++) { float y = v[i] * inv; v[i] = y * w[i]; }
            for (int j = 0; j < half; j++) {
                float a = v[j], b = v[j + half];
                float ac = a * cs[j], bs = b * sn[j];
                float bc = b * cs[j], as = a * sn[j];
                v[j] = ac - bs;
                v[j + half] = bc + as;
            }
            for (int i = 0; i < hd; i++) st(base, dt, off + i, v[i]);
        }
    }
    free(inv_freq); free(cs); free(sn); free(v);
}

/* apply_rope_cached without tables: the reference's on-the-fly fallback,
 * core/cpu_ops.cpp:66-77 (taken when cos_row or sin_row is NULL), on fp32
 * heads in place: for each pair (i, i+1), i = 2j < rot_dim,
 *   freq = 1 / powf(theta, i / rot_dim), angle = pos * freq,
 *   v[i]   = v0 * cos - v1 * sin
 *   v[i+1] = v0 * sin + v1 * cos                    (unfused)
 * with powf / cosf / sinf taken as the pinned inv_freq and sincos above. */
void or_apply_rope_interleaved(float* q, float* k, int nq, int nkv, int qhs, int khs, int rot,
                               int pos, float theta) {
    int half = rot / 2;
    float* inv_freq = (float*)malloc((size_t)(half > 0 ? half : 1) * sizeof(float));
    or_rope_inv_freq(inv_freq, rot, theta);
    for (int h = 0; h < nq + nkv; h++) {
        float* v = h < nq ? q + (int64_t)h * qhs : k + (int64_t)(h - nq) * khs;
        for (int j = 0; j < half; j++) {
            float c, s;
            or_sincosf((float)pos * inv_freq[j], &s, &c);
            float v0 = v[2 * j], v1 = v[2 * j + 1];
            float a = v0 * c, b = v1 * s, d = v0 * s, e = v1 * c;
            v[2 * j] = a - b;
            v[2 * j + 1] = d + e;
        }
    }
    free(inv_freq);
}

/* QK-norm + RoPE followed by the KV-cache write of the decode step,
 * models/llm/qwen3.cpp:470-488: after RoPE, the token's k heads and its v
 * heads are copied (memcpy) into ring slot slots[r] of the caches
 * [slot][n_kv][hd] at cache + r * crs; slots[r] < 0 copies nothing. */
void or_qk_norm_rope_kv(int dt, void* q, void* k, const void* v, int64_t qrs, int64_t krs,
                        int64_t vrs, int qhs, int khs, int vhs, int nq, int nkv, int hd,
                        const float* qw, const float* kw, const int32_t* pos, void* k_cache,
                        void* v_cache, int64_t crs, const int32_t* slots, int64_t rows,
                        float theta, float eps) {
    or_qk_norm_rope(dt, q, k, qrs, krs, qhs, khs, nq, nkv, hd, hd, qw, kw, pos, rows, theta, eps);
    const size_t es = dt == OR_F32 ? 4 : 2;
    for (int64_t r = 0; r < rows; r++) {
        if (slots[r] < 0) continue;
        for (int j = 0; j < nkv; j++) {
            const int64_t dst = (r * crs + ((int64_t)slots[r] * nkv + j) * hd) * (int64_t)es;
            memcpy((char*)k_cache + dst, (const char*)k + (r * krs + (int64_t)j * khs) * (int64_t)es, hd * es);
            memcpy((char*)v_cache + dst, (const char*)v + (r * vrs + (int64_t)j * vhs) * (int64_t)es, hd * es);
        }
    }
}

/* SiLU-gated activation: silu_vec_inplace (core/cpu_ops.cpp:7-14,
 * x / (1 + exp(-x))) times up, the gate*sigmoid(gate)*up of the fused FFN
 * (core/ane_runtime.cpp:393-395) evaluated in fp32. */
void or_silu_mul(int dt, void* out, int64_t os, const void* g, int64_t gs,
                 const void* u, int64_t us, int64_t rows, int n) {
    for (int64_t r = 0; r < rows; r++) {
        for (int i = 0; i < n; i++) {
            float gv = ld(g, dt, r * gs + i);
            float den = 1.0f + or_expf(-gv);
            float s = gv / den;
            float h = s * ld(u, dt, r * us + i);
            st(out, dt, r * os + i, h);
        }
    }
}

/* Embedding gather, models/llm/qwen3.cpp:498 (memcpy of row token*hidden),
 * batched.  Rows whose id is outside [0, vocab) are written as zeros and
 * counted.  out_dtype is the table's dtype (byte copy) or F32 from an
 * F16/BF16 table (exact widening). */
int64_t or_embedding_gather(void* out, int odt, const void* table, int tdt,
                            const int32_t* ids, int64_t rows, int vocab, int hidden) {
    int64_t bad = 0;
    size_t tes = tdt == OR_F32 ? 4 : 2, oes = odt == OR_F32 ? 4 : 2;
    for (int64_t r = 0; r < rows; r++) {
        int32_t id = ids[r];
        char* o = (char*)out + (size_t)r * hidden * oes;
        if (id < 0 || id >= vocab) { memset(o, 0, (size_t)hidden * oes); bad++; continue; }
        const char* t = (const char*)table + (size_t)id * hidden * tes;
        if (odt == tdt) memcpy(o, t, (size_t)hidden * tes);
        else for (int i = 0; i < hidden; i++) ((float*)o)[i] = ld(t, tdt, i);
    }
    return bad;
}

/* softmax, core/cpu_ops.cpp:83-99, in place over rows:
 * max (vDSP_maxv), x + (-max) (vDSP_vsadd), exp (vvexpf), sum (vDSP_sve,
 * pinned order), x * (1 / sum) (vDSP_vsmul). */
void or_softmax_rows(float* x, int64_t rows, int n, int64_t stride) {
    for (int64_t r = 0; r < rows; r++) {
        float* v = x + r * stride;
        float mx = v[0];
        for (int i = 1; i < n; i++) if (v[i] > mx) mx = v[i];
        float nmx = -mx;
        for (int i = 0; i < n; i++) v[i] = or_expf(v[i] + nmx);
        float inv = 1.0f / or_softmax_sum(v, n);
        for (int i = 0; i < n; i++) v[i] *= inv;
    }
}

/* ------------------------------------------------------------------ */
/* Decode attention over a ring KV cache, core/cpu_ops.cpp:173-240      */
/* ------------------------------------------------------------------ */

/* xor butterfly over n values (offsets n/2 .. 1); every slot ends equal. */
static float butterfly(float* a, int n) {
    float nx[64];
    for (int off = n >> 1; off >= 1; off >>= 1) {
        for (int l = 0; l < n; l++) nx[l] = a[l] + a[l ^ off];
        memcpy(a, nx, (size_t)n * sizeof(float));
    }
    return a[0];
}

/* One query token per sequence against its ring cache.  The reference
 * (core/cpu_ops.cpp:173-240) computes, per q head h of kv head h / groups,
 *   s_t = dot(q_h, k_t) * (1/sqrtf(head_dim)),   t over the cache_len
 *         slots from cache_start, wrapping at cache_capacity (:188-205);
 *   p   = softmax(s) (:207, core/cpu_ops.cpp:83-99);
 *   out = sum_t p_t v_t (:209-219);
 * and zeros when cache_len <= 0 (:176-179).  The summation orders are
 * pinned here (the CUDA kernel does the same operations in the same order):
 *   - dot: EPL = max(16 / element size, head_dim / 32) consecutive elements
 *     per lane, GL = head_dim / EPL lanes; each lane an fmaf chain over its
 *     elements; xor butterfly over the GL lane sums.
 *   - keys in splits of 64; per split j: m_j = max s, e_t = expf(s_t - m_j),
 *     l_j = two 32-lane butterflies (local keys 0-31, 32-63) added;
 *     o_j[d] = U = 4 * (32 / GL) accumulators, accumulator u an fmaf chain
 *     over local keys u, u+U, ...; xor butterfly over each warp's 32/GL
 *     accumulators; the four warp results added in order.
 *   - combine: M = max m_j, f_j = expf(m_j - M); O[d] and L each as four
 *     fmaf chains over splits j = w mod 4, added in order; out = O * (1/L).
 * The result is the reference's softmax-weighted sum with the
 * normalisation applied once at the end (the split-softmax identity). */
#define OR_ATTN_KEYS 64
void or_decode_attention(int dt, void* out, int64_t out_stride,
                         const void* q, int64_t q_stride, int q_head_stride,
                         const void* k_cache, const void* v_cache, int64_t cache_stride,
                         const int32_t* cache_start, const int32_t* cache_len, int capacity,
                         int64_t batch, int n_heads, int n_kv_heads, int head_dim) {
    const int es = dt == OR_F32 ? 4 : 2;
    const int epl = (head_dim / 32 > 16 / es) ? head_dim / 32 : 16 / es;
    const int gl = head_dim / epl;
    const int kpw = 32 / gl;
    const int U = 4 * kpw;
    const int groups = n_heads / n_kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    const int64_t kv_step = (int64_t)n_kv_heads * head_dim;
    float* qf = (float*)malloc((size_t)head_dim * sizeof(float));
    float* kbuf = (float*)malloc((size_t)OR_ATTN_KEYS * head_dim * sizeof(float));
    float* vbuf = (float*)malloc((size_t)OR_ATTN_KEYS * head_dim * sizeof(float));
    float* acc = (float*)malloc((size_t)U * head_dim * sizeof(float));
    float* O = (float*)malloc((size_t)4 * head_dim * sizeof(float));
    for (int64_t b = 0; b < batch; b++) {
        const int len = cache_len[b], start = cache_start[b];
        const int nsplit = len > 0 ? (len + OR_ATTN_KEYS - 1) / OR_ATTN_KEYS : 0;
        float* pm = (float*)malloc((size_t)(nsplit ? nsplit : 1) * sizeof(float));
        float* pl = (float*)malloc((size_t)(nsplit ? nsplit : 1) * sizeof(float));
        float* po = (float*)malloc((size_t)(nsplit ? nsplit : 1) * head_dim * sizeof(float));
        for (int h = 0; h < n_heads; h++) {
            const int kvh = h / groups;
            for (int d = 0; d < head_dim; d++)
                qf[d] = ld(q, dt, b * q_stride + (int64_t)h * q_head_stride + d);
            if (len <= 0) {
                for (int d = 0; d < head_dim; d++) st(out, dt, b * out_stride + (int64_t)h * head_dim + d, 0.0f);
                continue;
            }
            for (int j = 0; j < nsplit; j++) {
                const int t0 = j * OR_ATTN_KEYS;
                const int n = len - t0 < OR_ATTN_KEYS ? len - t0 : OR_ATTN_KEYS;
                float s[OR_ATTN_KEYS], e[OR_ATTN_KEYS];
                for (int i = 0; i < n; i++) {
                    int slot = start + t0 + i;
                    if (slot >= capacity) slot -= capacity;
                    const int64_t off = b * cache_stride + (int64_t)slot * kv_step + (int64_t)kvh * head_dim;
                    for (int d = 0; d < head_dim; d++) {
                        kbuf[i * head_dim + d] = ld(k_cache, dt, off + d);
                        vbuf[i * head_dim + d] = ld(v_cache, dt, off + d);
                    }
                    float lanes[32];
                    for (int l = 0; l < gl; l++) {
                        float a = 0.0f;
                        for (int x = 0; x < epl; x++)
                            a = fmaf(qf[l * epl + x], kbuf[i * head_dim + l * epl + x], a);
                        lanes[l] = a;
                    }
                    s[i] = butterfly(lanes, gl) * scale;
                }
                float m = -INFINITY;
                for (int i = 0; i < n; i++) m = fmaxf(m, s[i]);
                float w32[2][32];
                for (int i = 0; i < OR_ATTN_KEYS; i++) {
                    e[i] = i < n ? or_expf(s[i] - m) : 0.0f;
                    w32[i / 32][i % 32] = e[i];
                }
                const float l0 = butterfly(w32[0], 32), l1 = butterfly(w32[1], 32);
                pm[j] = m;
                pl[j] = l0 + l1;
                for (int u = 0; u < U; u++) {
                    for (int d = 0; d < head_dim; d++) {
                        float a = 0.0f;
                        for (int i = u; i < n; i += U) a = fmaf(e[i], vbuf[i * head_dim + d], a);
                        acc[u * head_dim + d] = a;
                    }
                }
                for (int d = 0; d < head_dim; d++) {
                    float r[4];
                    for (int w = 0; w < 4; w++) {
                        float g[32];
                        for (int x = 0; x < kpw; x++) g[x] = acc[(w * kpw + x) * head_dim + d];
                        r[w] = butterfly(g, kpw);
                    }
                    po[(int64_t)j * head_dim + d] = ((r[0] + r[1]) + r[2]) + r[3];
                }
            }
            float M = -INFINITY;
            for (int j = 0; j < nsplit; j++) M = fmaxf(M, pm[j]);
            float L[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int d = 0; d < 4 * head_dim; d++) O[d] = 0.0f;
            for (int j = 0; j < nsplit; j++) {
                const float f = or_expf(pm[j] - M);
                const int w = j & 3;
                L[w] = fmaf(pl[j], f, L[w]);
                for (int d = 0; d < head_dim; d++)
                    O[w * head_dim + d] = fmaf(po[(int64_t)j * head_dim + d], f, O[w * head_dim + d]);
            }
            const float inv = 1.0f / (((L[0] + L[1]) + L[2]) + L[3]);
            for (int d = 0; d < head_dim; d++) {
                const float o = ((O[d] + O[head_dim + d]) + O[2 * head_dim + d]) + O[3 * head_dim + d];
                st(out, dt, b * out_stride + (int64_t)h * head_dim + d, o * inv);
            }
        }
        free(pm);
        free(pl);
        free(po);
    }
    free(qf);
    free(kbuf);
    free(vbuf);
    free(acc);
    free(O);
}

/* ------------------------------------------------------------------ */
/* fp32 <-> fp16 packing at the ANE boundary, core/ane_runtime.cpp:611-653 */
/* ------------------------------------------------------------------ */

/* ane_matvec writes channel c of its one token to element c * ANE_SPATIAL of
 * the fp16 input surface [channels][32] (:622-629) and reads channel c of the
 * output from element c * ANE_SPATIAL (:643-650).  Batched: token t of
 * `tokens` goes to surface t / spatial, spatial slot t % spatial; elements of
 * other slots are left as they are.  round_mode 0 = round to nearest even
 * (the native __fp16 store on arm64, :604-609), NaN -> quiet NaN 0x7E00
 * with the sign; 1 = the truncating f32_to_f16 of the x86 branch. */
void or_ane_pack(int round_mode, uint16_t* surface, const float* in, int64_t in_stride,
                 int64_t tokens, int channels, int spatial) {
    for (int64_t t = 0; t < tokens; t++) {
        uint16_t* sf = surface + (t / spatial) * (int64_t)channels * spatial + t % spatial;
        for (int c = 0; c < channels; c++) {
            const float x = in[t * in_stride + c];
            sf[(int64_t)c * spatial] = round_mode ? or_f32_to_f16_trunc(x) : or_f32_to_f16_rne(x);
        }
    }
}

/* The output side: out[t][c] = (float) surface element (exact). */
void or_ane_unpack(float* out, int64_t out_stride, const uint16_t* surface, int64_t tokens,
                   int channels, int spatial) {
    for (int64_t t = 0; t < tokens; t++) {
        const uint16_t* sf = surface + (t / spatial) * (int64_t)channels * spatial + t % spatial;
        for (int c = 0; c < channels; c++) out[t * out_stride + c] = or_f16_to_f32(sf[(int64_t)c * spatial]);
    }
}

/* models/llm/qwen3.cpp:475-484: append while the ring has room, else
 * overwrite the oldest slot and advance the start. */
int or_kv_ring_advance(int32_t* start, int32_t* len, int capacity) {
    int slot;
    if (*len < capacity) {
        slot = *start + *len;
        if (slot >= capacity) slot -= capacity;
        (*len)++;
    } else {
        slot = *start;
        (*start)++;
        if (*start >= capacity) *start = 0;
    }
    return slot;
}

/* ------------------------------------------------------------------ */
/* Sampler, core/sampling.cpp:10-66 and softmax core/cpu_ops.cpp:83-99  */
/* ------------------------------------------------------------------ */
static int32_t sample_one(const float* logits, int vocab, const int32_t* hist,
                          int hl, float u, float temperature, float rep,
                          int ctx, float freq, float* adj, int32_t* cnt,
                          int32_t* uniq) {
    memcpy(adj, logits, (size_t)vocab * sizeof(float));
    if (hl > 0) {
        /* window = last `ctx` ids (sampling.cpp:17), ids outside the vocab
         * are ignored (:22) */
        int start = hl - ctx;
        if (start < 0) start = 0;
        int nu = 0;
        for (int j = start; j < hl; j++) {
            int32_t t = hist[j];
            if (t >= 0 && t < vocab) {
                if (cnt[t] == 0) uniq[nu++] = t;
                cnt[t]++;
            }
        }
        /* per distinct id: repetition penalty then frequency penalty (:29-42) */
        for (int i = 0; i < nu; i++) {
            int32_t t = uniq[i];
            if (rep > 1.0f) adj[t] = adj[t] > 0.0f ? adj[t] / rep : adj[t] * rep;
            if (freq > 0.0f) adj[t] -= freq * (float)cnt[t];
            cnt[t] = 0;
        }
    }
    if (temperature <= 0.0f) {                                    /* :45-52 */
        int mi = 0;
        for (int i = 1; i < vocab; i++) if (adj[i] > adj[mi]) mi = i;
        return mi;
    }
    float inv_t = 1.0f / temperature;                             /* :54-55 */
    for (int i = 0; i < vocab; i++) adj[i] *= inv_t;
    float mx = adj[0];                                            /* softmax */
    for (int i = 1; i < vocab; i++) if (adj[i] > mx) mx = adj[i];
    float nmx = -mx;
    for (int i = 0; i < vocab; i++) adj[i] = or_expf(adj[i] + nmx);
    float sum = or_softmax_sum(adj, vocab);
    float inv = 1.0f / sum;
    for (int i = 0; i < vocab; i++) adj[i] *= inv;
    float cum = 0.0f;                                             /* :58-65 */
    for (int i = 0; i < vocab; i++) {
        cum += adj[i];
        if (cum >= u) return i;
    }
    return vocab - 1;
}

void or_sample_rows(const float* logits, int64_t rows, int vocab, int64_t ls,
                    const int32_t* history, const int32_t* history_len,
                    int64_t hs, const float* uniforms, float temperature,
                    float rep, int ctx, float freq, int32_t* out) {
    float* adj = (float*)malloc((size_t)vocab * sizeof(float));
    int32_t* cnt = (int32_t*)calloc((size_t)vocab, sizeof(int32_t));
    int32_t* uniq = (int32_t*)malloc((size_t)(hs > 0 ? hs : 1) * sizeof(int32_t));
    for (int64_t r = 0; r < rows; r++) {
        int hl = history_len ? history_len[r] : 0;
        out[r] = sample_one(logits + r * ls, vocab, history ? history + r * hs : NULL,
                            hl, uniforms[r], temperature, rep, ctx, freq, adj, cnt, uniq);
    }
    free(adj); free(cnt); free(uniq);
}
