// qk_rope.cu -- per-head QK RMSNorm + half-split RoPE, in place
// (models/llm/qwen3.cpp:444-473; core/cpu_ops.cpp:43-80).
//
// Fast path (rot_dim == head_dim, head_dim / kVec a power of two in
// [2, 32], 16-byte aligned rows): one warp per unit of about 8 heads of a
// row.  A head is served by
// GL = chunks/2 lanes; lane l of the group holds chunk l (elements
// [l*V, l*V+V), first half) and chunk l + GL (the RoPE partners j + half).
// With that layout
//   - the first butterfly stage of the pinned sum-of-squares order
//     (offset GL) is an add inside the lane, the rest are xor shuffles
//     inside the group; no shuffle is needed for RoPE;
//   - the lane's cos/sin for j in [l*V, l*V+V) serve every head of the unit,
//     so they are computed once per unit, in registers;
//   - the lane's norm weights are the same for every q (k) head: loaded
//     once per unit as 16-byte vectors.
// All of the unit's heads are loaded before any math.
//
// Generic path (partial RoPE, other head sizes, unaligned rows, or the
// caller-supplied cos/sin rows of apply_rope_cached): one warp per
// (row, head) with the head staged in shared memory.
#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

constexpr int kQkWarps = 4;
constexpr int kMaxHalfRot = 128;

struct RopeFreq {
    float f[kMaxHalfRot];
};

struct QkArgs {
    void* q;
    void* k;
    int64_t q_row_stride, k_row_stride;
    int q_head_stride, k_head_stride;
    int n_q, n_kv, head_dim, rot_dim;
    const float* qw;
    const float* kw;
    const int32_t* positions;  // per row; NULL -> `pos`
    int pos;
    int64_t rows;
    float eps;
    const float* cos_row;      // generic path only: caller tables
    const float* sin_row;
};

// A work unit is IPU head iterations (IPU * hpw heads) of one row; one
// warp per unit, 8 warps per CTA.  Small units keep the register footprint
// low (many warps per SM hide the load latency) while every unit still
// moves 2 KB or more with 16-byte accesses.
constexpr int kUnitWarps = 8;

template <typename T, int IPU>
__global__ void __launch_bounds__(kUnitWarps * kWarp)
qk_norm_rope_unit_kernel(const QkArgs a, const RopeFreq fr, const int gl_log2,
                         const int units_per_row, const bool pow2_dim) {
    using S = typename T::storage;
    constexpr int V = T::kVec;
    const int lane = threadIdx.x & 31;
    const int64_t unit = (int64_t)blockIdx.x * kUnitWarps + (threadIdx.x >> 5);
    if (unit >= a.rows * units_per_row) return;
    const int64_t row = unit / units_per_row;
    const int GL = 1 << gl_log2;           // lanes per head
    const int hpw = kWarp >> gl_log2;      // heads per iteration
    const int g = lane >> gl_log2;         // head slot of this lane
    const int l = lane & (GL - 1);         // lane within the head group
    const int half = GL * V;               // rot_dim / 2
    const int nh = a.n_q + a.n_kv;
    const int head0 = (int)(unit - row * units_per_row) * IPU * hpw;
    S* qrow = (S*)a.q + row * a.q_row_stride;
    S* krow = (S*)a.k + row * a.k_row_stride;

    uint4 lo[IPU], hi[IPU];
#pragma unroll
    for (int it = 0; it < IPU; it++) {
        const int h = head0 + it * hpw + g;
        if (h < nh) {
            const S* base = h < a.n_q ? qrow + (int64_t)h * a.q_head_stride
                                      : krow + (int64_t)(h - a.n_q) * a.k_head_stride;
            lo[it] = ld_stream(base + l * V);
            hi[it] = ld_stream(base + half + l * V);
        }
    }

    // cos/sin of the lane's V frequencies at the row's position.  The hpw
    // lanes sharing l need the same values: each computes cpl of them and
    // the rest arrive by shuffle.
    const float fpos = (float)(a.positions ? __ldg(a.positions + row) : a.pos);
    const int cpl = half >= 32 ? half / 32 : V;
    float cs[V], sn[V];
    if (cpl == V) {
#pragma unroll
        for (int e = 0; e < V; e++) pinned_sincosf(__fmul_rn(fpos, fr.f[l * V + e]), &sn[e], &cs[e]);
    } else {
        float mc[4], ms[4];
#pragma unroll
        for (int c = 0; c < 4; c++)
            if (c < cpl) pinned_sincosf(__fmul_rn(fpos, fr.f[l * V + g * cpl + c]), &ms[c], &mc[c]);
#pragma unroll
        for (int e = 0; e < V; e++) {
            const int src = (e / cpl) * GL + l;
            float vc = mc[0], vs = ms[0];
#pragma unroll
            for (int c = 1; c < 4; c++)
                if (e % cpl == c) { vc = mc[c]; vs = ms[c]; }
            cs[e] = __shfl_sync(0xffffffffu, vc, src);
            sn[e] = __shfl_sync(0xffffffffu, vs, src);
        }
    }

    const bool norm = a.qw != nullptr;
    float w0[V], w1[V];
    int wtype = -1;  // 0: q weights loaded, 1: k weights loaded
    const float inv_dim = 1.0f / (float)a.head_dim;
#pragma unroll
    for (int it = 0; it < IPU; it++) {
        const int h = head0 + it * hpw + g;
        if (head0 + it * hpw >= nh) break;  // warp-uniform
        const bool live = h < nh;
        float x0[V], x1[V];
        if (live) {
            unpack<T>(lo[it], x0);
            unpack<T>(hi[it], x1);
        } else {
#pragma unroll
            for (int e = 0; e < V; e++) { x0[e] = 0.0f; x1[e] = 0.0f; }
        }
        if (norm) {
            float acc = __fadd_rn(sumsq_chain<V>(x0, 0.0f), sumsq_chain<V>(x1, 0.0f));
            for (int off = GL >> 1; off >= 1; off >>= 1)
                acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
            // ss / dim is exact as a multiply when dim is a power of two
            const float mean = pow2_dim ? __fmul_rn(acc, inv_dim) : __fdiv_rn(acc, (float)a.head_dim);
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
            const int want = h < a.n_q ? 0 : 1;
            if (want != wtype) {
                const float* wsrc = want == 0 ? a.qw : a.kw;
#pragma unroll
                for (int q4 = 0; q4 < V / 4; q4++) {
                    const float4 t0 = __ldg(reinterpret_cast<const float4*>(wsrc + l * V) + q4);
                    const float4 t1 = __ldg(reinterpret_cast<const float4*>(wsrc + half + l * V) + q4);
                    w0[4 * q4] = t0.x; w0[4 * q4 + 1] = t0.y; w0[4 * q4 + 2] = t0.z; w0[4 * q4 + 3] = t0.w;
                    w1[4 * q4] = t1.x; w1[4 * q4 + 1] = t1.y; w1[4 * q4 + 2] = t1.z; w1[4 * q4 + 3] = t1.w;
                }
                wtype = want;
            }
#pragma unroll
            for (int e = 0; e < V; e++) {
                x0[e] = __fmul_rn(__fmul_rn(x0[e], inv), w0[e]);
                x1[e] = __fmul_rn(__fmul_rn(x1[e], inv), w1[e]);
            }
        }
        if (live) {
            float y0[V], y1[V];
#pragma unroll
            for (int e = 0; e < V; e++) {
                y0[e] = __fsub_rn(__fmul_rn(x0[e], cs[e]), __fmul_rn(x1[e], sn[e]));
                y1[e] = __fadd_rn(__fmul_rn(x1[e], cs[e]), __fmul_rn(x0[e], sn[e]));
            }
            S* base = h < a.n_q ? qrow + (int64_t)h * a.q_head_stride
                                : krow + (int64_t)(h - a.n_q) * a.k_head_stride;
            st_stream(base + l * V, pack<T>(y0));
            st_stream(base + half + l * V, pack<T>(y1));
        }
    }
}

// One warp per (row, head); head staged in shared memory as fp32.
constexpr int kGenericMaxHead = 1024;

template <typename T>
__global__ void __launch_bounds__(kQkWarps * kWarp)
qk_norm_rope_generic_kernel(const QkArgs a, const RopeFreq fr) {
    using S = typename T::storage;
    constexpr int V = T::kVec;
    __shared__ float sm[kQkWarps][kGenericMaxHead];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int nh = a.n_q + a.n_kv;
    const int64_t item = (int64_t)blockIdx.x * kQkWarps + wid;
    if (item >= a.rows * nh) return;
    const int64_t row = item / nh;
    const int h = (int)(item - row * nh);
    S* base = h < a.n_q ? (S*)a.q + row * a.q_row_stride + (int64_t)h * a.q_head_stride
                        : (S*)a.k + row * a.k_row_stride + (int64_t)(h - a.n_q) * a.k_head_stride;
    float* v = sm[wid];
    const int hd = a.head_dim;
    const int nchunk = (hd + V - 1) / V;
    float acc = 0.0f;
    for (int c = lane; c < nchunk; c += kWarp) {
        const int n = min(V, hd - c * V);
        for (int e = 0; e < n; e++) {
            const float x = T::to_f(base[c * V + e]);
            v[c * V + e] = x;
            acc = __fmaf_rn(x, x, acc);
        }
    }
    __syncwarp();
    if (a.qw) {
        const float inv = rms_inv(butterfly_sum(acc, kWarp), hd, a.eps);
        const float* w = h < a.n_q ? a.qw : a.kw;
        for (int i = lane; i < hd; i += kWarp) v[i] = __fmul_rn(__fmul_rn(v[i], inv), __ldg(w + i));
        __syncwarp();
    }
    const int half = a.rot_dim / 2;
    const float fpos = (float)(a.positions ? __ldg(a.positions + row) : a.pos);
    for (int j = lane; j < half; j += kWarp) {
        float c, s;
        if (a.cos_row) {
            c = __ldg(a.cos_row + j);
            s = __ldg(a.sin_row + j);
        } else {
            pinned_sincosf(__fmul_rn(fpos, fr.f[j]), &s, &c);
        }
        const float x0 = v[j], x1 = v[j + half];
        base[j] = T::from_f(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
        base[j + half] = T::from_f(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s)));
    }
    for (int i = a.rot_dim + lane; i < hd; i += kWarp) base[i] = T::from_f(v[i]);
}

// inv_freq[j] = 1.0f / powf(theta, (float)(2j) / (float)rot_dim)
// (models/llm/qwen3.cpp:205-208), powf as the float rounding of the double pow.
static void make_freq(RopeFreq* fr, int rot_dim, float theta) {
    for (int j = 0; 2 * j < rot_dim && j < kMaxHalfRot; j++) {
        const float e = (float)(2 * j) / (float)rot_dim;
        const float p = (float)pow((double)theta, (double)e);
        fr->f[j] = 1.0f / p;
    }
}

static int ilog2_exact(int v) {
    if (v <= 0 || (v & (v - 1))) return -1;
    int r = 0;
    while ((1 << r) < v) r++;
    return r;
}

template <typename T>
static int launch_qk(const QkArgs& a, const RopeFreq& fr, cudaStream_t s) {
    constexpr int V = T::kVec;
    const int es = (int)sizeof(typename T::storage);
    const int nh = a.n_q + a.n_kv;
    const int nchunk = a.head_dim / V;
    const int gl_log2 = ilog2_exact(nchunk) - 1;
    bool fast = a.cos_row == nullptr && a.rot_dim == a.head_dim && a.head_dim % V == 0 &&
                gl_log2 >= 0 && nchunk <= 32 && is_aligned(a.q, 16) && is_aligned(a.k, 16) &&
                (a.q_row_stride * es) % 16 == 0 && (a.k_row_stride * es) % 16 == 0 &&
                (a.q_head_stride * es) % 16 == 0 && (a.k_head_stride * es) % 16 == 0;
    if (fast && (!a.qw || (is_aligned(a.qw, 16) && is_aligned(a.kw, 16)))) {
        const int hpw = kWarp >> gl_log2;
        const int ipu = hpw >= 8 ? 1 : 8 / hpw;   // about 8 heads per unit
        const int units_per_row = (nh + ipu * hpw - 1) / (ipu * hpw);
        const int64_t units = a.rows * units_per_row;
        const unsigned blocks = (unsigned)((units + kUnitWarps - 1) / kUnitWarps);
        const bool pow2 = (a.head_dim & (a.head_dim - 1)) == 0;
#define ANE_QK_UNIT(N) \
    qk_norm_rope_unit_kernel<T, N><<<blocks, kUnitWarps * kWarp, 0, s>>>(a, fr, gl_log2, units_per_row, pow2)
        if (ipu == 1) ANE_QK_UNIT(1);
        else if (ipu == 2) ANE_QK_UNIT(2);
        else if (ipu == 4) ANE_QK_UNIT(4);
        else ANE_QK_UNIT(8);
#undef ANE_QK_UNIT
    } else {
        if (a.head_dim > kGenericMaxHead)
            return fail(ANE_CUDA_ERR_UNSUPPORTED, "qk_norm_rope: head_dim %d > %d", a.head_dim,
                        kGenericMaxHead);
        const int64_t items = a.rows * nh;
        const unsigned blocks = (unsigned)((items + kQkWarps - 1) / kQkWarps);
        qk_norm_rope_generic_kernel<T><<<blocks, kQkWarps * kWarp, 0, s>>>(a, fr);
    }
    return check_launch("qk_norm_rope");
}

static int run_qk(int dtype, const QkArgs& a, float theta, cudaStream_t s) {
    RopeFreq fr;
    make_freq(&fr, a.rot_dim, theta);
    if (dtype == ANE_CUDA_F32) return launch_qk<F32>(a, fr, s);
    if (dtype == ANE_CUDA_F16) return launch_qk<F16>(a, fr, s);
    return launch_qk<BF16>(a, fr, s);
}

static int validate(const char* fn, const QkArgs& a) {
    if (a.n_q < 0 || a.n_kv < 0 || a.n_q + a.n_kv <= 0 || a.head_dim <= 0 || a.rows < 0)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: n_q=%d n_kv=%d head_dim=%d rows=%lld", fn, a.n_q,
                    a.n_kv, a.head_dim, (long long)a.rows);
    if (a.rot_dim < 0 || a.rot_dim > a.head_dim || (a.rot_dim & 1))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: rot_dim %d (head_dim %d)", fn, a.rot_dim, a.head_dim);
    if (a.rot_dim / 2 > kMaxHalfRot)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "%s: rot_dim %d > %d", fn, a.rot_dim, 2 * kMaxHalfRot);
    if ((a.n_q > 0 && !a.q) || (a.n_kv > 0 && !a.k))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: null q/k", fn);
    if ((a.qw == nullptr) != (a.kw == nullptr))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: give both q_weight and k_weight or neither", fn);
    if ((a.cos_row == nullptr) != (a.sin_row == nullptr))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: give both cos_row and sin_row or neither", fn);
    return ANE_CUDA_OK;
}

}  // namespace ane

extern "C" {

int ane_cuda_qk_norm_rope(int dtype, void* q, void* k, int64_t q_row_stride,
                          int64_t k_row_stride, int q_head_stride, int k_head_stride,
                          int n_q_heads, int n_kv_heads, int head_dim, int rot_dim,
                          const float* q_weight, const float* k_weight,
                          const int32_t* positions, int64_t rows, float theta, float eps,
                          void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "qk_norm_rope: bad dtype %d", dtype);
    QkArgs a{q, k, q_row_stride, k_row_stride, q_head_stride, k_head_stride, n_q_heads, n_kv_heads,
             head_dim, rot_dim, q_weight, k_weight, positions, 0, rows, eps, nullptr, nullptr};
    int st = validate("qk_norm_rope", a);
    if (st) return st;
    if (rows == 0) return ANE_CUDA_OK;
    if (!positions) return fail(ANE_CUDA_ERR_INVALID_ARG, "qk_norm_rope: positions is NULL");
    return run_qk(dtype, a, theta, as_stream(stream));
}

int ane_cuda_apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads, int head_dim,
                               int q_head_stride, int k_head_stride, int rot_dim, int pos,
                               float theta, const float* cos_row, const float* sin_row,
                               void* stream) {
    using namespace ane;
    QkArgs a{q, k, 0, 0, q_head_stride, k_head_stride, n_q_heads, n_kv_heads, head_dim, rot_dim,
             nullptr, nullptr, nullptr, pos, 1, 0.0f, cos_row, sin_row};
    int st = validate("apply_rope_cached", a);
    if (st) return st;
    return run_qk(ANE_CUDA_F32, a, theta, as_stream(stream));
}

}  // extern "C"
