// rmsnorm.cu -- residual add + RMSNorm over rows (core/cpu_ops.cpp:25-31
// with the vDSP_vadd residual of models/llm/qwen3.cpp:516-518, :527).
//
// One warp per row.  Lane l owns the 16-byte chunks c = l, l+32, l+64, ...
// of the row; it accumulates fmaf(x, x, acc) over its chunks in increasing
// order, and the 32 lane sums meet in an xor butterfly 16, 8, 4, 2, 1.
// That order is the pinned definition of the reference's vDSP_svesq, so the
// result does not depend on the launch shape.
//
// Rows of up to 16 chunks per lane (4096 fp16 / 2048 fp32 elements) stay in
// registers: one HBM read of x and d, one write of x and of out.  Wider or
// unaligned rows use a two-pass form that re-reads the just-written x.
#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

constexpr int kNormWarps = 4;

template <typename T, int VPL, bool HAS_D>
__global__ void __launch_bounds__(kNormWarps * kWarp)
rmsnorm_reg_kernel(typename T::storage* x, int64_t xs,
                   const typename T::storage* __restrict__ d, int64_t ds,
                   typename T::storage* out, int64_t os, const float* __restrict__ w,
                   int64_t rows, int dim, float eps) {
    pdl_begin();
    constexpr int V = T::kVec;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int nvec = dim / V;
    typename T::storage* xr = x + row * xs;
    typename T::storage* orow = out + row * os;

    uint4 xv[VPL];
    uint4 dv[HAS_D ? VPL : 1];
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) {
            xv[i] = ld_stream(xr + c * V);
            if constexpr (HAS_D) dv[i] = ld_stream(d + row * ds + c * V);
        }
    }
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) {
            float a[V];
            unpack<T>(xv[i], a);
            if constexpr (HAS_D) {
                float b[V];
                unpack<T>(dv[i], b);
#pragma unroll
                for (int e = 0; e < V; e++) a[e] = __fadd_rn(a[e], b[e]);
                xv[i] = pack<T>(a);
                st_stream(xr + c * V, xv[i]);
                unpack<T>(xv[i], a);  // the norm reads the stored value
            }
            acc = sumsq_chain<V>(a, acc);
        }
    }
    const float inv = rms_inv(butterfly_sum(acc, kWarp), dim, eps);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) {
            float a[V], wv[V];
            unpack<T>(xv[i], a);
            const float4* wp = reinterpret_cast<const float4*>(w + c * V);
#pragma unroll
            for (int q = 0; q < V / 4; q++) {
                const float4 t = __ldg(wp + q);
                wv[4 * q] = t.x; wv[4 * q + 1] = t.y; wv[4 * q + 2] = t.z; wv[4 * q + 3] = t.w;
            }
#pragma unroll
            for (int e = 0; e < V; e++) a[e] = __fmul_rn(__fmul_rn(a[e], inv), wv[e]);
            st_stream(orow + c * V, pack<T>(a));
        }
    }
}

// Any width / alignment.  Pass A: residual add, store x, accumulate in the
// pinned order; pass B: re-read x and write out.  VEC selects 16-byte
// vectors (dim % kVec == 0 and aligned rows) or element accesses.
template <typename T, bool VEC, bool HAS_D>
__global__ void __launch_bounds__(kNormWarps * kWarp)
rmsnorm_2pass_kernel(typename T::storage* x, int64_t xs,
                     const typename T::storage* __restrict__ d, int64_t ds,
                     typename T::storage* out, int64_t os, const float* __restrict__ w,
                     int64_t rows, int dim, float eps) {
    pdl_begin();
    constexpr int V = T::kVec;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int nchunk = (dim + V - 1) / V;
    typename T::storage* xr = x + row * xs;
    const typename T::storage* dr = HAS_D ? d + row * ds : nullptr;
    typename T::storage* orow = out + row * os;
    float acc = 0.0f;
    for (int c = lane; c < nchunk; c += kWarp) {
        float a[V];
        if constexpr (VEC) {
            unpack<T>(ld_stream(xr + c * V), a);
            if constexpr (HAS_D) {
                float b[V];
                unpack<T>(ld_stream(dr + c * V), b);
#pragma unroll
                for (int e = 0; e < V; e++) a[e] = __fadd_rn(a[e], b[e]);
                const uint4 sv = pack<T>(a);
                *reinterpret_cast<uint4*>(xr + c * V) = sv;
                unpack<T>(sv, a);
            }
            acc = sumsq_chain<V>(a, acc);
        } else {
            const int n = min(V, dim - c * V);
            for (int e = 0; e < n; e++) {
                float v = T::to_f(xr[c * V + e]);
                if constexpr (HAS_D) {
                    const typename T::storage s = T::from_f(__fadd_rn(v, T::to_f(dr[c * V + e])));
                    xr[c * V + e] = s;
                    v = T::to_f(s);
                }
                acc = __fmaf_rn(v, v, acc);
            }
        }
    }
    const float inv = rms_inv(butterfly_sum(acc, kWarp), dim, eps);
    __syncwarp();
    for (int c = lane; c < nchunk; c += kWarp) {
        const int n = min(V, dim - c * V);
        if constexpr (VEC) {
            float a[V];
            unpack<T>(*reinterpret_cast<const uint4*>(xr + c * V), a);
#pragma unroll
            for (int e = 0; e < V; e++) a[e] = __fmul_rn(__fmul_rn(a[e], inv), __ldg(w + c * V + e));
            st_stream(orow + c * V, pack<T>(a));
        } else {
            for (int e = 0; e < n; e++) {
                const float v = T::to_f(xr[c * V + e]);
                orow[c * V + e] = T::from_f(__fmul_rn(__fmul_rn(v, inv), __ldg(w + c * V + e)));
            }
        }
    }
}

template <typename T, bool HAS_D>
static void launch_rmsnorm(void* x, int64_t xs, const void* d, int64_t ds, void* out, int64_t os,
                           const float* w, int64_t rows, int dim, float eps, cudaStream_t s) {
    using S = typename T::storage;
    constexpr int V = T::kVec;
    const unsigned blocks = (unsigned)((rows + kNormWarps - 1) / kNormWarps);
    const int es = (int)sizeof(S);
    const bool vec = dim % V == 0 && is_aligned(x, 16) && is_aligned(out, 16) &&
                     is_aligned(w, 16) && (xs * es) % 16 == 0 && (os * es) % 16 == 0 &&
                     (!HAS_D || (is_aligned(d, 16) && (ds * es) % 16 == 0));
    S* xp = (S*)x;
    const S* dp = (const S*)d;
    S* op = (S*)out;
    const int per_lane = (dim / V + kWarp - 1) / kWarp;
#define ANE_NORM_REG(VPL) \
    launch_pdl(rmsnorm_reg_kernel<T, VPL, HAS_D>, blocks, kNormWarps * kWarp, 0, s, xp, xs, dp, ds, op, os, w, rows, dim, eps)
    if (vec && per_lane <= 1) ANE_NORM_REG(1);
    else if (vec && per_lane <= 2) ANE_NORM_REG(2);
    else if (vec && per_lane <= 4) ANE_NORM_REG(4);
    else if (vec && per_lane <= 8) ANE_NORM_REG(8);
    else if (vec && per_lane <= 16) ANE_NORM_REG(16);
    else if (vec)
        launch_pdl(rmsnorm_2pass_kernel<T, true, HAS_D>, blocks, kNormWarps * kWarp, 0, s, xp, xs, dp, ds, op, os, w, rows, dim, eps);
    else
        launch_pdl(rmsnorm_2pass_kernel<T, false, HAS_D>, blocks, kNormWarps * kWarp, 0, s, xp, xs, dp, ds, op, os, w, rows, dim, eps);
#undef ANE_NORM_REG
}

}  // namespace ane

extern "C" int ane_cuda_residual_rmsnorm(int dtype, void* x, int64_t x_stride, const void* d,
                                         int64_t d_stride, void* out, int64_t out_stride,
                                         const float* weight, int64_t rows, int dim, float eps,
                                         void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "residual_rmsnorm: bad dtype %d", dtype);
    if (rows < 0 || dim <= 0)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "residual_rmsnorm: rows=%lld dim=%d", (long long)rows, dim);
    if (rows == 0) return ANE_CUDA_OK;
    if (!x || !out || !weight) return fail(ANE_CUDA_ERR_INVALID_ARG, "residual_rmsnorm: null pointer");
    if (x_stride < dim || out_stride < dim || (d && d_stride < dim))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "residual_rmsnorm: row stride below dim");
    cudaStream_t s = as_stream(stream);
    if (d) {
        if (dtype == ANE_CUDA_F32) launch_rmsnorm<F32, true>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
        else if (dtype == ANE_CUDA_F16) launch_rmsnorm<F16, true>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
        else launch_rmsnorm<BF16, true>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
    } else {
        if (dtype == ANE_CUDA_F32) launch_rmsnorm<F32, false>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
        else if (dtype == ANE_CUDA_F16) launch_rmsnorm<F16, false>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
        else launch_rmsnorm<BF16, false>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
    }
    return check_launch("residual_rmsnorm");
}
