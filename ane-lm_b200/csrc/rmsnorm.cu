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
    constexpr int V = T::kVec;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    // the row's x and d toward L2 while the previous grid drains (16-byte
    // aligned rows, dim * size a multiple of 16 on this path)
    if (lane == 0 && row < rows) {
        const uint32_t bytes = (uint32_t)dim * sizeof(typename T::storage);
        prefetch_l2(x + row * xs, bytes);
        if constexpr (HAS_D) prefetch_l2(d + row * ds, bytes);
    }
    pdl_begin();
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

// rmsnorm_reg_kernel for rows that fit in a wave or so: d is staged in
// shared memory by cp.async (each lane its own slots: no barrier), x in
// registers, so a thread holds 16 chunks instead of 32 and five CTAs fit per
// SM instead of three.  The same operations in the same order: the same
// bits.
template <typename T, int VPL>
__global__ void __launch_bounds__(kNormWarps * kWarp, 5)
rmsnorm_dsm_kernel(typename T::storage* x, int64_t xs,
                   const typename T::storage* __restrict__ d, int64_t ds,
                   typename T::storage* out, int64_t os, const float* __restrict__ w,
                   int64_t rows, int dim, float eps) {
    constexpr int V = T::kVec;
    __shared__ __align__(16) uint4 sd[kNormWarps][VPL][kWarp];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + wid;
    if (lane == 0 && row < rows) {
        const uint32_t bytes = (uint32_t)dim * sizeof(typename T::storage);
        prefetch_l2(x + row * xs, bytes);
        prefetch_l2(d + row * ds, bytes);
    }
    pdl_begin();
    if (row >= rows) return;
    const int nvec = dim / V;
    typename T::storage* xr = x + row * xs;
    typename T::storage* orow = out + row * os;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) cp_async16(&sd[wid][i][lane], d + row * ds + c * V);
    }
    cp_async_commit();
    uint4 xv[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) xv[i] = ld_stream(xr + c * V);
    }
    cp_async_wait_pending(0);
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) {
            float a[V], b[V];
            unpack<T>(xv[i], a);
            unpack<T>(sd[wid][i][lane], b);
#pragma unroll
            for (int e = 0; e < V; e++) a[e] = __fadd_rn(a[e], b[e]);
            xv[i] = pack<T>(a);
            st_stream(xr + c * V, xv[i]);
            unpack<T>(xv[i], a);  // the norm reads the stored value
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

// Embedding gather fused with the residual add and RMSNorm after it (the
// decode step's first op, models/llm/qwen3.cpp:498 then :503 / :516-518):
// one warp per row, the row in registers.  e = table[id] widened to x's
// type (exact), x = e or x + e, stored; the norm of the stored x in the
// pinned order; out = (x * inv) * w.  The same operations in the same order
// as ane_cuda_embedding_gather then ane_cuda_residual_rmsnorm, so the same
// bits, in one launch.  An id outside [0, vocab) reads as a zero row and
// raises ANE_CUDA_FLAG_BAD_TOKEN_ID, as the gather does.
template <typename TI, int N>
__device__ __forceinline__ void load_widen(const typename TI::storage* p, float (&a)[N]) {
    using SI = typename TI::storage;
    if constexpr (sizeof(SI) * N == 16) {
        unpack<TI>(__ldg(reinterpret_cast<const uint4*>(p)), a);
    } else {
        static_assert(sizeof(SI) * N == 8, "8- or 16-byte table chunks");
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
        const SI* e = reinterpret_cast<const SI*>(&v);
#pragma unroll
        for (int k = 0; k < N; k++) a[k] = TI::to_f(e[k]);
    }
}

template <typename TI, typename TO, int VPL, bool ACC>
__global__ void __launch_bounds__(kNormWarps * kWarp)
embed_rmsnorm_kernel(typename TO::storage* x, int64_t xs, typename TO::storage* out, int64_t os,
                     const typename TI::storage* __restrict__ table,
                     const int32_t* __restrict__ ids, int vocab, int64_t rows, int dim,
                     const float* __restrict__ w, float eps, unsigned int* flags) {
    pdl_begin();
    constexpr int V = TO::kVec;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int nvec = dim / V;
    const int32_t id = __ldg(ids + row);
    const bool bad = id < 0 || id >= vocab;
    if (bad && lane == 0 && flags) atomicOr(flags, ANE_CUDA_FLAG_BAD_TOKEN_ID);
    const typename TI::storage* t = table + (int64_t)(bad ? 0 : id) * dim;
    typename TO::storage* xr = x + row * xs;
    typename TO::storage* orow = out + row * os;
    uint4 xv[VPL];
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) {
            float a[V];
            if (bad) {
#pragma unroll
                for (int e = 0; e < V; e++) a[e] = 0.0f;
            } else {
                load_widen<TI, V>(t + c * V, a);
            }
            if constexpr (ACC) {
                float b[V];
                unpack<TO>(ld_stream(xr + c * V), b);
#pragma unroll
                for (int e = 0; e < V; e++) a[e] = __fadd_rn(b[e], a[e]);
            }
            xv[i] = pack<TO>(a);
            st_stream(xr + c * V, xv[i]);
            unpack<TO>(xv[i], a);  // the norm reads the stored value
            acc = sumsq_chain<V>(a, acc);
        }
    }
    const float inv = rms_inv(butterfly_sum(acc, kWarp), dim, eps);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) {
            float a[V], wv[V];
            unpack<TO>(xv[i], a);
            const float4* wp = reinterpret_cast<const float4*>(w + c * V);
#pragma unroll
            for (int q = 0; q < V / 4; q++) {
                const float4 tq = __ldg(wp + q);
                wv[4 * q] = tq.x; wv[4 * q + 1] = tq.y; wv[4 * q + 2] = tq.z; wv[4 * q + 3] = tq.w;
            }
#pragma unroll
            for (int e = 0; e < V; e++) a[e] = __fmul_rn(__fmul_rn(a[e], inv), wv[e]);
            st_stream(orow + c * V, pack<TO>(a));
        }
    }
}

template <typename TI, typename TO, bool ACC>
static int launch_embed_norm(void* x, int64_t xs, void* out, int64_t os, const void* table,
                             const int32_t* ids, int vocab, int64_t rows, int dim, const float* w,
                             float eps, cudaStream_t s) {
    using SO = typename TO::storage;
    using SI = typename TI::storage;
    constexpr int V = TO::kVec;
    const unsigned blocks = (unsigned)((rows + kNormWarps - 1) / kNormWarps);
    const int per_lane = (dim / V + kWarp - 1) / kWarp;
    SO* xp = (SO*)x;
    SO* op = (SO*)out;
    const SI* tp = (const SI*)table;
    unsigned int* fl = status_flags_device();
#define ANE_EMB(VPL) \
    launch_pdl(embed_rmsnorm_kernel<TI, TO, VPL, ACC>, blocks, kNormWarps * kWarp, 0, s, xp, xs, op, os, tp, ids, vocab, rows, dim, w, eps, fl)
    if (per_lane <= 1) ANE_EMB(1);
    else if (per_lane <= 2) ANE_EMB(2);
    else if (per_lane <= 4) ANE_EMB(4);
    else if (per_lane <= 8) ANE_EMB(8);
    else if (per_lane <= 16) ANE_EMB(16);
    else return fail(ANE_CUDA_ERR_UNSUPPORTED, "embedding_rmsnorm: hidden %d too wide", dim);
#undef ANE_EMB
    return ANE_CUDA_OK;
}

template <typename TI, typename TO>
static int launch_embed_norm_acc(int acc, void* x, int64_t xs, void* out, int64_t os,
                                 const void* table, const int32_t* ids, int vocab, int64_t rows,
                                 int dim, const float* w, float eps, cudaStream_t s) {
    return acc ? launch_embed_norm<TI, TO, true>(x, xs, out, os, table, ids, vocab, rows, dim, w, eps, s)
               : launch_embed_norm<TI, TO, false>(x, xs, out, os, table, ids, vocab, rows, dim, w, eps, s);
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
static int launch_rmsnorm(void* x, int64_t xs, const void* d, int64_t ds, void* out, int64_t os,
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
    // a grid of at most 1.5 waves of the shared-memory form (five CTAs per
    // SM): there rows in flight and an early start beside the previous
    // kernel's CTAs count for more than the form's extra shared-memory
    // accesses (the Qwen3-8B chain at 4,096 rows per GPU +1.2%; 8,192 rows,
    // 2.8 waves, is faster in registers)
    if (vec && HAS_D && per_lane == 16 && 2u * blocks <= 3u * 5u * (unsigned)sm_count()) {
        launch_pdl(rmsnorm_dsm_kernel<T, 16>, blocks, kNormWarps * kWarp, 0, s, xp, xs, dp, ds, op, os, w, rows, dim, eps);
        return ANE_CUDA_OK;
    }
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
    return ANE_CUDA_OK;
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
    int st;
    if (d) {
        if (dtype == ANE_CUDA_F32) st = launch_rmsnorm<F32, true>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
        else if (dtype == ANE_CUDA_F16) st = launch_rmsnorm<F16, true>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
        else st = launch_rmsnorm<BF16, true>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
    } else {
        if (dtype == ANE_CUDA_F32) st = launch_rmsnorm<F32, false>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
        else if (dtype == ANE_CUDA_F16) st = launch_rmsnorm<F16, false>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
        else st = launch_rmsnorm<BF16, false>(x, x_stride, d, d_stride, out, out_stride, weight, rows, dim, eps, s);
    }
    if (st) return st;
    return check_launch("residual_rmsnorm");
}

extern "C" int ane_cuda_embedding_rmsnorm(int out_dtype, void* x, int64_t x_stride, void* out,
                                          int64_t out_stride, const void* table, int table_dtype,
                                          const int32_t* ids, int64_t rows, int vocab, int hidden,
                                          int accumulate, const float* weight, float eps,
                                          void* stream) {
    using namespace ane;
    const char* fn = "embedding_rmsnorm";
    if (!valid_dtype(out_dtype) || !valid_dtype(table_dtype))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: bad dtype", fn);
    if (rows < 0 || vocab <= 0 || hidden <= 0 || x_stride < hidden || out_stride < hidden)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: rows=%lld vocab=%d hidden=%d strides %lld %lld", fn,
                    (long long)rows, vocab, hidden, (long long)x_stride, (long long)out_stride);
    if (rows == 0) return ANE_CUDA_OK;
    if (!x || !out || !table || !ids || !weight)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: null pointer", fn);
    if (out_dtype != table_dtype && out_dtype != ANE_CUDA_F32)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "%s: out dtype %d from table dtype %d", fn, out_dtype,
                    table_dtype);
    // 16-byte chunks of x / out; the table read in 16-byte (same type) or
    // 8-byte (16-bit table widened to fp32) pieces of the same elements
    const int es = elem_size(out_dtype), tes = elem_size(table_dtype);
    const int v = 16 / es;
    if (hidden % v || !is_aligned(x, 16) || !is_aligned(out, 16) || !is_aligned(weight, 16) ||
        (x_stride * es) % 16 || (out_stride * es) % 16 || !is_aligned(table, (uintptr_t)(v * tes)))
        return fail(ANE_CUDA_ERR_UNSUPPORTED,
                    "%s: needs hidden a multiple of %d and 16-byte aligned rows, weight and table", fn, v);
    cudaStream_t s = as_stream(stream);
    int st;
    if (out_dtype == ANE_CUDA_F32) {
        if (table_dtype == ANE_CUDA_F32) st = launch_embed_norm_acc<F32, F32>(accumulate, x, x_stride, out, out_stride, table, ids, vocab, rows, hidden, weight, eps, s);
        else if (table_dtype == ANE_CUDA_F16) st = launch_embed_norm_acc<F16, F32>(accumulate, x, x_stride, out, out_stride, table, ids, vocab, rows, hidden, weight, eps, s);
        else st = launch_embed_norm_acc<BF16, F32>(accumulate, x, x_stride, out, out_stride, table, ids, vocab, rows, hidden, weight, eps, s);
    } else if (out_dtype == ANE_CUDA_F16) {
        st = launch_embed_norm_acc<F16, F16>(accumulate, x, x_stride, out, out_stride, table, ids, vocab, rows, hidden, weight, eps, s);
    } else {
        st = launch_embed_norm_acc<BF16, BF16>(accumulate, x, x_stride, out, out_stride, table, ids, vocab, rows, hidden, weight, eps, s);
    }
    if (st) return st;
    return check_launch(fn);
}
