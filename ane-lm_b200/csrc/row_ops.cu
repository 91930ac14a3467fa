// row_ops.cu -- the remaining row ops of core/cpu_ops used by the hybrid
// (linear-attention) Qwen3.5 layers, and its norm-weight loading:
//   rmsnorm_gated   core/cpu_ops.cpp:33-39   y = rmsnorm(x) * w / (1 + exp(-z)) * z
//   l2_normalize    core/cpu_ops.cpp:106-111 x = x / sqrtf(sum(x^2) + 1e-12) (* scale,
//                   the q scaling of models/llm/qwen3_5.cpp:530-531)
//   bf16 -> fp32 weights, plain or (1 + w)   core/safetensors.cpp:264-306
//
// One warp per row, as the RMSNorm kernel: lane l owns the 16-byte chunks
// l, l+32, ... and accumulates fmaf(x, x, acc) over them in order, then the
// 32 lane sums meet in an xor butterfly -- the pinned order of vDSP_svesq.
// Rows of up to 16 chunks per lane stay in registers; other rows are read
// twice.  All arithmetic is fp32 with explicit rounding; exp is the pinned
// exp, so every result is reproducible bit for bit.
#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

constexpr int kRowWarps = 4;

enum RowMode { kGated = 0, kL2 = 1 };

struct RowArgs {
    void* out;       // gated: output rows; l2: the rows themselves (in place)
    int64_t os;
    const void* x;
    int64_t xs;
    const void* z;   // gated only
    int64_t zs;
    const float* w;  // gated only
    int64_t rows;
    int dim;
    float eps;       // gated: rmsnorm eps
    float scale;     // l2: factor applied after the normalisation
};

template <int MODE>
__device__ __forceinline__ float row_inv(float ss, const RowArgs& a) {
    if constexpr (MODE == kGated) return rms_inv(ss, a.dim, a.eps);
    else return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, 1e-12f)));
}

// element i of a row: x value, its z (gated), weight (gated)
template <int MODE>
__device__ __forceinline__ float row_out(float x, float inv, float z, float w, float scale) {
    if constexpr (MODE == kGated) {
        float y = __fmul_rn(__fmul_rn(x, inv), w);
        y = __fdiv_rn(y, __fadd_rn(1.0f, pinned_expf(-z)));
        return __fmul_rn(y, z);
    } else {
        return __fmul_rn(__fmul_rn(x, inv), scale);
    }
}

template <typename T, int MODE, int VPL>
__global__ void __launch_bounds__(kRowWarps * kWarp)
row_reg_kernel(const RowArgs a) {
    pdl_begin();
    using S = typename T::storage;
    constexpr int V = T::kVec;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    if (row >= a.rows) return;
    const int nvec = a.dim / V;
    const S* xr = static_cast<const S*>(a.x) + row * a.xs;
    uint4 xv[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) xv[i] = ld_stream(xr + c * V);
    }
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        if (lane + i * kWarp < nvec) {
            float f[V];
            unpack<T>(xv[i], f);
            acc = sumsq_chain<V>(f, acc);
        }
    }
    const float inv = row_inv<MODE>(butterfly_sum(acc, kWarp), a);
    S* orow = static_cast<S*>(a.out) + row * a.os;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = lane + i * kWarp;
        if (c < nvec) {
            float f[V], zf[V], wf[V];
            unpack<T>(xv[i], f);
            if constexpr (MODE == kGated) {
                unpack<T>(ld_stream(static_cast<const S*>(a.z) + row * a.zs + c * V), zf);
#pragma unroll
                for (int q = 0; q < V / 4; q++) {
                    const float4 t = __ldg(reinterpret_cast<const float4*>(a.w + c * V) + q);
                    wf[4 * q] = t.x; wf[4 * q + 1] = t.y; wf[4 * q + 2] = t.z; wf[4 * q + 3] = t.w;
                }
            }
#pragma unroll
            for (int e = 0; e < V; e++) f[e] = row_out<MODE>(f[e], inv, zf[e], wf[e], a.scale);
            st_stream(orow + c * V, pack<T>(f));
        }
    }
}

// Any width or alignment: the same order with element accesses, two reads.
template <typename T, int MODE>
__global__ void __launch_bounds__(kRowWarps * kWarp)
row_any_kernel(const RowArgs a) {
    pdl_begin();
    using S = typename T::storage;
    constexpr int V = T::kVec;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    if (row >= a.rows) return;
    const S* xr = static_cast<const S*>(a.x) + row * a.xs;
    const int nchunk = (a.dim + V - 1) / V;
    float acc = 0.0f;
    for (int c = lane; c < nchunk; c += kWarp) {
        const int n = min(V, a.dim - c * V);
        for (int e = 0; e < n; e++) {
            const float v = T::to_f(xr[c * V + e]);
            acc = __fmaf_rn(v, v, acc);
        }
    }
    const float inv = row_inv<MODE>(butterfly_sum(acc, kWarp), a);
    __syncwarp();  // l2 is in place: every lane has read its chunks
    S* orow = static_cast<S*>(a.out) + row * a.os;
    for (int c = lane; c < nchunk; c += kWarp) {
        const int n = min(V, a.dim - c * V);
        for (int e = 0; e < n; e++) {
            const int i = c * V + e;
            const float x = T::to_f(xr[i]);
            float z = 0.0f, w = 0.0f;
            if constexpr (MODE == kGated) {
                z = T::to_f(static_cast<const S*>(a.z)[row * a.zs + i]);
                w = __ldg(a.w + i);
            }
            orow[i] = T::from_f(row_out<MODE>(x, inv, z, w, a.scale));
        }
    }
}

template <typename T, int MODE>
static int launch_row(const RowArgs& a, cudaStream_t s) {
    constexpr int V = T::kVec;
    const int es = (int)sizeof(typename T::storage);
    const unsigned blocks = (unsigned)((a.rows + kRowWarps - 1) / kRowWarps);
    bool vec = a.dim % V == 0 && is_aligned(a.x, 16) && is_aligned(a.out, 16) &&
               (a.xs * es) % 16 == 0 && (a.os * es) % 16 == 0;
    if (MODE == kGated)
        vec = vec && is_aligned(a.z, 16) && is_aligned(a.w, 16) && (a.zs * es) % 16 == 0;
    const int per_lane = (a.dim / V + kWarp - 1) / kWarp;
    const int threads = kRowWarps * kWarp;
    if (vec && per_lane <= 1) launch_pdl(row_reg_kernel<T, MODE, 1>, blocks, threads, 0, s, a);
    else if (vec && per_lane <= 2) launch_pdl(row_reg_kernel<T, MODE, 2>, blocks, threads, 0, s, a);
    else if (vec && per_lane <= 4) launch_pdl(row_reg_kernel<T, MODE, 4>, blocks, threads, 0, s, a);
    else if (vec && per_lane <= 8) launch_pdl(row_reg_kernel<T, MODE, 8>, blocks, threads, 0, s, a);
    else if (vec && per_lane <= 16) launch_pdl(row_reg_kernel<T, MODE, 16>, blocks, threads, 0, s, a);
    else launch_pdl(row_any_kernel<T, MODE>, blocks, threads, 0, s, a);
    return check_launch(MODE == kGated ? "rmsnorm_gated" : "l2_normalize");
}

template <int MODE>
static int run_row(int dtype, const RowArgs& a, cudaStream_t s) {
    if (dtype == ANE_CUDA_F32) return launch_row<F32, MODE>(a, s);
    if (dtype == ANE_CUDA_F16) return launch_row<F16, MODE>(a, s);
    return launch_row<BF16, MODE>(a, s);
}

// bf16 bits -> f32, optionally + 1.0f; 8 elements per thread step.
__global__ void bf16_to_f32_kernel(float* __restrict__ out, const uint16_t* __restrict__ in,
                                   int64_t n, int add_one, int vec) {
    pdl_begin();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    // NaN + 1 keeps the (quieted) NaN operand on the CPU; the GPU adder
    // returns its canonical NaN instead, so NaN is passed through here.
    auto cv = [add_one](uint32_t b) {
        const uint32_t u = b << 16;
        const float w = __uint_as_float(u);
        if (!add_one) return w;
        return (u & 0x7FFFFFFFu) > 0x7F800000u ? __uint_as_float(u | 0x400000u) : __fadd_rn(w, 1.0f);
    };
    int64_t done = 0;
    if (vec) {
        const int64_t nv = n / 8;
        for (int64_t i = t; i < nv; i += stride) {
            const uint4 v = __ldcs(reinterpret_cast<const uint4*>(in) + i);
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
            float f[8];
#pragma unroll
            for (int k = 0; k < 8; k++) f[k] = cv((wd[k >> 1] >> (16 * (k & 1))) & 0xFFFFu);
            float4* o = reinterpret_cast<float4*>(out) + 2 * i;
            __stcs(o, make_float4(f[0], f[1], f[2], f[3]));
            __stcs(o + 1, make_float4(f[4], f[5], f[6], f[7]));
        }
        done = nv * 8;
    }
    for (int64_t i = done + t; i < n; i += stride) out[i] = cv(in[i]);
}

}  // namespace ane

extern "C" {

int ane_cuda_rmsnorm_gated(int dtype, void* out, int64_t out_stride, const void* x,
                           int64_t x_stride, const void* z, int64_t z_stride, const float* weight,
                           int64_t rows, int dim, float eps, void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "rmsnorm_gated: bad dtype %d", dtype);
    if (rows < 0 || dim <= 0 || x_stride < dim || z_stride < dim || out_stride < dim)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "rmsnorm_gated: rows=%lld dim=%d or a stride below dim",
                    (long long)rows, dim);
    if (rows == 0) return ANE_CUDA_OK;
    if (!out || !x || !z || !weight) return fail(ANE_CUDA_ERR_INVALID_ARG, "rmsnorm_gated: null pointer");
    const RowArgs a{out, out_stride, x, x_stride, z, z_stride, weight, rows, dim, eps, 1.0f};
    return run_row<kGated>(dtype, a, as_stream(stream));
}

int ane_cuda_l2_normalize(int dtype, void* x, int64_t x_stride, int64_t rows, int dim, float scale,
                          void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "l2_normalize: bad dtype %d", dtype);
    if (rows < 0 || dim <= 0 || x_stride < dim)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "l2_normalize: rows=%lld dim=%d stride=%lld", (long long)rows,
                    dim, (long long)x_stride);
    if (rows == 0) return ANE_CUDA_OK;
    if (!x) return fail(ANE_CUDA_ERR_INVALID_ARG, "l2_normalize: null pointer");
    const RowArgs a{x, x_stride, x, x_stride, nullptr, 0, nullptr, rows, dim, 0.0f, scale};
    return run_row<kL2>(dtype, a, as_stream(stream));
}

int ane_cuda_bf16_to_f32(float* out, const uint16_t* in, int64_t n, int add_one, void* stream) {
    using namespace ane;
    if (n < 0) return fail(ANE_CUDA_ERR_INVALID_ARG, "bf16_to_f32: n=%lld", (long long)n);
    if (n == 0) return ANE_CUDA_OK;
    if (!out || !in) return fail(ANE_CUDA_ERR_INVALID_ARG, "bf16_to_f32: null pointer");
    const int vec = is_aligned(out, 16) && is_aligned(in, 16);
    const int blocks = resident_grid(reinterpret_cast<const void*>(bf16_to_f32_kernel), 256, 0,
                                     (n / 8 + 255) / 256 + 1);
    launch_pdl(bf16_to_f32_kernel, blocks, 256, 0, as_stream(stream), out, in, n, add_one != 0, vec);
    return check_launch("bf16_to_f32");
}

}  // extern "C"
