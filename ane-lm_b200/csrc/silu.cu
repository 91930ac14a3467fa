// silu.cu -- SiLU-gated activation and its sigmoid relatives
// (core/cpu_ops.cpp:7-23; the fused FFN gate of core/ane_runtime.cpp:393-395).
//
//   SILU_MUL    out = (g / (1 + exp(-g))) * u
//   SILU        x   =  x / (1 + exp(-x))                 silu_vec_inplace
//   MUL_SIGMOID y   =  y / (1 + exp(-z))                 mul_sigmoid_inplace
//
// Element-wise and HBM-bound: long contiguous inputs stream through a
// bulk-copy ring in shared memory (act_bulk_kernel); the rest use 16-byte
// vectors with evict-first accesses and a grid sized to the SM count.  fp32 rows use the pinned Cody-Waite/Taylor exp and
// an IEEE divide, each step rounded on its own, as the reference's vneg /
// vvexpf / vsadd / vdiv sequence (bit-exact).  fp16 / bf16 rows use the
// special-function unit's exp2 and reciprocal: the pinned form costs about
// 40 instructions per element, which at 6 bytes per element would make the
// kernel issue-bound well below the HBM roofline.
#include "ane_common.cuh"
#include "ane_internal.h"

#include <type_traits>

namespace ane {

enum ActMode { SILU_MUL = 0, SILU = 1, MUL_SIGMOID = 2 };

// fp32 results: the pinned exp and an IEEE divide, bit-exact with the
// reference's vneg / vvexpf / vsadd / vdiv sequence.
template <int MODE>
__device__ __forceinline__ float act_exact(float a, float b) {
    if constexpr (MODE == SILU_MUL) {
        const float s = __fdiv_rn(a, __fadd_rn(1.0f, pinned_expf(-a)));
        return __fmul_rn(s, b);
    } else if constexpr (MODE == SILU) {
        return __fdiv_rn(a, __fadd_rn(1.0f, pinned_expf(-a)));
    } else {  // a = y, b = z
        return __fdiv_rn(a, __fadd_rn(1.0f, pinned_expf(-b)));
    }
}

// fp16 / bf16 results: exp2 and reciprocal from the special-function unit.
// The fp32 value is within a few 1e-6 (relative) of the exact one, far
// below half an fp16 / bf16 unit in the last place, so the stored result
// matches the exact one or is one unit away.  e^-x overflowing to +inf
// gives x * 0 = -0 for large negative x, as x / inf does.  fp16 (FTZ)
// cannot hold the fp32 subnormals that the flushing forms drop; bf16 can.
template <bool FTZ>
__device__ __forceinline__ float sigmoid_den_fast(float x) {
    return __fadd_rn(1.0f, exp2f_approx<FTZ>(__fmul_rn(x, -1.44269504088896340736f)));
}
template <int MODE, bool FTZ>
__device__ __forceinline__ float act_fast(float a, float b) {
    if constexpr (MODE == SILU_MUL) {
        return __fmul_rn(__fmul_rn(a, rcp_approx<FTZ>(sigmoid_den_fast<FTZ>(a))), b);
    } else if constexpr (MODE == SILU) {
        return __fmul_rn(a, rcp_approx<FTZ>(sigmoid_den_fast<FTZ>(a)));
    } else {
        return __fmul_rn(a, rcp_approx<FTZ>(sigmoid_den_fast<FTZ>(b)));
    }
}

template <typename T, int MODE>
__device__ __forceinline__ float act(float a, float b) {
    if constexpr (sizeof(typename T::storage) == 4) return act_exact<MODE>(a, b);
    else return act_fast<MODE, std::is_same<T, F16>::value>(a, b);
}

constexpr int kActThreads = 256;
constexpr int kActUnroll = 2;  // 16-byte vectors per thread in flight, per input

struct ActArgs {
    void* out;
    const void* a;
    const void* b;
    int64_t out_stride, a_stride, b_stride;
    int64_t rows;
    int64_t n;
};

// Vector path: n % kVec == 0, every row 16-byte aligned.  Work item i is
// vector (i % nvec) of row (i / nvec).
template <typename T, int MODE, bool FLAT>
__global__ void __launch_bounds__(kActThreads)
act_vec_kernel(const ActArgs p) {
    pdl_begin();
    using S = typename T::storage;
    constexpr int V = T::kVec;
    const int64_t nvec = p.n / V;
    const int64_t total = p.rows * nvec;
    const int64_t stride = (int64_t)gridDim.x * kActThreads;
    for (int64_t i = (int64_t)blockIdx.x * kActThreads + threadIdx.x; i < total;
         i += kActUnroll * stride) {
        uint4 av[kActUnroll], bv[kActUnroll];
        int64_t r[kActUnroll], c[kActUnroll];
        bool ok[kActUnroll];
#pragma unroll
        for (int u = 0; u < kActUnroll; u++) {
            const int64_t j = i + u * stride;
            ok[u] = j < total;
            if constexpr (FLAT) {
                r[u] = 0;
                c[u] = j * V;
            } else {
                r[u] = ok[u] ? j / nvec : 0;
                c[u] = ok[u] ? (j - r[u] * nvec) * V : 0;
            }
            if (ok[u]) {
                av[u] = ld_stream((const S*)p.a + r[u] * p.a_stride + c[u]);
                if constexpr (MODE != SILU) bv[u] = ld_stream((const S*)p.b + r[u] * p.b_stride + c[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < kActUnroll; u++) {
            if (!ok[u]) continue;
            float x[V], y[V];
            unpack<T>(av[u], x);
            if constexpr (MODE != SILU) unpack<T>(bv[u], y);
#pragma unroll
            for (int e = 0; e < V; e++) x[e] = act<T, MODE>(x[e], MODE != SILU ? y[e] : 0.0f);
            st_stream((S*)p.out + r[u] * p.out_stride + c[u], pack<T>(x));
        }
    }
}


// Long contiguous inputs: a persistent CTA per SM streams 32 KB tiles of
// each input through a two-stage ring in shared memory, filled by one bulk
// copy (TMA) per input and tile, while the previous tile is computed from
// shared memory and stored with 16-byte streaming stores.  Few, large
// copies keep the DRAM request stream long and sequential; measured on the
// Qwen3-8B shapes this reaches the copy roofline where the grid-stride
// 16-byte loads above stop about 10% short.  Results are the same
// element-wise functions, so the same bits.
constexpr int kBulkTile = 32768;  // bytes per input per tile
constexpr int kBulkStages = 2;
template <int NIN>
constexpr size_t act_bulk_smem() { return (size_t)kBulkStages * NIN * kBulkTile; }

template <typename T, int MODE>
__global__ void __launch_bounds__(kActThreads)
act_bulk_kernel(const ActArgs p, int64_t ntiles, unsigned int* flags) {
    using S = typename T::storage;
    constexpr int V = T::kVec;
    constexpr int NIN = MODE == SILU ? 1 : 2;
    // the CTA's first tiles toward L2 while the previous grid drains
    if (threadIdx.x == 0)
        for (int k = 0; k < kBulkStages; k++)
            if (blockIdx.x + (int64_t)k * gridDim.x < ntiles) {
                const int64_t off = (blockIdx.x + (int64_t)k * gridDim.x) * kBulkTile;
                prefetch_l2(static_cast<const char*>(p.a) + off, kBulkTile);
                if constexpr (NIN == 2) prefetch_l2(static_cast<const char*>(p.b) + off, kBulkTile);
            }
    pdl_begin();
    constexpr int STEPS = kBulkTile / (kActThreads * 16);  // 16-byte vectors per thread and tile
    extern __shared__ __align__(128) unsigned char smem[];  // [stage][input][kBulkTile]
    __shared__ __align__(8) uint64_t full[kBulkStages];
    const int tid = threadIdx.x;
    const int64_t G = gridDim.x;
    const char* const src0 = static_cast<const char*>(p.a);
    const char* const src1 = static_cast<const char*>(p.b);
    char* const dst = static_cast<char*>(p.out);
    if (tid == 0) {
        for (int s = 0; s < kBulkStages; s++) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    // thread 0: tile -> stage s.  The stage was last read through the
    // generic proxy (before the barrier that precedes the call); the proxy
    // fence orders those reads before the copy's writes.
    auto issue = [&](int64_t tile, int s) {
        fence_proxy_async();
        mbar_expect_tx(&full[s], NIN * kBulkTile);
        bulk_load(smem + (s * NIN) * kBulkTile, src0 + tile * kBulkTile, kBulkTile, &full[s]);
        if constexpr (NIN == 2)
            bulk_load(smem + (s * NIN + 1) * kBulkTile, src1 + tile * kBulkTile, kBulkTile, &full[s]);
    };
    if (tid == 0)
        for (int s = 0; s < kBulkStages; s++)
            if (blockIdx.x + s * G < ntiles) issue(blockIdx.x + s * G, s);
    int s = 0;
    uint32_t ph = 0u;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += G) {
        if (!__syncthreads_and(mbar_wait_bounded(&full[s], (ph >> s) & 1u))) {
            // a copy did not land in time: flag it, wait (bounded) once more
            // for every stage still in flight, and stop
            if (tid == 0) {
                if (flags) atomicOr(flags, ANE_CUDA_FLAG_WAIT_TIMEOUT);
                for (int k = 0; k < kBulkStages; k++) {
                    const int sk = (s + k) % kBulkStages;
                    if (tile + k * G < ntiles) mbar_wait_bounded(&full[sk], (ph >> sk) & 1u);
                }
            }
            return;
        }
        ph ^= 1u << s;
        const unsigned char* const in0 = smem + (s * NIN) * kBulkTile;
#pragma unroll
        for (int st = 0; st < STEPS; st++) {
            const int off = (st * kActThreads + tid) * 16;
            float x[V], y[V];
            unpack<T>(*reinterpret_cast<const uint4*>(in0 + off), x);
            if constexpr (NIN == 2) unpack<T>(*reinterpret_cast<const uint4*>(in0 + kBulkTile + off), y);
#pragma unroll
            for (int e = 0; e < V; e++) x[e] = act<T, MODE>(x[e], NIN == 2 ? y[e] : 0.0f);
            st_stream(reinterpret_cast<S*>(dst + tile * kBulkTile + off), pack<T>(x));
        }
        __syncthreads();  // stage s consumed by every thread
        if (tid == 0 && tile + kBulkStages * G < ntiles) issue(tile + kBulkStages * G, s);
        s = s + 1 == kBulkStages ? 0 : s + 1;
    }
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kActThreads)
act_scalar_kernel(const ActArgs p) {
    pdl_begin();
    using S = typename T::storage;
    const int64_t total = p.rows * p.n;
    const int64_t stride = (int64_t)gridDim.x * kActThreads;
    for (int64_t i = (int64_t)blockIdx.x * kActThreads + threadIdx.x; i < total; i += stride) {
        const int64_t r = i / p.n, c = i - r * p.n;
        const float x = T::to_f(((const S*)p.a)[r * p.a_stride + c]);
        const float y = MODE != SILU ? T::to_f(((const S*)p.b)[r * p.b_stride + c]) : 0.0f;
        ((S*)p.out)[r * p.out_stride + c] = T::from_f(act<T, MODE>(x, y));
    }
}

template <typename T, int MODE>
static int launch_act(ActArgs p, cudaStream_t s) {
    constexpr int V = T::kVec;
    const int es = (int)sizeof(typename T::storage);
    bool vec = p.n % V == 0 && is_aligned(p.out, 16) && is_aligned(p.a, 16) &&
               (p.out_stride * es) % 16 == 0 && (p.a_stride * es) % 16 == 0;
    if (MODE != SILU) vec = vec && is_aligned(p.b, 16) && (p.b_stride * es) % 16 == 0;
    // rows stored back to back: one flat run of rows * n elements
    if (p.out_stride == p.n && p.a_stride == p.n && (MODE == SILU || p.b_stride == p.n)) {
        p.n *= p.rows;
        p.out_stride = p.a_stride = p.b_stride = p.n;
        p.rows = 1;
    }
    // long contiguous inputs: the bulk-copy ring over whole tiles, the
    // remainder (less than a tile) by the kernels below
    if (vec && p.rows == 1) {
        const int64_t ntiles = p.n * es / kBulkTile;
        if (ntiles >= 2 * (int64_t)sm_count()) {
            constexpr int nin = MODE == SILU ? 1 : 2;
            const void* kb = reinterpret_cast<const void*>(act_bulk_kernel<T, MODE>);
            const cudaError_t e = cudaFuncSetAttribute(act_bulk_kernel<T, MODE>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       (int)act_bulk_smem<nin>());
            if (e != cudaSuccess) return fail(ANE_CUDA_ERR_CUDA, "activation: %s", cudaGetErrorString(e));
            const int blocks = resident_grid(kb, kActThreads, act_bulk_smem<nin>(), ntiles);
            launch_pdl(act_bulk_kernel<T, MODE>, blocks, kActThreads, act_bulk_smem<nin>(), s, p, ntiles, status_flags_device());
            const int64_t done = ntiles * (kBulkTile / es);
            if (done == p.n) return check_launch("activation");
            const int st = check_launch("activation");
            if (st) return st;
            ActArgs t = p;
            t.out = static_cast<char*>(p.out) + done * es;
            t.a = static_cast<const char*>(p.a) + done * es;
            if (p.b) t.b = static_cast<const char*>(p.b) + done * es;
            t.n = p.n - done;
            t.out_stride = t.a_stride = t.b_stride = t.n;
            return launch_act<T, MODE>(t, s);
        }
    }
    const int64_t items = vec ? p.rows * (p.n / V) : p.rows * p.n;
    const int64_t want = (items + kActUnroll * kActThreads - 1) / (kActUnroll * kActThreads);
    const void* k = vec ? (p.rows == 1 ? (const void*)act_vec_kernel<T, MODE, true>
                                       : (const void*)act_vec_kernel<T, MODE, false>)
                        : (const void*)act_scalar_kernel<T, MODE>;
    const int blocks = resident_grid(k, kActThreads, 0, want);
    if (vec && p.rows == 1) launch_pdl(act_vec_kernel<T, MODE, true>, blocks, kActThreads, 0, s, p);
    else if (vec) launch_pdl(act_vec_kernel<T, MODE, false>, blocks, kActThreads, 0, s, p);
    else launch_pdl(act_scalar_kernel<T, MODE>, blocks, kActThreads, 0, s, p);
    return check_launch("activation");
}

template <int MODE>
static int dispatch_act(int dtype, const ActArgs& p, cudaStream_t s) {
    if (dtype == ANE_CUDA_F32) return launch_act<F32, MODE>(p, s);
    if (dtype == ANE_CUDA_F16) return launch_act<F16, MODE>(p, s);
    return launch_act<BF16, MODE>(p, s);
}

}  // namespace ane

extern "C" {

int ane_cuda_silu_mul(int dtype, void* out, int64_t out_stride, const void* gate,
                      int64_t gate_stride, const void* up, int64_t up_stride, int64_t rows,
                      int n, void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "silu_mul: bad dtype %d", dtype);
    if (rows < 0 || n <= 0)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "silu_mul: rows=%lld n=%d", (long long)rows, n);
    if (rows == 0) return ANE_CUDA_OK;
    if (!out || !gate || !up) return fail(ANE_CUDA_ERR_INVALID_ARG, "silu_mul: null pointer");
    if (out_stride < n || gate_stride < n || up_stride < n)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "silu_mul: row stride below n");
    ActArgs p{out, gate, up, out_stride, gate_stride, up_stride, rows, n};
    return dispatch_act<SILU_MUL>(dtype, p, as_stream(stream));
}

int ane_cuda_silu_inplace(int dtype, void* x, int64_t n, void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "silu_inplace: bad dtype %d", dtype);
    if (n < 0) return fail(ANE_CUDA_ERR_INVALID_ARG, "silu_inplace: n=%lld", (long long)n);
    if (n == 0) return ANE_CUDA_OK;
    if (!x) return fail(ANE_CUDA_ERR_INVALID_ARG, "silu_inplace: null pointer");
    ActArgs p{x, x, nullptr, n, n, 0, 1, n};
    return dispatch_act<SILU>(dtype, p, as_stream(stream));
}

int ane_cuda_mul_sigmoid_inplace(int dtype, void* y, const void* z, int64_t n, void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "mul_sigmoid_inplace: bad dtype %d", dtype);
    if (n < 0) return fail(ANE_CUDA_ERR_INVALID_ARG, "mul_sigmoid_inplace: n=%lld", (long long)n);
    if (n == 0) return ANE_CUDA_OK;
    if (!y || !z) return fail(ANE_CUDA_ERR_INVALID_ARG, "mul_sigmoid_inplace: null pointer");
    ActArgs p{y, y, z, n, n, n, 1, n};
    return dispatch_act<MUL_SIGMOID>(dtype, p, as_stream(stream));
}

}  // extern "C"
