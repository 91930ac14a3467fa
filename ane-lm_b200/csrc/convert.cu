// convert.cu -- BF16 -> FP16 weight conversion, bit-exact with the
// reference's truncating bf16_to_f16 (include/ane_lm/common.h:58-75).
//
// HBM-bound streaming kernel: 2 bytes read + 2 bytes written per element.
// Long inputs stream through a bulk-copy ring in shared memory
// (bf16_to_f16_bulk_kernel); shorter or unaligned ones use 16-byte vectors
// (8 elements) with evict-first loads and stores, kConvUnroll vectors in
// flight, over a grid of one resident wave.
#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

// One element (scalar tail): exponent re-bias by -112; e >= 31 (Inf/NaN included) ->
// signed Inf; 1 <= e <= 30 -> e<<10 | top 7 mantissa bits << 3;
// -10 <= e <= 0 -> (1.m << 16) >> (14 - e), i.e. the hidden-bit mantissa
// shifted right by (1 - e) and then by 13, truncating; below -> signed 0.
__device__ __forceinline__ uint32_t bf16_to_f16_bits(uint32_t b) {
    const uint32_t sign = b & 0x8000u;
    const int e = (int)((b >> 7) & 0xFFu) - 112;
    const uint32_t m7 = b & 0x7Fu;
    uint32_t r;
    if (e >= 31)
        r = 0x7C00u;
    else if (e >= 1)
        r = ((uint32_t)e << 10) | (m7 << 3);
    else if (e >= -10)
        r = ((m7 | 0x80u) << 16) >> (14 - e);
    else
        r = 0u;
    return sign | r;
}

// Two elements at once.  Round-toward-zero conversion of the exact fp32
// value is the reference's truncation, subnormals included (it drops the
// bits below 2^-24, and below 2^-25 nothing is left); it differs only where
// the reference saturates: |x| >= 65536, Inf and NaN become signed Inf
// (round-toward-zero would give 65504 or NaN), fixed up with a mask.
__device__ __forceinline__ uint32_t cvt_pair(uint32_t w) {
    const float lo = __uint_as_float(w << 16);
    const float hi = __uint_as_float(w & 0xFFFF0000u);
    uint32_t r;
    asm("cvt.rz.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    const uint32_t big = __vcmpgeu2(w & 0x7FFF7FFFu, 0x47804780u);  // 0xFFFF per saturating half
    return (r & ~big) | (((w & 0x80008000u) | 0x7C007C00u) & big);
}

__device__ __forceinline__ uint4 cvt_vec(uint4 v) {
    return make_uint4(cvt_pair(v.x), cvt_pair(v.y), cvt_pair(v.z), cvt_pair(v.w));
}

constexpr int kConvThreads = 256;
constexpr int kConvUnroll = 4;

// Vector path: in/out 16-byte aligned, nvec 8-element vectors.
__global__ void __launch_bounds__(kConvThreads)
bf16_to_f16_vec_kernel(uint4* __restrict__ out, const uint4* __restrict__ in, int64_t nvec) {
    pdl_begin();
    const int64_t stride = (int64_t)gridDim.x * kConvThreads;
    int64_t i = (int64_t)blockIdx.x * kConvThreads + threadIdx.x;
    // Main loop: kConvUnroll independent vectors per thread in flight.
    for (; i + (kConvUnroll - 1) * stride < nvec; i += kConvUnroll * stride) {
        uint4 v[kConvUnroll];
#pragma unroll
        for (int u = 0; u < kConvUnroll; u++) v[u] = ld_stream(in + i + u * stride);
#pragma unroll
        for (int u = 0; u < kConvUnroll; u++) st_stream(out + i + u * stride, cvt_vec(v[u]));
    }
    for (; i < nvec; i += stride) st_stream(out + i, cvt_vec(ld_stream(in + i)));
}


// Long inputs: a persistent CTA per SM streams 64 KB tiles through a
// two-stage ring in shared memory filled by one bulk copy (TMA) per tile,
// converting the previous tile from shared memory with 16-byte streaming
// stores (the same pattern as the activation kernels: few, large copies
// keep the DRAM request stream long and sequential; 16-64 KB tiles and 2-4
// stages were measured, 64 KB x 2 was fastest).
constexpr int kConvTile = 65536;  // bytes per tile
constexpr int kConvStages = 2;
constexpr size_t kConvSmem = (size_t)kConvStages * kConvTile;

__global__ void __launch_bounds__(kConvThreads)
bf16_to_f16_bulk_kernel(uint4* __restrict__ out, const uint4* __restrict__ in, int64_t ntiles,
                        unsigned int* flags) {
    pdl_begin();
    constexpr int VPT = kConvTile / 16;          // 16-byte vectors per tile
    constexpr int STEPS = VPT / kConvThreads;    // per thread
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full[kConvStages];
    const int tid = threadIdx.x;
    const int64_t G = gridDim.x;
    if (tid == 0) {
        for (int s = 0; s < kConvStages; s++) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    // thread 0: tile -> stage s (the stage's earlier generic reads are
    // ordered before the copy by the barrier before the call and the fence)
    auto issue = [&](int64_t tile, int s) {
        fence_proxy_async();
        mbar_expect_tx(&full[s], kConvTile);
        bulk_load(smem + s * kConvTile, in + tile * VPT, kConvTile, &full[s]);
    };
    if (tid == 0)
        for (int s = 0; s < kConvStages; s++)
            if (blockIdx.x + s * G < ntiles) issue(blockIdx.x + s * G, s);
    int s = 0;
    uint32_t ph = 0u;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += G) {
        if (!__syncthreads_and(mbar_wait_bounded(&full[s], (ph >> s) & 1u))) {
            // a copy did not land in time: flag it, wait (bounded) once more
            // for every stage still in flight, and stop
            if (tid == 0) {
                if (flags) atomicOr(flags, ANE_CUDA_FLAG_WAIT_TIMEOUT);
                for (int k = 0; k < kConvStages; k++) {
                    const int sk = (s + k) % kConvStages;
                    if (tile + k * G < ntiles) mbar_wait_bounded(&full[sk], (ph >> sk) & 1u);
                }
            }
            return;
        }
        ph ^= 1u << s;
        const uint4* const src = reinterpret_cast<const uint4*>(smem + s * kConvTile);
#pragma unroll
        for (int st = 0; st < STEPS; st++) {
            const int v = st * kConvThreads + tid;
            st_stream(out + tile * VPT + v, cvt_vec(src[v]));
        }
        __syncthreads();  // stage s consumed by every thread
        if (tid == 0 && tile + kConvStages * G < ntiles) issue(tile + kConvStages * G, s);
        s = s + 1 == kConvStages ? 0 : s + 1;
    }
}

// Scalar path for the ragged tail or unaligned buffers.
__global__ void bf16_to_f16_scalar_kernel(uint16_t* __restrict__ out,
                                          const uint16_t* __restrict__ in, int64_t n) {
    pdl_begin();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = (uint16_t)bf16_to_f16_bits(in[i]);
}

}  // namespace ane

extern "C" int ane_cuda_bf16_to_f16(uint16_t* out, const uint16_t* in, int64_t n, void* stream) {
    using namespace ane;
    if (n < 0) return fail(ANE_CUDA_ERR_INVALID_ARG, "bf16_to_f16: n = %lld < 0", (long long)n);
    if (n == 0) return ANE_CUDA_OK;
    if (!out || !in) return fail(ANE_CUDA_ERR_INVALID_ARG, "bf16_to_f16: null pointer");
    cudaStream_t s = as_stream(stream);
    const int sms = sm_count();
    int64_t done = 0;
    const int64_t ntiles = is_aligned(out, 16) && is_aligned(in, 16) ? n * 2 / kConvTile : 0;
    if (ntiles >= 2 * (int64_t)sms) {  // long inputs: the bulk-copy ring over whole tiles
        const cudaError_t e = cudaFuncSetAttribute(bf16_to_f16_bulk_kernel,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kConvSmem);
        if (e != cudaSuccess) return fail(ANE_CUDA_ERR_CUDA, "bf16_to_f16: %s", cudaGetErrorString(e));
        const int blocks = resident_grid((const void*)bf16_to_f16_bulk_kernel, kConvThreads, kConvSmem, ntiles);
        launch_pdl(bf16_to_f16_bulk_kernel, blocks, kConvThreads, kConvSmem, s,
            reinterpret_cast<uint4*>(out), reinterpret_cast<const uint4*>(in), ntiles, status_flags_device());
        done = ntiles * (kConvTile / 2);
    }
    if (is_aligned(out + done, 16) && is_aligned(in + done, 16) && n - done >= 8) {
        const int64_t nvec = (n - done) / 8;
        const int64_t want = (nvec + kConvThreads * kConvUnroll - 1) / (kConvThreads * kConvUnroll);
        const int blocks = resident_grid((const void*)bf16_to_f16_vec_kernel, kConvThreads, 0, want);
        launch_pdl(bf16_to_f16_vec_kernel, blocks, kConvThreads, 0, s,
            reinterpret_cast<uint4*>(out + done), reinterpret_cast<const uint4*>(in + done), nvec);
        done += nvec * 8;
    }
    if (done < n) {
        const int64_t rest = n - done;
        const int blocks = (int)((rest + 255) / 256 < (int64_t)sms * 4 ? (rest + 255) / 256 : (int64_t)sms * 4);
        launch_pdl(bf16_to_f16_scalar_kernel, blocks, 256, 0, s, out + done, in + done, rest);
    }
    return check_launch("bf16_to_f16");
}
