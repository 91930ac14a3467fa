// ane_pack.cu -- fp32 <-> fp16 activation packing at the ANE boundary
// (core/ane_runtime.cpp:611-653, ANE_SPATIAL = 32 at core/ane_runtime.h:10).
//
// ane_matvec writes channel c of its token to element c * 32 of the fp16
// input surface [channels][32] and reads channel c of the result from
// element c * 32 of the output surface.  Batched here: token t goes to
// surface t / 32, spatial slot t % 32, so a full surface carries 32 tokens
// (the 1x1 convolutions the ANE runs treat spatial slots independently).
// Elements of slots without a token are left untouched, as the reference
// leaves slots 1-31.
//
// Both directions are transposes: one CTA takes one surface (32 tokens) and
// a chunk of kPackCh channels, stages the fp32 tile in shared memory and
// moves rows of the other layout with 16-byte accesses: token rows of
// kPackCh floats, surface rows of 32 halves (64 bytes).  The tile keeps
// 16-byte aligned token rows and swizzles their 4-channel chunks by the
// token's group of 8 (chunk ^ (t / 8) % 8), so that the float4 row accesses
// and the per-channel column accesses are both free of bank conflicts.
#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

constexpr int kSpatial = 32;
constexpr int kPackCh = 128;      // channels per CTA
constexpr int kPackThreads = 256;

// tile slot of (token t, channel c)
__device__ __forceinline__ int tslot(int t, int c) {
    return t * kPackCh + ((((c >> 2) ^ ((t >> 3) & 7))) << 2) + (c & 3);
}

// f32 -> f16 bits.  Round to nearest even as the arm64 __fp16 store does
// (core/ane_runtime.cpp:624), NaN -> quiet NaN 0x7E00 with the sign.
__device__ __forceinline__ uint16_t f2h_rne(float x) {
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7E00u);
    return __half_as_ushort(__float2half_rn(x));
}

// f32 -> f16 bits, the truncating f32_to_f16 of include/ane_lm/common.h:58-71
// (the x86 branch at core/ane_runtime.cpp:626): exponent re-bias by -112;
// >= 31 (Inf and NaN too) -> signed Inf; <= 0 -> hidden bit and mantissa
// shifted right, low bits dropped; below 2^-25 -> signed zero.
__device__ __forceinline__ uint16_t f2h_trunc(float x) {
    const uint32_t u = __float_as_uint(x);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const int e = (int)((u >> 23) & 0xFFu) - 112;
    const uint32_t frac = u & 0x7FFFFFu;
    if (e <= 0) return e < -10 ? sign : sign | (((frac | 0x800000u) >> (1 - e)) >> 13);
    if (e >= 31) return sign | 0x7C00u;
    return sign | ((uint32_t)e << 10) | (frac >> 13);
}

// f16 bits -> f32, exact, NaN payloads kept (include/ane_lm/common.h:35-56):
// the hardware conversion is exact for every non-NaN half; a NaN is rebuilt
// with its payload.
__device__ __forceinline__ float h2f_fast(uint32_t h) {
    const float f = __half2float(__ushort_as_half((unsigned short)h));
    const bool nan = (h & 0x7C00u) == 0x7C00u && (h & 0x3FFu) != 0u;
    return nan ? __uint_as_float(((h & 0x8000u) << 16) | 0x7F800000u | ((h & 0x3FFu) << 13)) : f;
}

// The same by integer operations (the generic path).
__device__ __forceinline__ float h2f_exact(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        const float v = __fmul_rn((float)m, 5.9604644775390625e-08f);  // m * 2^-24, exact
        return __uint_as_float(__float_as_uint(v) | sign);
    }
    if (e == 31) return __uint_as_float(sign | 0x7F800000u | (m << 13));
    return __uint_as_float(sign | ((e + 112u) << 23) | (m << 13));
}

template <bool TRUNC>
__device__ __forceinline__ uint32_t f2h(float x) {
    if constexpr (TRUNC) return f2h_trunc(x);
    else return f2h_rne(x);
}

// two values -> a packed pair of f16 bits (a in the low half), by one
// paired hardware conversion.  Round to nearest: NaNs then replaced as in
// f2h_rne.  Truncating: round-toward-zero conversion is f2h_trunc's
// truncation, subnormals included, except where f2h_trunc saturates
// (|x| >= 65536, Inf and NaN -> signed Inf), replaced after.
template <bool TRUNC>
__device__ __forceinline__ uint32_t f2h_pair(float a, float b) {
    if constexpr (TRUNC) {
        uint32_t h;
        asm("cvt.rz.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));  // b -> high half
        const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
        if ((ua & 0x7FFFFFFFu) >= 0x47800000u) h = (h & 0xFFFF0000u) | ((ua >> 16) & 0x8000u) | 0x7C00u;
        if ((ub & 0x7FFFFFFFu) >= 0x47800000u) h = (h & 0x0000FFFFu) | (ub & 0x80000000u) | 0x7C000000u;
        return h;
    } else {
        const __half2 hh = __floats2half2_rn(a, b);
        uint32_t h = *reinterpret_cast<const uint32_t*>(&hh);
        if (a != a) h = (h & 0xFFFF0000u) | ((__float_as_uint(a) >> 16) & 0x8000u) | 0x7E00u;
        if (b != b) h = (h & 0x0000FFFFu) | ((__float_as_uint(b) & 0x80000000u) | 0x7E000000u);
        return h;
    }
}

// in [tokens][in_stride] f32 -> surface [ceil(tokens/32)][channels][32] f16.
template <bool TRUNC, bool VEC>
__global__ void __launch_bounds__(kPackThreads)
ane_pack_kernel(uint16_t* __restrict__ surface, const float* __restrict__ in, int64_t in_stride,
                int64_t tokens, int channels) {
    pdl_begin();
    __shared__ __align__(16) float tile[kSpatial * kPackCh];
    const int64_t s = blockIdx.x;
    const int c0 = blockIdx.y * kPackCh;
    const int nc = min(kPackCh, channels - c0);
    const int64_t t0 = s * kSpatial;
    const int nt = (int)min((int64_t)kSpatial, tokens - t0);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    // token rows -> tile[t][c]; a full tile's four rows per warp are all
    // loaded before any is stored, so they are in flight together
    constexpr int RPW = kSpatial / (kPackThreads / kWarp);  // rows per warp
    if (VEC && nc == kPackCh && nt == kSpatial) {
        float4 v[RPW];
#pragma unroll
        for (int k = 0; k < RPW; k++)
            v[k] = __ldcs(reinterpret_cast<const float4*>(in + (t0 + w + 8 * k) * in_stride + c0) + lane);
#pragma unroll
        for (int k = 0; k < RPW; k++) *reinterpret_cast<float4*>(tile + tslot(w + 8 * k, 4 * lane)) = v[k];
    } else {
        for (int r = w; r < nt; r += kPackThreads / kWarp) {
            const float* row = in + (t0 + r) * in_stride + c0;
            if (VEC && nc == kPackCh) {
                const float4 v = __ldcs(reinterpret_cast<const float4*>(row) + lane);
                *reinterpret_cast<float4*>(tile + tslot(r, 4 * lane)) = v;
            } else {
                for (int c = lane; c < nc; c += kWarp) tile[tslot(r, c)] = __ldcs(row + c);
            }
        }
    }
    __syncthreads();
    // tile -> surface rows: item (c, q) = 8 slots 8q .. 8q+7 of channel c
    uint16_t* const sbase = surface + (s * channels + c0) * kSpatial;
    for (int item = tid; item < nc * 4; item += kPackThreads) {
        const int c = item >> 2, q = item & 3;
        uint16_t* dst = sbase + c * kSpatial + 8 * q;
        const float* col = tile + tslot(8 * q, c);  // tokens 8q .. 8q+7 share the swizzle
        if (nt == kSpatial) {
            uint32_t h[4];
#pragma unroll
            for (int i = 0; i < 4; i++) h[i] = f2h_pair<TRUNC>(col[2 * i * kPackCh], col[(2 * i + 1) * kPackCh]);
            __stcs(reinterpret_cast<uint4*>(dst), make_uint4(h[0], h[1], h[2], h[3]));
        } else {
            for (int i = 0; i < 8 && 8 * q + i < nt; i++)
                dst[i] = (uint16_t)f2h<TRUNC>(col[i * kPackCh]);
        }
    }
}

// surface [ceil(tokens/32)][channels][32] f16 -> out [tokens][out_stride] f32.
template <bool VEC>
__global__ void __launch_bounds__(kPackThreads)
ane_unpack_kernel(float* __restrict__ out, int64_t out_stride, const uint16_t* __restrict__ surface,
                  int64_t tokens, int channels) {
    pdl_begin();
    __shared__ __align__(16) float tile[kSpatial * kPackCh];
    const int64_t s = blockIdx.x;
    const int c0 = blockIdx.y * kPackCh;
    const int nc = min(kPackCh, channels - c0);
    const int64_t t0 = s * kSpatial;
    const int nt = (int)min((int64_t)kSpatial, tokens - t0);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const uint16_t* const sbase = surface + (s * channels + c0) * kSpatial;
    auto put = [&](int item, const uint4 v) {  // 8 slots of a channel -> the tile
        const int c = item >> 2, q = item & 3;
        const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
        float* col = tile + tslot(8 * q, c);  // tokens 8q .. 8q+7 share the swizzle
#pragma unroll
        for (int i = 0; i < 8; i++) col[i * kPackCh] = h2f_fast((wd[i >> 1] >> (16 * (i & 1))) & 0xFFFFu);
    };
    constexpr int IPT = kPackCh * 4 / kPackThreads;  // items per thread of a full tile
    if (nc == kPackCh && nt == kSpatial) {
        uint4 v[IPT];  // all loaded before any is converted
#pragma unroll
        for (int k = 0; k < IPT; k++) {
            const int item = tid + k * kPackThreads;
            v[k] = __ldcs(reinterpret_cast<const uint4*>(sbase + (item >> 2) * kSpatial + 8 * (item & 3)));
        }
#pragma unroll
        for (int k = 0; k < IPT; k++) put(tid + k * kPackThreads, v[k]);
    } else {
        for (int item = tid; item < nc * 4; item += kPackThreads) {
            if (8 * (item & 3) >= nt) continue;
            put(item, __ldcs(reinterpret_cast<const uint4*>(sbase + (item >> 2) * kSpatial + 8 * (item & 3))));
        }
    }
    __syncthreads();
    for (int r = w; r < nt; r += kPackThreads / kWarp) {
        float* row = out + (t0 + r) * out_stride + c0;
        if (VEC && nc == kPackCh) {
            __stcs(reinterpret_cast<float4*>(row) + lane,
                   *reinterpret_cast<const float4*>(tile + tslot(r, 4 * lane)));
        } else {
            for (int c = lane; c < nc; c += kWarp) __stcs(row + c, tile[tslot(r, c)]);
        }
    }
}

// Any spatial size: one thread per (token, channel).
template <bool TRUNC>
__global__ void ane_pack_any_kernel(uint16_t* surface, const float* in, int64_t in_stride,
                                    int64_t tokens, int channels, int spatial) {
    pdl_begin();
    const int64_t total = tokens * channels;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / channels;
        const int c = (int)(i - t * channels);
        surface[((t / spatial) * channels + c) * spatial + t % spatial] =
            (uint16_t)f2h<TRUNC>(in[t * in_stride + c]);
    }
}

__global__ void ane_unpack_any_kernel(float* out, int64_t out_stride, const uint16_t* surface,
                                      int64_t tokens, int channels, int spatial) {
    pdl_begin();
    const int64_t total = tokens * channels;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / channels;
        const int c = (int)(i - t * channels);
        out[t * out_stride + c] = h2f_exact(surface[((t / spatial) * channels + c) * spatial + t % spatial]);
    }
}

static int check_pack(const char* fn, const void* a, const void* b, int64_t stride, int64_t tokens,
                      int channels, int spatial) {
    if (tokens < 0 || channels <= 0 || spatial <= 0 || stride < channels)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: tokens=%lld channels=%d spatial=%d stride=%lld", fn,
                    (long long)tokens, channels, spatial, (long long)stride);
    if (tokens > 0 && (!a || !b)) return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: null pointer", fn);
    if ((tokens + spatial - 1) / spatial > 0x7FFFFFFFll)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "%s: %lld tokens", fn, (long long)tokens);
    return ANE_CUDA_OK;
}

}  // namespace ane

extern "C" {

int ane_cuda_ane_pack(int round_mode, uint16_t* surface, const float* in, int64_t in_stride,
                      int64_t tokens, int channels, int spatial, void* stream) {
    using namespace ane;
    if (round_mode != ANE_CUDA_ROUND_NEAREST && round_mode != ANE_CUDA_ROUND_TRUNCATE)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "ane_pack: round_mode %d", round_mode);
    int st = check_pack("ane_pack", surface, in, in_stride, tokens, channels, spatial);
    if (st || tokens == 0) return st;
    const bool trunc = round_mode == ANE_CUDA_ROUND_TRUNCATE;
    cudaStream_t s = as_stream(stream);
    if (spatial == kSpatial && is_aligned(surface, 16)) {
        const dim3 grid((unsigned)((tokens + kSpatial - 1) / kSpatial),
                        (unsigned)((channels + kPackCh - 1) / kPackCh));
        if (grid.y > 65535) return fail(ANE_CUDA_ERR_UNSUPPORTED, "ane_pack: %d channels", channels);
        const bool vec = is_aligned(in, 16) && in_stride % 4 == 0;
        if (trunc) {
            if (vec) launch_pdl(ane_pack_kernel<true, true>, grid, kPackThreads, 0, s, surface, in, in_stride, tokens, channels);
            else launch_pdl(ane_pack_kernel<true, false>, grid, kPackThreads, 0, s, surface, in, in_stride, tokens, channels);
        } else {
            if (vec) launch_pdl(ane_pack_kernel<false, true>, grid, kPackThreads, 0, s, surface, in, in_stride, tokens, channels);
            else launch_pdl(ane_pack_kernel<false, false>, grid, kPackThreads, 0, s, surface, in, in_stride, tokens, channels);
        }
    } else {
        const int blocks = resident_grid(reinterpret_cast<const void*>(ane_pack_any_kernel<false>), 256, 0,
                                         (tokens * channels + 255) / 256);
        if (trunc) launch_pdl(ane_pack_any_kernel<true>, blocks, 256, 0, s, surface, in, in_stride, tokens, channels, spatial);
        else launch_pdl(ane_pack_any_kernel<false>, blocks, 256, 0, s, surface, in, in_stride, tokens, channels, spatial);
    }
    return check_launch("ane_pack");
}

int ane_cuda_ane_unpack(float* out, int64_t out_stride, const uint16_t* surface, int64_t tokens,
                        int channels, int spatial, void* stream) {
    using namespace ane;
    int st = check_pack("ane_unpack", out, surface, out_stride, tokens, channels, spatial);
    if (st || tokens == 0) return st;
    cudaStream_t s = as_stream(stream);
    if (spatial == kSpatial && is_aligned(surface, 16)) {
        const dim3 grid((unsigned)((tokens + kSpatial - 1) / kSpatial),
                        (unsigned)((channels + kPackCh - 1) / kPackCh));
        if (grid.y > 65535) return fail(ANE_CUDA_ERR_UNSUPPORTED, "ane_unpack: %d channels", channels);
        if (is_aligned(out, 16) && out_stride % 4 == 0)
            launch_pdl(ane_unpack_kernel<true>, grid, kPackThreads, 0, s, out, out_stride, surface, tokens, channels);
        else
            launch_pdl(ane_unpack_kernel<false>, grid, kPackThreads, 0, s, out, out_stride, surface, tokens, channels);
    } else {
        const int blocks = resident_grid(reinterpret_cast<const void*>(ane_unpack_any_kernel), 256, 0,
                                         (tokens * channels + 255) / 256);
        launch_pdl(ane_unpack_any_kernel, blocks, 256, 0, s, out, out_stride, surface, tokens, channels, spatial);
    }
    return check_launch("ane_unpack");
}

}  // extern "C"
