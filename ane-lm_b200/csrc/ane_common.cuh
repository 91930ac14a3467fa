// ane_common.cuh -- device helpers shared by the sm_100a kernels of the
// ANE-LM layer-op / sampler / convert path.
//
// Every floating-point step that the result depends on is written with an
// explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn, __fmaf_rn,
// __fdiv_rn, __fsqrt_rn) so that nvcc cannot contract or reassociate it;
// the CPU restatement used by the tests performs the same operations in the
// same order, which is what makes the results reproducible bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "ane_cuda.h"

namespace ane {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------
struct F32 {
    using storage = float;
    static constexpr int kVec = 4;  // elements per 16-byte vector
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};
struct F16 {
    using storage = __half;
    static constexpr int kVec = 8;
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
struct BF16 {
    using storage = __nv_bfloat16;
    static constexpr int kVec = 8;
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// Unpack / pack one 16-byte vector of T into / from kVec floats.
template <typename T>
__device__ __forceinline__ void unpack(const uint4& v, float* f) {
    const typename T::storage* p = reinterpret_cast<const typename T::storage*>(&v);
#pragma unroll
    for (int i = 0; i < T::kVec; i++) f[i] = T::to_f(p[i]);
}
template <typename T>
__device__ __forceinline__ uint4 pack(const float* f) {
    uint4 v;
    typename T::storage* p = reinterpret_cast<typename T::storage*>(&v);
#pragma unroll
    for (int i = 0; i < T::kVec; i++) p[i] = T::from_f(f[i]);
    return v;
}

// 16-byte global accesses.  ld_stream / st_stream mark lines as touched
// once (evict-first), for rows that are read or written exactly once.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
    __stcs(reinterpret_cast<uint4*>(p), v);
}
__device__ __forceinline__ uint4 ld_keep(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}

// ---------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------
// Every kernel of the library is launched with programmatic stream
// serialisation (launch_pdl): the next kernel on the stream may be
// dispatched while this one drains, which hides most of the launch gap
// between the short kernels of a decode step.  A kernel so launched calls
// pdl_begin() before its first global-memory access: griddepcontrol.wait
// returns once the previous grid on the stream has completed and its
// writes are visible (immediately when the launch had no such attribute),
// so ordering and memory visibility are as with a plain launch.  Then
// launch_dependents lets the next kernel be dispatched; the hardware holds
// it back until every CTA of this grid has started, so it never takes SM
// slots this grid still needs.
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
}

// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes a
// multiple of 16).  A kernel issues it for its first inputs BEFORE
// pdl_begin(), so those bytes start to come from DRAM while the previous
// grid on the stream drains.  This is safe whatever that grid writes: a
// prefetch only fills L2, the point of coherence of the GPU's global memory,
// so a line fetched before the previous grid wrote it is updated there by
// that write, and the kernel's own loads, all issued after
// griddepcontrol.wait, see the written value.  Nothing is loaded into the
// SM (no L1 fill, no register), and no value a thread reads changes.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// ---------------------------------------------------------------------
// exp: Cody & Waite (1980) reduction x = k ln2 + r, k = rint(x log2 e),
// ln 2 as a float head + tail; Taylor series of e^r to degree 7 by Horner;
// scaling by 2^k with at most two multiplies (the second one rounds once
// into the subnormal range).  Constants: ln 2, log2 e and 1/n! rounded to
// float.  Used where the result must be reproducible bit for bit (the
// sampler's softmax).
// ---------------------------------------------------------------------
__device__ __forceinline__ float pow2i(int k) { return u2f((uint32_t)(k + 127) << 23); }

__device__ __forceinline__ float pinned_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return u2f(0x7F800000u);
    if (x < -104.0f) return 0.0f;
    const float k = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = __fmaf_rn(-k, 0.693147182464599609375f, x);
    r = __fmaf_rn(-k, -1.904654212125933608e-09f, r);
    float p = __fmaf_rn(0.00019841270113829523324966431f, r, 0.0013888889225199818611145020f);
    p = __fmaf_rn(p, r, 0.0083333337679505348205566406f);
    p = __fmaf_rn(p, r, 0.041666667908430099487304688f);
    p = __fmaf_rn(p, r, 0.16666667163372039794921875f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ki = (int)k;
    if (ki > 127) return __fmul_rn(__fmul_rn(p, 2.0f), pow2i(127));
    if (ki < -126) return __fmul_rn(__fmul_rn(p, pow2i(ki + 64)), pow2i(-64));
    return __fmul_rn(p, pow2i(ki));
}

// 2^x and 1/x from the special-function unit (ex2.approx, rcp.approx): a few
// ulp of fp32, used only where the result is rounded to 16 bits.  FTZ picks
// the flush-to-zero forms, cheaper, and exact enough when the stored type
// cannot represent fp32 subnormals anyway (fp16); bf16 keeps fp32's
// exponent range and needs the subnormal-preserving forms.
template <bool FTZ>
__device__ __forceinline__ float exp2f_approx(float x) {
    float y;
    if constexpr (FTZ) asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    else asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <bool FTZ>
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    if constexpr (FTZ) asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    else asm("rcp.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32 pairs (sm_100 f32x2): two independent IEEE operations per
// instruction, each rounded to nearest even with subnormals kept -- the same
// bits as __fmul_rn / __fmaf_rn element by element (checked on the B200 over
// 2^20 random pairs, specials included).
// The pairs are built and split inside the asm (mov.b64 {lo, hi}), so no
// value is reinterpreted through a pointer.  There is no packed add here on
// purpose: the compiler contracts a packed multiply feeding a packed add or
// subtract into a packed fma despite the .rn modifiers (seen as 1-ulp and
// cancellation differences against the reference), so sums after a packed
// multiply are taken with scalar __fadd_rn / __fsub_rn.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mov.b64 rc, {%6, %7};\n fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// pinned_expf for x <= 0 (softmax arguments x - max), without branches:
// the same operations in the same order as pinned_expf, so the same bits for
// every x in [-inf, 0]; the two-step subnormal scaling is selected, not
// branched.  NaN arguments are outside its contract.
__device__ __forceinline__ float pinned_expf_nonpos(float x) {
    const float xc = fmaxf(x, -104.0f);
    const float k = rintf(__fmul_rn(xc, 1.44269502162933349609375f));
    float r = __fmaf_rn(-k, 0.693147182464599609375f, xc);
    r = __fmaf_rn(-k, -1.904654212125933608e-09f, r);
    float p = __fmaf_rn(0.00019841270113829523324966431f, r, 0.0013888889225199818611145020f);
    p = __fmaf_rn(p, r, 0.0083333337679505348205566406f);
    p = __fmaf_rn(p, r, 0.041666667908430099487304688f);
    p = __fmaf_rn(p, r, 0.16666667163372039794921875f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ki = (int)k;
    const bool sub = ki < -126;
    float y = __fmul_rn(p, pow2i(sub ? ki + 64 : ki));
    y = sub ? __fmul_rn(y, pow2i(-64)) : y;
    return x < -104.0f ? 0.0f : y;
}

// pinned_expf_nonpos of two arguments: the same operations, the multiplies
// and fmas two at a time (packed f32x2, the same bits element by element).
// No packed multiply here feeds an add, so nothing can be contracted.
__device__ __forceinline__ float2 pinned_expf_nonpos2(float2 x) {
    const float2 xc = make_float2(fmaxf(x.x, -104.0f), fmaxf(x.y, -104.0f));
    const float2 t = mul2_rn(xc, make_float2(1.44269502162933349609375f, 1.44269502162933349609375f));
    const float2 k = make_float2(rintf(t.x), rintf(t.y));
    const float2 nk = make_float2(-k.x, -k.y);
    float2 r = fma2_rn(nk, make_float2(0.693147182464599609375f, 0.693147182464599609375f), xc);
    r = fma2_rn(nk, make_float2(-1.904654212125933608e-09f, -1.904654212125933608e-09f), r);
    const auto c2 = [](float c) { return make_float2(c, c); };
    float2 p = fma2_rn(c2(0.00019841270113829523324966431f), r, c2(0.0013888889225199818611145020f));
    p = fma2_rn(p, r, c2(0.0083333337679505348205566406f));
    p = fma2_rn(p, r, c2(0.041666667908430099487304688f));
    p = fma2_rn(p, r, c2(0.16666667163372039794921875f));
    p = fma2_rn(p, r, c2(0.5f));
    p = fma2_rn(p, r, c2(1.0f));
    p = fma2_rn(p, r, c2(1.0f));
    const int k0 = (int)k.x, k1 = (int)k.y;
    const bool s0 = k0 < -126, s1 = k1 < -126;
    float2 y = mul2_rn(p, make_float2(pow2i(s0 ? k0 + 64 : k0), pow2i(s1 ? k1 + 64 : k1)));
    y.x = s0 ? __fmul_rn(y.x, pow2i(-64)) : y.x;
    y.y = s1 ? __fmul_rn(y.y, pow2i(-64)) : y.y;
    return make_float2(x.x < -104.0f ? 0.0f : y.x, x.y < -104.0f ? 0.0f : y.y);
}

// ---------------------------------------------------------------------
// sin / cos for RoPE: reduction by pi/2 in double (pi/2 as double head +
// tail, two fma), reduced argument rounded to float, Taylor polynomials of
// sin (degree 9) and cos (degree 10) in float by Horner, quadrant rotation.
// ---------------------------------------------------------------------
__device__ __forceinline__ void pinned_sincosf(float x, float* s, float* c) {
    const double xd = (double)x;
    const double kd = rint(__dmul_rn(xd, 0x1.45f306dc9c883p-1));
    double rd = __fma_rn(-kd, 0x1.921fb54442d18p+0, xd);
    rd = __fma_rn(-kd, 0x1.1a62633145c07p-54, rd);
    const float r = __double2float_rn(rd);
    const int q = (int)__dsub_rn(kd, __dmul_rn(4.0, floor(__dmul_rn(kd, 0.25))));
    const float r2 = __fmul_rn(r, r);
    float t = __fmaf_rn(2.7557318844628753e-06f, r2, -0.00019841270113829523324966431f);
    t = __fmaf_rn(t, r2, 0.0083333337679505348205566406f);
    t = __fmaf_rn(t, r2, -0.16666667163372039794921875f);
    t = __fmul_rn(t, r2);
    const float sp = __fmaf_rn(t, r, r);
    float u = __fmaf_rn(-2.755731998149713e-07f, r2, 2.4801587642286904e-05f);
    u = __fmaf_rn(u, r2, -0.0013888889225199818611145020f);
    u = __fmaf_rn(u, r2, 0.041666667908430099487304688f);
    u = __fmaf_rn(u, r2, -0.5f);
    const float cp = __fmaf_rn(u, r2, 1.0f);
    switch (q) {
        case 0:  *s = sp;  *c = cp;  break;
        case 1:  *s = cp;  *c = -sp; break;
        case 2:  *s = -sp; *c = -cp; break;
        default: *s = -cp; *c = sp;  break;
    }
}

// ---------------------------------------------------------------------
// Bulk async copies (TMA engine, no tensor map) and mbarriers.  Loads are
// plain per-CTA copies: no cluster multicast anywhere in this library.
// ---------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes) : "memory");
}
// one arrival (release semantics) on a CTA-local mbarrier
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// global -> shared, `bytes` a multiple of 16, both addresses 16-byte aligned
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// 16-byte asynchronous global -> shared copy (both addresses 16-byte
// aligned), completed by cp_async_commit / cp_async_wait_pending
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// waits until at most n (0-3) of this thread's latest commit groups are pending
__device__ __forceinline__ void cp_async_wait_pending(int n) {
    switch (n) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    }
}
// orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// Waits for `phase` of `bar` for at most ~2^32 SM clock cycles (about 2 s);
// false on timeout.  Every wait in this library is bounded.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, phase)) {
        if (clock64() - t0 > (1ll << 32)) return false;
    }
    return true;
}

// Lane-partial fmaf chain of the pinned sum of squares (one chunk).
template <int N>
__device__ __forceinline__ float sumsq_chain(const float* v, float acc) {
#pragma unroll
    for (int i = 0; i < N; i++) acc = __fmaf_rn(v[i], v[i], acc);
    return acc;
}

// xor butterfly over `width` lanes (offsets width/2 .. 1); every lane ends
// with the same bits because IEEE addition is commutative.
__device__ __forceinline__ float butterfly_sum(float v, int width) {
    for (int off = width >> 1; off >= 1; off >>= 1)
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// inv = 1 / sqrtf(ss / dim + eps)   (core/cpu_ops.cpp:28)
__device__ __forceinline__ float rms_inv(float ss, int dim, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
}

__device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace ane
