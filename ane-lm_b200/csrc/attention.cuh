// attention.cuh -- decode attention over a ring KV cache, the kernel
// (core/cpu_ops.cpp:173-240 gqa_attention; ring bookkeeping
// models/llm/qwen3.cpp:475-488).
//
// One query token per sequence.  The keys of a sequence are cut into splits
// of kAttnKeys; one CTA takes one (split, kv head, sequence) and serves all
// the q heads of that kv head, so every K and V row is read from HBM once.
// (The 16-bit kernel further down takes several consecutive splits per CTA
// through a copy pipeline.)  The fp32 kernel's CTA
//   1. stages its K rows and V rows in shared memory with one bulk copy per
//      row (TMA engine, 16-byte aligned rows; the ring wrap is per row),
//      on two mbarriers so the score pass starts while V is in flight;
//   2. computes the scores (a lane group per key, q in registers), the
//      split's max, exp and sum, and its un-normalised P.V;
//   3. with one split: writes the output; otherwise writes the split's
//      (m, l, o) to the workspace, and a second kernel (decode_attention_
//      merge_kernel, launched right behind it with programmatic dependent
//      launch) combines the splits of each (kv head, sequence) and writes
//      the output.  No state survives a call: the workspace holds only the
//      partials of the call in flight, so it needs no clearing, whatever
//      calls of other shapes, graph replays or interrupted calls used it
//      before.
// Every summation order of the fp32 kernel is fixed, so a CPU restatement
// doing the same operations in the same order reproduces it bit for bit:
//   dot   EPL = max(16 B / element, head_dim / 32) consecutive elements per
//         lane, GL = head_dim / EPL lanes per key: an fmaf chain per lane,
//         then an xor butterfly over the GL lanes;
//   sum   local keys 0-31 and 32-63 each by a 32-lane butterfly, added;
//   P.V   U = 4 warps x (32 / GL) key groups: group u takes keys u, u+U, ...
//         (fmaf chain), a butterfly over the key groups of a warp, then the
//         four warps added in order;
//   merge M = max m_j, f_j = exp(m_j - M); O and L each as four fmaf chains
//         over the splits j = w (mod 4), added in order; out = O * (1 / L).
// exp is the pinned pinned_expf of ane_common.cuh.
#pragma once

#include <atomic>
#include <type_traits>

#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

constexpr int kAttnKeys = 64;  // keys per split (per CTA)
constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * kWarp;
constexpr int kAttnMaxGroup = 8;  // q heads per kv head
constexpr int kAttnMaxDevices = 64;
static_assert(kAttnThreads == 2 * kAttnKeys, "one copy-issuing thread per K row and per V row");

struct AttnArgs {
    void* out;
    int64_t out_stride;  // elements between sequences; heads are head_dim apart
    const void* q;
    int64_t q_stride;
    int q_head_stride;
    const void* k_cache;  // [batch][capacity][n_kv][head_dim]
    const void* v_cache;
    int64_t cache_stride;  // elements between sequences
    const int32_t* start;  // [batch] ring start
    const int32_t* len;    // [batch] keys in the ring
    int capacity;
    int n_heads, n_kv;
    int max_len, max_splits;
    int chunks;            // 64-key chunks per CTA (16-bit kernel; 1 for fp32)
    int stages;            // copy stages per warp (16-bit kernel)
    float scale;           // 1 / sqrtf(head_dim)
    float* part_ml;        // [batch][n_heads][max_splits][2]
    float* part_o;         // [batch][n_heads][max_splits][head_dim]
    unsigned int* flags;   // device status word
};

template <typename T, int HD>
struct AttnShape {
    static constexpr int V = T::kVec;
    static constexpr int EPL = HD / 32 > V ? HD / 32 : V;  // elements per lane
    static constexpr int NV = EPL / V;                     // 16-byte vectors per lane
    static constexpr int GL = HD / EPL;                    // lanes per key
    static constexpr int KPW = kWarp / GL;                 // keys per warp step
    static constexpr int U = kAttnWarps * KPW;             // key groups per CTA
    static constexpr int NKEY = kAttnKeys / U;             // keys per group in P.V
    // fp32 V rows go straight to registers (prefetched at the start) when a
    // lane's share is at most 16 vectors: that halves the shared memory of
    // a CTA, so a batch-1 launch fits in one wave.  16-bit rows are staged
    // in shared memory like K: their kernels are issue-bound at large
    // batch, and the extra registers would cost occupancy.
    static constexpr bool VREG = sizeof(typename T::storage) == 4 && NKEY * NV <= 16;
    static_assert(EPL % V == 0 && GL * EPL == HD && KPW * GL == kWarp, "head_dim layout");
};

// floats per key row of the probabilities in shared memory (vector loads)
template <int G>
__host__ __device__ constexpr int attn_prow() { return G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; }

template <typename T, int HD>
__host__ __device__ constexpr size_t attn_rows_bytes() {  // K rows, and V rows unless they live in registers
    return (AttnShape<T, HD>::VREG ? 1 : 2) * (size_t)kAttnKeys * HD * sizeof(typename T::storage);
}

// The warp partials of P.V ([warp][G][HD] floats) reuse the K rows, which
// are dead once the scores are taken: 4 G HD floats <= 64 HD elements.
template <typename T, int HD, int G>
__host__ __device__ constexpr size_t attn_smem_bytes() {
    static_assert((size_t)kAttnWarps * G * HD * sizeof(float) <=
                      (size_t)kAttnKeys * HD * sizeof(typename T::storage),
                  "warp partials must fit over the K rows");
    return attn_rows_bytes<T, HD>()
           + (size_t)kAttnKeys * attn_prow<G>() * sizeof(float);  // P, key-major
}

// Dots of one 32-key block (keys kb*32 ..) with GC q heads held in registers.
// The lanes of a key group (GL lanes, GL keys) hold partial dots of every
// key of the group and reduce them by a reduce-scatter: at each stage of
// the xor butterfly (offsets GL/2 .. 1) a lane keeps the half of the keys
// matching its lane bit and adds the partner's partial for them, so lane l
// ends with the full dot of key l of the group.  Each add pairs the same two
// partial sums as the plain butterfly, so the result is the same, with
// GL - 1 shuffles per head instead of GL * log2(GL).
template <typename T, int HD, int GC>
__device__ __forceinline__ void score_block(const typename T::storage* sK,
                                            const float (&qf)[GC][AttnShape<T, HD>::EPL], int kb,
                                            int lane, float (&dot)[GC]) {
    using Sh = AttnShape<T, HD>;
    constexpr int V = Sh::V, EPL = Sh::EPL, NV = Sh::NV, GL = Sh::GL, H2 = GL / 2;
    const int l = lane % GL;
    const typename T::storage* base = sK + (kb * kWarp + (lane / GL) * GL) * HD + l * EPL;
    float v[H2][GC];
    const bool up0 = (l & H2) != 0;
#pragma unroll
    for (int k = 0; k < H2; k++) {
        float klo[EPL], khi[EPL];
#pragma unroll
        for (int c = 0; c < NV; c++) {
            unpack<T>(*reinterpret_cast<const uint4*>(base + k * HD + c * V), &klo[c * V]);
            unpack<T>(*reinterpret_cast<const uint4*>(base + (k + H2) * HD + c * V), &khi[c * V]);
        }
#pragma unroll
        for (int g = 0; g < GC; g++) {
            float plo = 0.0f, phi = 0.0f;
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                plo = __fmaf_rn(qf[g][e], klo[e], plo);
                phi = __fmaf_rn(qf[g][e], khi[e], phi);
            }
            const float send = up0 ? plo : phi;
            const float keep = up0 ? phi : plo;
            v[k][g] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, H2));
        }
    }
#pragma unroll
    for (int off = H2 / 2; off >= 1; off >>= 1) {
        const bool up = (l & off) != 0;
#pragma unroll
        for (int k = 0; k < off; k++) {
#pragma unroll
            for (int g = 0; g < GC; g++) {
                const float send = up ? v[k][g] : v[k + off][g];
                const float keep = up ? v[k + off][g] : v[k][g];
                v[k][g] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
            }
        }
    }
#pragma unroll
    for (int g = 0; g < GC; g++) dot[g] = v[0][g];
}

// The end of a split, shared by the kernels: s_red holds the four warp
// partials of P.V ([warp][G][HD]), s_m / s_l the split's max and exp-sum as
// two halves each.  One split: write the output.  Otherwise write the
// split's (m, l, o) to the workspace for decode_attention_merge_kernel.
template <typename T, int HD, int G>
__device__ __forceinline__ void attn_finish(const AttnArgs& a, const float* s_red,
                                            const float (&s_m)[G][2], const float (&s_l)[G][2],
                                            int nsplit, int split, int kvh, int64_t b,
                                            typename T::storage* out) {
    const int tid = threadIdx.x;
    const int h0 = kvh * G;
    // the split's o = ((R0 + R1) + R2) + R3 over the warps
    auto sum4 = [&](int g, int d) {
        const float* r = s_red + g * HD + d;
        return __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[G * HD]), r[2 * G * HD]), r[3 * G * HD]);
    };

    if (nsplit == 1) {
        // the merge with one split: f = exp(m - m), chains 1-3 empty
        for (int idx = tid; idx < G * HD; idx += kAttnThreads) {
            const int g = idx / HD, d = idx % HD;
            const float m = fmaxf(s_m[g][0], s_m[g][1]);
            const float f = pinned_expf(__fsub_rn(m, m));
            const float lsum = __fadd_rn(s_l[g][0], s_l[g][1]);
            const float L = __fadd_rn(__fadd_rn(__fadd_rn(__fmaf_rn(lsum, f, 0.0f), 0.0f), 0.0f), 0.0f);
            const float O = __fadd_rn(__fadd_rn(__fadd_rn(__fmaf_rn(sum4(g, d), f, 0.0f), 0.0f), 0.0f), 0.0f);
            out[idx] = T::from_f(__fmul_rn(O, __fdiv_rn(1.0f, L)));
        }
        return;
    }

    const int64_t pbase = (b * a.n_heads + h0) * (int64_t)a.max_splits;  // (seq, head h0, split 0)
    for (int idx = tid; idx < G * HD; idx += kAttnThreads) {
        const int g = idx / HD, d = idx % HD;
        a.part_o[(pbase + (int64_t)g * a.max_splits + split) * HD + d] = sum4(g, d);
    }
    if (tid < G) {
        float2* ml = reinterpret_cast<float2*>(a.part_ml) + pbase + (int64_t)tid * a.max_splits + split;
        *ml = make_float2(fmaxf(s_m[tid][0], s_m[tid][1]), __fadd_rn(s_l[tid][0], s_l[tid][1]));
    }
}

// ---- the merge of the splits ------------------------------------------------
// One CTA per (block of CPB float4 columns of the head dimension, kv head,
// sequence), serving the G q heads of the kv head.  Launched behind the
// split kernel with programmatic dependent launch: it is resident and
// waiting (griddepcontrol.wait) when the last split finishes, and the
// wait makes every split's partials visible.  The arithmetic is the merge's
// pinned order: M = max m_j, f_j = exp(m_j - M); O and L each as four fmaf
// chains over the splits j = c (mod 4), in order of j; the chains added in
// order; out = O * (1 / L).  Each thread's first PRE partial-o loads are
// issued before the (m, l) round trip, so the two overlap.
constexpr int kMergeThreads = 128;
constexpr int kMergeTile = 256;  // splits per (m, l) tile in shared memory

template <int HD, int G>
struct MergeShape {
    static constexpr int COLS = HD / 4;  // float4 columns of a head
    static constexpr int ALL = G * 4 * COLS;  // (head, chain, column) items of a kv head
    static constexpr int fp2(int v) { return v >= 2 ? 2 * fp2(v / 2) : 1; }  // power of 2 <= v
    static constexpr int NB0 = fp2(ALL / kMergeThreads > 0 ? ALL / kMergeThreads : 1);
    static constexpr int NB = NB0 < COLS ? NB0 : COLS;  // column blocks (CTAs per kv head)
    static constexpr int CPB = COLS / NB;               // columns per block
    static constexpr int ITEMS = G * 4 * CPB;
    static constexpr int IPT = (ITEMS + kMergeThreads - 1) / kMergeThreads;
    static constexpr int PRE = 16 / IPT;  // partial-o loads issued ahead per item
    static_assert(COLS % NB == 0 && IPT <= 2, "merge layout");
};

template <typename T, int HD, int G>
__global__ void __launch_bounds__(kMergeThreads)
decode_attention_merge_kernel(const AttnArgs a) {
    pdl_begin();
    using MS = MergeShape<HD, G>;
    constexpr int COLS = MS::COLS, CPB = MS::CPB, ITEMS = MS::ITEMS, IPT = MS::IPT, PRE = MS::PRE;
    constexpr int FT = kMergeTile;
    __shared__ float2 s_ml[G][FT];
    __shared__ float s_M[G], s_L[G][4];
    __shared__ __align__(16) float s_o[4][G][CPB * 4];

    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int cb = blockIdx.x, kvh = blockIdx.y;
    const int64_t b = blockIdx.z;
    const int len = a.len[b], start = a.start[b];
    const bool bad = len > a.capacity || len > a.max_len ||
                     (len > 0 && (start < 0 || start >= a.capacity));
    if (len <= 0 || bad) return;  // the split kernel wrote zeros
    const int nchunk = (len + kAttnKeys - 1) / kAttnKeys;
    const int nsplit = (nchunk + a.chunks - 1) / a.chunks;
    if (nsplit <= 1) return;  // the split kernel wrote the output
    const int h0 = kvh * G;
    const int64_t pbase = (b * a.n_heads + h0) * (int64_t)a.max_splits;
    const float2* const ml_all = reinterpret_cast<const float2*>(a.part_ml) + pbase;  // [g][max_splits]
    const float4* const o_all = reinterpret_cast<const float4*>(a.part_o) + pbase * COLS;

    // this thread's items: (head g, chain c4, column col of the block)
    int it_g[IPT], it_c4[IPT], it_col[IPT];
    bool it_on[IPT];
#pragma unroll
    for (int it = 0; it < IPT; it++) {
        const int idx = tid + it * kMergeThreads;
        it_on[it] = ITEMS % kMergeThreads == 0 || idx < ITEMS;
        const int i = it_on[it] ? idx : 0;
        it_col[it] = i % CPB;
        it_c4[it] = (i / CPB) & 3;
        it_g[it] = i / (4 * CPB);
    }
    auto o_ptr = [&](int it) {  // partial o of split 0 of this item's head and column
        return o_all + (int64_t)it_g[it] * a.max_splits * COLS + cb * CPB + it_col[it];
    };
    const int ns0 = min(nsplit, FT);
    float4 pre[IPT][PRE];
#pragma unroll
    for (int it = 0; it < IPT; it++) {
        const float4* po = o_ptr(it);
#pragma unroll
        for (int r = 0; r < PRE; r++) {
            const int s = it_c4[it] + 4 * r;
            if (it_on[it] && s < ns0) pre[it][r] = __ldcg(po + (int64_t)s * COLS);
        }
    }

    // M = max over all splits; the first tile's (m, l) kept in shared memory
    for (int idx = tid; idx < G * ns0; idx += kMergeThreads) {
        const int g = idx / ns0, s = idx % ns0;
        s_ml[g][s] = __ldcg(ml_all + (int64_t)g * a.max_splits + s);
    }
    __syncthreads();
    for (int g = w; g < G; g += kMergeThreads / kWarp) {
        float mx = -INFINITY;
        for (int s = lane; s < ns0; s += kWarp) mx = fmaxf(mx, s_ml[g][s].x);
        for (int s = FT + lane; s < nsplit; s += kWarp)
            mx = fmaxf(mx, __ldcg(ml_all + (int64_t)g * a.max_splits + s).x);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        if (lane == 0) s_M[g] = mx;
    }
    __syncthreads();

    float4 o[IPT];
#pragma unroll
    for (int it = 0; it < IPT; it++) o[it] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float Lc = 0.0f;
    for (int s0 = 0; s0 < nsplit; s0 += FT) {
        const int s1 = min(nsplit, s0 + FT), ns = s1 - s0;
        if (s0 > 0) {
            __syncthreads();  // the previous tile consumed
            for (int idx = tid; idx < G * ns; idx += kMergeThreads) {
                const int g = idx / ns, s = idx % ns;
                s_ml[g][s] = __ldcg(ml_all + (int64_t)g * a.max_splits + s0 + s);
            }
            __syncthreads();
        }
        for (int idx = tid; idx < G * ns; idx += kMergeThreads) {
            float2& e = s_ml[idx / ns][idx % ns];
            e.x = pinned_expf(__fsub_rn(e.x, s_M[idx / ns]));
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < IPT; it++) {
            if (!it_on[it]) continue;
            const float2* f = s_ml[it_g[it]] - s0;
            int s = s0 + it_c4[it];
            if (s0 == 0) {
#pragma unroll
                for (int r = 0; r < PRE; r++, s += 4) {
                    if (s < s1) {
                        const float fs = f[s].x;
                        o[it].x = __fmaf_rn(pre[it][r].x, fs, o[it].x);
                        o[it].y = __fmaf_rn(pre[it][r].y, fs, o[it].y);
                        o[it].z = __fmaf_rn(pre[it][r].z, fs, o[it].z);
                        o[it].w = __fmaf_rn(pre[it][r].w, fs, o[it].w);
                    }
                }
            }
            const float4* po = o_ptr(it);
#pragma unroll 16
            for (; s < s1; s += 4) {
                const float4 v = __ldcg(po + (int64_t)s * COLS);
                const float fs = f[s].x;
                o[it].x = __fmaf_rn(v.x, fs, o[it].x);
                o[it].y = __fmaf_rn(v.y, fs, o[it].y);
                o[it].z = __fmaf_rn(v.z, fs, o[it].z);
                o[it].w = __fmaf_rn(v.w, fs, o[it].w);
            }
        }
        if (tid < 4 * G) {
            const int c4 = tid & 3, g = tid >> 2;
            const float2* f = s_ml[g] - s0;
            for (int s = s0 + c4; s < s1; s += 4) Lc = __fmaf_rn(f[s].y, f[s].x, Lc);
        }
    }
#pragma unroll
    for (int it = 0; it < IPT; it++)
        if (it_on[it]) reinterpret_cast<float4*>(s_o[it_c4[it]][it_g[it]])[it_col[it]] = o[it];
    if (tid < 4 * G) s_L[tid >> 2][tid & 3] = Lc;
    __syncthreads();
    typename T::storage* const out =
        static_cast<typename T::storage*>(a.out) + b * a.out_stride + (int64_t)h0 * HD + cb * CPB * 4;
    for (int idx = tid; idx < G * CPB * 4; idx += kMergeThreads) {
        const int g = idx / (CPB * 4), d = idx % (CPB * 4);
        const float L = __fadd_rn(__fadd_rn(__fadd_rn(s_L[g][0], s_L[g][1]), s_L[g][2]), s_L[g][3]);
        const float O = __fadd_rn(__fadd_rn(__fadd_rn(s_o[0][g][d], s_o[1][g][d]), s_o[2][g][d]), s_o[3][g][d]);
        out[(int64_t)g * HD + d] = T::from_f(__fmul_rn(O, __fdiv_rn(1.0f, L)));
    }
}

template <typename T, int HD, int G>
__global__ void __launch_bounds__(kAttnThreads)
decode_attention_kernel(const AttnArgs a) {
    pdl_begin();
    using S = typename T::storage;
    using Sh = AttnShape<T, HD>;
    constexpr int V = Sh::V, EPL = Sh::EPL, NV = Sh::NV, GL = Sh::GL, KPW = Sh::KPW, U = Sh::U;
    constexpr int NKEY = Sh::NKEY;
    constexpr bool VREG = Sh::VREG;
    constexpr int PROW = attn_prow<G>();
    constexpr int GA = (G + 1) / 2;  // heads of warps 0-1; warps 2-3 take the other G - GA
    constexpr uint32_t ROW = HD * sizeof(S);
    extern __shared__ __align__(16) unsigned char smem[];
    S* const sK = reinterpret_cast<S*>(smem);
    S* const sV = sK + kAttnKeys * HD;  // only when !VREG
    float* const s_p = reinterpret_cast<float*>(smem + attn_rows_bytes<T, HD>());  // [key][PROW]
    float* const s_red = reinterpret_cast<float*>(smem);  // [warp][G][HD], over the K rows
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float s_m[G][2], s_l[G][2];

    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int split = blockIdx.x, kvh = blockIdx.y;
    const int64_t b = blockIdx.z;
    const int len = __ldg(a.len + b), start = __ldg(a.start + b);
    const int h0 = kvh * G;
    S* const out = static_cast<S*>(a.out) + b * a.out_stride + (int64_t)h0 * HD;

    const bool bad = len > a.capacity || len > a.max_len ||
                     (len > 0 && (start < 0 || start >= a.capacity));
    if (len <= 0 || bad) {  // core/cpu_ops.cpp:176-179: no keys -> zeros
        if (split == 0) {
            for (int i = tid; i < G * HD; i += kAttnThreads) out[i] = T::from_f(0.0f);
            if (bad && tid == 0 && a.flags) atomicOr(a.flags, ANE_CUDA_FLAG_BAD_CACHE);
        }
        return;
    }
    const int nsplit = (len + kAttnKeys - 1) / kAttnKeys;
    if (split >= nsplit) return;
    const int t0 = split * kAttnKeys;
    const int n = min(kAttnKeys, len - t0);

    // ---- 1. stage K and V rows -------------------------------------------
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_expect_tx(&bars[0], (uint32_t)n * ROW);
        if constexpr (!VREG) mbar_expect_tx(&bars[1], (uint32_t)n * ROW);
    }
    __syncthreads();  // byte counts registered before any copy is issued
    // ring position of local key i (models/llm/qwen3.cpp:190-204)
    auto row_off = [&](int i) {
        int slot = start + t0 + i;
        if (slot >= a.capacity) slot -= a.capacity;
        return b * a.cache_stride + ((int64_t)slot * a.n_kv + kvh) * HD;
    };
    {
        const int i = tid & (kAttnKeys - 1);  // threads 0-63 copy K rows, 64-127 V rows
        if (i < n) {
            if (tid < kAttnKeys)
                bulk_load(sK + i * HD, static_cast<const S*>(a.k_cache) + row_off(i), ROW, &bars[0]);
            else if constexpr (!VREG)
                bulk_load(sV + i * HD, static_cast<const S*>(a.v_cache) + row_off(i), ROW, &bars[1]);
        }
    }
    // P.V layout: key group u (lanes j*GL .. of warp w) takes keys u, u+U, ...
    const int j = lane / GL, l = lane % GL;
    const int u = w * KPW + j;
    uint4 vreg[VREG ? NKEY : 1][NV];
    if constexpr (VREG) {  // this lane's V chunks of its P.V keys, in flight during the scores
#pragma unroll
        for (int r = 0; r < NKEY; r++) {
            const int k = u + r * U;
            if (k < n) {
                const S* vp = static_cast<const S*>(a.v_cache) + row_off(k) + l * EPL;
#pragma unroll
                for (int c = 0; c < NV; c++) vreg[r][c] = ld_stream(vp + c * V);
            }
        }
    }

    // Warp w scores keys kb*32 .. kb*32+31 (kb = w & 1) for the heads
    // g0 .. g0+gc-1 (warps 2-3 the second half; with G odd they carry one
    // unused head).  q is loaded while the copies fly.
    const int kb = w & 1;
    const int g0 = (w >> 1) * GA, gc = (w >> 1) ? G - GA : GA;
    float qf[GA][EPL];
#pragma unroll
    for (int g = 0; g < GA; g++) {
        const int h = h0 + min(g0 + g, G - 1);
        const S* qp = static_cast<const S*>(a.q) + b * a.q_stride + (int64_t)h * a.q_head_stride +
                      (lane % GL) * EPL;
#pragma unroll
        for (int c = 0; c < NV; c++) unpack<T>(ld_keep(qp + c * V), &qf[g][c * V]);
    }

    // A wait that gives up raises the flag, waits once more (bounded) for
    // the CTA's copies still in flight into its shared memory, and leaves
    // without output; the flag marks the call's results as invalid.
    auto give_up = [&]() {
        if (tid == 0 && a.flags) atomicOr(a.flags, ANE_CUDA_FLAG_WAIT_TIMEOUT);
        mbar_wait_bounded(&bars[0], 0);
        if constexpr (!VREG) mbar_wait_bounded(&bars[1], 0);
    };
    if (!__syncthreads_and(mbar_wait_bounded(&bars[0], 0))) {
        give_up();
        return;
    }

    // ---- 2a. scores, split max / exp / sum (lane = key within the block) ---
    const int i = kb * kWarp + lane;  // this lane's key in the split
    float x[GA];
    {
        float dot[GA];
        score_block<T, HD, GA>(sK, qf, kb, lane, dot);
#pragma unroll
        for (int g = 0; g < GA; g++) {
            x[g] = i < n ? __fmul_rn(dot[g], a.scale) : -INFINITY;
            float mx = x[g];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            if (lane == 0 && g < gc) s_m[g0 + g][kb] = mx;
        }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GA; g++) {
        if (g < gc) {  // warp-uniform
            const float m = fmaxf(s_m[g0 + g][0], s_m[g0 + g][1]);
            const float e = i < n ? pinned_expf(__fsub_rn(x[g], m)) : 0.0f;
            const float sum = butterfly_sum(e, kWarp);
            if (lane == 0) s_l[g0 + g][kb] = sum;
            s_p[i * PROW + g0 + g] = e;
        }
    }
    if constexpr (VREG) {
        __syncthreads();
    } else if (!__syncthreads_and(mbar_wait_bounded(&bars[1], 0))) {
        give_up();
        return;
    }

    // ---- 2b. un-normalised P.V: key group u takes keys u, u+U, ... -------
    float acc[G][EPL];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[g][e] = 0.0f;
#pragma unroll
    for (int r = 0; r < NKEY; r++) {
        const int k = u + r * U;
        if (k >= n) break;  // keys of a group ascend
        float vf[EPL];
#pragma unroll
        for (int c = 0; c < NV; c++) {
            if constexpr (VREG) unpack<T>(vreg[r][c], &vf[c * V]);
            else unpack<T>(*reinterpret_cast<const uint4*>(sV + k * HD + l * EPL + c * V), &vf[c * V]);
        }
        float p[PROW];
        if constexpr (PROW >= 4) {
#pragma unroll
            for (int c = 0; c < PROW / 4; c++) {
                const float4 t = reinterpret_cast<const float4*>(s_p + k * PROW)[c];
                p[4 * c] = t.x; p[4 * c + 1] = t.y; p[4 * c + 2] = t.z; p[4 * c + 3] = t.w;
            }
        } else if constexpr (PROW == 2) {
            const float2 t = reinterpret_cast<const float2*>(s_p + k * PROW)[0];
            p[0] = t.x; p[1] = t.y;
        } else {
            p[0] = s_p[k];
        }
#pragma unroll
        for (int g = 0; g < G; g++)
#pragma unroll
            for (int e = 0; e < EPL; e++) acc[g][e] = __fmaf_rn(p[g], vf[e], acc[g][e]);
    }
#pragma unroll
    for (int off = kWarp / 2; off >= GL; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; g++)
#pragma unroll
            for (int e = 0; e < EPL; e++)
                acc[g][e] = __fadd_rn(acc[g][e], __shfl_xor_sync(0xffffffffu, acc[g][e], off));
    }
    if (j == 0) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            float4* dst = reinterpret_cast<float4*>(s_red + (w * G + g) * HD + l * EPL);
#pragma unroll
            for (int e = 0; e < EPL / 4; e++)
                dst[e] = make_float4(acc[g][4 * e], acc[g][4 * e + 1], acc[g][4 * e + 2], acc[g][4 * e + 3]);
        }
    }
    __syncthreads();

    attn_finish<T, HD, G>(a, s_red, s_m, s_l, nsplit, split, kvh, b, out);
}


// ---------------------------------------------------------------------------
// 16-bit caches: the two contractions on the tensor cores (mma.sync
// m16n8k16, fp32 accumulation), and a pipelined split.  Both are taken
// transposed so that the 16 rows of an MMA tile are all used: S^T = K Q^T
// has a warp's 16 keys as rows and the kv head's q heads as the 8 columns
// (G <= 8; the rest are zero), one MMA per 16 dims; O^T = V^T P^T has 16
// dims as rows, one MMA per 16 dims and part of P.  The exps stay in
// registers: movmatrix transposes them from the accumulator layout of the
// first product into the operand layout of the second.  P is split into a
// high and a low part in the cache's type (fp16 scaled by 2^12 so the low
// part stays normal), so P.V keeps about 16 (bf16) / 22 (fp16) significant
// bits of each weight.
//
// A CTA takes `chunks` consecutive 64-key chunks of one (kv head,
// sequence); warp w takes keys 16w .. 16w+15 of every chunk.  Each warp
// runs its own copy pipeline: its lanes copy the chunk's K and V rows in
// 16-byte pieces (cp.async; the ring wrap is per row) into a ring of
// `stages` buffers, one commit group per chunk, so the copies of the next
// chunks are in flight while the current one is computed, and no block
// barrier is taken until the end of the split.  (One bulk copy per 256-byte
// row, as in the fp32 kernel, held this kernel to about 60% of the HBM
// bandwidth: many small bulk copies cost more than the same bytes in
// 16-byte pieces.)  The warp keeps a running
// max m, sum l and o per head (online softmax: when m grows, l and o are
// scaled by exp(m_old - m_new)); at the end the four warps are merged with
// f_w = exp(m_w - M) into the split's (M, L, O), which attn_finish writes
// out, or leaves for the merge kernel, like the fp32 kernel's.  The
// summation orders differ from the fp32 kernel's (the MMA's internal order
// is the hardware's): results agree with the fp32 order to within the
// output type's rounding.
// K and V rows sit in shared memory with a 16-byte pad per row, which makes
// the fragment loads (ldmatrix for K, ldmatrix.trans for V) free of bank
// conflicts.
template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    if constexpr (std::is_same<T, F16>::value)
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, "
                     "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
                     "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

// transposes an 8x8 matrix of 16-bit values held one pair per lane (row
// lane / 4, columns 2 (lane % 4) and + 1)
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t v) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(v));
    return d;
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

// two floats -> a packed pair of T (element 0 in the low half)
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x0, float x1) {
    if constexpr (std::is_same<T, F16>::value) {
        const __half2 h = __floats2half2_rn(x0, x1);
        return *reinterpret_cast<const uint32_t*>(&h);
    } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
}
template <typename T>
__device__ __forceinline__ float low_f(uint32_t v) {  // element 0 of a packed pair
    return T::to_f(*reinterpret_cast<const typename T::storage*>(&v));
}
template <typename T>
__device__ __forceinline__ float high_f(uint32_t v) {
    const uint32_t hi = v >> 16;
    return T::to_f(*reinterpret_cast<const typename T::storage*>(&hi));
}

template <int HD>
__host__ __device__ constexpr int attn_mma_rs() { return HD + 8; }  // padded row, elements

constexpr int kAttnWarpKeys = kAttnKeys / kAttnWarps;  // keys of a warp in one chunk
constexpr int kAttnMaxStages = 4;

template <int HD>
__host__ __device__ constexpr size_t attn_mma_stage_bytes() {  // one warp's K and V rows of a chunk
    return 2 * (size_t)kAttnWarpKeys * attn_mma_rs<HD>() * 2;
}
template <int HD>
__host__ __device__ constexpr size_t attn_mma_smem_bytes(int stages) {
    return (size_t)kAttnWarps * stages * attn_mma_stage_bytes<HD>();
}
// ring stages per warp: two to three chunks in flight per warp and two CTAs
// per SM (one at head_dim 256) cover the HBM latency
template <int HD>
__host__ __device__ constexpr int attn_mma_max_stages() { return HD <= 64 ? 4 : 3; }

template <typename T, int HD, int G>
__global__ void __launch_bounds__(kAttnThreads)
decode_attention_mma_kernel(const AttnArgs a) {
    pdl_begin();
    using S = typename T::storage;
    static_assert(sizeof(S) == 2, "16-bit caches");
    static_assert(G <= 8, "at most 8 q heads per kv head");
    constexpr int RS = attn_mma_rs<HD>();
    constexpr int WK = kAttnWarpKeys;
    constexpr int STAGE = 2 * WK * RS;  // elements: K rows, then V rows
    constexpr uint32_t ROW = HD * sizeof(S);
    constexpr int KSTEPS = HD / 16;
    constexpr bool F16S = std::is_same<T, F16>::value;
    constexpr float PSCALE = F16S ? 4096.0f : 1.0f;  // 2^12: fp16 low parts stay normal
    static_assert(WK == 16, "one 16-deep k-step of P.V per warp and chunk");
    // the warp partials fit in one stage set
    static_assert((size_t)kAttnWarps * G * HD * sizeof(float) <= attn_mma_smem_bytes<HD>(1),
                  "warp partials");
    extern __shared__ __align__(16) unsigned char smem[];
    float* const s_red = reinterpret_cast<float*>(smem);  // [warp][G][HD], after the pipelines
    __shared__ float s_m[G][2], s_l[G][2];
    __shared__ float s_wm[G][kAttnWarps], s_wl[G][kAttnWarps];

    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int gid = lane >> 2, tq = lane & 3;  // MMA fragment row / column pair
    const int split = blockIdx.x, kvh = blockIdx.y;
    const int64_t b = blockIdx.z;
    const int len = __ldg(a.len + b), start = __ldg(a.start + b);
    const int h0 = kvh * G;
    S* const out = static_cast<S*>(a.out) + b * a.out_stride + (int64_t)h0 * HD;

    const bool bad = len > a.capacity || len > a.max_len ||
                     (len > 0 && (start < 0 || start >= a.capacity));
    if (len <= 0 || bad) {  // core/cpu_ops.cpp:176-179: no keys -> zeros
        if (split == 0) {
            for (int i = tid; i < G * HD; i += kAttnThreads) out[i] = T::from_f(0.0f);
            if (bad && tid == 0 && a.flags) atomicOr(a.flags, ANE_CUDA_FLAG_BAD_CACHE);
        }
        return;
    }
    const int nchunk = (len + kAttnKeys - 1) / kAttnKeys;
    const int nsplit = (nchunk + a.chunks - 1) / a.chunks;
    if (split >= nsplit) return;
    const int c0 = split * a.chunks;              // first chunk of this CTA
    const int nc = min(nchunk - c0, a.chunks);    // its chunks, >= 1
    const int ns = a.stages;                      // 1 .. kAttnMaxStages

    // ---- the warp's copy ring -----------------------------------------------
    S* const ring = reinterpret_cast<S*>(smem) + (size_t)w * ns * STAGE;
    constexpr int CPR = ROW / 16;  // 16-byte pieces per row
    const S* const kbase = static_cast<const S*>(a.k_cache) + b * a.cache_stride + (int64_t)kvh * HD;
    const S* const vbase = static_cast<const S*>(a.v_cache) + b * a.cache_stride + (int64_t)kvh * HD;
    // the warp's keys of chunk j of the CTA: first key, and how many exist
    auto warp_keys = [&](int j, int& kb) {
        kb = (c0 + j) * kAttnKeys + WK * w;
        return min(WK, max(0, len - kb));
    };
    // chunk j into stage st: 16-byte asynchronous copies, CPR consecutive
    // lanes on the pieces of a key's K row and V row (rows 0-15 K, 16-31 V),
    // one commit group per chunk (an empty one past the last chunk keeps
    // the count)
    static_assert(CPR <= kWarp && kWarp % CPR == 0, "row pieces per lane");
    const int px = lane % CPR;
    auto issue = [&](int j, int st) {
        int kb;
        const int nw = j < nc ? warp_keys(j, kb) : 0;
        S* const dst = ring + st * STAGE + 8 * px;
#pragma unroll 4
        for (int key = lane / CPR; key < WK; key += kWarp / CPR) {
            if (key < nw) {
                int slot = start + kb + key;  // ring position (models/llm/qwen3.cpp:190-204)
                if (slot >= a.capacity) slot -= a.capacity;
                const int64_t off = (int64_t)slot * a.n_kv * HD + 8 * px;
                cp_async16(dst + key * RS, kbase + off);
                cp_async16(dst + (WK + key) * RS, vbase + off);
            }
        }
        cp_async_commit();
    };
    for (int j = 0; j < ns; j++) issue(j, j);

    // q fragments: the B operand of S^T = K Q^T (column gid = head gid < G;
    // other columns zero), loaded while the copies fly
    uint32_t qb[KSTEPS][2];
    {
        const bool hv = gid < G;
        const S* qp = static_cast<const S*>(a.q) + b * a.q_stride +
                      (int64_t)(h0 + (hv ? gid : 0)) * a.q_head_stride + 2 * tq;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ks++) {
            qb[ks][0] = hv ? __ldg(reinterpret_cast<const uint32_t*>(qp + 16 * ks)) : 0u;
            qb[ks][1] = hv ? __ldg(reinterpret_cast<const uint32_t*>(qp + 16 * ks + 8)) : 0u;
        }
    }

    // ---- 2. the chunks: scores, online softmax, P.V --------------------------
    // Transposed products fill the 16-row MMA tiles: S^T = K Q^T (rows: the
    // warp's 16 keys) and O^T = V^T P^T (rows: 16 dims), with P^T moved from
    // the accumulator layout of the first to the operand layout of the
    // second by movmatrix.  This thread: keys gid and gid + 8, heads
    // hA = 2 tq and hB = 2 tq + 1.
    const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: matrix, row
    const int koffK = ((mi & 1) * 8 + rr) * RS + (mi >> 1) * 8;  // keys (mi&1)*8+rr, dims +0/+8
    const int koffV = ((mi >> 1) * 8 + rr) * RS + (mi & 1) * 8;  // keys (mi>>1)*8+rr, dims +0/+8
    float o[HD / 16][4];  // O^T: dims 16t + gid (+8) x heads hA, hB
#pragma unroll
    for (int t = 0; t < HD / 16; t++) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.0f, lB = 0.0f;
    int st = 0;
    for (int j = 0; j < nc; j++) {
        cp_async_wait_pending(ns - 1);  // chunk j's group has landed (this lane's copies)
        __syncwarp();                   // ... and every lane's
        int kb;
        const int nw = warp_keys(j, kb);  // warp-uniform
        if (nw > 0) {
            const S* const sK = ring + st * STAGE;
            const S* const sV = sK + WK * RS;
            float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int ks = 0; ks < KSTEPS; ks++) {
                uint32_t ka[4];
                ldsm_x4(ka, sK + koffK + 16 * ks);
                mma16816<T>(sc, ka, qb[ks][0], qb[ks][1]);
            }
            // rows past the keys hold stale data: their scores become -inf
            // by selection, and their V fragments are zeroed below
            const bool v0 = gid < nw, v1 = gid + 8 < nw;
            const float x0 = v0 ? __fmul_rn(sc[0], a.scale) : -INFINITY;  // key gid, hA
            const float x1 = v0 ? __fmul_rn(sc[1], a.scale) : -INFINITY;  // key gid, hB
            const float x2 = v1 ? __fmul_rn(sc[2], a.scale) : -INFINITY;  // key gid + 8, hA
            const float x3 = v1 ? __fmul_rn(sc[3], a.scale) : -INFINITY;  // key gid + 8, hB
            float cA = fmaxf(x0, x2), cB = fmaxf(x1, x3);
#pragma unroll
            for (int off = 4; off <= 16; off <<= 1) {  // over the 8 key rows (gid)
                cA = fmaxf(cA, __shfl_xor_sync(0xffffffffu, cA, off));
                cB = fmaxf(cB, __shfl_xor_sync(0xffffffffu, cB, off));
            }
            const float nA = fmaxf(mA, cA), nB = fmaxf(mB, cB);
            // exps of x - m (<= 0, or NaN); NaN arguments stay NaN, as in pinned_expf
            auto exp2v = [](float2 d) {
                const float2 e = pinned_expf_nonpos2(d);
                return make_float2(d.x != d.x ? d.x : e.x, d.y != d.y ? d.y : e.y);
            };
            const float2 e01 = exp2v(make_float2(__fsub_rn(x0, nA), __fsub_rn(x1, nB)));
            const float2 e23 = exp2v(make_float2(__fsub_rn(x2, nA), __fsub_rn(x3, nB)));
            const float2 f = exp2v(make_float2(__fsub_rn(mA, nA), __fsub_rn(mB, nB)));  // 0 at first
            lA = __fmaf_rn(lA, f.x, __fadd_rn(e01.x, e23.x));
            lB = __fmaf_rn(lB, f.y, __fadd_rn(e01.y, e23.y));
            if (__any_sync(0xffffffffu, nA != mA || nB != mB)) {
#pragma unroll
                for (int t = 0; t < HD / 16; t++) {
                    o[t][0] = __fmul_rn(o[t][0], f.x);
                    o[t][1] = __fmul_rn(o[t][1], f.y);
                    o[t][2] = __fmul_rn(o[t][2], f.x);
                    o[t][3] = __fmul_rn(o[t][3], f.y);
                }
            }
            mA = nA;
            mB = nB;
            // P^T (keys x heads) in high and low parts, then transposed into
            // the B operand of O^T = V^T P^T: column gid = head gid, rows =
            // keys 2 tq, 2 tq + 1 (+ 8)
            uint32_t bh[2], bl[2];
            {
                const float p0 = __fmul_rn(e01.x, PSCALE), p1 = __fmul_rn(e01.y, PSCALE);
                const float p2 = __fmul_rn(e23.x, PSCALE), p3 = __fmul_rn(e23.y, PSCALE);
                const uint32_t h01 = pack2<T>(p0, p1), h23 = pack2<T>(p2, p3);
                const uint32_t l01 = pack2<T>(__fsub_rn(p0, low_f<T>(h01)), __fsub_rn(p1, high_f<T>(h01)));
                const uint32_t l23 = pack2<T>(__fsub_rn(p2, low_f<T>(h23)), __fsub_rn(p3, high_f<T>(h23)));
                bh[0] = movmatrix_trans(h01);
                bh[1] = movmatrix_trans(h23);
                bl[0] = movmatrix_trans(l01);
                bl[1] = movmatrix_trans(l23);
            }
            // V^T fragments by ldmatrix.trans: this thread gets
            // V[keys 2tq, 2tq+1 (+8)][dim]; halves of keys >= nw are zeroed
            // (their weight is 0, the data stale)
            const S* const vb = sV + koffV;
            auto pv = [&](auto masked) {
                uint32_t vm0 = 0xffffffffu, vm1 = 0xffffffffu;
                if constexpr (decltype(masked)::value) {
                    const int k0 = 2 * tq;
                    vm0 = (k0 < nw ? 0x0000ffffu : 0u) | (k0 + 1 < nw ? 0xffff0000u : 0u);
                    vm1 = (k0 + 8 < nw ? 0x0000ffffu : 0u) | (k0 + 9 < nw ? 0xffff0000u : 0u);
                }
#pragma unroll
                for (int t = 0; t < HD / 16; t++) {
                    uint32_t va[4];
                    ldsm_x4_trans(va, vb + 16 * t);
                    if constexpr (decltype(masked)::value) {
                        va[0] &= vm0;
                        va[1] &= vm0;
                        va[2] &= vm1;
                        va[3] &= vm1;
                    }
                    mma16816<T>(o[t], va, bh[0], bh[1]);
                    mma16816<T>(o[t], va, bl[0], bl[1]);
                }
            };
            if (nw == WK)
                pv(std::integral_constant<bool, false>());
            else
                pv(std::integral_constant<bool, true>());
        }
        __syncwarp();  // every lane is done with stage st
        issue(j + ns, st);
        st = st + 1 == ns ? 0 : st + 1;
    }

    // ---- 3. merge the four warps into the split's (M, L, O) -------------------
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
        lA = __fadd_rn(lA, __shfl_xor_sync(0xffffffffu, lA, off));
        lB = __fadd_rn(lB, __shfl_xor_sync(0xffffffffu, lB, off));
    }
    const int hA = 2 * tq, hB = 2 * tq + 1;
    if (gid == 0) {
        if (hA < G) {
            s_wm[hA][w] = mA;
            s_wl[hA][w] = lA;
        }
        if (hB < G) {
            s_wm[hB][w] = mB;
            s_wl[hB][w] = lB;
        }
    }
    __syncthreads();  // the rings are dead: every chunk's copies were waited for
    auto wmax = [&](int h) {
        return fmaxf(fmaxf(s_wm[h][0], s_wm[h][1]), fmaxf(s_wm[h][2], s_wm[h][3]));
    };
    if (hA < G) {
        const float fw = __fmul_rn(pinned_expf(__fsub_rn(mA, wmax(hA))), 1.0f / PSCALE);
        float* const r = s_red + (w * G + hA) * HD + gid;
#pragma unroll
        for (int t = 0; t < HD / 16; t++) {
            r[16 * t] = __fmul_rn(o[t][0], fw);
            r[16 * t + 8] = __fmul_rn(o[t][2], fw);
        }
    }
    if (hB < G) {
        const float fw = __fmul_rn(pinned_expf(__fsub_rn(mB, wmax(hB))), 1.0f / PSCALE);
        float* const r = s_red + (w * G + hB) * HD + gid;
#pragma unroll
        for (int t = 0; t < HD / 16; t++) {
            r[16 * t] = __fmul_rn(o[t][1], fw);
            r[16 * t + 8] = __fmul_rn(o[t][3], fw);
        }
    }
    if (tid < G) {
        const float M = wmax(tid);
        float lw[kAttnWarps];
#pragma unroll
        for (int v = 0; v < kAttnWarps; v++)
            lw[v] = __fmul_rn(s_wl[tid][v], pinned_expf(__fsub_rn(s_wm[tid][v], M)));
        s_m[tid][0] = s_m[tid][1] = M;
        s_l[tid][0] = __fadd_rn(lw[0], lw[1]);
        s_l[tid][1] = __fadd_rn(lw[2], lw[3]);
    }
    __syncthreads();
    attn_finish<T, HD, G>(a, s_red, s_m, s_l, nsplit, split, kvh, b, out);
}

// Launches the kernel instance for (head_dim, group); ANE_CUDA_ERR_UNSUPPORTED
// for shapes without one.
template <typename T>
int launch_decode_attention(const AttnArgs& a, int head_dim, int group, int64_t batch,
                            cudaStream_t s);

}  // namespace ane

namespace ane {

template <typename T, int HD, int G>
int launch_attention_shape(const AttnArgs& a, int64_t batch, cudaStream_t s) {
    // 16-bit caches: the tensor-core kernel; fp32: the CUDA-core kernel
    AttnArgs la = a;
    size_t smem;
    unsigned gx = (unsigned)a.max_splits;
    void (*kern)(AttnArgs);
    if constexpr (sizeof(typename T::storage) == 2) {
        kern = decode_attention_mma_kernel<T, HD, G>;
        constexpr int smax = attn_mma_max_stages<HD>();
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)attn_mma_smem_bytes<HD>(smax));
        // CTAs resident per SM with rings of 1 .. smax stages, queried once
        // per device
        static std::atomic<int> occ_dev[kAttnMaxDevices][kAttnMaxStages + 1];
        int dev = 0;
        if (e == cudaSuccess) e = cudaGetDevice(&dev);
        if (e == cudaSuccess && (dev < 0 || dev >= kAttnMaxDevices))
            return fail(ANE_CUDA_ERR_UNSUPPORTED, "decode_attention: device %d", dev);
        std::atomic<int>* const occ = occ_dev[dev];
        for (int st = 1; st <= smax && e == cudaSuccess; st++) {
            if (occ[st].load(std::memory_order_relaxed) > 0) continue;
            int per_sm = 0;
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kAttnThreads,
                                                              attn_mma_smem_bytes<HD>(st));
            occ[st].store(per_sm < 1 ? 1 : per_sm, std::memory_order_relaxed);
        }
        if (e != cudaSuccess)
            return fail(ANE_CUDA_ERR_CUDA, "decode_attention: %s", cudaGetErrorString(e));
        // Split each (kv head, sequence) into just enough CTAs to fill the
        // resident slots once: long splits keep the copy rings busy and
        // leave few partials to merge.  The slots depend on the ring depth,
        // which follows the chunks per CTA (up to smax), so each depth is
        // tried and the choice that needs exactly that depth and gives the
        // most CTAs is kept (one chunk per CTA and one stage at batch 1,
        // a single split and smax stages at large batch).
        const int nchunk = a.max_splits;  // 64-key chunks of the longest sequence
        const int64_t pairs = batch * a.n_kv;
        int64_t best_ctas = 0;
        la.chunks = nchunk;
        la.stages = smax < nchunk ? smax : nchunk;
        for (int st = 1; st <= smax; st++) {
            const int64_t slots = (int64_t)sm_count() * occ[st].load(std::memory_order_relaxed);
            int64_t nsplit = pairs >= slots ? 1 : slots / pairs;
            if (nsplit > nchunk) nsplit = nchunk;
            const int chunks = (int)((nchunk + nsplit - 1) / nsplit);
            const int need = chunks < smax ? chunks : smax;
            const int64_t ctas = pairs * ((nchunk + chunks - 1) / chunks);
            if (need == st && ctas > best_ctas) {
                best_ctas = ctas;
                la.chunks = chunks;
                la.stages = st;
            }
        }
        // Many sequences of a few chunks (at least two waves of CTAs at the
        // full depth): one stage less, when that keeps two and fits more
        // CTAs per SM -- residency then hides more latency than the deeper
        // ring (measured at 256 x 1K keys: 5.7 against 5.2 TB/s; at 64 x 4K,
        // under two waves, the full depth stays ahead).
        if (la.stages == smax && smax > 2 &&
            best_ctas >= 2 * (int64_t)sm_count() * occ[smax].load(std::memory_order_relaxed) &&
            occ[smax - 1].load(std::memory_order_relaxed) > occ[smax].load(std::memory_order_relaxed))
            la.stages = smax - 1;
        gx = (unsigned)((nchunk + la.chunks - 1) / la.chunks);
        smem = attn_mma_smem_bytes<HD>(la.stages);
    } else {
        kern = decode_attention_kernel<T, HD, G>;
        la.chunks = 1;
        la.stages = 0;
        smem = attn_smem_bytes<T, HD, G>();
        if (smem > 48 * 1024) {
            const cudaError_t e =
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess)
                return fail(ANE_CUDA_ERR_CUDA, "decode_attention: %s", cudaGetErrorString(e));
        }
    }
    const dim3 grid(gx, (unsigned)a.n_kv, (unsigned)batch);
    launch_pdl(kern, grid, kAttnThreads, smem, s, la);
    if (gx > 1) {  // some (kv head, sequence) may have several splits
        const dim3 mgrid((unsigned)MergeShape<HD, G>::NB, (unsigned)a.n_kv, (unsigned)batch);
        launch_pdl(decode_attention_merge_kernel<T, HD, G>, mgrid, kMergeThreads, 0, s, la);
    }
    return check_launch("decode_attention");
}

template <typename T, int HD>
int launch_attention_hd(const AttnArgs& a, int group, int64_t batch, cudaStream_t s) {
    switch (group) {
        case 1: return launch_attention_shape<T, HD, 1>(a, batch, s);
        case 2: return launch_attention_shape<T, HD, 2>(a, batch, s);
        case 3: return launch_attention_shape<T, HD, 3>(a, batch, s);
        case 4: return launch_attention_shape<T, HD, 4>(a, batch, s);
        case 5: return launch_attention_shape<T, HD, 5>(a, batch, s);
        case 6: return launch_attention_shape<T, HD, 6>(a, batch, s);
        case 7: return launch_attention_shape<T, HD, 7>(a, batch, s);
        case 8: return launch_attention_shape<T, HD, 8>(a, batch, s);
        default: return fail(ANE_CUDA_ERR_UNSUPPORTED, "decode_attention: %d q heads per kv head", group);
    }
}

template <typename T>
int launch_decode_attention(const AttnArgs& a, int head_dim, int group, int64_t batch,
                            cudaStream_t s) {
    switch (head_dim) {
        case 64: return launch_attention_hd<T, 64>(a, group, batch, s);
        case 128: return launch_attention_hd<T, 128>(a, group, batch, s);
        case 256: return launch_attention_hd<T, 256>(a, group, batch, s);
        default: return fail(ANE_CUDA_ERR_UNSUPPORTED, "decode_attention: head_dim %d", head_dim);
    }
}

}  // namespace ane
