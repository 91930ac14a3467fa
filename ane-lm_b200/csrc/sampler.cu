// sampler.cu -- batched sample_token (core/sampling.cpp:10-66) and softmax
// (core/cpu_ops.cpp:83-99), one CTA per row: 512 threads, two CTAs per SM,
// so that a batch of up to 2 x SMs rows runs in a single wave; a batch of
// at most one row per SM (a row-sharded batch on several GPUs) takes one
// 1024-thread CTA per row instead.  The summation orders below are those of
// 1024 virtual threads whatever the CTA size, so both give the same bits.
//
// Pass 0  the row's repetition window goes into a shared-memory hash
//         (id -> count) and a vocabulary bitmap; each distinct id's logit is
//         penalised once (rep, then freq), as sampling.cpp:17-42 does.
// Pass 1  max of the penalised logits (argmax for temperature <= 0), back
//         to front, eight 16-byte groups in flight per thread; max.NaN
//         propagates a NaN logit into the result, which is all the NaN rule
//         needs.  max(fl(a * inv_t)) = fl(max(a) * inv_t) since rounding is
//         monotone.
// Pass 2  e = exp(d), d = fl(fl(a * inv_t) - max), summed in the pinned order
//         of 1024 "virtual threads": group g of 4 consecutive elements belongs
//         to virtual thread g % 1024, which adds its elements in increasing
//         order; an xor butterfly inside each virtual warp of 32, then over
//         the 32 virtual-warp sums.  Thread t of the CTA plays virtual threads
//         t and t + 512, so the bits do not depend on the CTA size.
// Pass 3  the inverse-CDF scan `cum += p[i]; if (cum >= r) return i`, with
//         p = fl(e * (1/sum)), reproduced bit for bit in parallel.  While cum
//         stays inside one binade [2^E, 2^(E+1)) (or below 2^-125), every fp32
//         add cum + p lands on a multiple of U = ulp(cum) and equals
//         cum + round(p / U) * U, unless p / U is an exact tie.  So over a
//         tile of 4096 elements the running sums are an integer prefix sum
//         in units of U.  The first element that is a tie, is larger than the
//         binade, or carries the sum out of the binade is added serially with
//         a real fp32 add, the binade is re-derived, and the tile resumes
//         after it.  The first element whose running sum reaches r (in
//         units: ceil(r / U)) is the token.
//         Elements with d < T(E) = ln(U / (2 inv)) - 1e-4 have p < U / 2:
//         they add 0 units, are no tie and cannot leave the binade.  U only
//         grows along the row, so an element found insignificant stays so.
//         A tile's elements are tested against a logit floor xl with
//         d(xl) < T(E) (a superset of the significant ones, one compare per
//         element); each warp compacts its candidates in element order into
//         shared memory and evaluates their p once.  The first tile, where
//         cum leaves its binade every few elements, is summed serially in
//         fp32 by one thread until the binade holds for 256 elements.
#include <atomic>

#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

constexpr int kSampThreads = 512;                 // softmax, and sampling with more rows than SMs
constexpr int kSampThreadsWide = 1024;            // sampling with at most one row per SM
constexpr int kMaxSampWarps = kSampThreadsWide / kWarp;
constexpr int kVirtThreads = 1024;                 // pinned softmax-sum order
constexpr int kPerThread = 8;                      // CDF elements per thread per tile
constexpr int kMaxSweep = 8;                       // groups of 4 in flight per thread, max pass
constexpr int kMaxWindow = 4096;
constexpr uint32_t kSat = 1u << 30;                // saturation of unit counts
constexpr uint32_t kBinadeUnits = 1u << 24;
constexpr uint32_t kNoEvent = 0xFFFFFFFFu;

struct SampArgs {
    const float* logits;
    int64_t rows;
    int vocab;
    int64_t ls;
    const int32_t* hist;
    const int32_t* hist_len;
    int64_t hs;
    const float* uniforms;
    float temperature, rep, freq;
    int ctx;
    int32_t* out;
    int slots_log2;
    bool vec;  // rows 16-byte aligned and vocab % 4 == 0
};

__device__ __forceinline__ float max_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) {
    const uint32_t s = a + b;  // a, b <= kSat, no wrap
    return s < kSat ? s : kSat;
}

// Shared state of one row.
struct RowSmem {
    float red_f[kVirtThreads / kWarp];
    uint32_t red_u[kMaxSampWarps];
    uint32_t wscan[2][kMaxSampWarps];  // warp totals, alternating by round
    float bcast_f;
    // CDF state
    uint32_t ucum;   // running sum in units of U
    int E;           // binade exponent; U = 2^(E-23)
    uint32_t tr;     // ceil(r / U), saturated
    int start;       // first element still to scan
    float xl;        // CDF candidates: logits above xl (a superset of the significant ones)
    int result;
    uint32_t ev_before[kMaxSampWarps];  // per warp: units before its first event
    float ev_p[kMaxSampWarps];          //           and that element's p
};

// --- penalties -------------------------------------------------------------
struct Penalty {
    const uint32_t* bitmap;
    const int32_t* keys;
    const float* vals;
    uint32_t mask;
    int shift;
};

__device__ __forceinline__ uint32_t slot_of(int32_t tok, int shift) {
    return ((uint32_t)tok * 2654435761u) >> shift;
}

__device__ __forceinline__ float penalised(const Penalty& P, int i, float x) {
    if (P.bitmap[i >> 5] & (1u << (i & 31))) {
        uint32_t h = slot_of(i, P.shift);
        while (P.keys[h] != i) h = (h + 1) & P.mask;  // present: the bit is set
        return P.vals[h];
    }
    return x;
}

// Elements base .. base+3 (base a multiple of 4) with penalties applied;
// past the vocabulary: -inf.  The group's 4 bits share one bitmap word.
__device__ __forceinline__ void load4(const SampArgs& a, const float* row, const Penalty& P,
                                      int base, float v[4]) {
    if (a.vec && base + 3 < a.vocab) {
        const float4 t = *reinterpret_cast<const float4*>(row + base);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
#pragma unroll
        for (int e = 0; e < 4; e++) v[e] = base + e < a.vocab ? row[base + e] : -INFINITY;
    }
    if (base < a.vocab && ((P.bitmap[base >> 5] >> (base & 31)) & 0xFu)) {
#pragma unroll
        for (int e = 0; e < 4; e++)
            if (base + e < a.vocab) v[e] = penalised(P, base + e, v[e]);
    }
}

// --- block reductions --------------------------------------------------------
template <int NT>
__device__ __forceinline__ float block_max(float v, RowSmem& S) {
    constexpr int kSampWarps = NT / kWarp;
    for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) S.red_f[w] = v;
    __syncthreads();
    if (w == 0) {
        v = lane < kSampWarps ? S.red_f[lane] : -INFINITY;
        for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) S.bcast_f = v;
    }
    __syncthreads();
    return S.bcast_f;
}

// The pinned order over 1024 virtual threads: thread t of an NT-thread CTA
// plays virtual threads t, t + NT, ... (acc[v] is virtual thread t + v NT).
// Butterfly inside each virtual warp (virtual warp w + v NT / 32 is real
// warp w's acc[v]), then over the 32 virtual-warp sums -- the same order for
// every NT.
template <int NT>
__device__ __forceinline__ float block_sum_pinned(const float (&acc)[kVirtThreads / NT], RowSmem& S) {
    constexpr int VPT = kVirtThreads / NT, NW = NT / kWarp;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int v = 0; v < VPT; v++) {
        const float s = butterfly_sum(acc[v], kWarp);
        if (lane == 0) S.red_f[w + v * NW] = s;
    }
    __syncthreads();
    if (w == 0) {
        const float v = butterfly_sum(S.red_f[lane], kWarp);
        if (lane == 0) S.bcast_f = v;
    }
    __syncthreads();
    return S.bcast_f;
}

// --- pass 0: window -> hash + bitmap ------------------------------------------
template <int NT>
__device__ Penalty build_penalties(const SampArgs& a, int64_t row, const float* lrow,
                                   uint32_t* bitmap, int32_t* keys, int32_t* counts, float* vals) {
    const int nwords = (a.vocab + 31) >> 5;
    const int slots = 1 << a.slots_log2;
    for (int i = threadIdx.x; i < nwords; i += NT) bitmap[i] = 0u;
    for (int i = threadIdx.x; i < slots; i += NT) { keys[i] = -1; counts[i] = 0; }
    __syncthreads();
    Penalty P{bitmap, keys, vals, (uint32_t)(slots - 1), 32 - a.slots_log2};
    if (a.hist && a.hist_len) {
        int hl = __ldg(a.hist_len + row);
        hl = hl < 0 ? 0 : (hl > a.hs ? (int)a.hs : hl);
        int start = hl - a.ctx;
        if (start < 0) start = 0;
        const int32_t* h = a.hist + row * a.hs;
        for (int j = start + threadIdx.x; j < hl; j += NT) {
            const int32_t tok = __ldg(h + j);
            if (tok < 0 || tok >= a.vocab) continue;
            uint32_t s = slot_of(tok, P.shift);
            while (true) {  // the table has at least twice the window's slots
                const int32_t prev = atomicCAS(&keys[s], -1, tok);
                if (prev == -1 || prev == tok) break;
                s = (s + 1) & P.mask;
            }
            atomicAdd(&counts[s], 1);
            atomicOr(&bitmap[tok >> 5], 1u << (tok & 31));
        }
    }
    __syncthreads();
    for (int s = threadIdx.x; s < slots; s += NT) {
        const int32_t tok = keys[s];
        if (tok < 0) continue;
        float x = lrow[tok];
        if (a.rep > 1.0f) x = x > 0.0f ? __fdiv_rn(x, a.rep) : __fmul_rn(x, a.rep);
        if (a.freq > 0.0f) x = __fsub_rn(x, __fmul_rn(a.freq, (float)counts[s]));
        vals[s] = x;
    }
    __syncthreads();
    return P;
}

// p in units of U = 2^(E-23): k = round(p / U); tie when p / U is an exact
// half; big when p >= 2^(E+1) (certain to leave the binade).  Branch-free:
// p / U = m * 2^s; for s <= 0 the shift sh = min(-s, 31) leaves q = m >> sh
// and a remainder rem; rounding to nearest adds 1 when rem > half, and
// rem == half (sh > 0) is a tie.  sh >= 25 gives q = 0 and rem < half
// because m < 2^24.
__device__ __forceinline__ void classify(float p, int E, uint32_t& k, bool& tie, bool& big) {
    const uint32_t b = __float_as_uint(p);
    const uint32_t pe = (b >> 23) & 0xFFu;
    const uint32_t m = (b & 0x7FFFFFu) | (pe ? 0x800000u : 0u);
    const int s = (int)(pe ? pe : 1u) - 127 - E;
    big = m != 0u && s >= 1;
    const uint32_t sh = (uint32_t)min(max(-s, 0), 31);
    const uint32_t q = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u);
    const uint32_t half = sh ? 1u << (sh - 1u) : 0u;
    tie = sh != 0u && rem == half && m != 0u;
    k = q + (rem > half ? 1u : 0u);
}

// The CDF scan's candidate floor for a binade: a logit xl with d(xl) < td,
// d(v) = fl(fl(v * inv_t) - max).  d does not decrease with v, so every
// logit v <= xl has d(v) < td: it is insignificant.  xl comes from td with a
// margin that covers the two roundings of d, and is checked; -inf (every
// element a candidate) if the check fails.  t_inv = 1 / inv_t in double.
__device__ __forceinline__ float candidate_floor(float td, float inv_t, float neg_m, double t_inv) {
    if (!(td > -INFINITY)) return -INFINITY;
    const double t = (double)td, n = (double)neg_m;
    const double delta = 0x1p-21 * (fabs(t - n) + fabs(n) + fabs(t)) + 0x1p-140;
    const double y = (t - n - delta) * t_inv;
    const float x = __double2float_rd(y - fabs(y) * 0x1p-40);
    if (!(x == x)) return -INFINITY;
    return __fadd_rn(__fmul_rn(x, inv_t), neg_m) < td ? x : -INFINITY;
}

// The scan state in one binade [2^E, 2^(E+1)) of the running sum.
struct Binade {
    uint32_t ucum;  // running sum in units of U = 2^(E-23)
    int E;
    uint32_t tr;    // ceil(r / U), saturated
    float td;       // significance threshold on d
    float xl;       // candidate floor on the logits
};

// The binade state of an exact fp32 running sum `cum`.
__device__ __forceinline__ Binade binade_of(float cum, float r, double ln_2inv, float inv_t, float neg_m,
                                            double t_inv) {
    Binade B;
    const uint32_t b = __float_as_uint(cum);
    int e = (int)((b >> 23) & 0xFFu) - 127;
    if (e < -126) e = -126;
    B.E = e;
    // cum / U: exact integer below 2^24
    const int pe = (int)((b >> 23) & 0xFFu);
    const uint32_t m = pe ? ((b & 0x7FFFFFu) | 0x800000u) : (b & 0x7FFFFFu);
    const int s = (pe ? pe : 1) - 127 - e;  // 0 for normals and for e = -126 subnormals
    B.ucum = m << s;
    // ceil(r / U)
    const uint32_t rb = __float_as_uint(r);
    const int re = (int)((rb >> 23) & 0xFFu);
    const uint32_t rm = re ? ((rb & 0x7FFFFFu) | 0x800000u) : (rb & 0x7FFFFFu);
    const int rs = (re ? re : 1) - 127 - e;
    uint32_t tr;
    if (rm == 0) tr = 0;
    else if (rs >= 7) tr = kSat;
    else if (rs >= 0) tr = rm << rs;
    else if (-rs >= 25) tr = 1;
    else tr = (rm + (1u << -rs) - 1u) >> -rs;
    B.tr = tr < kSat ? tr : kSat;
    // d < td  =>  exp(d) * inv < U / 2 with room for the exp's and the
    // product's rounding (relative 2^-21) and for rounding td itself.  Below
    // U / 2 = 2^-126 a product near U / 2 would be subnormal and its rounding
    // no longer relative: no element is skipped there.
    // ln(U / (2 inv)) = (E - 23) ln 2 - ln(2 inv), ln(2 inv) computed once per row
    B.td = e - 24 >= -126 ? (float)((double)(e - 23) * 0.69314718055994530942 - ln_2inv - 1e-4)
                          : -INFINITY;
    B.xl = candidate_floor(B.td, inv_t, neg_m, t_inv);
    return B;
}

__device__ __forceinline__ void set_binade(RowSmem& S, float cum, float r, double ln_2inv, float inv_t,
                                           float neg_m, double t_inv) {
    const Binade B = binade_of(cum, r, ln_2inv, inv_t, neg_m, t_inv);
    S.E = B.E;
    S.ucum = B.ucum;
    S.tr = B.tr;
    S.xl = B.xl;
}

// Dynamic shared memory of sample_rows_kernel: the window hash (keys,
// counts, values: 12 B per slot), the vocabulary bitmap, then (16-byte
// aligned) the per-warp candidate lists: NT / 32 x 256 logits-then-p (4 B)
// and tile-local indices (2 B).
__host__ __device__ constexpr size_t cand_offset(int slots, int vocab) {
    return (((size_t)slots * 12 + (size_t)((vocab + 31) / 32) * 4) + 15) & ~(size_t)15;
}
__host__ __device__ constexpr size_t samp_smem(int nt, int slots, int vocab) {
    return cand_offset(slots, vocab) + (size_t)(nt / kWarp) * kWarp * kPerThread * 6;
}

// NT = 512: two CTAs per SM (a batch of up to 2 x SMs rows in one wave);
// NT = 1024: one CTA per SM, for batches of at most one row per SM.  Every
// order the result depends on is the same for both.
template <int NT>
__global__ void __launch_bounds__(NT, NT == kSampThreads ? 2 : 1)
sample_rows_kernel(const SampArgs a) {
    constexpr int kSampThreads = NT;
    constexpr int kSampWarps = NT / kWarp;
    constexpr int kTile = NT * kPerThread;
    constexpr int VPT = kVirtThreads / NT;  // virtual threads of the pinned sum per thread
    pdl_begin();
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ RowSmem S;
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int slots = 1 << a.slots_log2;
    int32_t* keys = reinterpret_cast<int32_t*>(dyn);
    int32_t* counts = keys + slots;
    float* vals = reinterpret_cast<float*>(counts + slots);
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(vals + slots);
    // candidates (logit, then p) and their tile-local indices, after the bitmap
    const size_t cand_off = cand_offset(slots, a.vocab);
    float (*const cbuf)[kWarp * kPerThread] = reinterpret_cast<float (*)[kWarp * kPerThread]>(dyn + cand_off);
    uint16_t (*const cidx)[kWarp * kPerThread] = reinterpret_cast<uint16_t (*)[kWarp * kPerThread]>(
        dyn + cand_off + sizeof(float) * kSampWarps * kWarp * kPerThread);
    const float* lrow = a.logits + row * a.ls;
    const Penalty P = build_penalties<NT>(a, row, lrow, bitmap, keys, counts, vals);
    const int ngroups = (a.vocab + 3) >> 2;

    // ---- greedy: first maximum (core/sampling.cpp:45-52) ----
    // The reference keeps max_i = 0 and moves on `adjusted[i] >
    // adjusted[max_i]`: a NaN never wins a comparison, so element 0 being
    // NaN gives 0, and otherwise the result is the first index of the
    // largest non-NaN value (element 0 included).
    if (a.temperature <= 0.0f) {
        float v0[4];
        load4(a, lrow, P, 0, v0);
        if (v0[0] != v0[0]) {
            if (tid == 0) a.out[row] = 0;
            return;
        }
        float best = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int g = tid; g < ngroups; g += kSampThreads) {
            float v[4];
            load4(a, lrow, P, g * 4, v);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = g * 4 + e;
                if (i < a.vocab && v[e] == v[e] && (v[e] > best || (v[e] == best && i < bi))) {
                    best = v[e];
                    bi = i;
                }
            }
        }
        // larger value wins, equal values -> smaller index
        for (int off = 16; off >= 1; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (lane == 0) { S.red_f[w] = best; S.red_u[w] = (uint32_t)bi; }
        __syncthreads();
        if (w == 0) {
            best = lane < kSampWarps ? S.red_f[lane] : -INFINITY;
            bi = lane < kSampWarps ? (int)S.red_u[lane] : 0x7FFFFFFF;
            for (int off = 16; off >= 1; off >>= 1) {
                const float ob = __shfl_xor_sync(0xffffffffu, best, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
            }
            if (lane == 0) a.out[row] = bi == 0x7FFFFFFF ? 0 : bi;
        }
        return;
    }

    // ---- pass 1: max, four groups in flight per thread ----
    // fmaxf skips NaN like the reference's `>` scan (vDSP_maxv); NaNs are
    // counted on the side.
    // (back to front: the exp-sum pass then starts on the lines read last,
    // which are still in L2)
    // max.NaN: a NaN logit makes mx NaN (the NaN rule below); otherwise mx
    // is the largest penalised logit.  kMaxSweep groups in flight per thread.
    float mx = -INFINITY;
    const int nsweep = (ngroups + kMaxSweep * kSampThreads - 1) / (kMaxSweep * kSampThreads);
    for (int sw = nsweep - 1; sw >= 0; sw--) {
        const int g0 = sw * kMaxSweep * kSampThreads;
        float v[kMaxSweep][4];
#pragma unroll
        for (int u = 0; u < kMaxSweep; u++) {
            const int g = g0 + u * kSampThreads + tid;
            if (g < ngroups) load4(a, lrow, P, g * 4, v[u]);
            else v[u][0] = v[u][1] = v[u][2] = v[u][3] = -INFINITY;
        }
#pragma unroll
        for (int u = 0; u < kMaxSweep; u++)
#pragma unroll
            for (int e = 0; e < 4; e++) mx = max_nan(mx, v[u][e]);
    }
    bool nan_seen = mx != mx;
    nan_seen = __syncthreads_or(nan_seen);
    mx = block_max<NT>(mx, S);
    const float inv_t = __fdiv_rn(1.0f, a.temperature);
    const float neg_m = -__fmul_rn(mx, inv_t);
    const float r = __ldg(a.uniforms + row);
    // The reference's softmax sum is NaN exactly when a penalised logit is
    // NaN (exp(NaN) = NaN) or max * (1/T) is infinite (+inf - inf, or every
    // element -inf + inf); then every p is NaN, `cum >= r` never holds and
    // it returns vocab - 1 (core/sampling.cpp:58-65).  A NaN uniform never
    // compares true either.
    if (nan_seen || !(fabsf(neg_m) <= 3.402823466e38f) || r != r) {
        if (tid == 0) a.out[row] = a.vocab - 1;
        return;
    }

    // ---- pass 2: pinned sum of exp over the 1024 virtual threads ----
    // Two steps of 1024 groups per iteration, all four loads issued first
    // (64 bytes in flight per thread), then the exps and the adds in order.
    float acc[VPT];
#pragma unroll
    for (int v = 0; v < VPT; v++) acc[v] = 0.0f;
    auto add4 = [&](const float (&v)[4], int g, float& ac) {
        float d[4];
#pragma unroll
        for (int j = 0; j < 4; j++) d[j] = __fadd_rn(__fmul_rn(v[j], inv_t), neg_m);
        const float2 e01 = pinned_expf_nonpos2(make_float2(d[0], d[1]));
        const float2 e23 = pinned_expf_nonpos2(make_float2(d[2], d[3]));
        const float e[4] = {e01.x, e01.y, e23.x, e23.y};
        if (g * 4 + 3 < a.vocab) {
#pragma unroll
            for (int j = 0; j < 4; j++) ac = __fadd_rn(ac, e[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (g * 4 + j < a.vocab) ac = __fadd_rn(ac, e[j]);
        }
    };
    // Two steps of 1024 groups per iteration, every load issued first;
    // virtual thread tid + v NT takes group g0 + tid + v NT, then the same
    // group of the second step (its groups in increasing order).
    for (int g0 = 0; g0 < ngroups; g0 += 2 * kVirtThreads) {
        float vv[2][VPT][4];
#pragma unroll
        for (int st = 0; st < 2; st++)
#pragma unroll
            for (int v = 0; v < VPT; v++) {
                const int g = g0 + st * kVirtThreads + v * NT + tid;
                if (g < ngroups) load4(a, lrow, P, g * 4, vv[st][v]);
            }
#pragma unroll
        for (int st = 0; st < 2; st++)
#pragma unroll
            for (int v = 0; v < VPT; v++) {
                const int g = g0 + st * kVirtThreads + v * NT + tid;
                if (g < ngroups) add4(vv[st][v], g, acc[v]);
            }
    }
    const float inv = __fdiv_rn(1.0f, block_sum_pinned<NT>(acc, S));

    // ---- pass 3: exact parallel inverse-CDF scan over significant elements ----
    if (!(r > 0.0f)) {  // cum >= r holds after the first element
        if (tid == 0) a.out[row] = 0;
        return;
    }
    const double ln_2inv = log(2.0 * (double)inv);
    const double t_inv = 1.0 / (double)inv_t;
    if (tid == 0) {
        set_binade(S, 0.0f, r, ln_2inv, inv_t, neg_m, t_inv);
        S.start = 0;
        S.result = -1;
    }
    // ---- pass 3a: the first tile, serially -----------------------------------
    // While cum is small it leaves its binade every few elements, and each
    // crossing would cost a block-wide round.  So the CTA computes every p of
    // the first tile into shared memory and one thread adds them in fp32 --
    // the reference's own loop, eight elements per branch -- until a stretch
    // of 256 elements passes without a change of binade; from there the
    // block rounds below take over with the unit arithmetic.
    {
        const int t0end = min(kTile, a.vocab);
        float* const pt = &cbuf[0][0];  // kTile floats
#pragma unroll
        for (int h = 0; h < kPerThread / 4; h++) {
            float v[4];
            load4(a, lrow, P, tid * kPerThread + 4 * h, v);  // -inf past the vocabulary
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
                const float2 ex = pinned_expf_nonpos2(make_float2(__fadd_rn(__fmul_rn(v[e], inv_t), neg_m),
                                                                  __fadd_rn(__fmul_rn(v[e + 1], inv_t), neg_m)));
                pt[tid * kPerThread + 4 * h + e] = __fmul_rn(ex.x, inv);
                pt[tid * kPerThread + 4 * h + e + 1] = __fmul_rn(ex.y, inv);
            }
        }
        __syncthreads();
        if (tid == 0) {
            float cum = 0.0f;
            int j = 0, hit = -1;
            while (j < t0end) {
                const int jend = min(t0end, j + kWarp * kPerThread);
                const uint32_t e0 = __float_as_uint(cum) >> 23;
                // j is a multiple of 8 here; the next chunk's loads are
                // issued before this chunk's adds
                float4 n0 = *reinterpret_cast<const float4*>(pt + j);
                float4 n1 = *reinterpret_cast<const float4*>(pt + j + 4);
                for (; j + 8 <= jend; j += 8) {
                    const float pv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
                    const int jn = min(j + 8, kTile - 8);
                    n0 = *reinterpret_cast<const float4*>(pt + jn);
                    n1 = *reinterpret_cast<const float4*>(pt + jn + 4);
                    float cs[8];
                    cs[0] = __fadd_rn(cum, pv[0]);
#pragma unroll
                    for (int q = 1; q < 8; q++) cs[q] = __fadd_rn(cs[q - 1], pv[q]);
                    if (cs[7] >= r) {  // p >= 0: the running sums do not decrease
                        uint32_t m = 0;
#pragma unroll
                        for (int q = 0; q < 8; q++) m |= (cs[q] >= r ? 1u : 0u) << q;
                        hit = j + __ffs(m) - 1;
                        break;
                    }
                    cum = cs[7];
                }
                for (; hit < 0 && j < jend; j++) {
                    cum = __fadd_rn(cum, pt[j]);
                    if (cum >= r) hit = j;
                }
                if (hit >= 0) break;
                if ((__float_as_uint(cum) >> 23) == e0 && cum > 0.0f) break;  // a quiet stretch
            }
            if (hit >= 0) S.result = hit;
            else set_binade(S, cum, r, ln_2inv, inv_t, neg_m, t_inv);  // exact: the unit arithmetic resumes from cum
            S.start = j;
        }
        __syncthreads();
    }
    // ---- pass 3b: the other tiles, over candidate lists ------------------------
    // Per tile: each thread tests its 8 logits against the binade's floor
    // xl (every significant element is a candidate; most elements are not),
    // each warp compacts its candidates in element order into shared
    // memory, computes their p once and adds their units for the current
    // binade (a serial element -- tie or big -- saturates the sum).  One
    // block prefix of the 16 warp totals gives the tile's total: below tr
    // and inside the binade, nothing happens in the tile and the state
    // advances in every thread alike.  Otherwise the first event (serial
    // element, binade crossing or hit) lies in the first warp whose units
    // reach the limit; that warp walks its candidates in order to find it,
    // every thread applies it to its own copy of the state (the real fp32
    // add, as in the first tile), the warps from the event's on recount
    // their remaining candidates from the stored p in the new binade, and
    // so on until the tile is done.
    float* const cv = cbuf[w];
    uint16_t* const ci = cidx[w];
    const int ntiles = (a.vocab + kTile - 1) / kTile;
    uint32_t st_ucum = S.ucum, st_tr = S.tr;
    int st_E = S.E, st_start = S.start;
    float st_xl = S.xl;
    int res = S.result;
    int rp = 0;  // round parity: which wscan buffer
    auto units = [](float p, int E) {
        uint32_t k;
        bool tie, big;
        classify(p, E, k, tie, big);
        return (tie || big) ? kSat : k;
    };
    // sum of the warp's units (every lane gets it, in `mine`), then the block
    // prefix: wpre = units of the warps before this one; returns all 16
    // warps' total
    auto block_units = [&](uint32_t& mine, uint32_t& wpre) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) mine = sat_add(mine, __shfl_xor_sync(0xffffffffu, mine, off));
        if (lane == 0) S.wscan[rp][w] = mine;
        __syncthreads();
        uint32_t t = lane < kSampWarps ? S.wscan[rp][lane] : 0u;
        rp ^= 1;
#pragma unroll
        for (int off = 1; off < kSampWarps; off <<= 1) {
            const uint32_t o = __shfl_up_sync(0xffffffffu, t, off);
            if (lane >= off) t = sat_add(t, o);
        }
        wpre = __shfl_sync(0xffffffffu, t, (w + 31) & 31);
        if (w == 0) wpre = 0;
        return __shfl_sync(0xffffffffu, t, kSampWarps - 1);
    };
    for (int tile = st_start / kTile; tile < ntiles && res < 0; tile++) {
        const int tbase = tile * kTile;
        const int base = tbase + tid * kPerThread;
        const int tile_end = min(tbase + kTile, a.vocab);
        uint32_t msk = 0;
        {
            float v[kPerThread];
#pragma unroll
            for (int h = 0; h < kPerThread / 4; h++) load4(a, lrow, P, base + 4 * h, &v[4 * h]);
#pragma unroll
            for (int e = 0; e < kPerThread; e++) msk |= (v[e] > st_xl ? 1u : 0u) << e;
            const int lo = min(max(st_start - base, 0), kPerThread);
            const int hi = min(max(a.vocab - base, 0), kPerThread);
            msk &= ((1u << hi) - 1u) & ~((1u << lo) - 1u);
            const int cnt = __popc(msk);
            int incl = cnt;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += o;
            }
            int pos = incl - cnt;
#pragma unroll
            for (int e = 0; e < kPerThread; e++)
                if ((msk >> e) & 1u) {
                    cv[pos] = v[e];
                    ci[pos] = (uint16_t)(tid * kPerThread + e);
                    pos++;
                }
            msk = (uint32_t)__shfl_sync(0xffffffffu, incl, 31);  // the warp's candidate count
        }
        const int nw = (int)msk;
        __syncwarp();
        // p of each candidate (kept in cv), this lane's units: items lane, lane + 32, ...
        uint32_t mine = 0;
        for (int j0 = 0; j0 < nw; j0 += 2 * kWarp) {
            const int ja = j0 + lane, jb = ja + kWarp;
            const float da = ja < nw ? __fadd_rn(__fmul_rn(cv[ja], inv_t), neg_m) : -INFINITY;
            const float db = jb < nw ? __fadd_rn(__fmul_rn(cv[jb], inv_t), neg_m) : -INFINITY;
            const float2 ex = pinned_expf_nonpos2(make_float2(da, db));
            if (ja < nw) {
                const float p = __fmul_rn(ex.x, inv);
                cv[ja] = p;
                mine = sat_add(mine, units(p, st_E));
            }
            if (jb < nw) {
                const float p = __fmul_rn(ex.y, inv);
                cv[jb] = p;
                mine = sat_add(mine, units(p, st_E));
            }
        }
        __syncwarp();
        uint32_t wpre;
        uint32_t all = block_units(mine, wpre);
        while (true) {
            const uint32_t tot = sat_add(st_ucum, all);
            if (tot < st_tr && tot < kBinadeUnits) {  // no event in the rest of the tile
                st_ucum = tot;  // exact and < 2^24
                st_start = tile_end;
                break;
            }
            // The first event lies in the first warp whose units reach tr or
            // leave the binade (a serial element saturates them): only that
            // warp walks its candidates in order to find it.
            uint32_t run = sat_add(st_ucum, wpre);
            const uint32_t lim = st_tr < kBinadeUnits ? st_tr : kBinadeUnits;
            const bool ev_warp = run < lim && sat_add(run, mine) >= lim;
            uint32_t ev = kNoEvent, before = 0;
            float pe = 0.0f;
            for (int j0 = 0; ev_warp && j0 < nw; j0 += kWarp) {
                const int j = j0 + lane;
                const bool valid = j < nw && tbase + (int)ci[j] >= st_start;
                const float p = valid ? cv[j] : 0.0f;
                uint32_t k;
                bool tie, big;
                classify(p, st_E, k, tie, big);
                const bool ser = valid && (tie || big);
                const uint32_t kk = valid ? (ser ? kSat : k) : 0u;
                uint32_t inc = kk;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t o = __shfl_up_sync(0xffffffffu, inc, off);
                    if (lane >= off) inc = sat_add(inc, o);
                }
                uint32_t ex = __shfl_up_sync(0xffffffffu, inc, 1);
                if (lane == 0) ex = 0;
                const uint32_t r0 = sat_add(run, ex);  // units before this candidate
                uint32_t e = kNoEvent;
                if (valid) {
                    const uint32_t local = (uint32_t)ci[j] << 1;
                    if (ser) {
                        e = local;
                    } else {
                        const uint32_t nr = sat_add(r0, k);
                        if (nr >= kBinadeUnits) e = local;
                        else if (nr >= st_tr) e = local | 1u;
                    }
                }
                const uint32_t bal = __ballot_sync(0xffffffffu, e != kNoEvent);
                if (bal) {  // candidates ascend with the lanes: the lowest lane is first
                    const int src = __ffs(bal) - 1;
                    ev = __shfl_sync(0xffffffffu, e, src);
                    before = __shfl_sync(0xffffffffu, r0, src);
                    pe = __shfl_sync(0xffffffffu, p, src);
                    break;
                }
                run = sat_add(run, __shfl_sync(0xffffffffu, inc, 31));
            }
            if (lane == 0) {
                S.red_u[w] = ev;
                S.ev_before[w] = before;
                S.ev_p[w] = pe;
            }
            __syncthreads();
            // the first event over the warps, applied by every thread to its
            // own copy of the state (the next writes of these slots come
            // after the barrier of the recount below)
            const uint32_t wev = lane < kSampWarps ? S.red_u[lane] : kNoEvent;
            const uint32_t gev = __reduce_min_sync(0xffffffffu, wev);
            if (gev == kNoEvent) {  // cannot happen (the total above had one); kept safe
                st_ucum = tot < kBinadeUnits ? tot : st_ucum;
                st_start = tile_end;
                break;
            }
            const int i = tbase + (int)(gev >> 1);
            if (gev & 1u) {
                res = i;
                break;
            }
            const int ow = __ffs(__ballot_sync(0xffffffffu, wev == gev)) - 1;
            // before * 2^(E-23), exact: two power-of-two scalings; then a real fp32 add
            const float cum_prev =
                __fmul_rn(__fmul_rn((float)S.ev_before[ow], pow2i(st_E - 23 + 64)), pow2i(-64));
            const float cum = __fadd_rn(cum_prev, S.ev_p[ow]);
            if (cum >= r) {
                res = i;
                break;
            }
            {
                const Binade B = binade_of(cum, r, ln_2inv, inv_t, neg_m, t_inv);
                st_ucum = B.ucum;
                st_tr = B.tr;
                st_E = B.E;
                st_xl = B.xl;
                st_start = i + 1;
            }
            // the tile's remaining candidates recounted in the new binade
            // (the warps before the event's have none left)
            mine = 0;
            if (w >= ow)
                for (int j = lane; j < nw; j += kWarp)
                    if (tbase + (int)ci[j] >= st_start) mine = sat_add(mine, units(cv[j], st_E));
            all = block_units(mine, wpre);
        }
        if (res >= 0) break;
    }
    if (tid == 0) a.out[row] = res >= 0 ? res : a.vocab - 1;
}

// softmax over rows in place (core/cpu_ops.cpp:83-99) with the pinned sum.
__global__ void __launch_bounds__(kSampThreads, 2)
softmax_rows_kernel(float* x, int n, int64_t stride) {
    pdl_begin();
    __shared__ RowSmem S;
    float* row = x + (int64_t)blockIdx.x * stride;
    const int tid = threadIdx.x;
    const int ngroups = (n + 3) >> 2;
    float mx = -INFINITY;
    for (int g = tid; g < ngroups; g += kSampThreads)
        for (int e = 0; e < 4 && g * 4 + e < n; e++) mx = fmaxf(mx, row[g * 4 + e]);
    const float neg_m = -block_max<kSampThreads>(mx, S);
    // x - max is <= 0 or NaN (a NaN element, +inf - inf, or -inf + inf when
    // every element is -inf): NaN stays NaN through the exp, as in the
    // reference's vvexpf, and then makes the sum and every output NaN
    auto ex = [](float d) { return d != d ? d : pinned_expf_nonpos(d); };
    float acc_lo = 0.0f, acc_hi = 0.0f;
    for (int g0 = 0; g0 < ngroups; g0 += kVirtThreads) {
        const int ga = g0 + tid, gb = g0 + tid + kSampThreads;
        if (ga < ngroups)
            for (int e = 0; e < 4 && ga * 4 + e < n; e++) {
                const float v = ex(__fadd_rn(row[ga * 4 + e], neg_m));
                row[ga * 4 + e] = v;
                acc_lo = __fadd_rn(acc_lo, v);
            }
        if (gb < ngroups)
            for (int e = 0; e < 4 && gb * 4 + e < n; e++) {
                const float v = ex(__fadd_rn(row[gb * 4 + e], neg_m));
                row[gb * 4 + e] = v;
                acc_hi = __fadd_rn(acc_hi, v);
            }
    }
    const float accs[2] = {acc_lo, acc_hi};
    const float inv = __fdiv_rn(1.0f, block_sum_pinned<kSampThreads>(accs, S));
    for (int i = tid; i < n; i += kSampThreads) row[i] = __fmul_rn(row[i], inv);
}

}  // namespace ane

extern "C" {

int ane_cuda_sample_rows(const float* logits, int64_t rows, int vocab, int64_t logits_stride,
                         const int32_t* history, const int32_t* history_len,
                         int64_t history_stride, const float* uniforms, float temperature,
                         float repetition_penalty, int repetition_context,
                         float frequency_penalty, int32_t* out_tokens, void* stream) {
    using namespace ane;
    if (rows < 0 || vocab <= 0 || logits_stride < vocab)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "sample_rows: rows=%lld vocab=%d stride=%lld",
                    (long long)rows, vocab, (long long)logits_stride);
    if (rows == 0) return ANE_CUDA_OK;
    if (!logits || !uniforms || !out_tokens)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "sample_rows: null pointer");
    if ((history == nullptr) != (history_len == nullptr))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "sample_rows: give history and history_len together");
    if (history && history_stride < 0)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "sample_rows: history_stride < 0");
    if (rows > 0x7fffffffLL) return fail(ANE_CUDA_ERR_UNSUPPORTED, "sample_rows: too many rows");
    int64_t window = history ? history_stride : 0;
    if (window > repetition_context) window = repetition_context > 0 ? repetition_context : 0;
    if (window > kMaxWindow)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "sample_rows: repetition window %lld > %d",
                    (long long)window, kMaxWindow);
    int slots_log2 = 5;
    while ((1 << slots_log2) < 2 * window) slots_log2++;
    // at most one row per SM: one 1024-thread CTA each; else 512-thread CTAs,
    // two per SM (the results do not depend on the choice)
    constexpr size_t kMaxDyn = 225 * 1024;  // plus about 1 KB of static shared memory
    const bool wide = rows <= (int64_t)sm_count() &&
                      samp_smem(kSampThreadsWide, 1 << slots_log2, vocab) <= kMaxDyn;
    const size_t smem = samp_smem(wide ? kSampThreadsWide : kSampThreads, 1 << slots_log2, vocab);
    if (smem > kMaxDyn) return fail(ANE_CUDA_ERR_UNSUPPORTED, "sample_rows: vocab %d too large", vocab);
    // the attribute is set once per device and kernel (setting it twice is
    // harmless, so concurrent first calls need no lock)
    static std::atomic<int> configured[64][2];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return fail(ANE_CUDA_ERR_CUDA, "sample_rows: no current device");
    if (!configured[dev][wide].load(std::memory_order_acquire)) {
        cudaError_t e = wide ? cudaFuncSetAttribute(sample_rows_kernel<kSampThreadsWide>,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxDyn)
                             : cudaFuncSetAttribute(sample_rows_kernel<kSampThreads>,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxDyn);
        if (e != cudaSuccess)
            return fail(ANE_CUDA_ERR_CUDA, "sample_rows: %s", cudaGetErrorString(e));
        configured[dev][wide].store(1, std::memory_order_release);
    }
    SampArgs a{logits, rows, vocab, logits_stride, history, history_len, history_stride, uniforms,
               temperature, repetition_penalty, frequency_penalty, repetition_context, out_tokens,
               slots_log2, vocab % 4 == 0 && logits_stride % 4 == 0 && is_aligned(logits, 16)};
    if (wide) launch_pdl(sample_rows_kernel<kSampThreadsWide>, (unsigned)rows, kSampThreadsWide, smem, as_stream(stream), a);
    else launch_pdl(sample_rows_kernel<kSampThreads>, (unsigned)rows, kSampThreads, smem, as_stream(stream), a);
    return check_launch("sample_rows");
}

int ane_cuda_softmax_rows(float* x, int64_t rows, int n, int64_t stride, void* stream) {
    using namespace ane;
    if (rows < 0 || n <= 0 || stride < n)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "softmax_rows: rows=%lld n=%d stride=%lld",
                    (long long)rows, n, (long long)stride);
    if (rows == 0) return ANE_CUDA_OK;
    if (!x) return fail(ANE_CUDA_ERR_INVALID_ARG, "softmax_rows: null pointer");
    if (rows > 0x7fffffffLL) return fail(ANE_CUDA_ERR_UNSUPPORTED, "softmax_rows: too many rows");
    launch_pdl(softmax_rows_kernel, (unsigned)rows, kSampThreads, 0, as_stream(stream), x, n, stride);
    return check_launch("softmax_rows");
}

}  // extern "C"
