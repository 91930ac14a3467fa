// sampler.cu -- batched sample_token (core/sampling.cpp:10-66) and softmax
// (core/cpu_ops.cpp:83-99), one 1024-thread CTA per row.
//
// Pass 0  the row's repetition window goes into a shared-memory hash
//         (id -> count) and a vocabulary bitmap; each distinct id's logit is
//         penalised once (rep, then freq), as sampling.cpp:17-42 does.
// Pass 1  max of the penalised logits (argmax for temperature <= 0).
//         max(fl(a * inv_t)) = fl(max(a) * inv_t) since rounding is monotone.
// Pass 2  e = exp(fl(fl(a * inv_t) - max)) summed in the pinned order: group
//         g of 4 consecutive elements belongs to thread g % 1024, which adds
//         its elements in increasing order; an xor butterfly inside each warp,
//         then over the 32 warp sums.
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
#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / kWarp;
constexpr int kMaxWindow = 4096;
constexpr uint32_t kSat = 1u << 30;       // saturation of unit counts
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

__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) {
    const uint32_t s = a + b;  // a, b <= kSat, no wrap
    return s < kSat ? s : kSat;
}

// Shared state of one row.
struct RowSmem {
    float red_f[kSampWarps];
    uint32_t red_u[kSampWarps];
    uint32_t wscan[kSampWarps];
    float bcast_f;
    int bcast_i;
    // CDF state
    uint32_t ucum;   // running sum in units of U
    int E;           // binade exponent; U = 2^(E-23)
    uint32_t tr;     // ceil(r / U), saturated
    int start;       // first element still to scan
    uint32_t ev;     // event code of this round
    int result;
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
        while (P.keys[h] != i) h = (h + 1) & P.mask;
        return P.vals[h];
    }
    return x;
}

// Loads element group g (4 consecutive elements) with penalties applied;
// elements past the vocabulary read as -inf and are never counted.
__device__ __forceinline__ void load_group(const SampArgs& a, const float* row, const Penalty& P,
                                           int g, float v[4]) {
    const int base = g * 4;
    if (a.vec) {
        const float4 t = *reinterpret_cast<const float4*>(row + base);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
#pragma unroll
        for (int e = 0; e < 4; e++) v[e] = base + e < a.vocab ? row[base + e] : -INFINITY;
    }
#pragma unroll
    for (int e = 0; e < 4; e++)
        if (base + e < a.vocab) v[e] = penalised(P, base + e, v[e]);
}

// --- block reductions --------------------------------------------------------
__device__ __forceinline__ float block_max(float v, RowSmem& S) {
    for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) S.red_f[w] = v;
    __syncthreads();
    if (w == 0) {
        v = S.red_f[lane];
        for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) S.bcast_f = v;
    }
    __syncthreads();
    return S.bcast_f;
}

// The pinned order: xor butterfly in each warp, then over the warp sums.
__device__ __forceinline__ float block_sum_pinned(float v, RowSmem& S) {
    v = butterfly_sum(v, kWarp);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) S.red_f[w] = v;
    __syncthreads();
    if (w == 0) {
        v = butterfly_sum(S.red_f[lane], kWarp);
        if (lane == 0) S.bcast_f = v;
    }
    __syncthreads();
    return S.bcast_f;
}

// --- pass 0: window -> hash + bitmap ------------------------------------------
__device__ Penalty build_penalties(const SampArgs& a, int64_t row, const float* lrow,
                                   uint32_t* bitmap, int32_t* keys, int32_t* counts, float* vals) {
    const int nwords = (a.vocab + 31) >> 5;
    const int slots = 1 << a.slots_log2;
    for (int i = threadIdx.x; i < nwords; i += kSampThreads) bitmap[i] = 0u;
    for (int i = threadIdx.x; i < slots; i += kSampThreads) { keys[i] = -1; counts[i] = 0; }
    __syncthreads();
    Penalty P{bitmap, keys, vals, (uint32_t)(slots - 1), 32 - a.slots_log2};
    if (a.hist && a.hist_len) {
        int hl = __ldg(a.hist_len + row);
        hl = hl < 0 ? 0 : (hl > a.hs ? (int)a.hs : hl);
        int start = hl - a.ctx;
        if (start < 0) start = 0;
        const int32_t* h = a.hist + row * a.hs;
        for (int j = start + threadIdx.x; j < hl; j += kSampThreads) {
            const int32_t tok = __ldg(h + j);
            if (tok < 0 || tok >= a.vocab) continue;
            uint32_t s = slot_of(tok, P.shift);
            while (true) {
                const int32_t prev = atomicCAS(&keys[s], -1, tok);
                if (prev == -1 || prev == tok) break;
                s = (s + 1) & P.mask;
            }
            atomicAdd(&counts[s], 1);
            atomicOr(&bitmap[tok >> 5], 1u << (tok & 31));
        }
    }
    __syncthreads();
    for (int s = threadIdx.x; s < slots; s += kSampThreads) {
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
// half; big when p >= 2^(E+1) (certain to leave the binade).
__device__ __forceinline__ void classify(float p, int E, uint32_t& k, bool& tie, bool& big) {
    const uint32_t b = __float_as_uint(p);
    const int pe = (int)((b >> 23) & 0xFFu);
    const uint32_t m = pe ? ((b & 0x7FFFFFu) | 0x800000u) : (b & 0x7FFFFFu);
    const int s = (pe ? pe : 1) - 127 - E;
    k = 0; tie = false; big = false;
    if (m == 0) return;
    if (s >= 1) { big = true; return; }
    if (s == 0) { k = m; return; }
    const int sh = -s;
    if (sh >= 25) return;
    const uint32_t q = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
    tie = rem == half;
    k = q + (rem > half ? 1u : 0u);
}

// Sets the binade state of S from an exact fp32 running sum `cum`.
__device__ __forceinline__ void set_binade(RowSmem& S, float cum, float r) {
    const uint32_t b = __float_as_uint(cum);
    int e = (int)((b >> 23) & 0xFFu) - 127;
    if (e < -126) e = -126;
    S.E = e;
    // cum / U: exact integer below 2^24
    const int pe = (int)((b >> 23) & 0xFFu);
    const uint32_t m = pe ? ((b & 0x7FFFFFu) | 0x800000u) : (b & 0x7FFFFFu);
    const int s = (pe ? pe : 1) - 127 - e;  // 0 for normals; 0 for e = -126 subnormals
    S.ucum = m << s;
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
    S.tr = tr < kSat ? tr : kSat;
}

__global__ void __launch_bounds__(kSampThreads, 1)
sample_rows_kernel(const SampArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ RowSmem S;
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int slots = 1 << a.slots_log2;
    int32_t* keys = reinterpret_cast<int32_t*>(dyn);
    int32_t* counts = keys + slots;
    float* vals = reinterpret_cast<float*>(counts + slots);
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(vals + slots);
    const float* lrow = a.logits + row * a.ls;
    const Penalty P = build_penalties(a, row, lrow, bitmap, keys, counts, vals);
    const int ngroups = (a.vocab + 3) >> 2;

    // ---- pass 1: max / argmax ----
    if (a.temperature <= 0.0f) {
        float best = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int g = tid; g < ngroups; g += kSampThreads) {
            float v[4];
            load_group(a, lrow, P, g, v);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = g * 4 + e;
                if (i < a.vocab && (v[e] > best || bi == 0x7FFFFFFF)) { best = v[e]; bi = i; }
            }
        }
        // first maximum: larger value wins, equal values -> smaller index
        for (int off = 16; off >= 1; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (lane == 0) { S.red_f[w] = best; S.red_u[w] = (uint32_t)bi; }
        __syncthreads();
        if (w == 0) {
            best = S.red_f[lane];
            bi = (int)S.red_u[lane];
            for (int off = 16; off >= 1; off >>= 1) {
                const float ob = __shfl_xor_sync(0xffffffffu, best, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
            }
            if (lane == 0) a.out[row] = bi == 0x7FFFFFFF ? 0 : bi;
        }
        return;
    }
    float mx = -INFINITY;
    for (int g = tid; g < ngroups; g += kSampThreads) {
        float v[4];
        load_group(a, lrow, P, g, v);
#pragma unroll
        for (int e = 0; e < 4; e++) mx = fmaxf(mx, v[e]);
    }
    mx = block_max(mx, S);
    const float inv_t = __fdiv_rn(1.0f, a.temperature);
    const float neg_m = -__fmul_rn(mx, inv_t);

    // ---- pass 2: pinned sum of exp ----
    float acc = 0.0f;
    for (int g = tid; g < ngroups; g += kSampThreads) {
        float v[4];
        load_group(a, lrow, P, g, v);
#pragma unroll
        for (int e = 0; e < 4; e++)
            if (g * 4 + e < a.vocab)
                acc = __fadd_rn(acc, pinned_expf(__fadd_rn(__fmul_rn(v[e], inv_t), neg_m)));
    }
    const float inv = __fdiv_rn(1.0f, block_sum_pinned(acc, S));

    // ---- pass 3: exact parallel inverse-CDF scan ----
    const float r = __ldg(a.uniforms + row);
    if (tid == 0) {
        set_binade(S, 0.0f, r);
        S.start = 0;
        S.result = -1;
    }
    __syncthreads();
    const int ntiles = (ngroups + kSampThreads - 1) / kSampThreads;
    for (int tile = 0; tile < ntiles; tile++) {
        const int g = tile * kSampThreads + tid;
        float p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (g < ngroups) {
            float v[4];
            load_group(a, lrow, P, g, v);
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (g * 4 + e < a.vocab)
                    p[e] = __fmul_rn(pinned_expf(__fadd_rn(__fmul_rn(v[e], inv_t), neg_m)), inv);
        }
        const int tile_end = min((tile + 1) * kSampThreads * 4, a.vocab);
        while (true) {
            const uint32_t ucum = S.ucum;
            const int E = S.E, start = S.start;
            const uint32_t tr = S.tr;
            uint32_t k[4];
            bool ser[4], valid[4];
            uint32_t kt = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = g * 4 + e;
                valid[e] = g < ngroups && i < a.vocab && i >= start;
                bool tie, big;
                classify(p[e], E, k[e], tie, big);
                ser[e] = tie || big;
                if (!valid[e]) { k[e] = 0; ser[e] = false; }
                kt = sat_add(kt, ser[e] ? kSat : k[e]);
            }
            // block exclusive scan of kt (saturating)
            uint32_t inc = kt;
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t o = __shfl_up_sync(0xffffffffu, inc, off);
                if (lane >= off) inc = sat_add(inc, o);
            }
            if (lane == 31) S.wscan[w] = inc;
            __syncthreads();
            if (w == 0) {
                uint32_t t = S.wscan[lane];
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t o = __shfl_up_sync(0xffffffffu, t, off);
                    if (lane >= off) t = sat_add(t, o);
                }
                S.red_u[lane] = t;  // inclusive warp-total scan
            }
            __syncthreads();
            uint32_t excl = __shfl_up_sync(0xffffffffu, inc, 1);
            if (lane == 0) excl = 0;
            uint32_t run = sat_add(ucum, sat_add(w > 0 ? S.red_u[w - 1] : 0u, excl));
            const uint32_t total = S.red_u[kSampWarps - 1];
            // first event of this thread
            uint32_t ev = kNoEvent;
            uint32_t before = run;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                if (!valid[e] || ev != kNoEvent) continue;
                const uint32_t local = (uint32_t)(tid * 4 + e);
                if (ser[e]) { ev = local << 1; before = run; break; }
                const uint32_t nr = sat_add(run, k[e]);
                if (nr >= kBinadeUnits) { ev = local << 1; before = run; break; }
                if (nr >= tr) { ev = (local << 1) | 1u; break; }
                run = nr;
            }
            const uint32_t wmin = __reduce_min_sync(0xffffffffu, ev);
            if (lane == 0) S.wscan[w] = wmin;
            __syncthreads();
            if (w == 0) {
                const uint32_t m = __reduce_min_sync(0xffffffffu, S.wscan[lane]);
                if (lane == 0) S.ev = m;
            }
            __syncthreads();
            const uint32_t gev = S.ev;
            if (gev == kNoEvent) {
                if (tid == 0) {
                    S.ucum = ucum + total;  // no crossing: exact and < 2^24
                    S.start = tile_end;
                }
                __syncthreads();
                break;
            }
            const int local = (int)(gev >> 1);
            if (ev == gev) {  // owner of the first event
                const int i = tile * kSampThreads * 4 + local;
                if (gev & 1u) {
                    S.result = i;
                } else {
                    // exact running sum before element i, then a real fp32 add
                    // before * 2^(E-23), exact: two power-of-two scalings
                    const float cum_prev =
                        __fmul_rn(__fmul_rn((float)before, pow2i(E - 23 + 64)), pow2i(-64));
                    const float cum = __fadd_rn(cum_prev, p[local & 3]);
                    if (cum >= r) S.result = i;
                    else { set_binade(S, cum, r); S.start = i + 1; }
                }
            }
            __syncthreads();
            if (S.result >= 0) break;
        }
        if (S.result >= 0) break;
    }
    if (tid == 0) a.out[row] = S.result >= 0 ? S.result : a.vocab - 1;
}

// softmax over rows in place (core/cpu_ops.cpp:83-99) with the pinned sum.
__global__ void __launch_bounds__(kSampThreads, 1)
softmax_rows_kernel(float* x, int n, int64_t stride) {
    __shared__ RowSmem S;
    float* row = x + (int64_t)blockIdx.x * stride;
    const int ngroups = (n + 3) >> 2;
    float mx = -INFINITY;
    for (int g = threadIdx.x; g < ngroups; g += kSampThreads)
        for (int e = 0; e < 4 && g * 4 + e < n; e++) mx = fmaxf(mx, row[g * 4 + e]);
    const float neg_m = -block_max(mx, S);
    float acc = 0.0f;
    for (int g = threadIdx.x; g < ngroups; g += kSampThreads)
        for (int e = 0; e < 4 && g * 4 + e < n; e++) {
            const float v = pinned_expf(__fadd_rn(row[g * 4 + e], neg_m));
            row[g * 4 + e] = v;
            acc = __fadd_rn(acc, v);
        }
    const float inv = __fdiv_rn(1.0f, block_sum_pinned(acc, S));
    for (int g = threadIdx.x; g < ngroups; g += kSampThreads)
        for (int e = 0; e < 4 && g * 4 + e < n; e++) row[g * 4 + e] = __fmul_rn(row[g * 4 + e], inv);
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
    const size_t smem = (size_t)(1 << slots_log2) * 12 + (size_t)((vocab + 31) / 32) * 4;
    if (smem > 200 * 1024) return fail(ANE_CUDA_ERR_UNSUPPORTED, "sample_rows: vocab %d too large", vocab);
    static thread_local int configured_dev = -1;
    static thread_local size_t configured_smem = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev || configured_smem < smem) {
        cudaError_t e = cudaFuncSetAttribute(sample_rows_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess)
            return fail(ANE_CUDA_ERR_CUDA, "sample_rows: %s", cudaGetErrorString(e));
        configured_dev = dev;
        configured_smem = 200 * 1024;
    }
    SampArgs a{logits, rows, vocab, logits_stride, history, history_len, history_stride, uniforms,
               temperature, repetition_penalty, frequency_penalty, repetition_context, out_tokens,
               slots_log2, vocab % 4 == 0 && logits_stride % 4 == 0 && is_aligned(logits, 16)};
    sample_rows_kernel<<<(unsigned)rows, kSampThreads, smem, as_stream(stream)>>>(a);
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
    softmax_rows_kernel<<<(unsigned)rows, kSampThreads, 0, as_stream(stream)>>>(x, n, stride);
    return check_launch("softmax_rows");
}

}  // extern "C"
