// qk_rope.cu -- per-head QK RMSNorm + half-split RoPE, in place
// (models/llm/qwen3.cpp:444-473; core/cpu_ops.cpp:43-80).
//
// Fast path (rot_dim == head_dim, head_dim / kVec a power of two in
// [2, 32], 16-byte aligned rows): one warp per row, or, for a few rows (a
// decode step), one warp per group of HPW heads of a row.  A head is served by
// GL = chunks/2 lanes; lane l of the group holds chunk l (elements
// [l*V, l*V+V), first half) and chunk l + GL (the RoPE partners j + half).
// With that layout
//   - the first butterfly stage of the pinned sum-of-squares order
//     (offset GL) is an add inside the lane, the rest are xor shuffles
//     inside the group; no shuffle is needed for RoPE;
//   - the lane's cos/sin for j in [l*V, l*V+V) serve every head of the row,
//     so they are computed once per row, in registers;
//   - the lane's norm weights are the same for every q (k) head: staged
//     once per CTA in shared memory.
//
// Generic path (partial RoPE, other head sizes, unaligned rows, or the
// caller-supplied cos/sin rows of apply_rope_cached): one warp per
// (row, head) with the head staged in shared memory.
#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

constexpr int kQkWarps = 4;
constexpr int kMaxHalfRot = 128;

struct RopeFreq {
    float f[kMaxHalfRot];
};

struct QkArgs {
    void* q;
    void* k;
    int64_t q_row_stride, k_row_stride;
    int q_head_stride, k_head_stride;
    int n_q, n_kv, head_dim, rot_dim;
    const float* qw;
    const float* kw;
    const int32_t* positions;  // per row; NULL -> `pos`
    int pos;
    int64_t rows;
    float eps;
    const float* cos_row;      // generic path only: caller tables
    const float* sin_row;
    // KV-cache write (row kernel, KV = true): row r's k heads after norm and
    // RoPE, and its v heads unchanged, go to ring slot slots[r] (< 0: none)
    // of the caches [slot][n_kv][head_dim] at cache + r * cache_row_stride.
    const void* v;
    int64_t v_row_stride;
    int v_head_stride;
    void* k_cache;
    void* v_cache;
    int64_t cache_row_stride;
    const int32_t* slots;
    int cache_capacity;        // slots outside [0, capacity) write nothing and raise a flag
    unsigned int* flags;
    // generic path only: RoPE over interleaved pairs (2j, 2j + 1), the
    // reference's fallback without tables (core/cpu_ops.cpp:66-77)
    int interleaved;
};

// One warp per row.  The row's heads stream through a ring of D register
// slots: iteration `it` (HPW heads) is consumed from slot it % D, which is
// refilled with iteration it + D straight away, so D iterations of loads
// stay in flight while the warp computes.  The in-place kernel takes D = 1
// (eight resident CTAs per SM) when the rows span several waves of CTAs:
// measured 4-5% faster there than D = 2, whose extra registers cost a
// resident CTA; when every row's warp is resident at once (one wave of the
// D = 2 kernel's seven CTAs per SM, 4,096 Qwen3-8B rows on a B200) each warp
// works through its row alone and D = 2 keeps a second iteration of loads
// in flight (1.5% faster alone, the chain 1.6%).  A few rows (fewer CTAs
// than SMs: the batch-1 decode step) take D = 1 again: there the row's own
// latency decides, and the D = 2 kernel measured 0.6 us slower per token.
// The KV-writing kernel keeps 2.  Per-row setup (position,
// cos/sin) is paid once for all heads of the row.  GL (lanes per head) is a
// template parameter so that every index is a constant; the frequency table
// and the norm weights are staged once per CTA in shared memory.
constexpr int kRowWarps = 4;

template <typename T, int GL, int D, bool KV>
__global__ void __launch_bounds__(kRowWarps * kWarp, KV ? 4 : (D == 2 ? 7 : 8))
qk_norm_rope_row_kernel(const QkArgs a, const __grid_constant__ RopeFreq fr, const bool pow2_dim,
                        const int wpr) {
    using S = typename T::storage;
    constexpr int V = T::kVec;
    constexpr int HPW = kWarp / GL;                  // heads per iteration
    constexpr int HALF = GL * V;                     // rot_dim / 2 = head_dim / 2
    constexpr int CPL = HALF >= 32 ? HALF / 32 : V;  // cos/sin computed per lane
    {
        // the row's q and k heads toward L2 while the previous grid drains,
        // when they are contiguous (16-byte aligned, sizes multiples of 16
        // bytes on this path)
        const int64_t gw = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
        const int64_t r = gw / wpr;
        if ((threadIdx.x & 31) == 0 && r < a.rows && gw % wpr == 0) {
            if (a.n_q > 0 && a.q_head_stride == 2 * HALF)
                prefetch_l2((const S*)a.q + r * a.q_row_stride, (uint32_t)(a.n_q * 2 * HALF * sizeof(S)));
            if (a.n_kv > 0 && a.k_head_stride == 2 * HALF)
                prefetch_l2((const S*)a.k + r * a.k_row_stride, (uint32_t)(a.n_kv * 2 * HALF * sizeof(S)));
        }
    }
    pdl_begin();
    __shared__ __align__(16) float s_freq[HALF];
    __shared__ __align__(16) float s_w[2][2 * HALF];
    for (int i = threadIdx.x; i < HALF; i += blockDim.x) s_freq[i] = fr.f[i];
    if (a.qw != nullptr) {
        for (int i = threadIdx.x; i < 2 * HALF; i += blockDim.x) {
            s_w[0][i] = __ldg(a.qw + i);
            s_w[1][i] = __ldg(a.kw + i);
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    // a row is wpr warps: warp `part` of them takes the row's iterations
    // [part * per, part * per + per) (per = the iterations a warp takes)
    const int64_t gw = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    const int64_t row = gw / wpr;
    const int part = (int)(gw - row * wpr);
    if (row >= a.rows) return;
    const int g = lane / GL;  // head slot of this lane
    const int l = lane % GL;  // lane within the head group
    const int nq = a.n_q, nqk = a.n_q + a.n_kv;
    const int nh = KV ? nqk + a.n_kv : nqk;  // with KV the v heads follow, copy only
    const int nit_row = (nh + HPW - 1) / HPW;
    const int per = (nit_row + wpr - 1) / wpr;
    const int itb = part * per;                         // this warp's first iteration
    const int nit = min(nit_row, itb + per);            // one past its last
    S* const qrow = (S*)a.q + row * a.q_row_stride;
    S* const krow = (S*)a.k + row * a.k_row_stride;
    const int qhs = a.q_head_stride, khs = a.k_head_stride;
    auto head_ptr = [&](int h) -> S* {
        if (KV && h >= nqk) return (S*)a.v + row * a.v_row_stride + (int64_t)(h - nqk) * a.v_head_stride;
        return h < nq ? qrow + h * qhs : krow + (h - nq) * khs;
    };
    int slot = -1;
    if constexpr (KV) {
        slot = __ldg(a.slots + row);
        if (slot >= a.cache_capacity) {
            if (lane == 0 && a.flags) atomicOr(a.flags, ANE_CUDA_FLAG_BAD_CACHE);
            slot = -1;
        }
    }
    // cache row of kv head j in this row's slot
    auto cache_ptr = [&](void* cache, int j) -> S* {
        return (S*)cache + row * a.cache_row_stride + ((int64_t)slot * a.n_kv + j) * (2 * HALF);
    };

    uint4 lo[D], hi[D];
#pragma unroll
    for (int d = 0; d < D; d++) {
        const int h = (itb + d) * HPW + g;
        if (itb + d < nit && h < nh) {
            const S* p = head_ptr(h);
            lo[d] = ld_stream(p + l * V);
            hi[d] = ld_stream(p + HALF + l * V);
        }
    }

    // cos/sin of the lane's V frequencies at the row's position.  The HPW
    // lanes sharing l need the same values: each computes CPL of them and
    // the rest arrive by shuffle.
    const float fpos = (float)(a.positions ? __ldg(a.positions + row) : a.pos);
    float cs[V], sn[V];
    if constexpr (CPL == V) {
#pragma unroll
        for (int e = 0; e < V; e++) pinned_sincosf(__fmul_rn(fpos, s_freq[l * V + e]), &sn[e], &cs[e]);
    } else {
        float mc[CPL], ms[CPL];
#pragma unroll
        for (int c = 0; c < CPL; c++)
            pinned_sincosf(__fmul_rn(fpos, s_freq[l * V + g * CPL + c]), &ms[c], &mc[c]);
#pragma unroll
        for (int e = 0; e < V; e++) {
            cs[e] = __shfl_sync(0xffffffffu, mc[e % CPL], (e / CPL) * GL + l);
            sn[e] = __shfl_sync(0xffffffffu, ms[e % CPL], (e / CPL) * GL + l);
        }
    }

    const bool norm = a.qw != nullptr;
    const float inv_dim = 1.0f / (float)(2 * HALF);
    for (int it0 = itb; it0 < nit; it0 += D) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            if (it0 + d >= nit) break;  // warp-uniform
            const int h = (it0 + d) * HPW + g;
            const bool live = h < nh;
            const bool vhead = KV && h >= nqk;  // copied bit for bit, no norm / RoPE
            uint4 raw_lo, raw_hi;
            if constexpr (KV) {
                raw_lo = lo[d];
                raw_hi = hi[d];
            }
            float x0[V], x1[V];
            if (live) {
                unpack<T>(lo[d], x0);
                unpack<T>(hi[d], x1);
            } else {
#pragma unroll
                for (int e = 0; e < V; e++) { x0[e] = 0.0f; x1[e] = 0.0f; }
            }
            const int hn = h + D * HPW;  // refill the slot D iterations ahead
            if (it0 + d + D < nit && hn < nh) {
                const S* q = head_ptr(hn);
                lo[d] = ld_stream(q + l * V);
                hi[d] = ld_stream(q + HALF + l * V);
            }
            if (norm) {
                float acc = __fadd_rn(sumsq_chain<V>(x0, 0.0f), sumsq_chain<V>(x1, 0.0f));
#pragma unroll
                for (int off = GL / 2; off >= 1; off >>= 1)
                    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
                // ss / dim is exact as a multiply when dim is a power of two
                const float mean = pow2_dim ? __fmul_rn(acc, inv_dim) : __fdiv_rn(acc, (float)(2 * HALF));
                const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
                const float* w = s_w[h < nq ? 0 : 1];
#pragma unroll
                for (int q4 = 0; q4 < (vhead ? 0 : V / 4); q4++) {
                    const float4 t0 = reinterpret_cast<const float4*>(w + l * V)[q4];
                    const float4 t1 = reinterpret_cast<const float4*>(w + HALF + l * V)[q4];
                    const float w0[4] = {t0.x, t0.y, t0.z, t0.w};
                    const float w1[4] = {t1.x, t1.y, t1.z, t1.w};
#pragma unroll
                    for (int e = 0; e < 4; e += 2) {  // (x * inv) * w, neighbouring elements paired
                        const float2 t0 = mul2_rn(mul2_rn(make_float2(x0[4 * q4 + e], x0[4 * q4 + e + 1]),
                                                          make_float2(inv, inv)),
                                                  make_float2(w0[e], w0[e + 1]));
                        const float2 t1 = mul2_rn(mul2_rn(make_float2(x1[4 * q4 + e], x1[4 * q4 + e + 1]),
                                                          make_float2(inv, inv)),
                                                  make_float2(w1[e], w1[e + 1]));
                        x0[4 * q4 + e] = t0.x;
                        x0[4 * q4 + e + 1] = t0.y;
                        x1[4 * q4 + e] = t1.x;
                        x1[4 * q4 + e + 1] = t1.y;
                    }
                }
            }
            if (vhead) {
                if (live && slot >= 0) {
                    S* c = cache_ptr(a.v_cache, h - nqk);
                    st_stream(c + l * V, raw_lo);
                    st_stream(c + HALF + l * V, raw_hi);
                }
            } else if (live) {
                float y0[V], y1[V];
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    // v0 c - v1 s and v1 c + v0 s for elements e and e + 1:
                    // each product pairs neighbouring elements (operands that
                    // already sit in neighbouring registers), the sums and
                    // differences are scalar (a packed multiply feeding a
                    // packed add may be contracted)
                    const float2 c2 = make_float2(cs[e], cs[e + 1]), s2 = make_float2(sn[e], sn[e + 1]);
                    const float2 a0 = make_float2(x0[e], x0[e + 1]), a1 = make_float2(x1[e], x1[e + 1]);
                    const float2 p0c = mul2_rn(a0, c2), p1s = mul2_rn(a1, s2);
                    const float2 p1c = mul2_rn(a1, c2), p0s = mul2_rn(a0, s2);
                    y0[e] = __fsub_rn(p0c.x, p1s.x);
                    y0[e + 1] = __fsub_rn(p0c.y, p1s.y);
                    y1[e] = __fadd_rn(p1c.x, p0s.x);
                    y1[e + 1] = __fadd_rn(p1c.y, p0s.y);
                }
                const uint4 p0 = pack<T>(y0), p1 = pack<T>(y1);
                S* q = head_ptr(h);
                st_stream(q + l * V, p0);
                st_stream(q + HALF + l * V, p1);
                if (KV && h >= nq && slot >= 0) {  // k head after RoPE: also into the cache
                    S* c = cache_ptr(a.k_cache, h - nq);
                    st_stream(c + l * V, p0);
                    st_stream(c + HALF + l * V, p1);
                }
            }
        }
    }
}

// One warp per (row, head); head staged in shared memory as fp32.
constexpr int kGenericMaxHead = 1024;

template <typename T>
__global__ void __launch_bounds__(kQkWarps * kWarp)
qk_norm_rope_generic_kernel(const QkArgs a, const __grid_constant__ RopeFreq fr) {
    pdl_begin();
    using S = typename T::storage;
    constexpr int V = T::kVec;
    __shared__ float sm[kQkWarps][kGenericMaxHead];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int nh = a.n_q + a.n_kv;
    const int64_t item = (int64_t)blockIdx.x * kQkWarps + wid;
    if (item >= a.rows * nh) return;
    const int64_t row = item / nh;
    const int h = (int)(item - row * nh);
    S* base = h < a.n_q ? (S*)a.q + row * a.q_row_stride + (int64_t)h * a.q_head_stride
                        : (S*)a.k + row * a.k_row_stride + (int64_t)(h - a.n_q) * a.k_head_stride;
    float* v = sm[wid];
    const int hd = a.head_dim;
    const int nchunk = (hd + V - 1) / V;
    float acc = 0.0f;
    for (int c = lane; c < nchunk; c += kWarp) {
        const int n = min(V, hd - c * V);
        for (int e = 0; e < n; e++) {
            const float x = T::to_f(base[c * V + e]);
            v[c * V + e] = x;
            acc = __fmaf_rn(x, x, acc);
        }
    }
    __syncwarp();
    if (a.qw) {
        const float inv = rms_inv(butterfly_sum(acc, kWarp), hd, a.eps);
        const float* w = h < a.n_q ? a.qw : a.kw;
        for (int i = lane; i < hd; i += kWarp) v[i] = __fmul_rn(__fmul_rn(v[i], inv), __ldg(w + i));
        __syncwarp();
    }
    const int half = a.rot_dim / 2;
    const float fpos = (float)(a.positions ? __ldg(a.positions + row) : a.pos);
    if (a.interleaved) {
        // pair (2j, 2j + 1): angle = pos * inv_freq[j], unfused products
        for (int j = lane; j < half; j += kWarp) {
            float c, s;
            pinned_sincosf(__fmul_rn(fpos, fr.f[j]), &s, &c);
            const float x0 = v[2 * j], x1 = v[2 * j + 1];
            base[2 * j] = T::from_f(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
            base[2 * j + 1] = T::from_f(__fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
        }
        for (int i = a.rot_dim + lane; i < hd; i += kWarp) base[i] = T::from_f(v[i]);
        return;
    }
    for (int j = lane; j < half; j += kWarp) {
        float c, s;
        if (a.cos_row) {
            c = __ldg(a.cos_row + j);
            s = __ldg(a.sin_row + j);
        } else {
            pinned_sincosf(__fmul_rn(fpos, fr.f[j]), &s, &c);
        }
        const float x0 = v[j], x1 = v[j + half];
        base[j] = T::from_f(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
        base[j + half] = T::from_f(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s)));
    }
    for (int i = a.rot_dim + lane; i < hd; i += kWarp) base[i] = T::from_f(v[i]);
}

// inv_freq[j] = 1.0f / powf(theta, (float)(2j) / (float)rot_dim)
// (models/llm/qwen3.cpp:205-208), powf as the float rounding of the double pow.
static void make_freq(RopeFreq* fr, int rot_dim, float theta) {
    for (int j = 0; 2 * j < rot_dim && j < kMaxHalfRot; j++) {
        const float e = (float)(2 * j) / (float)rot_dim;
        const float p = (float)pow((double)theta, (double)e);
        fr->f[j] = 1.0f / p;
    }
}

static int ilog2_exact(int v) {
    if (v <= 0 || (v & (v - 1))) return -1;
    int r = 0;
    while ((1 << r) < v) r++;
    return r;
}

template <typename T>
static int launch_qk(const QkArgs& a, const RopeFreq& fr, cudaStream_t s, bool kv) {
    constexpr int V = T::kVec;
    const int es = (int)sizeof(typename T::storage);
    const int nh = a.n_q + a.n_kv;
    const int nchunk = a.head_dim / V;
    const int gl_log2 = ilog2_exact(nchunk) - 1;
    bool fast = a.cos_row == nullptr && !a.interleaved && a.rot_dim == a.head_dim && a.head_dim % V == 0 &&
                gl_log2 >= 0 && nchunk <= 32 && is_aligned(a.q, 16) && is_aligned(a.k, 16) &&
                (a.q_row_stride * es) % 16 == 0 && (a.k_row_stride * es) % 16 == 0 &&
                (a.q_head_stride * es) % 16 == 0 && (a.k_head_stride * es) % 16 == 0;
    if (kv) {
        const bool ok = fast && is_aligned(a.v, 16) && is_aligned(a.k_cache, 16) &&
                        is_aligned(a.v_cache, 16) && (a.v_row_stride * es) % 16 == 0 &&
                        (a.v_head_stride * es) % 16 == 0 && (a.cache_row_stride * es) % 16 == 0;
        if (!ok)
            return fail(ANE_CUDA_ERR_UNSUPPORTED,
                        "qk_norm_rope_kv: needs head_dim / %d a power of two <= 32 and 16-byte aligned "
                        "rows, heads and caches", V);
    }
    if (fast) {
        const bool pow2 = (a.head_dim & (a.head_dim - 1)) == 0;
        const unsigned sms = (unsigned)sm_count();
        // Few rows (a decode step): one warp per iteration of HPW heads, so
        // a row's iterations run side by side instead of one after another,
        // as long as all those warps fit in one wave of the D = 1 kernel
        // (eight CTAs of four warps per SM).  The per-row set-up (position,
        // cos/sin) is then repeated by each of the row's warps.
        const int hpw = kWarp >> gl_log2;
        const int nit = (nh + (kv ? a.n_kv : 0) + hpw - 1) / hpw;
        const int wpr = a.rows * nit <= (int64_t)kRowWarps * 8 * sms ? nit : 1;
        const unsigned blocks = (unsigned)((a.rows * wpr + kRowWarps - 1) / kRowWarps);
        // one full wave of whole rows: more CTAs than SMs, all resident in the D = 2 kernel
        const bool one_wave = wpr == 1 && blocks > sms && blocks <= 7u * sms;
#define ANE_QK_ROW(GLV)                                                                          \
    do {                                                                                          \
        if (kv) launch_pdl(qk_norm_rope_row_kernel<T, GLV, 2, true>, blocks, kRowWarps * kWarp, 0, s, a, fr, pow2, wpr); \
        else if (one_wave) launch_pdl(qk_norm_rope_row_kernel<T, GLV, 2, false>, blocks, kRowWarps * kWarp, 0, s, a, fr, pow2, wpr); \
        else launch_pdl(qk_norm_rope_row_kernel<T, GLV, 1, false>, blocks, kRowWarps * kWarp, 0, s, a, fr, pow2, wpr);   \
    } while (0)
        switch (gl_log2) {
            case 0: ANE_QK_ROW(1); break;
            case 1: ANE_QK_ROW(2); break;
            case 2: ANE_QK_ROW(4); break;
            case 3: ANE_QK_ROW(8); break;
            default: ANE_QK_ROW(16); break;
        }
#undef ANE_QK_ROW
    } else {
        if (a.head_dim > kGenericMaxHead)
            return fail(ANE_CUDA_ERR_UNSUPPORTED, "qk_norm_rope: head_dim %d > %d", a.head_dim,
                        kGenericMaxHead);
        const int64_t items = a.rows * nh;
        const unsigned blocks = (unsigned)((items + kQkWarps - 1) / kQkWarps);
        launch_pdl(qk_norm_rope_generic_kernel<T>, blocks, kQkWarps * kWarp, 0, s, a, fr);
    }
    return check_launch("qk_norm_rope");
}

static int run_qk(int dtype, const QkArgs& a, float theta, cudaStream_t s, bool kv = false) {
    RopeFreq fr;
    make_freq(&fr, a.rot_dim, theta);
    if (dtype == ANE_CUDA_F32) return launch_qk<F32>(a, fr, s, kv);
    if (dtype == ANE_CUDA_F16) return launch_qk<F16>(a, fr, s, kv);
    return launch_qk<BF16>(a, fr, s, kv);
}

static int validate(const char* fn, const QkArgs& a) {
    if (a.n_q < 0 || a.n_kv < 0 || a.n_q + a.n_kv <= 0 || a.head_dim <= 0 || a.rows < 0)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: n_q=%d n_kv=%d head_dim=%d rows=%lld", fn, a.n_q,
                    a.n_kv, a.head_dim, (long long)a.rows);
    if (a.rot_dim < 0 || a.rot_dim > a.head_dim || (a.rot_dim & 1))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: rot_dim %d (head_dim %d)", fn, a.rot_dim, a.head_dim);
    if (a.rot_dim / 2 > kMaxHalfRot)
        return fail(ANE_CUDA_ERR_UNSUPPORTED, "%s: rot_dim %d > %d", fn, a.rot_dim, 2 * kMaxHalfRot);
    if ((a.n_q > 0 && !a.q) || (a.n_kv > 0 && !a.k))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: null q/k", fn);
    if ((a.qw == nullptr) != (a.kw == nullptr))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: give both q_weight and k_weight or neither", fn);
    if ((a.cos_row == nullptr) != (a.sin_row == nullptr))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "%s: give both cos_row and sin_row or neither", fn);
    return ANE_CUDA_OK;
}

}  // namespace ane

extern "C" {

int ane_cuda_qk_norm_rope(int dtype, void* q, void* k, int64_t q_row_stride,
                          int64_t k_row_stride, int q_head_stride, int k_head_stride,
                          int n_q_heads, int n_kv_heads, int head_dim, int rot_dim,
                          const float* q_weight, const float* k_weight,
                          const int32_t* positions, int64_t rows, float theta, float eps,
                          void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "qk_norm_rope: bad dtype %d", dtype);
    QkArgs a{q, k, q_row_stride, k_row_stride, q_head_stride, k_head_stride, n_q_heads, n_kv_heads,
             head_dim, rot_dim, q_weight, k_weight, positions, 0, rows, eps, nullptr, nullptr};
    a.flags = status_flags_device();
    int st = validate("qk_norm_rope", a);
    if (st) return st;
    if (rows == 0) return ANE_CUDA_OK;
    if (!positions) return fail(ANE_CUDA_ERR_INVALID_ARG, "qk_norm_rope: positions is NULL");
    return run_qk(dtype, a, theta, as_stream(stream));
}

int ane_cuda_qk_norm_rope_kv(int dtype, void* q, void* k, const void* v, int64_t q_row_stride,
                             int64_t k_row_stride, int64_t v_row_stride, int q_head_stride,
                             int k_head_stride, int v_head_stride, int n_q_heads, int n_kv_heads,
                             int head_dim, const float* q_weight, const float* k_weight,
                             const int32_t* positions, void* k_cache, void* v_cache,
                             int64_t cache_row_stride, const int32_t* slots, int cache_capacity,
                             int64_t rows, float theta, float eps, void* stream) {
    using namespace ane;
    if (!valid_dtype(dtype)) return fail(ANE_CUDA_ERR_INVALID_ARG, "qk_norm_rope_kv: bad dtype %d", dtype);
    QkArgs a{q, k, q_row_stride, k_row_stride, q_head_stride, k_head_stride, n_q_heads, n_kv_heads,
             head_dim, head_dim, q_weight, k_weight, positions, 0, rows, eps, nullptr, nullptr,
             v, v_row_stride, v_head_stride, k_cache, v_cache, cache_row_stride, slots,
             cache_capacity, status_flags_device()};
    int st = validate("qk_norm_rope_kv", a);
    if (st) return st;
    if (rows == 0) return ANE_CUDA_OK;
    if (n_kv_heads <= 0 || !positions || !v || !k_cache || !v_cache || !slots)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "qk_norm_rope_kv: null pointer or no kv heads");
    if (cache_row_stride < 0 || cache_capacity <= 0 ||
        (cache_row_stride > 0 && cache_row_stride < (int64_t)cache_capacity * n_kv_heads * head_dim))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "qk_norm_rope_kv: cache_row_stride %lld capacity %d",
                    (long long)cache_row_stride, cache_capacity);
    return run_qk(dtype, a, theta, as_stream(stream), true);
}

int ane_cuda_apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads, int head_dim,
                               int q_head_stride, int k_head_stride, int rot_dim, int pos,
                               float theta, const float* cos_row, const float* sin_row,
                               void* stream) {
    using namespace ane;
    // core/cpu_ops.cpp:62-77: both tables -> the half-split fast path;
    // either one NULL -> the fallback over interleaved pairs
    const bool tables = cos_row != nullptr && sin_row != nullptr;
    QkArgs a{q, k, 0, 0, q_head_stride, k_head_stride, n_q_heads, n_kv_heads, head_dim, rot_dim,
             nullptr, nullptr, nullptr, pos, 1, 0.0f, tables ? cos_row : nullptr,
             tables ? sin_row : nullptr};
    a.interleaved = tables ? 0 : 1;
    int st = validate("apply_rope_cached", a);
    if (st) return st;
    return run_qk(ANE_CUDA_F32, a, theta, as_stream(stream));
}

}  // extern "C"
