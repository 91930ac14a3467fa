// gather.cu -- batched embedding gather (models/llm/qwen3.cpp:498) and the
// per-device status word the C ABI reports bad input through.
//
// One warp per output row; 16-byte vector copies when the row width and
// both base pointers allow it, element copies otherwise.  Out-of-range ids
// write a zero row and raise ANE_CUDA_FLAG_BAD_TOKEN_ID.
#include <atomic>

#include "ane_common.cuh"
#include "ane_internal.h"

namespace ane {

__device__ unsigned int g_status_flags;

constexpr int kGatherWarps = 4;

// Byte-row copy: row_vec 16-byte vectors per row.
__global__ void __launch_bounds__(kGatherWarps * kWarp)
gather_vec_kernel(uint4* __restrict__ out, const uint4* __restrict__ table,
                  const int32_t* __restrict__ ids, int64_t rows, int vocab, int64_t row_vec) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kGatherWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int32_t id = __ldg(ids + row);
    uint4* o = out + row * row_vec;
    if (id < 0 || id >= vocab) {
        for (int64_t c = lane; c < row_vec; c += kWarp) o[c] = make_uint4(0, 0, 0, 0);
        if (lane == 0) atomicOr(&g_status_flags, ANE_CUDA_FLAG_BAD_TOKEN_ID);
        return;
    }
    const uint4* t = table + (int64_t)id * row_vec;
    int64_t c = lane;
    for (; c + 3 * kWarp < row_vec; c += 4 * kWarp) {
        uint4 a = ld_keep(t + c), b = ld_keep(t + c + kWarp);
        uint4 d = ld_keep(t + c + 2 * kWarp), e = ld_keep(t + c + 3 * kWarp);
        st_stream(o + c, a); st_stream(o + c + kWarp, b);
        st_stream(o + c + 2 * kWarp, d); st_stream(o + c + 3 * kWarp, e);
    }
    for (; c < row_vec; c += kWarp) st_stream(o + c, ld_keep(t + c));
}

// Widening gather: F16/BF16 table -> F32 rows (exact), or same-type
// element copy for unaligned shapes.
template <typename TI, typename TO>
__global__ void __launch_bounds__(kGatherWarps * kWarp)
gather_elem_kernel(typename TO::storage* __restrict__ out,
                   const typename TI::storage* __restrict__ table,
                   const int32_t* __restrict__ ids, int64_t rows, int vocab, int hidden) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kGatherWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int32_t id = __ldg(ids + row);
    typename TO::storage* o = out + row * hidden;
    if (id < 0 || id >= vocab) {
        for (int c = lane; c < hidden; c += kWarp) o[c] = TO::from_f(0.0f);
        if (lane == 0) atomicOr(&g_status_flags, ANE_CUDA_FLAG_BAD_TOKEN_ID);
        return;
    }
    const typename TI::storage* t = table + (int64_t)id * hidden;
    for (int c = lane; c < hidden; c += kWarp) o[c] = TO::from_f(TI::to_f(t[c]));
}

// Looked up once per device (a failed lookup is retried); concurrent first
// calls store the same address (atomics, so there is no data race).
unsigned int* status_flags_device() {
    static std::atomic<unsigned int*> addr[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    unsigned int* a = addr[dev].load(std::memory_order_acquire);
    if (!a) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status_flags) != cudaSuccess) return nullptr;
        a = static_cast<unsigned int*>(p);
        addr[dev].store(a, std::memory_order_release);
    }
    return a;
}

}  // namespace ane

extern "C" {

int ane_cuda_read_status_flags(uint32_t* flags, int clear) {
    using namespace ane;
    if (!flags) return fail(ANE_CUDA_ERR_INVALID_ARG, "read_status_flags: flags is NULL");
    cudaError_t e = cudaDeviceSynchronize();
    unsigned int v = 0;
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_status_flags, sizeof(v));
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_status_flags, &zero, sizeof(zero));
    }
    if (e != cudaSuccess)
        return fail(ANE_CUDA_ERR_CUDA, "read_status_flags: %s", cudaGetErrorString(e));
    *flags = v;
    return ANE_CUDA_OK;
}

int ane_cuda_embedding_gather(void* out, int out_dtype, const void* table, int table_dtype,
                              const int32_t* ids, int64_t rows, int vocab, int hidden,
                              void* stream) {
    using namespace ane;
    if (rows < 0 || vocab <= 0 || hidden <= 0)
        return fail(ANE_CUDA_ERR_INVALID_ARG, "embedding_gather: rows=%lld vocab=%d hidden=%d",
                    (long long)rows, vocab, hidden);
    if (!valid_dtype(out_dtype) || !valid_dtype(table_dtype))
        return fail(ANE_CUDA_ERR_INVALID_ARG, "embedding_gather: bad dtype");
    if (rows == 0) return ANE_CUDA_OK;
    if (!out || !table || !ids) return fail(ANE_CUDA_ERR_INVALID_ARG, "embedding_gather: null pointer");
    cudaStream_t s = as_stream(stream);
    const unsigned blocks = (unsigned)((rows + kGatherWarps - 1) / kGatherWarps);
    const int tes = elem_size(table_dtype);
    if (out_dtype == table_dtype) {
        const int64_t row_bytes = (int64_t)hidden * tes;
        if (row_bytes % 16 == 0 && is_aligned(out, 16) && is_aligned(table, 16)) {
            launch_pdl(gather_vec_kernel, blocks, kGatherWarps * kWarp, 0, s,
                reinterpret_cast<uint4*>(out), reinterpret_cast<const uint4*>(table), ids, rows,
                vocab, row_bytes / 16);
        } else if (table_dtype == ANE_CUDA_F32) {
            launch_pdl(gather_elem_kernel<F32, F32>, blocks, kGatherWarps * kWarp, 0, s,
                (float*)out, (const float*)table, ids, rows, vocab, hidden);
        } else if (table_dtype == ANE_CUDA_F16) {
            launch_pdl(gather_elem_kernel<F16, F16>, blocks, kGatherWarps * kWarp, 0, s,
                (__half*)out, (const __half*)table, ids, rows, vocab, hidden);
        } else {
            launch_pdl(gather_elem_kernel<BF16, BF16>, blocks, kGatherWarps * kWarp, 0, s,
                (__nv_bfloat16*)out, (const __nv_bfloat16*)table, ids, rows, vocab, hidden);
        }
    } else if (out_dtype == ANE_CUDA_F32 && table_dtype == ANE_CUDA_F16) {
        launch_pdl(gather_elem_kernel<F16, F32>, blocks, kGatherWarps * kWarp, 0, s,
            (float*)out, (const __half*)table, ids, rows, vocab, hidden);
    } else if (out_dtype == ANE_CUDA_F32 && table_dtype == ANE_CUDA_BF16) {
        launch_pdl(gather_elem_kernel<BF16, F32>, blocks, kGatherWarps * kWarp, 0, s,
            (float*)out, (const __nv_bfloat16*)table, ids, rows, vocab, hidden);
    } else {
        return fail(ANE_CUDA_ERR_UNSUPPORTED,
                    "embedding_gather: out dtype %d from table dtype %d", out_dtype, table_dtype);
    }
    return check_launch("embedding_gather");
}

}  // extern "C"
