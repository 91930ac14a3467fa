// ane_internal.h -- host-side helpers shared by the C ABI entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "ane_cuda.h"

namespace ane {

// Records a one-line description for ane_cuda_last_error() (thread-local)
// and returns `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// ANE_CUDA_OK, or ANE_CUDA_ERR_CUDA with the launch error recorded.
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool is_aligned(const void* p, uintptr_t a) {
    return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

inline int elem_size(int dtype) { return dtype == ANE_CUDA_F32 ? 4 : 2; }
inline bool valid_dtype(int dtype) {
    return dtype == ANE_CUDA_F32 || dtype == ANE_CUDA_F16 || dtype == ANE_CUDA_BF16;
}

// Device address of the current device's status word (the flags of
// ane_cuda_read_status_flags), for kernels compiled in other files; NULL on
// a CUDA error.
unsigned int* status_flags_device();

// Number of SMs of the current device (cached per device).
int sm_count();

// Grid size for a grid-stride kernel: `want` blocks, capped at what is
// resident at once (SMs x blocks per SM), so the grid is a single wave.
int resident_grid(const void* kernel, int threads, size_t smem, int64_t want);

}  // namespace ane
