// convert_model.cpp -- `ane-lm convert` with the conversion on the GPU.
//
// For each shard (core/model_loader.cpp:163-171) and each BF16 tensor of it
// in header order (core/safetensors.cpp:345-383): create the parent
// directories, write the 128-byte blob header, and stream the tensor through
// two pinned staging slots: copy from the mapping into pinned memory, H2D,
// ane_cuda_bf16_to_f16, D2H, write.  While the GPU works on one slot the host
// fills or drains the other.  Non-BF16 tensors are skipped, as the reference
// does.  The output tree is byte-identical to the reference writer's.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <filesystem>
#include <string>

#include "ane_cuda.h"
#include "ane_internal.h"
#include "safetensors_io.h"

namespace ane_lm {
namespace cuda {
namespace {

constexpr size_t kChunkElems = (size_t)16 << 20;  // 32 MiB of BF16 per slot

int set_err(int st, const std::string& msg) { return ane::fail(st, "%s", msg.c_str()); }

struct Stage {
    uint16_t* h_in[2] = {nullptr, nullptr};
    uint16_t* h_out[2] = {nullptr, nullptr};
    uint16_t* d_in[2] = {nullptr, nullptr};
    uint16_t* d_out[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    size_t pending[2] = {0, 0};

    cudaError_t init() {
        cudaError_t e = cudaSuccess;
        for (int s = 0; s < 2 && e == cudaSuccess; s++) {
            e = cudaHostAlloc((void**)&h_in[s], kChunkElems * 2, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaHostAlloc((void**)&h_out[s], kChunkElems * 2, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaMalloc((void**)&d_in[s], kChunkElems * 2);
            if (e == cudaSuccess) e = cudaMalloc((void**)&d_out[s], kChunkElems * 2);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[s], cudaEventDisableTiming);
        }
        return e;
    }
    ~Stage() {
        for (int s = 0; s < 2; s++) {
            if (done[s]) cudaEventDestroy(done[s]);
            if (d_in[s]) cudaFree(d_in[s]);
            if (d_out[s]) cudaFree(d_out[s]);
            if (h_in[s]) cudaFreeHost(h_in[s]);
            if (h_out[s]) cudaFreeHost(h_out[s]);
        }
    }
};

// Writes one BF16 tensor as an ANE blob.
int write_blob(Stage& st, cudaStream_t s, const std::string& path, const uint16_t* src,
               int64_t n) {
    std::error_code ec;
    std::filesystem::create_directories(std::filesystem::path(path).parent_path(), ec);
    FILE* f = fopen(path.c_str(), "wb");
    if (!f) return set_err(ANE_CUDA_ERR_INVALID_ARG, "cannot write " + path);
    uint8_t header[128];
    ane_blob_header(header, (uint64_t)n * 2);
    bool ok = fwrite(header, 1, 128, f) == 128;
    int status = ANE_CUDA_OK;
    size_t chunk = 0;
    auto drain = [&](int slot) {
        if (!st.pending[slot]) return;
        const cudaError_t e = cudaEventSynchronize(st.done[slot]);
        if (e != cudaSuccess) {
            status = set_err(ANE_CUDA_ERR_CUDA, std::string("convert: ") + cudaGetErrorString(e));
        } else if (ok) {
            ok = fwrite(st.h_out[slot], 2, st.pending[slot], f) == st.pending[slot];
        }
        st.pending[slot] = 0;
    };
    for (int64_t off = 0; off < n && status == ANE_CUDA_OK; off += (int64_t)kChunkElems, chunk++) {
        const int slot = (int)(chunk & 1);
        drain(slot);  // the chunk two back, written in order
        const size_t m = (size_t)((n - off) < (int64_t)kChunkElems ? (n - off) : (int64_t)kChunkElems);
        memcpy(st.h_in[slot], src + off, m * 2);
        cudaError_t e = cudaMemcpyAsync(st.d_in[slot], st.h_in[slot], m * 2, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) { status = set_err(ANE_CUDA_ERR_CUDA, cudaGetErrorString(e)); break; }
        const int kst = ane_cuda_bf16_to_f16(st.d_out[slot], st.d_in[slot], (int64_t)m, s);
        if (kst != ANE_CUDA_OK) { status = kst; break; }
        e = cudaMemcpyAsync(st.h_out[slot], st.d_out[slot], m * 2, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaEventRecord(st.done[slot], s);
        if (e != cudaSuccess) { status = set_err(ANE_CUDA_ERR_CUDA, cudaGetErrorString(e)); break; }
        st.pending[slot] = m;
    }
    // the last two chunks, oldest first
    const int first = (int)(chunk & 1);
    drain(first);
    drain(first ^ 1);
    if (fclose(f) != 0) ok = false;
    if (status == ANE_CUDA_OK && !ok) status = set_err(ANE_CUDA_ERR_INVALID_ARG, "short write to " + path);
    return status;
}

int write_file_blobs(Stage& st, cudaStream_t s, const std::string& path,
                     const std::string& out_dir, int64_t* written) {
    SafetensorsFile sf;
    std::string err;
    if (!sf.open(path, &err)) return set_err(ANE_CUDA_ERR_INVALID_ARG, err);
    for (const TensorInfo& t : sf.tensors()) {
        if (t.dtype != TensorDtype::BF16) continue;
        const int64_t n = t.numel();
        if ((uint64_t)n * 2 > t.end - t.begin)
            return set_err(ANE_CUDA_ERR_INVALID_ARG, "tensor '" + t.name + "' is shorter than its shape");
        const int rc = write_blob(st, s, ane_blob_path(out_dir, t.name),
                                  reinterpret_cast<const uint16_t*>(sf.data(t)), n);
        if (rc != ANE_CUDA_OK) return rc;
        (*written)++;
    }
    return ANE_CUDA_OK;
}

}  // namespace
}  // namespace cuda
}  // namespace ane_lm

extern "C" {

int ane_cuda_write_ane_blobs(const char* safetensors_path, const char* output_dir,
                             int64_t* written, void* stream) {
    using namespace ane_lm::cuda;
    if (!safetensors_path || !output_dir || !written)
        return set_err(ANE_CUDA_ERR_INVALID_ARG, "write_ane_blobs: null argument");
    *written = 0;
    Stage st;
    const cudaError_t e = st.init();
    if (e != cudaSuccess)
        return set_err(ANE_CUDA_ERR_CUDA, std::string("write_ane_blobs: ") + cudaGetErrorString(e));
    return write_file_blobs(st, static_cast<cudaStream_t>(stream), safetensors_path, output_dir, written);
}

int ane_cuda_convert_model(const char* model_dir, const char* output_dir, int64_t* written,
                           void* stream) {
    using namespace ane_lm::cuda;
    if (!model_dir || !output_dir || !written)
        return set_err(ANE_CUDA_ERR_INVALID_ARG, "convert_model: null argument");
    *written = 0;
    std::vector<std::string> shards;
    std::string err;
    if (!discover_shards(model_dir, &shards, &err)) return set_err(ANE_CUDA_ERR_INVALID_ARG, err);
    Stage st;
    const cudaError_t e = st.init();
    if (e != cudaSuccess)
        return set_err(ANE_CUDA_ERR_CUDA, std::string("convert_model: ") + cudaGetErrorString(e));
    for (const std::string& shard : shards) {
        const int rc = write_file_blobs(st, static_cast<cudaStream_t>(stream), shard, output_dir, written);
        if (rc != ANE_CUDA_OK) return rc;
    }
    return ANE_CUDA_OK;
}

}  // extern "C"
