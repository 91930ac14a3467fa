// convert_model.cpp -- `ane-lm convert` with the conversion on the GPU.
//
// For each shard (core/model_loader.cpp:163-171) and each BF16 tensor of it
// (core/safetensors.cpp:345-383): create the parent directories, write the
// 128-byte blob header, and stream the tensor through two pinned staging
// slots: read from the shard into pinned memory (pread: no page faults on a
// shared mapping), H2D, ane_cuda_bf16_to_f16, D2H, write.  While the GPU works on one slot the
// host fills or drains the other.  Every tensor is its own output file, so
// the tensors are shared out among a few worker threads, each with its own
// stream and staging slots: the host copies and file writes, which bound
// the conversion, run in parallel.  Non-BF16 tensors are skipped, as the
// reference does.  The output tree is byte-identical to the reference
// writer's.
#include <cuda_runtime.h>

#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_set>
#include <vector>

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

// Reads `bytes` at `offset` of fd into dst; false on a short read or error.
bool read_at(int fd, void* dst, size_t bytes, uint64_t offset) {
    uint8_t* p = static_cast<uint8_t*>(dst);
    while (bytes > 0) {
        const ssize_t r = pread(fd, p, bytes, (off_t)offset);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        p += r;
        bytes -= (size_t)r;
        offset += (uint64_t)r;
    }
    return true;
}

// Writes one BF16 tensor (n elements at byte `src_offset` of shard fd) as an
// ANE blob.
int write_blob(Stage& st, cudaStream_t s, const std::string& path, int src_fd,
               uint64_t src_offset, int64_t n) {
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
        if (!read_at(src_fd, st.h_in[slot], m * 2, src_offset + (uint64_t)off * 2)) {
            status = set_err(ANE_CUDA_ERR_INVALID_ARG, "convert: short read of a tensor for " + path);
            break;
        }
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

// One blob to write: a BF16 tensor of a mapped shard.
struct Job {
    const std::string* file;  // the shard
    uint64_t offset;          // of the tensor's data in the shard
    int64_t n;
    std::string path;
};

// Adds the BF16 tensors of one opened shard to `jobs`, in header order.
int collect_jobs(const SafetensorsFile& sf, const std::string& out_dir, std::vector<Job>* jobs) {
    for (const TensorInfo& t : sf.tensors()) {
        if (t.dtype != TensorDtype::BF16) continue;
        const int64_t n = t.numel();
        if ((uint64_t)n * 2 > t.end - t.begin)
            return set_err(ANE_CUDA_ERR_INVALID_ARG, "tensor '" + t.name + "' is shorter than its shape");
        jobs->push_back({&sf.path(), sf.file_offset(t), n, ane_blob_path(out_dir, t.name)});
    }
    return ANE_CUDA_OK;
}

constexpr int kMaxWorkers = 4;

// Writes every job, on up to kMaxWorkers threads of the calling thread's
// device, each with its own stream and staging slots.  Work queued on
// `stream` before the call completes first.  The first failure stops the
// workers and is reported (with its message) on the calling thread.
int run_jobs(const std::vector<Job>& jobs, cudaStream_t stream, int64_t* written) {
    if (jobs.empty()) return ANE_CUDA_OK;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return set_err(ANE_CUDA_ERR_CUDA, std::string("convert: ") + cudaGetErrorString(e));
    const unsigned hw = std::thread::hardware_concurrency();
    const int nw = (int)std::min<size_t>(jobs.size(), std::max(1u, std::min<unsigned>(kMaxWorkers, hw ? hw : 1)));
    // A later job for the same output file (a tensor repeated in a later
    // shard) overwrites it in the reference, which writes in order: only the
    // last job per path runs, the earlier ones count as written.  So no two
    // workers ever write one file, and the tree is the reference's.
    std::vector<char> superseded(jobs.size(), 0);
    {
        std::unordered_set<std::string> seen;
        for (size_t i = jobs.size(); i-- > 0;)
            if (!seen.insert(jobs[i].path).second) superseded[i] = 1;
    }
    std::atomic<size_t> next{0};
    std::atomic<int64_t> done{0};
    std::atomic<bool> failed{false};
    std::mutex mu;
    int first_status = ANE_CUDA_OK;
    std::string first_msg;
    auto record = [&](int st, const std::string& msg) {
        std::lock_guard<std::mutex> lock(mu);
        if (first_status == ANE_CUDA_OK) {
            first_status = st;
            first_msg = msg;
        }
        failed = true;
    };
    auto worker = [&]() {
        cudaError_t we = cudaSetDevice(dev);
        cudaStream_t ws = nullptr;
        if (we == cudaSuccess) we = cudaStreamCreateWithFlags(&ws, cudaStreamNonBlocking);
        Stage st;
        if (we == cudaSuccess) we = st.init();
        if (we != cudaSuccess) {
            record(ANE_CUDA_ERR_CUDA, std::string("convert: ") + cudaGetErrorString(we));
        } else {
            for (size_t i = next++; i < jobs.size() && !failed; i = next++) {
                if (superseded[i]) {
                    done++;
                    continue;
                }
                const int fd = ::open(jobs[i].file->c_str(), O_RDONLY);
                if (fd < 0) {
                    record(ANE_CUDA_ERR_INVALID_ARG, "convert: cannot read " + *jobs[i].file);
                    break;
                }
                const int rc = write_blob(st, ws, jobs[i].path, fd, jobs[i].offset, jobs[i].n);
                ::close(fd);
                if (rc != ANE_CUDA_OK) {
                    record(rc, ane_cuda_last_error());  // the message is this thread's
                    break;
                }
                done++;
            }
        }
        if (ws) cudaStreamDestroy(ws);
    };
    std::vector<std::thread> pool;
    for (int w = 1; w < nw; w++) pool.emplace_back(worker);
    worker();  // the calling thread is worker 0
    for (std::thread& t : pool) t.join();
    *written += done;
    if (first_status != ANE_CUDA_OK) return set_err(first_status, first_msg);
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
    SafetensorsFile sf;
    std::string err;
    if (!sf.open(safetensors_path, &err)) return set_err(ANE_CUDA_ERR_INVALID_ARG, err);
    std::vector<Job> jobs;
    const int rc = collect_jobs(sf, output_dir, &jobs);
    if (rc != ANE_CUDA_OK) return rc;
    return run_jobs(jobs, static_cast<cudaStream_t>(stream), written);
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
    // every shard mapped for the whole conversion (address space only)
    std::vector<std::unique_ptr<SafetensorsFile>> files;
    std::vector<Job> jobs;
    for (const std::string& shard : shards) {
        files.push_back(std::make_unique<SafetensorsFile>());
        if (!files.back()->open(shard, &err)) return set_err(ANE_CUDA_ERR_INVALID_ARG, err);
        const int rc = collect_jobs(*files.back(), output_dir, &jobs);
        if (rc != ANE_CUDA_OK) return rc;
    }
    return run_jobs(jobs, static_cast<cudaStream_t>(stream), written);
}

}  // extern "C"
