// safetensors_io.h -- host side of `ane-lm convert` on the GPU: safetensors
// header parsing, shard discovery and the ANE blob writer.
//
// Follows core/safetensors.cpp (header parse :58-186, open :203-245, blob
// writer :316-383) and core/model_loader.cpp (shard discovery :14-90,
// write_ane_blobs over shards :163-171) of ANE-LM, with the conversion itself
// on the device (ane_cuda_bf16_to_f16).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ane_lm {
namespace cuda {

enum class TensorDtype { BF16, F16, F32, F64, I32, I64, U8, Unknown };

struct TensorInfo {
    std::string name;
    TensorDtype dtype = TensorDtype::Unknown;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // data_offsets, relative to the data section
    int64_t numel() const;
};

// A read-only mapping of one .safetensors file and its parsed header.
class SafetensorsFile {
public:
    ~SafetensorsFile();
    // false (with `err` set) when the file cannot be mapped or parsed.
    bool open(const std::string& path, std::string* err);
    const std::vector<TensorInfo>& tensors() const { return tensors_; }
    const uint8_t* data(const TensorInfo& t) const { return data_ + t.begin; }
    size_t data_bytes() const { return data_bytes_; }
    // byte offset of a tensor's data in the file, and the file's path
    uint64_t file_offset(const TensorInfo& t) const {
        return (uint64_t)(data_ - static_cast<const uint8_t*>(map_)) + t.begin;
    }
    const std::string& path() const { return path_; }

private:
    std::string path_;
    void* map_ = nullptr;
    size_t map_size_ = 0;
    const uint8_t* data_ = nullptr;
    size_t data_bytes_ = 0;
    std::vector<TensorInfo> tensors_;
};

// Shards of a model directory: the files named by
// model.safetensors.index.json's weight_map (unique, sorted), else every
// *.safetensors below the directory (sorted).
bool discover_shards(const std::string& model_dir, std::vector<std::string>* files,
                     std::string* err);

// The 128-byte ANE blob header for `data_bytes` of fp16 data.
void ane_blob_header(uint8_t header[128], uint64_t data_bytes);

// Blob path of a tensor: output_dir + "/" + name with '.' -> '/' + ".bin".
std::string ane_blob_path(const std::string& output_dir, const std::string& name);

}  // namespace cuda
}  // namespace ane_lm
