#pragma once

// Reader of OPWPACK1 tensor packs (OpWorks include/runtime/pack_reader.cuh:
// same magic, u64 manifest length, JSON manifest, 64-byte aligned blob,
// aliases, dtype float32 / bfloat16, and the same API). The file is mapped
// once (mmap) instead of reopened per tensor, and data() hands out pointers
// into the mapping so the loader can stream tensors to the GPU without an
// intermediate host copy.

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "json.cuh"

namespace opworks {

class PackReader {
  public:
    struct TensorMeta {
        uint64_t offset; // bytes, relative to the blob start
        std::vector<int64_t> shape;
        int64_t numel;
    };

    explicit PackReader(const std::string &path) : path_(path) {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0)
            throw std::runtime_error("cannot open pack " + path);
        struct stat st;
        if (::fstat(fd, &st) != 0) {
            ::close(fd);
            throw std::runtime_error("cannot stat pack " + path);
        }
        size_ = static_cast<uint64_t>(st.st_size);
        if (size_ < 16) {
            ::close(fd);
            throw std::runtime_error(path + ": not an OpWorks pack (bad magic)");
        }
        void *m = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED)
            throw std::runtime_error("cannot map pack " + path);
        map_ = std::shared_ptr<void>(m, [sz = size_](void *p) { ::munmap(p, sz); });
        const char *base = static_cast<const char *>(m);
        if (std::memcmp(base, "OPWPACK1", 8) != 0)
            throw std::runtime_error(path + ": not an OpWorks pack (bad magic)");
        uint64_t json_len = 0;
        std::memcpy(&json_len, base + 8, 8);
        if (json_len > (1ull << 30) || 16 + json_len > size_)
            throw std::runtime_error(path + ": corrupt manifest length");
        blob_offset_ = 16 + json_len;
        blob_size_ = size_ - blob_offset_;
        manifest_ = json::parse(std::string(base + 16, json_len));
        if (manifest_.at("format_version").as_int() != 1)
            throw std::runtime_error(path + ": unsupported format version");
        dtype_ = manifest_.at("dtype").as_string();
        if (dtype_ == "float32")
            elem_size_ = 4;
        else if (dtype_ == "bfloat16")
            elem_size_ = 2;
        else
            throw std::runtime_error(path + ": unsupported dtype " + dtype_);
        for (const auto &[name, meta] : manifest_.at("tensors").as_object()) {
            TensorMeta t;
            const int64_t offset = meta.at("offset").as_int();
            if (offset < 0)
                throw std::runtime_error(path + ": negative offset of " + name);
            t.offset = static_cast<uint64_t>(offset);
            t.numel = 1;
            for (const auto &d : meta.at("shape").as_array()) {
                const int64_t dim = d.as_int();
                if (dim <= 0)
                    throw std::runtime_error(path + ": non-positive dim in " + name);
                t.numel *= dim;
                if (t.numel > (1ll << 40))
                    throw std::runtime_error(path + ": absurd tensor size in " + name);
                t.shape.push_back(dim);
            }
            const uint64_t bytes = static_cast<uint64_t>(t.numel) * elem_size_;
            if (t.offset > blob_size_ || bytes > blob_size_ - t.offset) // no wrap-around
                throw std::runtime_error(path + ": tensor " + name + " overruns the data blob");
            tensors_.emplace(name, std::move(t));
        }
        if (const json::Value *aliases = manifest_.find("aliases")) {
            for (const auto &[alias, target] : aliases->as_object()) {
                const std::string &tname = target.as_string();
                if (tensors_.find(tname) == tensors_.end())
                    throw std::runtime_error(path + ": alias " + alias + " targets missing tensor " + tname);
                aliases_.emplace(alias, tname);
            }
        }
    }

    bool has(const std::string &name) const { return tensors_.count(name) != 0 || aliases_.count(name) != 0; }

    const TensorMeta &meta(const std::string &name) const {
        auto it = tensors_.find(resolve(name));
        if (it == tensors_.end())
            throw std::runtime_error(path_ + ": missing tensor " + name);
        return it->second;
    }

    const std::string &dtype() const { return dtype_; }
    size_t elem_size() const { return elem_size_; }

    // Pointer to a tensor's bytes inside the mapped file.
    const void *data(const std::string &name) const {
        return static_cast<const char *>(map_.get()) + blob_offset_ + meta(name).offset;
    }

    std::vector<uint8_t> read_raw(const std::string &name) const {
        const TensorMeta &m = meta(name);
        std::vector<uint8_t> out(static_cast<size_t>(m.numel) * elem_size_);
        std::memcpy(out.data(), data(name), out.size());
        return out;
    }

    std::vector<float> read(const std::string &name) const {
        if (dtype_ != "float32")
            throw std::runtime_error(path_ + ": read() requires a float32 pack; use read_raw for " + dtype_);
        const TensorMeta &m = meta(name);
        std::vector<float> out(static_cast<size_t>(m.numel));
        std::memcpy(out.data(), data(name), out.size() * 4);
        return out;
    }

    std::vector<float> read_bf16_as_float(const std::string &name) const {
        if (dtype_ != "bfloat16")
            throw std::runtime_error(path_ + ": read_bf16_as_float requires a bfloat16 pack");
        const TensorMeta &m = meta(name);
        const uint16_t *src = static_cast<const uint16_t *>(data(name));
        std::vector<float> out(static_cast<size_t>(m.numel));
        for (size_t i = 0; i < out.size(); ++i) {
            const uint32_t bits = static_cast<uint32_t>(src[i]) << 16;
            std::memcpy(&out[i], &bits, 4);
        }
        return out;
    }

    // int32 payload stored in a float32 pack (fixture ids).
    std::vector<int32_t> read_int32(const std::string &name) const {
        const TensorMeta &m = meta(name);
        std::vector<int32_t> out(static_cast<size_t>(m.numel));
        std::memcpy(out.data(), data(name), out.size() * 4);
        return out;
    }

    const json::Value &manifest() const { return manifest_; }
    const std::string &path() const { return path_; }

  private:
    const std::string &resolve(const std::string &name) const {
        auto it = aliases_.find(name);
        return it == aliases_.end() ? name : it->second;
    }

    std::string path_;
    std::shared_ptr<void> map_;
    uint64_t size_ = 0;
    std::string dtype_;
    size_t elem_size_ = 4;
    json::Value manifest_;
    std::map<std::string, TensorMeta> tensors_;
    std::map<std::string, std::string> aliases_;
    uint64_t blob_offset_ = 0;
    uint64_t blob_size_ = 0;
};

} // namespace opworks
