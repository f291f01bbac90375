#pragma once

// NCCL for the tensor-parallel Llama engine, bound at run time: the library
// (libnccl.so.2, the one already loaded in the process if any, e.g. by
// PyTorch) is opened only when a tensor-parallel engine is created, so the
// runtime has no link-time dependency on NCCL and request-partitioned or
// single-GPU use never touches it. Types come from the NCCL header.

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace opworks {

class NcclLite {
  public:
    static NcclLite &get() {
        static NcclLite n;
        return n;
    }
    // 128-byte communicator id created by one rank and shared with the others
    void unique_id(char *out) {
        ncclUniqueId id;
        check(get_id_(&id), "ncclGetUniqueId");
        std::memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
    }
    ncclComm_t init(const char *id_bytes, int world, int rank) {
        ncclUniqueId id;
        std::memcpy(id.internal, id_bytes, NCCL_UNIQUE_ID_BYTES);
        ncclComm_t comm = nullptr;
        check(init_rank_(&comm, world, id, rank), "ncclCommInitRank");
        return comm;
    }
    void allreduce_sum(float *buf, size_t count, ncclComm_t comm, cudaStream_t stream) {
        check(all_reduce_(buf, buf, count, ncclFloat, ncclSum, comm, stream), "ncclAllReduce");
    }
    void destroy(ncclComm_t comm) {
        if (comm)
            destroy_(comm);
    }

  private:
    NcclLite() {
        // prefer a copy that is already loaded, then the system library
        handle_ = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
        if (!handle_)
            handle_ = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!handle_)
            throw std::runtime_error("tensor parallelism needs NCCL: libnccl.so.2 could not be loaded");
        get_id_ = reinterpret_cast<decltype(get_id_)>(sym("ncclGetUniqueId"));
        init_rank_ = reinterpret_cast<decltype(init_rank_)>(sym("ncclCommInitRank"));
        all_reduce_ = reinterpret_cast<decltype(all_reduce_)>(sym("ncclAllReduce"));
        destroy_ = reinterpret_cast<decltype(destroy_)>(sym("ncclCommDestroy"));
        err_str_ = reinterpret_cast<decltype(err_str_)>(sym("ncclGetErrorString"));
    }
    void *sym(const char *name) {
        void *p = dlsym(handle_, name);
        if (!p)
            throw std::runtime_error(std::string("NCCL symbol missing: ") + name);
        return p;
    }
    void check(ncclResult_t r, const char *what) {
        if (r != ncclSuccess)
            throw std::runtime_error(std::string(what) + " failed: " + err_str_(r));
    }
    void *handle_ = nullptr;
    ncclResult_t (*get_id_)(ncclUniqueId *) = nullptr;
    ncclResult_t (*init_rank_)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce_)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                cudaStream_t) = nullptr;
    ncclResult_t (*destroy_)(ncclComm_t) = nullptr;
    const char *(*err_str_)(ncclResult_t) = nullptr;
};

} // namespace opworks
