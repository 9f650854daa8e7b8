// q38_nccl.cu -- the NCCL side of split-sequence decode (q38_full_decode_split)
// and the communicator helpers of the C ABI.
//
// The library does not link NCCL: it resolves the few functions it calls
// from libnccl.so.2 at run time, on first use. A process that has already
// loaded NCCL (a Rust host with its own NCCL, or PyTorch) shares that copy
// (dlopen by soname returns the loaded object), so a communicator the host
// created with its own ncclCommInitRank can be passed in as is. Hosts that
// never use split-sequence decode never load NCCL, and the library still
// loads on machines without it.
//
// The exchange is one ncclAllGather of every rank's (o, m, l) partials into
// a buffer in this GPU's own memory; no kernel of this library reads another
// GPU's memory.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "q38_internal.h"

namespace q38 {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int *) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    std::string why;  // empty when every function resolved
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW);
        if (!h) {
            const char *e = dlerror();
            api.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
            return;
        }
        auto sym = [&](const char *name, auto &fn) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn && api.why.empty()) api.why = std::string("libnccl.so.2 lacks ") + name;
        };
        sym("ncclGetUniqueId", api.get_unique_id);
        sym("ncclCommInitRank", api.comm_init_rank);
        sym("ncclCommDestroy", api.comm_destroy);
        sym("ncclCommCount", api.comm_count);
        sym("ncclAllGather", api.all_gather);
        sym("ncclGetErrorString", api.error_string);
    });
    return api;
}

int api_fail(const NcclApi &api) {
    record_error(api.why.c_str());
    return Q38_ERR_CUDA;
}

int nccl_fail(const NcclApi &api, ncclResult_t r, const char *what) {
    char buf[256];
    std::snprintf(buf, sizeof buf, "%s: %s", what,
                  api.error_string ? api.error_string(r) : "NCCL error");
    record_error(buf);
    return Q38_ERR_CUDA;
}

}  // namespace

int nccl_comm_ranks(void *comm, int *nranks) {
    const NcclApi &api = nccl();
    if (!api.why.empty()) return api_fail(api);
    const ncclResult_t r = api.comm_count(static_cast<ncclComm_t>(comm), nranks);
    if (r != ncclSuccess) return nccl_fail(api, r, "ncclCommCount");
    return Q38_OK;
}

int nccl_all_gather_f32(void *comm, const float *send, float *recv, size_t count,
                        cudaStream_t stream) {
    const NcclApi &api = nccl();
    if (!api.why.empty()) return api_fail(api);
    const ncclResult_t r =
        api.all_gather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(comm), stream);
    if (r != ncclSuccess) return nccl_fail(api, r, "ncclAllGather");
    return Q38_OK;
}

}  // namespace q38

extern "C" {

int q38_nccl_unique_id(void *id) {
    if (!id) {
        q38::record_error("null id buffer");
        return Q38_ERR_ARG;
    }
    const q38::NcclApi &api = q38::nccl();
    if (!api.why.empty()) return q38::api_fail(api);
    static_assert(sizeof(ncclUniqueId) == Q38_NCCL_ID_BYTES, "NCCL unique id size");
    ncclUniqueId u;
    const ncclResult_t r = api.get_unique_id(&u);
    if (r != ncclSuccess) return q38::nccl_fail(api, r, "ncclGetUniqueId");
    std::memcpy(id, &u, sizeof u);
    return Q38_OK;
}

int q38_nccl_comm_create(const void *id, int nranks, int rank, int device, void **comm) {
    if (!id || !comm || nranks <= 0 || rank < 0 || rank >= nranks || device < 0) {
        q38::record_error("bad communicator arguments");
        return Q38_ERR_ARG;
    }
    *comm = nullptr;
    const q38::NcclApi &api = q38::nccl();
    if (!api.why.empty()) return q38::api_fail(api);
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        q38::record_error("cannot select the communicator's device");
        return Q38_ERR_CUDA;
    }
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof u);
    ncclComm_t c = nullptr;
    const ncclResult_t r = api.comm_init_rank(&c, nranks, u, rank);
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (r != ncclSuccess) return q38::nccl_fail(api, r, "ncclCommInitRank");
    *comm = c;
    return Q38_OK;
}

int q38_nccl_comm_destroy(void *comm) {
    if (!comm) return Q38_OK;
    const q38::NcclApi &api = q38::nccl();
    if (!api.why.empty()) return q38::api_fail(api);
    const ncclResult_t r = api.comm_destroy(static_cast<ncclComm_t>(comm));
    if (r != ncclSuccess) return q38::nccl_fail(api, r, "ncclCommDestroy");
    return Q38_OK;
}

}  // extern "C"
