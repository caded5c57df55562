// Collectives and communicators behind the C ABI.
//
// The reference runtime is single-device per process (gpu-compute/src/
// cuda.rs:80-86), so a caller that shards rows, images or heads across GPUs
// needs the one real exchange of this path - the global sum's all-reduce -
// from the backend itself.  NCCL is resolved at run time instead of linked:
// a process that already loaded NCCL (a framework's own communicator) shares
// that copy, and a process without NCCL pays nothing until it asks for a
// collective.  As the reference does for its run-time libraries
// (compute-cuda/src/libraries.rs:100-117), every symbol this file uses is
// checked before the first call, and a missing one is reported by name.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "host.h"
#include "kernels.h"

namespace fb {
namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclCommInitAll) init_all = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommCuDevice) cu_device = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

std::mutex g_nccl_mutex;
NcclApi g_nccl;
bool g_nccl_ready = false;

// Opens the NCCL library: $FB_NCCL_LIBRARY when set, else the copy this
// process already loaded, else the default search for libnccl.so.2.
void* open_nccl(std::string* where) {
    if (const char* path = std::getenv("FB_NCCL_LIBRARY"); path && *path) {
        *where = path;
        return dlopen(path, RTLD_NOW | RTLD_LOCAL);
    }
    *where = "libnccl.so.2";
    if (void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD)) return h;
    return dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
}

// The resolved API, or a status with the reason.  Success is cached; a
// failure is not, so a later call may find a library loaded in between.
int nccl_api(const NcclApi** out) {
    std::lock_guard<std::mutex> lock(g_nccl_mutex);
    if (g_nccl_ready) {
        *out = &g_nccl;
        return FB_OK;
    }
    std::string where;
    void* h = open_nccl(&where);
    if (!h) {
        const char* why = dlerror();
        return fail(FB_ERR_DRIVER, "NCCL is unavailable: cannot open " + where + (why ? std::string(": ") + why : ""));
    }
    NcclApi api;
    struct Entry {
        const char* name;
        void** slot;
    };
    const Entry entries[] = {
        {"ncclGetUniqueId", reinterpret_cast<void**>(&api.get_unique_id)},
        {"ncclCommInitRank", reinterpret_cast<void**>(&api.init_rank)},
        {"ncclCommInitAll", reinterpret_cast<void**>(&api.init_all)},
        {"ncclCommDestroy", reinterpret_cast<void**>(&api.destroy)},
        {"ncclCommCuDevice", reinterpret_cast<void**>(&api.cu_device)},
        {"ncclAllReduce", reinterpret_cast<void**>(&api.all_reduce)},
        {"ncclGetErrorString", reinterpret_cast<void**>(&api.error_string)},
    };
    for (const Entry& e : entries) {
        *e.slot = dlsym(h, e.name);
        if (!*e.slot) {
            dlclose(h);
            return fail(FB_ERR_MISSING_SYMBOL, std::string("incompatible NCCL library (") + where +
                                                   "): missing symbol " + e.name);
        }
    }
    g_nccl = api;
    g_nccl_ready = true;  // the handle stays open for the process's lifetime
    *out = &g_nccl;
    return FB_OK;
}

int nccl_status(const NcclApi* api, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return FB_OK;
    return fail(FB_ERR_DRIVER, std::string(what) + ": " + api->error_string(r));
}

}  // namespace

int nccl_all_reduce_sum_f64(double* buf, uint64_t count, void* comm, void* stream) {
    const NcclApi* api = nullptr;
    if (int rc = nccl_api(&api); rc != FB_OK) return rc;
    int comm_dev = -1, dev = -1;
    if (int rc = nccl_status(api, api->cu_device(static_cast<ncclComm_t>(comm), &comm_dev), "ncclCommCuDevice");
        rc != FB_OK)
        return rc;
    cudaGetDevice(&dev);
    if (comm_dev != dev)
        return fail(FB_ERR_FOREIGN_RUNTIME, "the communicator belongs to device " + std::to_string(comm_dev) +
                                                ", the call runs on device " + std::to_string(dev));
    return nccl_status(api,
                       api->all_reduce(buf, buf, count, ncclFloat64, ncclSum, static_cast<ncclComm_t>(comm),
                                       static_cast<cudaStream_t>(stream)),
                       "ncclAllReduce");
}

}  // namespace fb

using namespace fb;

extern "C" {

int fb_nccl_unique_id(void* id) {
    if (!id) return fail(FB_ERR_INVALID_INPUT, "null unique-id buffer");
    const NcclApi* api = nullptr;
    if (int rc = nccl_api(&api); rc != FB_OK) return rc;
    ncclUniqueId uid;
    if (int rc = nccl_status(api, api->get_unique_id(&uid), "ncclGetUniqueId"); rc != FB_OK) return rc;
    std::memcpy(id, &uid, sizeof(uid));
    return FB_OK;
}

int fb_nccl_comm_init_rank(void** comm, int nranks, const void* id, int rank) {
    if (!comm || !id) return fail(FB_ERR_INVALID_INPUT, "null communicator or unique-id pointer");
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return fail(FB_ERR_INVALID_INPUT, "rank " + std::to_string(rank) + " outside 0.." + std::to_string(nranks - 1));
    const NcclApi* api = nullptr;
    if (int rc = nccl_api(&api); rc != FB_OK) return rc;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    if (int rc = nccl_status(api, api->init_rank(&c, nranks, uid, rank), "ncclCommInitRank"); rc != FB_OK) return rc;
    *comm = c;
    return FB_OK;
}

int fb_nccl_comm_init_all(void** comms, int ndev, const int* devices) {
    if (!comms || ndev < 1) return fail(FB_ERR_INVALID_INPUT, "need at least one device and a communicator array");
    const NcclApi* api = nullptr;
    if (int rc = nccl_api(&api); rc != FB_OK) return rc;
    return nccl_status(api, api->init_all(reinterpret_cast<ncclComm_t*>(comms), ndev, devices), "ncclCommInitAll");
}

int fb_nccl_comm_destroy(void* comm) {
    if (!comm) return FB_OK;
    const NcclApi* api = nullptr;
    if (int rc = nccl_api(&api); rc != FB_OK) return rc;
    return nccl_status(api, api->destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

}  // extern "C"
