// tp_comm.cu — the multi-GPU control path reachable from C: NCCL
// communicators for the row-split decode stack and the expert-parallel MoE.
//
// Communicators are created non-blocking (ncclCommInitRankConfig with
// config.blocking = 0), and every wait on one (its initialisation, a
// collective's completion on the stream) is polled against a wall-clock
// limit through ncclCommGetAsyncError and cudaStreamQuery; when the limit
// runs out the communicator is aborted (ncclCommAbort) and the call returns
// BH_ETIMEDOUT, so a rank that never joins, or stops, makes the others fail
// in bounded time instead of hanging. A communicator is passed as void* (an
// ncclComm_t); one created by the caller works too, with the same timeouts if
// it was created non-blocking.
//
// NCCL is opened at run time (dlopen of $BH_NCCL_LIB, else libnccl.so.2; in a
// process that already loaded NCCL, for instance through PyTorch, that same
// library), so the library has no link-time dependency on it; the entry
// points return BH_ENODEV when it cannot be found. nccl.h supplies the types
// only.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>

#include "bh_ctx.cuh"
#include "bh_kernels.cuh"

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*finalize)(ncclComm_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    bool ok = false;
};

template <class F>
bool sym(void* lib, const char* name, F& fn) {
    fn = reinterpret_cast<F>(dlsym(lib, name));
    return fn != nullptr;
}

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* path = std::getenv("BH_NCCL_LIB");
        void* lib = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) return;
        api.ok = sym(lib, "ncclGetUniqueId", api.get_unique_id) &&
                 sym(lib, "ncclCommInitRankConfig", api.init_rank_config) &&
                 sym(lib, "ncclCommGetAsyncError", api.get_async_error) && sym(lib, "ncclCommAbort", api.abort) &&
                 sym(lib, "ncclCommFinalize", api.finalize) && sym(lib, "ncclCommDestroy", api.destroy) &&
                 sym(lib, "ncclCommCount", api.count) && sym(lib, "ncclCommUserRank", api.user_rank) &&
                 sym(lib, "ncclAllGather", api.all_gather) && sym(lib, "ncclAllReduce", api.all_reduce);
    });
    return api;
}

using Clock = std::chrono::steady_clock;

Clock::time_point deadline_of(int timeout_ms) {
    return Clock::now() + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 1);
}

// Until the communicator's asynchronous state leaves ncclInProgress: BH_OK on
// ncclSuccess; on an error or at the deadline the communicator is aborted.
int wait_comm(const NcclApi& api, ncclComm_t comm, Clock::time_point deadline) {
    for (;;) {
        ncclResult_t st = ncclInProgress;
        if (api.get_async_error(comm, &st) != ncclSuccess) st = ncclInternalError;
        if (st == ncclSuccess) return BH_OK;
        if (st != ncclInProgress) {
            api.abort(comm);
            return BH_EIO;
        }
        if (Clock::now() > deadline) {
            api.abort(comm);
            return BH_ETIMEDOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

// Until the work enqueued on stream (a collective) has completed, watching the
// communicator for errors; aborted at the deadline.
int wait_stream(const NcclApi& api, ncclComm_t comm, cudaStream_t s, Clock::time_point deadline) {
    for (;;) {
        const cudaError_t q = cudaStreamQuery(s);
        if (q == cudaSuccess) return BH_OK;
        if (q != cudaErrorNotReady) {
            cudaGetLastError();
            api.abort(comm);
            return BH_EIO;
        }
        ncclResult_t st = ncclSuccess;
        if (api.get_async_error(comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
            api.abort(comm);
            return BH_EIO;
        }
        if (Clock::now() > deadline) {
            api.abort(comm);
            return BH_ETIMEDOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// A collective call on a non-blocking communicator may return ncclInProgress
// while it is being enqueued; wait for the communicator, then for the stream.
int finish_collective(const NcclApi& api, ncclComm_t comm, ncclResult_t r, cudaStream_t s, int timeout_ms) {
    const Clock::time_point dl = deadline_of(timeout_ms);
    if (r != ncclSuccess && r != ncclInProgress) return BH_EIO;
    int rc = wait_comm(api, comm, dl);
    if (rc != BH_OK) return rc;
    return wait_stream(api, comm, s, dl);
}

}  // namespace

extern "C" {

int bh_tp_unique_id(void* id_out) {
    if (!id_out) return BH_EINVAL;
    const NcclApi& api = nccl();
    if (!api.ok) return BH_ENODEV;
    ncclUniqueId id;
    if (api.get_unique_id(&id) != ncclSuccess) return BH_EIO;
    static_assert(sizeof(id) == 128, "ncclUniqueId size");
    std::memcpy(id_out, &id, sizeof(id));
    return BH_OK;
}

int bh_tp_comm_init(int device, const void* unique_id, int world, int rank, int timeout_ms, void** comm_out) {
    if (!unique_id || !comm_out || world < 1 || rank < 0 || rank >= world || timeout_ms < 1) return BH_EINVAL;
    *comm_out = nullptr;
    const NcclApi& api = nccl();
    if (!api.ok) return BH_ENODEV;
    if (device >= 0 && cudaSetDevice(device) != cudaSuccess) return BH_ENODEV;
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // calls return at once; completion is polled below
    ncclComm_t comm = nullptr;
    const ncclResult_t r = api.init_rank_config(&comm, world, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (comm) api.abort(comm);
        return BH_EIO;
    }
    const int rc = wait_comm(api, comm, deadline_of(timeout_ms));
    if (rc != BH_OK) return rc;  // (aborted)
    *comm_out = comm;
    return BH_OK;
}

int bh_tp_comm_abort(void* comm) {
    if (!comm) return BH_EINVAL;
    const NcclApi& api = nccl();
    if (!api.ok) return BH_ENODEV;
    return api.abort(static_cast<ncclComm_t>(comm)) == ncclSuccess ? BH_OK : BH_EIO;
}

int bh_tp_comm_free(void* comm, int timeout_ms) {
    if (!comm || timeout_ms < 1) return BH_EINVAL;
    const NcclApi& api = nccl();
    if (!api.ok) return BH_ENODEV;
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    const ncclResult_t r = api.finalize(c);
    if (r != ncclSuccess && r != ncclInProgress) {
        api.abort(c);
        return BH_EIO;
    }
    const int rc = wait_comm(api, c, deadline_of(timeout_ms));
    if (rc != BH_OK) return rc;  // (aborted)
    return api.destroy(c) == ncclSuccess ? BH_OK : BH_EIO;
}

int bh_tp_comm_info(void* comm, int* rank, int* world) {
    if (!comm) return BH_EINVAL;
    const NcclApi& api = nccl();
    if (!api.ok) return BH_ENODEV;
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    if (rank && api.user_rank(c, rank) != ncclSuccess) return BH_EIO;
    if (world && api.count(c, world) != ncclSuccess) return BH_EIO;
    return BH_OK;
}

int bh_tp_allgather(void* comm, const void* send, void* recv, size_t bytes_per_rank, void* stream, int timeout_ms) {
    if (!comm || !send || !recv || bytes_per_rank == 0 || timeout_ms < 1) return BH_EINVAL;
    const NcclApi& api = nccl();
    if (!api.ok) return BH_ENODEV;
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return finish_collective(api, c, api.all_gather(send, recv, bytes_per_rank, ncclUint8, c, s), s, timeout_ms);
}

int bh_tp_allreduce_sum_f32(void* comm, float* buf, size_t count, void* stream, int timeout_ms) {
    if (!comm || !buf || count == 0 || timeout_ms < 1) return BH_EINVAL;
    const NcclApi& api = nccl();
    if (!api.ok) return BH_ENODEV;
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return finish_collective(api, c, api.all_reduce(buf, buf, count, ncclFloat32, ncclSum, c, s), s, timeout_ms);
}

int bh_stack_tp_connect_comm(bh_stack* st, void* comm, int timeout_ms) {
    if (!st || !comm || timeout_ms < 1) return BH_EINVAL;
    int rank = 0, world = 0, nrank = -1, nworld = -1;
    int rc = bh_stack_tp_info(st, &rank, &world, nullptr);
    if (rc != BH_OK) return rc;
    if ((rc = bh_tp_comm_info(comm, &nrank, &nworld)) != BH_OK) return rc;
    if (nrank != rank || nworld != world) return BH_EINVAL;
    // every rank's 64-byte IPC handle, all-gathered over the communicator
    unsigned char own[64];
    if ((rc = bh_stack_tp_handle(st, own)) != BH_OK) return rc;
    void* dbuf = nullptr;
    cudaStream_t s = nullptr;
    if (cudaMalloc(&dbuf, 64 * (size_t)(world + 1)) != cudaSuccess) {
        cudaGetLastError();
        return BH_ENOMEM;
    }
    unsigned char* send = static_cast<unsigned char*>(dbuf) + 64 * (size_t)world;
    unsigned char* recv = static_cast<unsigned char*>(dbuf);
    std::unique_ptr<unsigned char[]> all(new unsigned char[64 * (size_t)world]);
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMemcpy(send, own, 64, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = BH_EIO;
    if (rc == BH_OK) rc = bh_tp_allgather(comm, send, recv, 64, s, timeout_ms);
    if (rc == BH_OK && cudaMemcpy(all.get(), recv, 64 * (size_t)world, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = BH_EIO;
    if (s) cudaStreamDestroy(s);
    cudaFree(dbuf);
    if (rc != BH_OK) return rc;
    return bh_stack_tp_connect(st, all.get());
}

}  // extern "C"
