// comm.cpp -- acb_comm: NCCL over NVLink / NVSwitch for the sharded jobs, loaded with dlopen
// (libnccl.so.2: the copy a host process already loaded, e.g. PyTorch's, else the system's).
//
// The reference has no collectives (one GPU per process; ace-server pins workers with
// CUDA_VISIBLE_DEVICES, tools/ace-server.cpp:2095-2120). This library adds the two transfers its
// sharded DiT job needs: an all-gather of the finished latents and, when one GPU holds one CFG half,
// the per-step exchange of the velocity with the GPU holding the other half.
//
// Failure handling: the communicator is created non-blocking (ncclConfig_t.blocking = 0), every
// NCCL call that reports ncclInProgress is polled with ncclCommGetAsyncError, and every wait for a
// stream that holds NCCL work polls cudaStreamQuery; a deadline (the caller's timeout) ends each
// wait. On a timeout or an asynchronous NCCL error the communicator is aborted (ncclCommAbort, which
// also stops its kernels) and the call returns ACB_ERR_TIMEOUT / ACB_ERR_CUDA with the reason in
// acb_last_error.
#include "comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>

#include "host_common.h"

using namespace acb;

namespace {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *)                                                   = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *)      = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *)                                 = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t)                                                         = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t)                                                       = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t)      = nullptr;
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t)            = nullptr;
    ncclResult_t (*GroupStart)()                                                                  = nullptr;
    ncclResult_t (*GroupEnd)()                                                                    = nullptr;
    const char * (*GetErrorString)(ncclResult_t)                                                  = nullptr;
    std::string error;
};

NcclApi &  nccl() {
    static NcclApi    api;
    static std::once_flag once;
    std::call_once(once, [] {
        void * h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        }
        if (!h) {
            api.error = std::string("libnccl.so.2 not found: ") + dlerror();
            return;
        }
        auto sym = [&](const char * n) { return dlsym(h, n); };
        api.GetUniqueId        = (decltype(api.GetUniqueId)) sym("ncclGetUniqueId");
        api.CommInitRankConfig = (decltype(api.CommInitRankConfig)) sym("ncclCommInitRankConfig");
        api.CommGetAsyncError  = (decltype(api.CommGetAsyncError)) sym("ncclCommGetAsyncError");
        api.CommAbort          = (decltype(api.CommAbort)) sym("ncclCommAbort");
        api.CommDestroy        = (decltype(api.CommDestroy)) sym("ncclCommDestroy");
        api.AllGather          = (decltype(api.AllGather)) sym("ncclAllGather");
        api.Send               = (decltype(api.Send)) sym("ncclSend");
        api.Recv               = (decltype(api.Recv)) sym("ncclRecv");
        api.GroupStart         = (decltype(api.GroupStart)) sym("ncclGroupStart");
        api.GroupEnd           = (decltype(api.GroupEnd)) sym("ncclGroupEnd");
        api.GetErrorString     = (decltype(api.GetErrorString)) sym("ncclGetErrorString");
        api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommGetAsyncError && api.CommAbort &&
                 api.CommDestroy && api.AllGather && api.Send && api.Recv && api.GroupStart && api.GroupEnd &&
                 api.GetErrorString;
        if (!api.ok) {
            api.error = "libnccl.so.2 lacks a required symbol";
        }
    });
    return api;
}

using Clock = std::chrono::steady_clock;

}  // namespace

struct acb_comm {
    ncclComm_t comm    = nullptr;
    int        rank    = 0;
    int        world   = 1;
    int        device  = 0;
    int        timeout = 60000;  // ms
    bool       broken  = false;

    // abort the communicator (its kernels stop; the other ranks' waits then end by their deadline)
    acb_status fail(acb_status s, const std::string & why) {
        set_last_error("acb_comm (rank " + std::to_string(rank) + "): " + why);
        if (comm && !broken) {
            nccl().CommAbort(comm);
            comm = nullptr;
        }
        broken = true;
        return s;
    }

    // poll the communicator until its pending operation is done (non-blocking mode)
    acb_status settle(ncclResult_t r, const char * what) {
        NcclApi &  n  = nccl();
        const auto t0 = Clock::now();
        while (r == ncclInProgress) {
            if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > timeout) {
                return fail(ACB_ERR_TIMEOUT, std::string(what) + ": no progress within the timeout");
            }
            std::this_thread::yield();
            n.CommGetAsyncError(comm, &r);
        }
        if (r != ncclSuccess) {
            return fail(ACB_ERR_CUDA, std::string(what) + ": " + n.GetErrorString(r));
        }
        return ACB_OK;
    }
};

namespace acb {

int comm_rank(const acb_comm * c) {
    return c ? c->rank : 0;
}

int comm_world(const acb_comm * c) {
    return c ? c->world : 1;
}

acb_status comm_all_gather(acb_comm * c, const void * in, void * out, size_t bytes, cudaStream_t stream) {
    if (!c || c->broken) {
        return ACB_ERR_INVALID_ARG;
    }
    return c->settle(nccl().AllGather(in, out, bytes, ncclUint8, c->comm, stream), "all-gather");
}

acb_status comm_exchange(acb_comm * c, int peer, const void * send, void * recv, size_t bytes, cudaStream_t stream) {
    if (!c || c->broken || peer < 0 || peer >= c->world) {
        return ACB_ERR_INVALID_ARG;
    }
    NcclApi & n = nccl();
    ACB_TRY(c->settle(n.GroupStart(), "group start"));
    n.Send(send, bytes, ncclUint8, peer, c->comm, stream);
    n.Recv(recv, bytes, ncclUint8, peer, c->comm, stream);
    return c->settle(n.GroupEnd(), "send/recv");
}

acb_status comm_wait(acb_comm * c, cudaStream_t stream) {
    if (!c || c->broken) {
        return ACB_ERR_INVALID_ARG;
    }
    NcclApi &  n  = nccl();
    const auto t0 = Clock::now();
    for (;;) {
        const cudaError_t e = cudaStreamQuery(stream);
        if (e == cudaSuccess) {
            return ACB_OK;
        }
        if (e != cudaErrorNotReady) {
            return c->fail(ACB_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(e));
        }
        ncclResult_t r = ncclSuccess;
        n.CommGetAsyncError(c->comm, &r);
        if (r != ncclSuccess && r != ncclInProgress) {
            return c->fail(ACB_ERR_CUDA, std::string("asynchronous NCCL error: ") + n.GetErrorString(r));
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > c->timeout) {
            return c->fail(ACB_ERR_TIMEOUT, "a peer did not take part within the timeout");
        }
        std::this_thread::yield();
    }
}

}  // namespace acb

extern "C" acb_status acb_comm_unique_id(void * id) {
    if (!id) {
        return ACB_ERR_INVALID_ARG;
    }
    NcclApi & n = nccl();
    if (!n.ok) {
        set_last_error(n.error);
        return ACB_ERR_UNSUPPORTED;
    }
    ncclUniqueId u;
    const ncclResult_t r = n.GetUniqueId(&u);
    if (r != ncclSuccess) {
        set_last_error(std::string("ncclGetUniqueId: ") + n.GetErrorString(r));
        return ACB_ERR_CUDA;
    }
    memcpy(id, &u, sizeof(u));
    return ACB_OK;
}

extern "C" acb_status acb_comm_init(const void * id, int world, int rank, int device, int timeout_ms, acb_comm ** out) {
    if (!id || !out || world <= 0 || rank < 0 || rank >= world || timeout_ms <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    *out        = nullptr;
    NcclApi & n = nccl();
    if (!n.ok) {
        set_last_error(n.error);
        return ACB_ERR_UNSUPPORTED;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        set_last_error("acb_comm_init: cannot select the device");
        return ACB_ERR_CUDA;
    }
    auto c     = new acb_comm();
    c->rank    = rank;
    c->world   = world;
    c->device  = device;
    c->timeout = timeout_ms;
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking     = 0;
    ncclResult_t r   = n.CommInitRankConfig(&c->comm, world, u, rank, &cfg);
    if (r == ncclSuccess || r == ncclInProgress) {
        if (r == ncclInProgress) {
            n.CommGetAsyncError(c->comm, &r);
        }
        const acb_status s = c->settle(r, "communicator init");
        if (s != ACB_OK) {
            delete c;
            return s;
        }
    } else {
        set_last_error(std::string("ncclCommInitRankConfig: ") + n.GetErrorString(r));
        delete c;
        return ACB_ERR_CUDA;
    }
    *out = c;
    return ACB_OK;
}

extern "C" int acb_comm_rank(const acb_comm * c) {
    return comm_rank(c);
}

extern "C" int acb_comm_world(const acb_comm * c) {
    return comm_world(c);
}

extern "C" void acb_comm_free(acb_comm * c) {
    if (!c) {
        return;
    }
    if (c->comm) {
        cudaSetDevice(c->device);
        if (c->broken) {
            nccl().CommAbort(c->comm);
        } else {
            nccl().CommDestroy(c->comm);
        }
    }
    delete c;
}
