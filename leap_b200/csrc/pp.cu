// pp.cu — stage-to-stage transport for layer-range pipelines inside one box.
//
// The reference hands the activation x[dim] from one device of its ring to
// the next over TCP, UDP or its kernel-module transport
// (src/inference/FloatTransformer.cpp:772-793 master side, :800-946
// worker_loop; src/inference/Transformer.h:17-23).  Between the GPUs of one
// B200 box the same hop is a point-to-point NCCL send over NVLink, ordered
// on the caller's stream so a stage never waits on its host.
//
// NCCL is loaded at run time (dlopen): a process that already holds an NCCL
// library (torch's) shares it, so the two never disagree on versions; no
// link-time dependency is added.  The communicator is non-blocking, so
// creation and every enqueue are bounded by the caller's timeout, and
// leap_pp_abort ends transfers whose peer has gone.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>

#include "ctx.h"

namespace {

struct NcclApi {
    bool ok = false;
    char why[256] = {};
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

template <class F>
bool resolve(void *h, const char *name, F &fn) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = nullptr;
        for (const char *name : {"libnccl.so.2", "libnccl.so"}) {
            h = dlopen(name, RTLD_NOW | RTLD_NOLOAD);  // already in the process
            if (!h) h = dlopen(name, RTLD_NOW | RTLD_LOCAL);
            if (h) break;
        }
        if (!h) {
            snprintf(api.why, sizeof(api.why), "cannot load libnccl.so.2: %s", dlerror());
            return;
        }
        bool ok = resolve(h, "ncclGetUniqueId", api.GetUniqueId) &&
                  resolve(h, "ncclCommInitRankConfig", api.CommInitRankConfig) &&
                  resolve(h, "ncclCommGetAsyncError", api.CommGetAsyncError) &&
                  resolve(h, "ncclSend", api.Send) && resolve(h, "ncclRecv", api.Recv) &&
                  resolve(h, "ncclCommFinalize", api.CommFinalize) &&
                  resolve(h, "ncclCommDestroy", api.CommDestroy) &&
                  resolve(h, "ncclCommAbort", api.CommAbort) &&
                  resolve(h, "ncclGetErrorString", api.GetErrorString);
        if (!ok) {
            snprintf(api.why, sizeof(api.why), "libnccl lacks a needed symbol");
            return;
        }
        api.ok = true;
    });
    return api;
}

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(d);
    }
    ~DevGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

struct leap_pp {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1, device = 0;
    int timeout_ms = 60000;
    bool broken = false;  // aborted, or a transfer failed
};

namespace {

using clk = std::chrono::steady_clock;

// Poll the non-blocking communicator until its pending operation is done.
int settle(leap_pp *pp, ncclResult_t first, const char *what) {
    const NcclApi &api = nccl();
    if (first != ncclSuccess && first != ncclInProgress) {
        pp->broken = true;
        leap::set_error("%s: %s", what, api.GetErrorString(first));
        return LEAP_ERR_COMM;
    }
    // An enqueue on a non-blocking communicator usually settles within
    // microseconds: poll without sleeping at first (a sleep here delays the
    // stage's next launches and shows up as hop latency), then yield, then
    // back off to short sleeps; all bounded by the deadline.
    const auto start = clk::now();
    const auto deadline = start + std::chrono::milliseconds(pp->timeout_ms);
    for (unsigned polls = 0;; ++polls) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t q = api.CommGetAsyncError(pp->comm, &st);
        if (q != ncclSuccess) st = q;
        if (st == ncclSuccess) return LEAP_OK;
        if (st != ncclInProgress) {
            pp->broken = true;
            leap::set_error("%s: %s", what, api.GetErrorString(st));
            return LEAP_ERR_COMM;
        }
        if (clk::now() > deadline) {
            pp->broken = true;
            api.CommAbort(pp->comm);
            pp->comm = nullptr;
            leap::set_error("%s: no progress within %d ms (communicator aborted)", what,
                            pp->timeout_ms);
            return LEAP_ERR_COMM;
        }
        if (polls < 4096) continue;
        if (clk::now() - start < std::chrono::milliseconds(2))
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int check_pp(leap_pp *pp, const void *buf, size_t bytes) {
    if (!pp || !buf || bytes == 0) {
        leap::set_error("pp: null argument or empty transfer");
        return LEAP_ERR_INVALID;
    }
    if (pp->broken || !pp->comm) {
        leap::set_error("pp: the communicator was aborted or failed");
        return LEAP_ERR_COMM;
    }
    return LEAP_OK;
}

int transfer(leap_pp *pp, bool send, int peer, void *buf, size_t bytes, void *stream) {
    int st = check_pp(pp, buf, bytes);
    if (st != LEAP_OK) return st;
    if (peer < 0 || peer >= pp->world || peer == pp->rank) {
        leap::set_error("pp: peer %d invalid for rank %d of %d", peer, pp->rank, pp->world);
        return LEAP_ERR_INVALID;
    }
    DevGuard g(pp->device);
    const NcclApi &api = nccl();
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const ncclResult_t r = send ? api.Send(buf, bytes, ncclInt8, peer, pp->comm, s)
                                : api.Recv(buf, bytes, ncclInt8, peer, pp->comm, s);
    return settle(pp, r, send ? "pp send" : "pp recv");
}

}  // namespace

extern "C" {

int leap_pp_unique_id(void *id_out) {
    leap::clear_error();
    if (!id_out) {
        leap::set_error("pp: null argument");
        return LEAP_ERR_INVALID;
    }
    const NcclApi &api = nccl();
    if (!api.ok) {
        leap::set_error("pp: %s", api.why);
        return LEAP_ERR_COMM;
    }
    ncclUniqueId id;
    const ncclResult_t r = api.GetUniqueId(&id);
    if (r != ncclSuccess) {
        leap::set_error("pp: ncclGetUniqueId: %s", api.GetErrorString(r));
        return LEAP_ERR_COMM;
    }
    memcpy(id_out, &id, sizeof(id));
    return LEAP_OK;
}

int leap_pp_init(const void *id, int rank, int world, int device, int timeout_ms, leap_pp **out) {
    leap::clear_error();
    if (!id || !out || world < 1 || rank < 0 || rank >= world || device < 0) {
        leap::set_error("pp: bad arguments (rank %d of %d, device %d)", rank, world, device);
        return LEAP_ERR_INVALID;
    }
    *out = nullptr;
    const NcclApi &api = nccl();
    if (!api.ok) {
        leap::set_error("pp: %s", api.why);
        return LEAP_ERR_COMM;
    }
    leap_pp *pp = new (std::nothrow) leap_pp();
    if (!pp) {
        leap::set_error("pp: host allocation failed");
        return LEAP_ERR_NOMEM;
    }
    pp->rank = rank;
    pp->world = world;
    pp->device = device;
    pp->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
    DevGuard g(device);
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // bounded by settle(); abortable
    const ncclResult_t r = api.CommInitRankConfig(&pp->comm, world, uid, rank, &cfg);
    const int st = settle(pp, r, "pp init");
    if (st != LEAP_OK) {
        if (pp->comm) api.CommAbort(pp->comm);
        delete pp;
        return st;
    }
    *out = pp;
    return LEAP_OK;
}

int leap_pp_send(leap_pp *pp, int peer, const void *buf, size_t bytes, void *stream) {
    leap::clear_error();
    return transfer(pp, true, peer, const_cast<void *>(buf), bytes, stream);
}

int leap_pp_recv(leap_pp *pp, int peer, void *buf, size_t bytes, void *stream) {
    leap::clear_error();
    return transfer(pp, false, peer, buf, bytes, stream);
}

int leap_pp_send_next(leap_pp *pp, const void *buf, size_t bytes, void *stream) {
    leap::clear_error();
    if (!pp) {
        leap::set_error("pp: null communicator");
        return LEAP_ERR_INVALID;
    }
    return transfer(pp, true, pp->rank + 1, const_cast<void *>(buf), bytes, stream);
}

int leap_pp_recv_prev(leap_pp *pp, void *buf, size_t bytes, void *stream) {
    leap::clear_error();
    if (!pp) {
        leap::set_error("pp: null communicator");
        return LEAP_ERR_INVALID;
    }
    return transfer(pp, false, pp->rank - 1, buf, bytes, stream);
}

int leap_pp_abort(leap_pp *pp) {
    leap::clear_error();
    if (!pp) {
        leap::set_error("pp: null communicator");
        return LEAP_ERR_INVALID;
    }
    if (pp->comm) {
        DevGuard g(pp->device);
        nccl().CommAbort(pp->comm);
        pp->comm = nullptr;
    }
    pp->broken = true;
    return LEAP_OK;
}

int leap_pp_destroy(leap_pp *pp) {
    leap::clear_error();
    if (!pp) return LEAP_OK;
    int st = LEAP_OK;
    if (pp->comm) {
        DevGuard g(pp->device);
        const NcclApi &api = nccl();
        // flush what was issued, then free; a failed flush aborts instead
        st = settle(pp, api.CommFinalize(pp->comm), "pp finalize");
        if (st == LEAP_OK)
            api.CommDestroy(pp->comm);
        else if (pp->comm)
            api.CommAbort(pp->comm);
        pp->comm = nullptr;
    }
    delete pp;
    return st;
}

}  // extern "C"
