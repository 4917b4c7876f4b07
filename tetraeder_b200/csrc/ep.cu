// Expert parallelism: the communicator of a rank and the exchange of the reference's EP mode
// (qwen3moe_shard.rs:1038-1056): every rank routes the same tokens, computes the contributions of
// the experts it holds (the others map to -1), and the partial outputs are summed across ranks
// (b.reduce -> Executor::all_reduce, crates/executor/src/exec.rs:326-351 -> Comm::all_reduce,
// crates/ggml-sys/src/comm.rs:69-87).  NCCL over NVLink does the sum.
//
// Communicators are created non-blocking, so that every host wait on NCCL has a deadline: a
// rank that never joins ends tmoe_comm_init with TMOE_E_COMM instead of a hang, and
// tmoe_comm_abort lets a host watchdog end a communicator whose peer died.
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>

#include "../../include/tmoe.h"
#include "kernels.cuh"

struct tmoe_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = 0;
    double timeout_s = 60.0;
};

namespace tmoe {

// Polls the communicator until its pending operation leaves ncclInProgress; after `timeout_s`
// it aborts the communicator (which is then unusable: c->comm = NULL).  An enqueue of a step's
// exchange normally completes within microseconds, so the first 200 us only yield the thread
// between polls; longer waits (communicator setup, a slow peer) sleep 20 us at a time.
static ncclResult_t nccl_wait(tmoe_comm *c) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = ncclCommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) return r;
        if (st != ncclInProgress) return st;
        const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (dt > c->timeout_s) {
            ncclCommAbort(c->comm);
            c->comm = nullptr;
            return ncclInternalError;
        }
        if (dt < 200e-6)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int ep_comm_device(const tmoe_comm *c) { return c->device; }

int ep_allreduce_sum(tmoe_comm *c, float *buf, size_t n, cudaStream_t st, char *msg, size_t msg_len) {
    if (!c->comm) {
        snprintf(msg, msg_len, "the communicator was aborted");
        return TMOE_E_COMM;
    }
    ncclResult_t r = ncclAllReduce(buf, buf, n, ncclFloat, ncclSum, c->comm, st);
    if (r == ncclInProgress) r = nccl_wait(c);
    if (r != ncclSuccess) {
        snprintf(msg, msg_len, "ncclAllReduce: %s", ncclGetErrorString(r));
        return TMOE_E_COMM;
    }
    return TMOE_OK;
}

int ep_comm_ranks(const tmoe_comm *c, int *rank) {
    if (rank) *rank = c->rank;
    return c->nranks;
}

// recv[p * bytes ...] = rank p's `send` bytes (device buffers), for every rank p: the one-time
// exchange of the all-to-all mode's buffer handles.
int ep_allgather_bytes(tmoe_comm *c, const void *send, void *recv, size_t bytes, cudaStream_t st, char *msg,
                       size_t msg_len) {
    if (!c->comm) {
        snprintf(msg, msg_len, "the communicator was aborted");
        return TMOE_E_COMM;
    }
    ncclResult_t r = ncclAllGather(send, recv, bytes, ncclUint8, c->comm, st);
    if (r == ncclInProgress) r = nccl_wait(c);
    if (r != ncclSuccess) {
        snprintf(msg, msg_len, "ncclAllGather: %s", ncclGetErrorString(r));
        return TMOE_E_COMM;
    }
    return TMOE_OK;
}

// All-to-all of fixed-size blocks: block p of every buffer's `send` goes to rank p, whose block
// `rank` of `recv` receives it.  The local block is a device copy; the others are one NCCL group
// of sends and receives, so the exchange is one collective step for the ranks.
int ep_alltoall(tmoe_comm *c, const EpBuf *bufs, int nbufs, cudaStream_t st, char *msg, size_t msg_len,
                bool copy_self) {
    if (!c->comm) {
        snprintf(msg, msg_len, "the communicator was aborted");
        return TMOE_E_COMM;
    }
    for (int b = 0; b < nbufs && copy_self; b++) {
        const size_t n = bufs[b].bytes_per_peer;
        const cudaError_t e = cudaMemcpyAsync((char *)bufs[b].recv + (size_t)c->rank * n,
                                              (const char *)bufs[b].send + (size_t)c->rank * n, n,
                                              cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) {
            snprintf(msg, msg_len, "local block copy: %s", cudaGetErrorString(e));
            return TMOE_E_CUDA;
        }
    }
    ncclResult_t r = ncclGroupStart();
    for (int b = 0; b < nbufs && (r == ncclSuccess || r == ncclInProgress); b++) {
        const size_t n = bufs[b].bytes_per_peer;
        for (int p = 0; p < c->nranks; p++) {
            if (p == c->rank) continue;
            r = ncclSend((const char *)bufs[b].send + (size_t)p * n, n, ncclUint8, p, c->comm, st);
            if (r != ncclSuccess && r != ncclInProgress) break;
            r = ncclRecv((char *)bufs[b].recv + (size_t)p * n, n, ncclUint8, p, c->comm, st);
            if (r != ncclSuccess && r != ncclInProgress) break;
        }
    }
    const ncclResult_t re = ncclGroupEnd();
    if (r == ncclSuccess || r == ncclInProgress) r = re;
    if (r == ncclInProgress) r = nccl_wait(c);
    if (r != ncclSuccess) {
        snprintf(msg, msg_len, "all-to-all: %s", ncclGetErrorString(r));
        return TMOE_E_COMM;
    }
    return TMOE_OK;
}

}  // namespace tmoe

namespace {
thread_local char g_comm_error[256] = "";

int comm_fail(const char *what, ncclResult_t r) {
    snprintf(g_comm_error, sizeof g_comm_error, "%s: %s", what, ncclGetErrorString(r));
    return TMOE_E_COMM;
}
}  // namespace

extern "C" {

const char *tmoe_comm_last_error(void) { return g_comm_error; }

int tmoe_comm_unique_id(void *id_out) {
    if (!id_out) return TMOE_E_INVALID;
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return comm_fail("ncclGetUniqueId", r);
    static_assert(sizeof(ncclUniqueId) == TMOE_COMM_ID_BYTES, "unique id size");
    memcpy(id_out, &id, sizeof id);
    return TMOE_OK;
}

int tmoe_comm_init(const void *id, int32_t nranks, int32_t rank, int32_t device, double timeout_s,
                   tmoe_comm **out) {
    if (!id || !out || nranks < 1 || rank < 0 || rank >= nranks || timeout_s <= 0) return TMOE_E_INVALID;
    *out = nullptr;
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return TMOE_E_CUDA;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    tmoe_comm *c = new tmoe_comm;
    c->nranks = nranks, c->rank = rank, c->device = device, c->timeout_s = timeout_s;
    ncclResult_t r = ncclCommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
    if (r == ncclInProgress) r = tmoe::nccl_wait(c);
    cudaSetDevice(prev);
    if (r != ncclSuccess) {
        if (c->comm) ncclCommAbort(c->comm);
        delete c;
        return comm_fail("ncclCommInitRankConfig", r);
    }
    *out = c;
    return TMOE_OK;
}

int tmoe_comm_abort(tmoe_comm *c) {
    if (!c || !c->comm) return TMOE_E_INVALID;
    const ncclResult_t r = ncclCommAbort(c->comm);
    c->comm = nullptr;
    return r == ncclSuccess ? TMOE_OK : comm_fail("ncclCommAbort", r);
}

void tmoe_comm_destroy(tmoe_comm *c) {
    if (!c) return;
    if (c->comm) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(c->device);
        ncclResult_t r = ncclCommFinalize(c->comm);
        if (r == ncclInProgress) r = tmoe::nccl_wait(c);
        if (c->comm) {
            if (r == ncclSuccess)
                ncclCommDestroy(c->comm);
            else
                ncclCommAbort(c->comm);
        }
        cudaSetDevice(prev);
    }
    delete c;
}

}  // extern "C"
