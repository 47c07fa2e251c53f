/* sb_dist.c -- the multi-GPU SGEMM from C: row panels over the ranks of one
 * node, and an in-place NCCL all-gather of C over NVLink.
 *
 * The reference has no multi-GPU path (gpu_workload.c:66-67 uses device 0
 * only).  The sharding rule is this package's own: rank p of P computes rows
 * [p R, p R + R) of C = A B (R = ceil(M / P)) with the CUDA-core kernel of
 * sb_sgemm_rows, B replicated and nothing crossing NVLink during the
 * product; when the caller wants the whole C on every rank, one
 * ncclAllGather follows on the same stream.  Row-major panels are
 * contiguous, so the gather runs in place (send buffer = this rank's panel
 * inside the receive buffer) and needs no reshuffle.
 *
 * NCCL is loaded with dlopen on first use, so the library has no link-time
 * dependency on it.  Communicators are created non-blocking
 * (ncclConfig_t.blocking = 0): every wait -- initialisation, a collective in
 * flight -- polls ncclCommGetAsyncError against a host-side deadline and,
 * when a peer never arrives or a collective never completes, aborts the
 * communicator (ncclCommAbort) and returns an error instead of hanging. */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <nccl.h>
#include <pthread.h>
#include <string.h>
#include <time.h>

#include "sb_internal.h"

typedef ncclResult_t (*fn_uid)(ncclUniqueId *);
typedef ncclResult_t (*fn_init)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
typedef ncclResult_t (*fn_comm)(ncclComm_t);
typedef ncclResult_t (*fn_async)(ncclComm_t, ncclResult_t *);
typedef ncclResult_t (*fn_ag)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
typedef const char *(*fn_str)(ncclResult_t);

static struct {
    int loaded;
    fn_uid get_unique_id;
    fn_init init_rank_config;
    fn_async get_async_error;
    fn_comm abort_comm, finalize, destroy;
    fn_ag all_gather;
    fn_str error_string;
} nccl;
static pthread_mutex_t nccl_lock = PTHREAD_MUTEX_INITIALIZER;

static int nccl_load(void) {
    pthread_mutex_lock(&nccl_lock);
    if (!nccl.loaded) {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            nccl.get_unique_id = (fn_uid)dlsym(h, "ncclGetUniqueId");
            nccl.init_rank_config = (fn_init)dlsym(h, "ncclCommInitRankConfig");
            nccl.get_async_error = (fn_async)dlsym(h, "ncclCommGetAsyncError");
            nccl.abort_comm = (fn_comm)dlsym(h, "ncclCommAbort");
            nccl.finalize = (fn_comm)dlsym(h, "ncclCommFinalize");
            nccl.destroy = (fn_comm)dlsym(h, "ncclCommDestroy");
            nccl.all_gather = (fn_ag)dlsym(h, "ncclAllGather");
            nccl.error_string = (fn_str)dlsym(h, "ncclGetErrorString");
            if (nccl.get_unique_id && nccl.init_rank_config && nccl.get_async_error && nccl.abort_comm &&
                nccl.finalize && nccl.destroy && nccl.all_gather && nccl.error_string)
                nccl.loaded = 1;
        }
    }
    const int ok = nccl.loaded;
    pthread_mutex_unlock(&nccl_lock);
    return ok ? 0 : sb_fail(SB_ERR_STATE, "NCCL (libnccl.so.2) could not be loaded", __FILE__, __LINE__);
}

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec / 1e9;
}

static int nccl_fail(ncclResult_t r, const char *what, int line) {
    return sb_fail(SB_ERR_STATE, nccl.error_string ? nccl.error_string(r) : what, what, line);
}

/* Poll the communicator until its pending operation (initialisation,
 * finalisation) is done; abort it on an error or at the deadline. */
static int comm_settle(ncclComm_t comm, double deadline, const char *what) {
    for (;;) {
        ncclResult_t st = ncclInProgress;
        ncclResult_t r = nccl.get_async_error(comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return 0;
        if (st != ncclInProgress) {
            nccl.abort_comm(comm);
            return nccl_fail(st, what, __LINE__);
        }
        if (now_s() > deadline) {
            nccl.abort_comm(comm);
            return sb_fail(SB_ERR_STATE, "NCCL wait timed out (a peer never arrived); communicator aborted", what,
                           __LINE__);
        }
        struct timespec ts = {0, 200000};
        nanosleep(&ts, NULL);
    }
}

int sb_nccl_unique_id(void *id) {
    SB_ARG(id, "null id buffer");
    int rc = nccl_load();
    if (rc) return rc;
    ncclResult_t r = nccl.get_unique_id((ncclUniqueId *)id);
    return r == ncclSuccess ? 0 : nccl_fail(r, "ncclGetUniqueId", __LINE__);
}

int sb_nccl_comm_init(void **comm, int world, const void *id, int rank, double timeout_s) {
    SB_ARG(comm && id && world >= 1 && rank >= 0 && rank < world && timeout_s > 0, "bad communicator arguments");
    int rc = nccl_load();
    if (rc) return rc;
    if (!sb_ctx_get()) return SB_ERR_STATE; /* NCCL binds to the device of the current context */
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t c = NULL;
    ncclResult_t r = nccl.init_rank_config(&c, world, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (c) nccl.abort_comm(c);
        return nccl_fail(r, "ncclCommInitRankConfig", __LINE__);
    }
    rc = comm_settle(c, now_s() + timeout_s, "ncclCommInitRankConfig");
    if (rc) return rc;
    *comm = c;
    return 0;
}

int sb_nccl_comm_destroy(void *comm, double timeout_s) {
    if (!comm) return 0;
    int rc = nccl_load();
    if (rc) return rc;
    ncclComm_t c = (ncclComm_t)comm;
    ncclResult_t r = nccl.finalize(c);
    if (r != ncclSuccess && r != ncclInProgress) {
        nccl.abort_comm(c);
        return nccl_fail(r, "ncclCommFinalize", __LINE__);
    }
    rc = comm_settle(c, now_s() + timeout_s, "ncclCommFinalize"); /* aborts on failure */
    if (rc) return rc;
    r = nccl.destroy(c);
    return r == ncclSuccess ? 0 : nccl_fail(r, "ncclCommDestroy", __LINE__);
}

int sb_nccl_abort(void *comm) {
    if (!comm) return 0;
    int rc = nccl_load();
    if (rc) return rc;
    ncclResult_t r = nccl.abort_comm((ncclComm_t)comm);
    return r == ncclSuccess ? 0 : nccl_fail(r, "ncclCommAbort", __LINE__);
}

int sb_sgemm_panel_allgather(const float *A, const float *B, float *C, int M, int N, int K, int rank, int world,
                             void *comm, int gather, void *stream) {
    SB_ARG(world >= 1 && rank >= 0 && rank < world, "bad rank / world");
    SB_ARG(!gather || comm || world == 1, "all-gather needs a communicator");
    const int R = (M + world - 1) / world;
    const int row0 = rank * R < M ? rank * R : M;
    const int row1 = row0 + R < M ? row0 + R : M;
    int rc = sb_sgemm_rows(A, B, C, M, N, K, row0, row1, stream);
    if (rc || !gather || world == 1) return rc;
    if ((rc = nccl_load())) return rc;
    /* in place: this rank's R rows of the (world * R) x N buffer C */
    const size_t count = (size_t)R * N;
    ncclResult_t r = nccl.all_gather(C + (size_t)rank * count, C, count, ncclFloat32, (ncclComm_t)comm,
                                     (cudaStream_t)stream);
    if (r == ncclInProgress) /* a non-blocking communicator may still be enqueueing (first-use connection
                              * set-up): it must settle before the next NCCL call on it */
        return comm_settle((ncclComm_t)comm, now_s() + 120.0, "ncclAllGather");
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather", __LINE__);
    return 0;
}

int sb_nccl_wait(void *comm, void *stream, double timeout_s) {
    SB_ARG(timeout_s > 0, "bad timeout");
    const double deadline = now_s() + timeout_s;
    int rc = comm ? nccl_load() : 0;
    if (rc) return rc;
    for (;;) {
        CUresult q = cuStreamQuery((CUstream)stream);
        if (q == CUDA_SUCCESS) return 0;
        if (q != CUDA_ERROR_NOT_READY) return sb_fail((int)q, "cuStreamQuery", __FILE__, __LINE__);
        if (comm) {
            ncclResult_t st = ncclSuccess;
            ncclResult_t r = nccl.get_async_error((ncclComm_t)comm, &st);
            if (r != ncclSuccess) st = r;
            if (st != ncclSuccess && st != ncclInProgress) {
                nccl.abort_comm((ncclComm_t)comm);
                return nccl_fail(st, "collective failed; communicator aborted", __LINE__);
            }
        }
        if (now_s() > deadline) {
            if (comm) nccl.abort_comm((ncclComm_t)comm);
            return sb_fail(SB_ERR_STATE, "stream did not finish in time; communicator aborted", __FILE__, __LINE__);
        }
        struct timespec ts = {0, 50000};
        nanosleep(&ts, NULL);
    }
}

/* ---- CUDA IPC: the C of every rank mapped into every other rank's process,
 * so sb_sgemm_multi can store a panel's tiles straight into all of them. */
int sb_ipc_export(const void *ptr, void *handle64, size_t *offset) {
    SB_ARG(ptr && handle64 && offset, "bad ipc export arguments");
    if (!sb_ctx_get()) return SB_ERR_STATE;
    CUdeviceptr base = 0;
    size_t size = 0;
    SB_CK(cuMemGetAddressRange(&base, &size, (CUdeviceptr)(uintptr_t)ptr));
    CUipcMemHandle h;
    SB_CK(cuIpcGetMemHandle(&h, base));
    memcpy(handle64, &h, sizeof h);
    *offset = (size_t)((CUdeviceptr)(uintptr_t)ptr - base);
    return 0;
}

int sb_ipc_open(const void *handle64, size_t offset, void **ptr) {
    SB_ARG(handle64 && ptr, "bad ipc open arguments");
    if (!sb_ctx_get()) return SB_ERR_STATE;
    CUipcMemHandle h;
    memcpy(&h, handle64, sizeof h);
    CUdeviceptr base = 0;
    SB_CK(cuIpcOpenMemHandle(&base, h, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS));
    *ptr = (void *)(uintptr_t)(base + offset);
    return 0;
}

int sb_ipc_close(void *ptr, size_t offset) {
    SB_ARG(ptr, "bad ipc close arguments");
    SB_CK(cuIpcCloseMemHandle((CUdeviceptr)(uintptr_t)ptr - offset));
    return 0;
}
