/* NCCL for the sharding layer, loaded at run time.
 *
 * libm3cuda.so does not link NCCL: a process that already holds one (PyTorch
 * loads its own copy) keeps it, and a process that never shards never maps
 * it.  The first use looks for an already loaded libnccl.so.2 (RTLD_NOLOAD),
 * else loads it from the default search path, and resolves the six entry
 * points used here.  Communicators are created non-blocking and every wait
 * on them is bounded, so a rank that never joins makes the others fail with
 * an error instead of hanging. */

#include "m3c_internal.h"

#include <dlfcn.h>
#include <stdio.h>
#include <nccl.h>
#include <pthread.h>
#include <string.h>
#include <time.h>

typedef ncclResult_t (*get_unique_id_fn)(ncclUniqueId *);
typedef ncclResult_t (*init_rank_config_fn)(ncclComm_t *, int, ncclUniqueId,
                                            int, ncclConfig_t *);
typedef ncclResult_t (*all_reduce_fn)(const void *, void *, size_t,
                                      ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                      cudaStream_t);
typedef ncclResult_t (*comm_fn)(ncclComm_t);
typedef ncclResult_t (*async_error_fn)(ncclComm_t, ncclResult_t *);
typedef const char *(*error_string_fn)(ncclResult_t);

static struct {
    pthread_once_t once;
    bool loaded;
    char why[160];
    get_unique_id_fn get_unique_id;
    init_rank_config_fn init_rank_config;
    all_reduce_fn all_reduce;
    comm_fn destroy;
    comm_fn abort_comm;
    async_error_fn async_error;
    error_string_fn error_string;
} nccl = {PTHREAD_ONCE_INIT, false, "", NULL, NULL, NULL, NULL, NULL, NULL,
          NULL};

static void load_nccl(void)
{
    void *handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);

    if (handle == NULL) {
        handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    }
    if (handle == NULL) {
        const char *reason = dlerror();

        snprintf(nccl.why, sizeof(nccl.why), "cannot load libnccl.so.2: %s",
                 reason != NULL ? reason : "not found");
        return;
    }
    nccl.get_unique_id = (get_unique_id_fn)dlsym(handle, "ncclGetUniqueId");
    nccl.init_rank_config =
        (init_rank_config_fn)dlsym(handle, "ncclCommInitRankConfig");
    nccl.all_reduce = (all_reduce_fn)dlsym(handle, "ncclAllReduce");
    nccl.destroy = (comm_fn)dlsym(handle, "ncclCommDestroy");
    nccl.abort_comm = (comm_fn)dlsym(handle, "ncclCommAbort");
    nccl.async_error = (async_error_fn)dlsym(handle, "ncclCommGetAsyncError");
    nccl.error_string = (error_string_fn)dlsym(handle, "ncclGetErrorString");
    if (nccl.get_unique_id == NULL || nccl.init_rank_config == NULL ||
        nccl.all_reduce == NULL || nccl.destroy == NULL ||
        nccl.abort_comm == NULL || nccl.async_error == NULL ||
        nccl.error_string == NULL) {
        snprintf(nccl.why, sizeof(nccl.why),
                 "libnccl.so.2 lacks an entry point this library needs");
        return;
    }
    nccl.loaded = true;
}

static m3_status nccl_ready(m3_error *error)
{
    (void)pthread_once(&nccl.once, load_nccl);
    if (!nccl.loaded) {
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED, "%s", nccl.why);
    }
    return M3_STATUS_OK;
}

static double seconds_now(void)
{
    struct timespec t;

    (void)clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

static m3_status nccl_failure(m3_error *error, ncclResult_t result,
                              const char *what)
{
    return m3c_error_set(error, M3_STATUS_INTERNAL, "%s: %s", what,
                         nccl.error_string(result));
}

/* Wait (bounded) until the communicator's pending operation has finished.
 * An enqueue on a non-blocking communicator usually settles within
 * microseconds, so the first polls spin; later ones back off to sleeps of up
 * to 200 us (communicator set-up takes milliseconds). */
static m3_status settle_comm(ncclComm_t comm, double limit_seconds,
                             const char *what, m3_error *error)
{
    double deadline = seconds_now() + limit_seconds;
    ncclResult_t state = ncclInProgress;
    long pause_ns = 1000;
    unsigned polls;

    for (polls = 0U;; ++polls) {
        ncclResult_t result = nccl.async_error(comm, &state);

        if (result != ncclSuccess) {
            return nccl_failure(error, result, what);
        }
        if (state != ncclInProgress) {
            break;
        }
        if (seconds_now() > deadline) {
            return m3c_error_set(error, M3_STATUS_CANCELLED,
                                 "%s: no answer within %.0f s", what,
                                 limit_seconds);
        }
        if (polls >= 256U) {
            struct timespec pause = {0, pause_ns};

            (void)nanosleep(&pause, NULL);
            if (pause_ns < 200000) {
                pause_ns *= 2;
            }
        }
    }
    if (state != ncclSuccess) {
        return nccl_failure(error, state, what);
    }
    return M3_STATUS_OK;
}

m3_status m3_cuda_shard_id_create(m3_cuda_shard_id *id, m3_error *error)
{
    ncclUniqueId unique;
    ncclResult_t result;
    m3_status status;

    if (id == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "shard id output is null");
    }
    status = nccl_ready(error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    result = nccl.get_unique_id(&unique);
    if (result != ncclSuccess) {
        return nccl_failure(error, result, "cannot create a communicator id");
    }
    memcpy(id->bytes, unique.internal, sizeof(id->bytes));
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3c_comm_create(const m3_cuda_shard_id *id, int rank, int count,
                          double limit_seconds, void **comm_out,
                          m3_error *error)
{
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    ncclUniqueId unique;
    ncclComm_t comm = NULL;
    ncclResult_t result;
    m3_status status;

    *comm_out = NULL;
    status = nccl_ready(error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    memcpy(unique.internal, id->bytes, sizeof(unique.internal));
    config.blocking = 0;
    result = nccl.init_rank_config(&comm, count, unique, rank, &config);
    if (result != ncclSuccess && result != ncclInProgress) {
        return nccl_failure(error, result, "cannot create the communicator");
    }
    status = settle_comm(comm, limit_seconds, "communicator set-up", error);
    if (status != M3_STATUS_OK) {
        if (comm != NULL) {
            (void)nccl.abort_comm(comm);
        }
        return status;
    }
    *comm_out = comm;
    return M3_STATUS_OK;
}

void m3c_comm_destroy(void *comm)
{
    if (comm != NULL && nccl.loaded) {
        (void)nccl.destroy((ncclComm_t)comm);
    }
}

m3_status m3c_comm_max_u32(void *comm, uint32_t *words, size_t count,
                           void *stream, double limit_seconds,
                           m3_error *error)
{
    ncclResult_t result = nccl.all_reduce(words, words, count, ncclUint32,
                                          ncclMax, (ncclComm_t)comm,
                                          (cudaStream_t)stream);

    if (result == ncclInProgress) {
        return settle_comm((ncclComm_t)comm, limit_seconds,
                           "all-reduce enqueue", error);
    }
    if (result != ncclSuccess) {
        return nccl_failure(error, result, "all-reduce failed");
    }
    return M3_STATUS_OK;
}
