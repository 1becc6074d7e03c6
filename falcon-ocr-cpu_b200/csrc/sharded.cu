// sharded.cu -- the head-sharded prefill of one long page over the ranks of an
// NCCL communicator (one process per GPU), host side.
//
// Rank i holds the query heads of its KV groups (Q FP32, K and V BF16, its
// sinks) and computes them with the BF16 tensor-core prefill in bands of
// query rows, latest rows first (under a causal or prefix-LM mask the later
// rows see more keys, so the light band comes last and leaves the shortest
// gather exposed).  Each band's kernel writes its BF16 output straight into
// this rank's slot of the band's gathered block [world][rows][heads][64],
// and an in-place ncclAllGather of the block, issued on the context's comm
// stream behind the band's event, overlaps the next band's computation.  No
// copy kernel runs, and no kernel reads another GPU's memory: peers' rows
// arrive only through NCCL.
//
// There is no counterpart in the reference, which prefills a page on one
// host; the per-rank computation is kernels::attention_prefill_bf16
// (src/kernels/attention/mod.rs:321-349) on a subset of heads.
//
// NCCL is resolved at run time from the libnccl.so.2 the process already has
// loaded (the one that made the caller's communicator), or else loaded by
// that name; the library itself does not link it.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "fo_kernels.h"

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

std::mutex g_nccl_mutex;
NcclApi g_nccl;

}  // namespace

// The process's NCCL, resolved once; null with a message when absent.
static const NcclApi *nccl_api(char *msg, size_t n) {
    std::lock_guard<std::mutex> lock(g_nccl_mutex);
    if (g_nccl.ok) return &g_nccl;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        snprintf(msg, n, "libnccl.so.2 is not available: %s", dlerror());
        return nullptr;
    }
    NcclApi a;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.all_gather || !a.all_reduce ||
        !a.error_string) {
        snprintf(msg, n, "libnccl.so.2 lacks an entry point the sharded prefill needs");
        return nullptr;
    }
    a.ok = true;
    g_nccl = a;
    return &g_nccl;
}

// ---------------------------------------------------- helpers for fo_abi.cu
// Each returns 0, or -1 with a message in msg.

int fo_nccl_unique_id_impl(uint8_t *id, char *msg, size_t n) {
    const NcclApi *a = nccl_api(msg, n);
    if (!a) return -1;
    ncclUniqueId u;
    const ncclResult_t r = a->get_unique_id(&u);
    if (r != ncclSuccess) {
        snprintf(msg, n, "ncclGetUniqueId: %s", a->error_string(r));
        return -1;
    }
    static_assert(sizeof(u) == FO_NCCL_ID_BYTES, "ncclUniqueId size");
    memcpy(id, &u, sizeof(u));
    return 0;
}

// A communicator of `world` ranks on the current device.
int fo_nccl_comm_init_impl(int world, int rank, const uint8_t *id, void **comm, char *msg, size_t n) {
    const NcclApi *a = nccl_api(msg, n);
    if (!a) return -1;
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    const ncclResult_t r = a->comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) {
        snprintf(msg, n, "ncclCommInitRank: %s", a->error_string(r));
        return -1;
    }
    *comm = c;
    return 0;
}

int fo_nccl_comm_destroy_impl(void *comm, char *msg, size_t n) {
    const NcclApi *a = nccl_api(msg, n);
    if (!a) return -1;
    const ncclResult_t r = a->comm_destroy(static_cast<ncclComm_t>(comm));
    if (r != ncclSuccess) {
        snprintf(msg, n, "ncclCommDestroy: %s", a->error_string(r));
        return -1;
    }
    return 0;
}

// The in-place all-gather of one band's block [world][count] BF16 values:
// this rank's part is already at block + rank * count.
int fo_nccl_gather_bf16(void *comm, uint16_t *block, size_t count, int rank, cudaStream_t stream, char *msg,
                        size_t n) {
    const NcclApi *a = nccl_api(msg, n);
    if (!a) return -1;
    const ncclResult_t r = a->all_gather(block + (size_t)rank * count, block, count, ncclBfloat16,
                                         static_cast<ncclComm_t>(comm), stream);
    if (r != ncclSuccess) {
        snprintf(msg, n, "ncclAllGather: %s", a->error_string(r));
        return -1;
    }
    return 0;
}

// Every rank's `bytes` bytes at send gathered into recv [world][bytes] (the
// peer-block registration's handle exchange).
int fo_nccl_allgather_bytes(void *comm, const void *send, void *recv, size_t bytes, cudaStream_t stream, char *msg,
                            size_t n) {
    const NcclApi *a = nccl_api(msg, n);
    if (!a) return -1;
    const ncclResult_t r = a->all_gather(send, recv, bytes, ncclUint8, static_cast<ncclComm_t>(comm), stream);
    if (r != ncclSuccess) {
        snprintf(msg, n, "ncclAllGather: %s", a->error_string(r));
        return -1;
    }
    return 0;
}

// A barrier of the communicator's ranks on `stream`: an all-reduce of one
// word.  Once it completes on a rank, every rank's work queued before it on
// its own stream has completed (the peer-store gather's end).
int fo_nccl_barrier(void *comm, int32_t *word, cudaStream_t stream, char *msg, size_t n) {
    const NcclApi *a = nccl_api(msg, n);
    if (!a) return -1;
    const ncclResult_t r = a->all_reduce(word, word, 1, ncclInt32, ncclSum, static_cast<ncclComm_t>(comm), stream);
    if (r != ncclSuccess) {
        snprintf(msg, n, "ncclAllReduce: %s", a->error_string(r));
        return -1;
    }
    return 0;
}
