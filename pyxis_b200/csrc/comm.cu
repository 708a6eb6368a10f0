// comm.cu -- NCCL communicator and the vocab-parallel greedy head (include/pyxis_comm.h).
//
// The lm_head of src/output_head.rs:21-44 split by vocabulary rows: every rank multiplies the
// same hidden rows with its shard of the head (pyxis_cuda_matmul_dev's kernels), reduces each
// row's logits to one 64-bit key (argmax.cu: order-preserving value bits, then the inverted
// global index, so the largest key is the first maximum), the ranks all-gather the keys (8 bytes
// per row and rank over NVLink), and a small kernel takes the largest key of each row.  Nothing
// goes through the host; the whole sequence can be captured in a CUDA graph.
//
// NCCL is loaded with dlopen on first use: libnccl.so.2 resolves to the copy a process already
// has (PyTorch's, for instance), else the system one.
#include <dlfcn.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include "argmax.h"
#include "comm.h"
#include "common.cuh"
#include "kernels.h"

namespace pyxis {
namespace {

struct NcclApi {
    bool ok = false;
    char why[256] = {0};
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char *e = dlerror();
            snprintf(api.why, sizeof api.why, "cannot load NCCL: %s", e ? e : "not found");
            return;
        }
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.error_string;
        if (!api.ok) snprintf(api.why, sizeof api.why, "NCCL library lacks a required symbol");
    });
    return api;
}

int fail(int code, const char *msg) { return record_error(code, msg); }

int nccl_fail(const NcclApi &api, ncclResult_t r, const char *what) {
    char buf[384];
    snprintf(buf, sizeof buf, "%s: %s", what, api.error_string ? api.error_string(r) : "NCCL error");
    return record_error(PYXIS_ENCCL, buf);
}

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DevGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

int comm_allgather(pyxis_cuda_comm *c, const void *send, void *recv, size_t count, bool u64, cudaStream_t st) {
    const NcclApi &api = nccl();
    if (!api.ok) return fail(PYXIS_EUNSUPPORTED, api.why);
    const ncclResult_t r = api.all_gather(send, recv, count, u64 ? ncclUint64 : ncclFloat32, c->nccl, st);
    if (r != ncclSuccess) return nccl_fail(api, r, "ncclAllGather");
    return PYXIS_OK;
}

int head_reserve(pyxis_cuda_comm *c, size_t M, size_t shard_rows) {
    const size_t nl = M * shard_rows, nk = M * (size_t)(c->nranks + 1);
    if (nl > c->logits_cap) {
        cudaFree(c->logits);
        c->logits = nullptr;
        c->logits_cap = 0;
        if (cudaMalloc(&c->logits, nl * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return fail(PYXIS_ENOMEM, "head: cudaMalloc(logits) failed");
        }
        c->logits_cap = nl;
    }
    if (nk > c->keys_cap) {
        cudaFree(c->keys);
        c->keys = nullptr;
        c->keys_cap = 0;
        if (cudaMalloc(&c->keys, nk * sizeof(uint64_t)) != cudaSuccess) {
            cudaGetLastError();
            return fail(PYXIS_ENOMEM, "head: cudaMalloc(keys) failed");
        }
        c->keys_cap = nk;
    }
    return PYXIS_OK;
}

int head_greedy_enqueue(pyxis_cuda_comm *c, const pyxis_cuda_weights *shard, size_t vocab_lo, size_t shard_rows,
                        size_t hidden, const float *X, size_t M, size_t ldx, int row0, int nrows, int32_t *tokens,
                        void *ws, size_t ws_bytes, cudaStream_t st) {
    if (M * shard_rows > c->logits_cap || M * (size_t)(c->nranks + 1) > c->keys_cap)
        return fail(PYXIS_EINVAL, "head: buffers not reserved for this many rows");
    pyxis_cuda_ctx *ctx = c->ctx;
    int rc = run_matmul(ctx, shard, X, M, ldx, shard_rows, hidden, c->logits, shard_rows, ws, ws_bytes, st);
    if (rc) return rc;
    uint64_t *mine = c->keys, *all = c->keys + M;
    cudaError_t e = launch_argmax_keys(c->logits, M, shard_rows, shard_rows, (int64_t)vocab_lo, mine, ctx->amax,
                                       ctx->num_sms, st);
    if (e != cudaSuccess) return fail(PYXIS_ECUDA, cudaGetErrorString(e));
    rc = comm_allgather(c, mine, all, M, true, st);
    if (rc) return rc;
    e = launch_pick_keys(all, c->nranks, (int)M, row0, nrows, tokens, st);
    if (e != cudaSuccess) return fail(PYXIS_ECUDA, cudaGetErrorString(e));
    return PYXIS_OK;
}

}  // namespace pyxis

using namespace pyxis;

extern "C" {

int pyxis_cuda_comm_unique_id(uint8_t id[PYXIS_COMM_ID_BYTES]) {
    if (!id) return fail(PYXIS_EINVAL, "null id");
    const NcclApi &api = nccl();
    if (!api.ok) return fail(PYXIS_EUNSUPPORTED, api.why);
    static_assert(sizeof(ncclUniqueId) == PYXIS_COMM_ID_BYTES, "NCCL id size");
    ncclUniqueId u;
    const ncclResult_t r = api.get_unique_id(&u);
    if (r != ncclSuccess) return nccl_fail(api, r, "ncclGetUniqueId");
    memcpy(id, &u, sizeof u);
    return PYXIS_OK;
}

int pyxis_cuda_comm_init(pyxis_cuda_ctx *ctx, const uint8_t id[PYXIS_COMM_ID_BYTES], int nranks, int rank,
                         pyxis_cuda_comm **out) {
    if (!ctx || !id || !out) return fail(PYXIS_EINVAL, "null argument");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(PYXIS_EINVAL, "comm_init: bad nranks / rank");
    const NcclApi &api = nccl();
    if (!api.ok) return fail(PYXIS_EUNSUPPORTED, api.why);
    DevGuard g(ctx->device);
    auto *c = new (std::nothrow) pyxis_cuda_comm();
    if (!c) return fail(PYXIS_ENOMEM, "host allocation failed");
    c->ctx = ctx;
    c->nranks = nranks;
    c->rank = rank;
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    const ncclResult_t r = api.comm_init_rank(&c->nccl, nranks, u, rank);
    if (r != ncclSuccess) {
        delete c;
        return nccl_fail(api, r, "ncclCommInitRank");
    }
    *out = c;
    return PYXIS_OK;
}

int pyxis_cuda_comm_info(const pyxis_cuda_comm *c, int *nranks, int *rank) {
    if (!c) return fail(PYXIS_EINVAL, "null communicator");
    if (nranks) *nranks = c->nranks;
    if (rank) *rank = c->rank;
    return PYXIS_OK;
}

int pyxis_cuda_comm_free(pyxis_cuda_comm *c) {
    if (!c) return PYXIS_OK;
    DevGuard g(c->ctx->device);
    cudaStreamSynchronize(c->ctx->stream);
    if (c->nccl) nccl().comm_destroy(c->nccl);
    cudaFree(c->logits);
    cudaFree(c->keys);
    delete c;
    return PYXIS_OK;
}

int pyxis_cuda_head_reserve(pyxis_cuda_comm *c, size_t M, size_t shard_rows) {
    if (!c) return fail(PYXIS_EINVAL, "null communicator");
    DevGuard g(c->ctx->device);
    return head_reserve(c, M, shard_rows);
}

int pyxis_cuda_head_greedy_dev(pyxis_cuda_comm *c, const pyxis_cuda_weights *shard, size_t vocab, size_t vocab_lo,
                               size_t shard_rows, size_t hidden, const float *X, size_t M, size_t ldx, int32_t *tokens,
                               void *stream) {
    if (!c || !shard) return fail(PYXIS_EINVAL, "null communicator or shard");
    if (M == 0) return PYXIS_OK;
    if (!X || !tokens) return fail(PYXIS_EINVAL, "null X or tokens");
    if (M > (size_t)kArgmaxMaxRows) return fail(PYXIS_EINVAL, "head: more than 1024 rows per call");
    if (vocab == 0 || vocab >= 0x7FFFFFFFull || shard_rows == 0 || vocab_lo + shard_rows > vocab)
        return fail(PYXIS_EINVAL, "head: the shard's rows are not inside [0, vocab)");
    if (shard->device != c->ctx->device) return fail(PYXIS_EINVAL, "head: the shard lives on another device");
    if (shard->num_elements != shard_rows * hidden)
        return fail(PYXIS_EINVAL, "head: shard length != shard_rows * hidden");
    if (M > 1 && ldx < hidden) return fail(PYXIS_EINVAL, "row stride smaller than the row");
    DevGuard g(c->ctx->device);
    int rc = head_reserve(c, M, shard_rows);
    if (rc) return rc;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->ctx->stream;
    return head_greedy_enqueue(c, shard, vocab_lo, shard_rows, hidden, X, M, ldx, 0, (int)M, tokens, nullptr, 0, st);
}

}  // extern "C"
