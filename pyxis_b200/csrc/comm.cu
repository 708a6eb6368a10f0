// comm.cu -- NCCL communicator and the vocab-parallel greedy head (include/pyxis_comm.h).
//
// The lm_head of src/output_head.rs:21-44 split by vocabulary rows: every rank multiplies the
// same hidden rows with its shard of the head (pyxis_cuda_matmul_dev's kernels), reduces each
// row's logits to one 64-bit key (argmax.cu: order-preserving value bits, then the inverted
// global index, so the largest key is the first maximum), the ranks exchange the keys (8 bytes
// per row and rank over NVLink), and each takes the largest key of each row.  Nothing goes through
// the host; the whole sequence can be captured in a CUDA graph.
//
// The exchange is one small kernel over peer memory when the ranks' GPUs can map each other's
// memory (CUDA IPC, one process per GPU): every rank stores its keys straight into each peer's
// receive buffer, publishes an epoch flag there with a system-scope release, waits (bounded) for
// every peer's flag in its own buffer and picks the tokens -- no collective launch, which on these
// 8-bytes-per-row messages cost more than the stores.  Keys go to one of two buffers by epoch
// parity: a rank cannot begin call e + 2 before every peer has published call e + 1, i.e. finished
// reading call e.  Otherwise (IPC unavailable) an NCCL all-gather and a pick kernel do the same.
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
#include "tc_ptx.cuh"

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

constexpr int kXMaxRows = kArgmaxMaxRows;   // rows per exchange
constexpr int kXMaxRanks = 8;
constexpr uint64_t kXTimeoutNs = 2000000000ull;
constexpr int kErrExchange = 0x701;
// Layout of a rank's receive buffer: keys [2][kXMaxRanks][kXMaxRows] u64, flags [kXMaxRanks] u32
// (the epoch each rank last published here), this rank's own epoch counter (u32).
constexpr size_t kXKeyBytes = 2ull * kXMaxRanks * kXMaxRows * sizeof(uint64_t);
constexpr size_t kXBytes = kXKeyBytes + 64 + 64;

PYXIS_DEVINL void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
PYXIS_DEVINL unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One CTA: mine [M] keys -> every rank's buffer (slot of this call's epoch parity, row block of
// this rank), then mine zeroed for the next call, flags, a bounded wait for all ranks' flags here,
// then tokens[r] for rows [row0, row0 + nrows).  A wait that runs out records kErrExchange and
// leaves the tokens unwritten.
__global__ void __launch_bounds__(256)
    exchange_pick_kernel(uint64_t *__restrict__ mine, int M, int rank, int nranks, void *const *xtable,
                         int row0, int nrows, int32_t *__restrict__ tokens, int *err) {
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    pdl_wait();
    pdl_trigger();
    uint8_t *local = static_cast<uint8_t *>(xtable[rank]);
    unsigned *epoch_ctr = reinterpret_cast<unsigned *>(local + kXKeyBytes + 64);
    if (threadIdx.x == 0) {
        s_epoch = *epoch_ctr + 1;  // every rank makes the same calls: the epochs agree
        *epoch_ctr = s_epoch;
        s_ok = 1;
    }
    __syncthreads();
    const unsigned e = s_epoch;
    const int slot = e & 1;
    for (int p = 0; p < nranks; ++p) {
        uint64_t *dst = reinterpret_cast<uint64_t *>(static_cast<uint8_t *>(xtable[p])) +
                        ((size_t)slot * kXMaxRanks + rank) * kXMaxRows;
        for (int r = threadIdx.x; r < M; r += blockDim.x) dst[r] = mine[r];
    }
    __syncthreads();
    // the tensor-core GEMV's epilogue max-reduces the next call's keys into mine
    for (int r = threadIdx.x; r < M; r += blockDim.x) mine[r] = 0;
    if (threadIdx.x == 0) {
        __threadfence_system();  // the keys above before the flags, for every peer
        for (int p = 0; p < nranks; ++p)
            st_release_sys(reinterpret_cast<unsigned *>(static_cast<uint8_t *>(xtable[p]) + kXKeyBytes) + rank, e);
        const unsigned *flags = reinterpret_cast<const unsigned *>(local + kXKeyBytes);
        const uint64_t t0 = tc::globaltimer_ns();
        for (int q = 0; q < nranks && s_ok; ++q) {
            while ((int)(ld_acquire_sys(flags + q) - e) < 0) {
                if (tc::globaltimer_ns() - t0 > kXTimeoutNs) {
                    atomicCAS(err, 0, kErrExchange);
                    s_ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
    }
    __syncthreads();
    if (!s_ok) return;
    const uint64_t *keys = reinterpret_cast<const uint64_t *>(local) + (size_t)slot * kXMaxRanks * kXMaxRows;
    for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
        uint64_t m = 0;
        for (int q = 0; q < nranks; ++q) {
            const uint64_t k = __ldcv(keys + (size_t)q * kXMaxRows + row0 + r);
            m = k > m ? k : m;
        }
        tokens[r] = m == 0 ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFu));
    }
}

// Maps every rank's receive buffer into every other rank (collective: all ranks call it in
// comm_init, and every rank makes the same NCCL calls whatever its own verdict, so none is left
// waiting).  Leaves c->p2p false, and frees what it made, unless every rank can map every other.
void setup_p2p(pyxis_cuda_comm *c) {
    if (c->nranks < 2 || c->nranks > kXMaxRanks) return;
    const NcclApi &api = nccl();
    cudaStream_t st = c->ctx->stream;
    const size_t R = (size_t)c->nranks;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    uint8_t *scratch = nullptr;  // [R] verdicts (int), then [R] IPC handles of 64 bytes
    if (cudaMalloc(&scratch, 16 * R + 64 * R) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    int *dv = reinterpret_cast<int *>(scratch);
    uint8_t *hbuf = scratch + 16 * R;
    cudaIpcMemHandle_t mine{};
    int ok = cudaMalloc(&c->xbuf, kXBytes) == cudaSuccess && cudaMemset(c->xbuf, 0, kXBytes) == cudaSuccess &&
             cudaIpcGetMemHandle(&mine, c->xbuf) == cudaSuccess;
    cudaGetLastError();
    auto exchange_verdict = [&](int mine_ok) -> bool {
        int v = mine_ok, all[kXMaxRanks] = {0};
        bool good = cudaMemcpy(dv + c->rank, &v, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess;
        good = api.all_gather(dv + c->rank, dv, 1, ncclInt32, c->nccl, st) == ncclSuccess && good;
        good = cudaStreamSynchronize(st) == cudaSuccess && good;
        good = good && cudaMemcpy(all, dv, sizeof(int) * R, cudaMemcpyDeviceToHost) == cudaSuccess;
        for (size_t q = 0; q < R; ++q) good = good && all[q] != 0;
        return good;
    };
    cudaMemcpy(hbuf + 64 * (size_t)c->rank, &mine, 64, cudaMemcpyHostToDevice);
    const bool sent = api.all_gather(hbuf + 64 * (size_t)c->rank, hbuf, 64, ncclUint8, c->nccl, st) == ncclSuccess;
    ok = exchange_verdict(ok && sent);
    void *bases[kXMaxRanks] = {nullptr};
    if (ok) {
        cudaIpcMemHandle_t h[kXMaxRanks];
        ok = cudaMemcpy(h, hbuf, 64 * R, cudaMemcpyDeviceToHost) == cudaSuccess;
        for (int q = 0; q < c->nranks && ok; ++q) {
            if (q == c->rank) {
                bases[q] = c->xbuf;
                continue;
            }
            ok = cudaIpcOpenMemHandle(&c->peer_base[q], h[q], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
            bases[q] = c->peer_base[q];
        }
        ok = ok && cudaMalloc(&c->xtable, sizeof(void *) * R) == cudaSuccess &&
             cudaMemcpy(c->xtable, bases, sizeof(void *) * R, cudaMemcpyHostToDevice) == cudaSuccess;
        cudaGetLastError();
    }
    // the ranks must agree on the path
    ok = exchange_verdict(ok);
    cudaFree(scratch);
    cudaGetLastError();
    if (ok) {
        c->p2p = true;
        return;
    }
    for (int q = 0; q < kXMaxRanks; ++q)
        if (c->peer_base[q]) {
            cudaIpcCloseMemHandle(c->peer_base[q]);
            c->peer_base[q] = nullptr;
        }
    cudaFree(c->xtable);
    cudaFree(c->xbuf);
    c->xtable = nullptr;
    c->xbuf = nullptr;
    cudaGetLastError();
}

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
        // zero: the fused head GEMV max-reduces into it (and every call leaves it zero again)
        if (cudaMemset(c->keys, 0, nk * sizeof(uint64_t)) != cudaSuccess) {
            cudaGetLastError();
            return fail(PYXIS_ECUDA, "head: cudaMemset(keys) failed");
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
    uint64_t *mine = c->keys, *all = c->keys + M;
    // int8 shards on the tensor-core GEMV write the keys from its epilogue (into mine, which the
    // consumers below leave zero); other shards take the GEMV, then the argmax scan over the logits
    cudaError_t e = cudaSuccess;
    if (!head_gemv_keys(ctx, shard, X, M, ldx, shard_rows, hidden, c->logits, shard_rows, (int64_t)vocab_lo, mine,
                        st, &e)) {
        int rc = run_matmul(ctx, shard, X, M, ldx, shard_rows, hidden, c->logits, shard_rows, ws, ws_bytes, st);
        if (rc) return rc;
        e = launch_argmax_keys(c->logits, M, shard_rows, shard_rows, (int64_t)vocab_lo, mine, ctx->amax, ctx->num_sms,
                               st);
    }
    if (e != cudaSuccess) return fail(PYXIS_ECUDA, cudaGetErrorString(e));
    if (c->p2p && M <= (size_t)kXMaxRows) {
        e = launch_kernel(exchange_pick_kernel, dim3(1), dim3(256), 0, st, mine, (int)M, c->rank, c->nranks,
                          (void *const *)c->xtable, row0, nrows, tokens, ctx->d_err);
        if (e != cudaSuccess) return fail(PYXIS_ECUDA, cudaGetErrorString(e));
        return PYXIS_OK;
    }
    int rc = comm_allgather(c, mine, all, M, true, st);
    if (rc) return rc;
    e = launch_pick_keys(all, c->nranks, (int)M, row0, nrows, tokens, mine, (int)M, st);
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
    setup_p2p(c);
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
    for (int q = 0; q < 8; ++q)
        if (c->peer_base[q]) cudaIpcCloseMemHandle(c->peer_base[q]);
    cudaFree(c->xtable);
    cudaFree(c->xbuf);
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
