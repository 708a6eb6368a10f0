// api.cu -- the extern "C" boundary (include/pyxis_cuda.h): contexts, device-resident weights,
// argument checks that mirror the reference's asserts, and kernel dispatch.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>

#include "../../include/pyxis_cuda.h"
#include "argmax.h"
#include "common.cuh"
#include "ctx.h"
#include "kernels.h"

using namespace pyxis;


namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(PYXIS_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define PYXIS_CUDA_TRY(expr, what)                      \
    do {                                                \
        cudaError_t e_ = (expr);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

// Makes ctx's device current for the call and restores the caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }

constexpr size_t kTcMinRows = 16;        // matmul_dev rows from which the tensor-core GEMM runs
constexpr size_t kTcGemvMinRows = 16384;  // out_features from which int8 GEMVs use tensor cores

bool is_dense(int qtype) { return qtype == PYXIS_QTYPE_F32 || qtype == PYXIS_QTYPE_BF16; }
bool is_qtype(int qtype) { return qtype >= PYXIS_QTYPE_INT8 && qtype <= PYXIS_QTYPE_BF16; }

size_t packed_bytes(int qtype, size_t n) {
    switch (qtype) {
    case PYXIS_QTYPE_INT8: return n;
    case PYXIS_QTYPE_INT4: return div_ceil(n, 2);
    case PYXIS_QTYPE_F32: return n * 4;
    default: return n * 2;  // BF16
    }
}

int grow(float **buf, size_t *cap, size_t need) {
    if (need <= *cap) return PYXIS_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    size_t n = need < 4096 ? 4096 : need;
    PYXIS_CUDA_TRY(cudaMalloc(buf, n * sizeof(float)), "cudaMalloc(staging)");
    *cap = n;
    return PYXIS_OK;
}

int alloc_weights(pyxis_cuda_ctx *ctx, int qtype, size_t n, size_t bs, pyxis_cuda_weights **out) {
    auto *w = new (std::nothrow) pyxis_cuda_weights{};
    if (!w) return fail(PYXIS_ENOMEM, "host allocation failed");
    w->device = ctx->device;
    w->qtype = qtype;
    w->num_elements = n;
    w->block_size = is_dense(qtype) ? 0 : bs;
    w->data_bytes = packed_bytes(qtype, n);
    w->num_scales = is_dense(qtype) ? 0 : div_ceil(n, bs);
    size_t off = div_ceil(w->data_bytes, 256) * 256;
    size_t total = off + w->num_scales * sizeof(float);
    void *mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, total ? total : 256);
    if (e != cudaSuccess) {
        delete w;
        if (e == cudaErrorMemoryAllocation) {
            cudaGetLastError();
            return fail(PYXIS_ENOMEM, "cudaMalloc(%zu bytes) for weights failed", total);
        }
        return cuda_fail(e, "cudaMalloc(weights)");
    }
    w->data = (uint8_t *)mem;
    w->scales = (float *)((uint8_t *)mem + off);
    *out = w;
    return PYXIS_OK;
}

cudaStream_t pick_stream(pyxis_cuda_ctx *ctx, void *stream) {
    return stream ? (cudaStream_t)stream : ctx->stream;
}

QMatrix qmatrix(const pyxis_cuda_weights *w, size_t N, size_t K) {
    return QMatrix{w->qtype, w->data, w->scales, w->block_size, N, K};
}

// The reference's matmul asserts (src/matmul.rs:27-50).
int check_matmul(const pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, size_t out_features,
                 size_t in_features) {
    if (!ctx || !w) return fail(PYXIS_EINVAL, "null context or weights");
    if (w->device != ctx->device)
        return fail(PYXIS_EINVAL, "weights live on device %d, context on device %d", w->device, ctx->device);
    if (w->num_elements != out_features * in_features)
        return fail(PYXIS_EINVAL, "weight.len() = %zu != out_features * in_features = %zu * %zu",
                    w->num_elements, out_features, in_features);
    if (!is_dense(w->qtype) && w->block_size == 0) return fail(PYXIS_EINVAL, "block_size must be > 0");
    return PYXIS_OK;
}

// The context's default workspace, allocated at init: it covers the weight-streaming matmul's x
// copies for 64 tokens of K <= 16384 plus kWsPartialCap of split-K partial sums, and the
// tensor-core GEMM's needs up to a few hundred tokens.  Larger needs grow it outside stream
// capture (pyxis_cuda_reserve_workspace, or the first call that needs it).
constexpr size_t kWsPartialCap = 12u << 20;
constexpr size_t kDefaultWorkspace = 20u << 20;
constexpr size_t kWsTickets = 16384;  // 128-row tiles: matrices of up to 2M rows

int grow_workspace(pyxis_cuda_ctx *ctx, size_t want) {
    if (ctx->ws_cap >= want) return PYXIS_OK;
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_cap = 0;
    PYXIS_CUDA_TRY(cudaMalloc(&ctx->ws, want), "cudaMalloc(workspace)");
    ctx->ws_cap = want;
    return PYXIS_OK;
}

// Grows the context workspace, refusing while `st` is being captured (an allocation there would
// be an error, and a graph would keep the old pointer).
int ensure_ctx_workspace(pyxis_cuda_ctx *ctx, size_t want, cudaStream_t st) {
    if (ctx->ws_cap >= want) return PYXIS_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
        return fail(PYXIS_EINVAL,
                    "the context workspace must grow to %zu bytes, which cannot happen during stream capture: "
                    "call pyxis_cuda_reserve_workspace first",
                    want);
    return grow_workspace(ctx, want);
}

}  // namespace

int pyxis::record_error(int code, const char *msg) { return fail(code, "%s", msg); }

namespace {
// Weight-streaming tensor-core matmul for decode-shaped batches of 9-64 tokens (int4 / int8 with
// group-32 scales, int8 with one scale per row).  Its MMAs are K = 16 fp16 instructions with x as hi
// and lo halves, 16 per 128 of K and 128 rows, and a tcgen05.mma costs about 128 cycles at any N up
// to 256 (measured per stage: 1.05 us at 16 token columns, 1.2 us at 64), so the instruction count,
// not the token count, sets its pace: it wins where the CUDA cores' FMAs per weight grow with the
// tokens (int4 gate|up 12288 x 2048 at 64 tokens: 22 us against 67 us on the prefill GEMM), while
// up to 8 tokens the batch GEMV streams faster.
bool use_gemm_ws(const QMatrix &q, size_t M) { return M >= 9 && gemm_ws_supported(q, M); }

bool use_gemm_tc(const QMatrix &q, size_t M, const float *X, size_t ldx) {
    return M >= kTcMinRows && gemm_tc_supported(q) && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && ldx % 4 == 0;
}

// Tensor cores for big matrices (the lm_head).  Below kTcGemvMinRows a GEMV is latency-bound:
// the CUDA-core batch kernel (all weight loads in flight at once, split-K over warps) finishes
// first at every batch size, and the tensor-core kernel's fixed start-up (digit operand, ring
// fill, TMEM) does not pay for itself.  Measured on B200 (graph replay, device time): int8
// 12288 x 2048 at batch 8 takes 22.9 us on the batch kernel vs 25.0 us on the tensor cores,
// 4096 x 2048 9.8 vs 18.1 us; the lm_head (151936 rows) is the other way round.
bool use_gemv_tc(const pyxis_cuda_ctx *ctx, const QMatrix &q, size_t b, const float *xb, size_t ldx) {
    const bool tc_ok = q.N >= kTcGemvMinRows || !gemv_batch_supported(q, b, ctx->num_sms);
    return tc_ok && gemv_tc_supported(q, b, ctx->num_sms) && (reinterpret_cast<uintptr_t>(xb) & 15) == 0 &&
           (b == 1 || ldx % 4 == 0);
}
}  // namespace

bool pyxis::head_gemv_keys(pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, const float *X, size_t M, size_t ldx,
                           size_t N, size_t K, float *Y, size_t ldy, int64_t index_base, uint64_t *keys,
                           cudaStream_t st, cudaError_t *err) {
    const QMatrix q = qmatrix(w, N, K);
    if (M == 0 || M > 8 || !use_gemv_tc(ctx, q, M, X, ldx)) return false;
    PdlScope pdl;
    *err = launch_gemv_tc(q, X, M, ldx, Y, ldy, ctx->tcg_scratch, ctx->tcg_scratch_bytes, ctx->d_err, ctx->num_sms,
                          st, keys, (long long)index_base);
    return true;
}

int pyxis::run_matmul(pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, const float *X, size_t M, size_t ldx,
                      size_t out_features, size_t in_features, float *Y, size_t ldy, void *workspace,
                      size_t workspace_bytes, cudaStream_t st) {
    // Programmatic dependent launch: a GEMV may start while the kernel before it on the stream
    // finishes, streaming its (immutable) weights; every kernel launched this way reads x and
    // writes y only after griddepcontrol.wait, i.e. after its predecessor has completed.
    PdlScope pdl;
    QMatrix q = qmatrix(w, out_features, in_features);
    if (use_gemm_ws(q, M)) {
        const size_t need = gemm_ws_workspace_bytes(M, out_features, in_features, ctx->num_sms, 0);
        if (!workspace) {
            // the context's workspace: x's fp16 copies, the rest for split-K partial sums
            const size_t want = gemm_ws_workspace_bytes(M, out_features, in_features, ctx->num_sms, kWsPartialCap);
            int rc = ensure_ctx_workspace(ctx, want, st);
            if (rc) return rc;
            workspace = ctx->ws;
            workspace_bytes = ctx->ws_cap;
        } else if (workspace_bytes < need) {
            return fail(PYXIS_EINVAL, "workspace of %zu bytes < %zu needed", workspace_bytes, need);
        } else if (reinterpret_cast<uintptr_t>(workspace) & 255) {
            return fail(PYXIS_EINVAL, "workspace must be 256-byte aligned");
        }
        cudaError_t e = launch_gemm_ws(q, X, M, ldx, Y, ldy, workspace, workspace_bytes, ctx->ws_tickets,
                                       ctx->ws_tickets_n, ctx->d_err, ctx->num_sms, st);
        if (e != cudaSuccess) return cuda_fail(e, "weight-streaming matmul launch");
        return PYXIS_OK;
    }
    if (use_gemm_tc(q, M, X, ldx)) {
        const size_t need = gemm_tc_workspace_bytes(M, in_features);
        if (!workspace) {
            // the context's own workspace also holds split-K partials when they help
            const size_t want = gemm_tc_workspace_bytes_splitk(M, out_features, in_features, w->block_size == in_features,
                                                               w->block_size, ctx->num_sms);
            int rc = ensure_ctx_workspace(ctx, want, st);
            if (rc) return rc;
            workspace = ctx->ws;
            workspace_bytes = ctx->ws_cap;
        } else if (workspace_bytes < need) {
            return fail(PYXIS_EINVAL, "workspace of %zu bytes < %zu needed", workspace_bytes, need);
        } else if (reinterpret_cast<uintptr_t>(workspace) & 255) {
            return fail(PYXIS_EINVAL, "workspace must be 256-byte aligned");
        }
        cudaError_t e = launch_gemm_tc(q, X, M, ldx, Y, ldy, workspace, workspace_bytes, ctx->d_err, ctx->num_sms, st);
        if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMM launch");
        return PYXIS_OK;
    }
    for (size_t m0 = 0; m0 < M; m0 += 8) {
        size_t b = M - m0 < 8 ? M - m0 : 8;
        const float *xb = X + m0 * ldx;
        cudaError_t e;
        if (use_gemv_tc(ctx, q, b, xb, ldx))
            e = launch_gemv_tc(q, xb, b, ldx, Y + m0 * ldy, ldy, ctx->tcg_scratch, ctx->tcg_scratch_bytes, ctx->d_err,
                               ctx->num_sms, st);
        else
            e = launch_gemv(q, xb, b, ldx, Y + m0 * ldy, ldy, ctx->d_err, ctx->num_sms, st);
        if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
    }
    return PYXIS_OK;
}


extern "C" {

const char *pyxis_cuda_last_error(void) { return g_last_error.c_str(); }

uint32_t pyxis_cuda_abi_version(void) { return (1u << 16) | 0u; }

int pyxis_cuda_init(int device, pyxis_cuda_ctx **out) {
    if (!out) return fail(PYXIS_EINVAL, "null output pointer");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(PYXIS_ENODEV, "no CUDA device (%s)", cudaGetErrorString(e));
    }
    if (device < 0 || device >= count) return fail(PYXIS_ENODEV, "device %d out of range (%d devices)", device, count);
    cudaDeviceProp prop;
    PYXIS_CUDA_TRY(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(PYXIS_ENODEV, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
                    prop.major, prop.minor);
    DeviceGuard g(device);
    auto *ctx = new (std::nothrow) pyxis_cuda_ctx{};
    if (!ctx) return fail(PYXIS_ENOMEM, "host allocation failed");
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete ctx;
        return cuda_fail(e, "cudaStreamCreate");
    }
    size_t ab = argmax_scratch_bytes(kArgmaxMaxRows);
    e = cudaMalloc(&ctx->amax_mem, ab);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->amax_mem, 0, ab, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        pyxis_cuda_destroy(ctx);
        return cuda_fail(e, "argmax scratch");
    }
    e = cudaMalloc(&ctx->d_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(int));
    ctx->tcg_scratch_bytes = gemv_tc_scratch_bytes(ctx->num_sms);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->tcg_scratch, ctx->tcg_scratch_bytes);
    if (e == cudaSuccess) e = cudaMemset(ctx->tcg_scratch, 0, ctx->tcg_scratch_bytes);
    if (e != cudaSuccess) {
        pyxis_cuda_destroy(ctx);
        return cuda_fail(e, "device error flag");
    }
    ctx->ws_tickets_n = kWsTickets;
    e = cudaMalloc(&ctx->ws_tickets, kWsTickets * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(ctx->ws_tickets, 0, kWsTickets * sizeof(unsigned));
    if (e == cudaSuccess) {
        const int rc = grow_workspace(ctx, kDefaultWorkspace);
        if (rc) {
            pyxis_cuda_destroy(ctx);
            return rc;
        }
    }
    if (e != cudaSuccess) {
        pyxis_cuda_destroy(ctx);
        return cuda_fail(e, "workspace tickets");
    }
    ctx->amax.partial = (uint64_t *)ctx->amax_mem;
    ctx->amax.ticket = (unsigned *)((uint8_t *)ctx->amax_mem + (size_t)kArgmaxMaxRows * kArgmaxMaxCtasPerRow * sizeof(uint64_t));
    *out = ctx;
    return PYXIS_OK;
}

int pyxis_cuda_destroy(pyxis_cuda_ctx *ctx) {
    if (!ctx) return PYXIS_OK;
    DeviceGuard g(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->dx);
    cudaFree(ctx->dy);
    cudaFree(ctx->ws);
    cudaFree(ctx->amax_mem);
    cudaFree(ctx->d_err);
    cudaFree(ctx->tcg_scratch);
    cudaFree(ctx->ws_tickets);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return PYXIS_OK;
}

void *pyxis_cuda_stream(pyxis_cuda_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int pyxis_cuda_synchronize(pyxis_cuda_ctx *ctx) {
    if (!ctx) return fail(PYXIS_EINVAL, "null context");
    DeviceGuard g(ctx->device);
    PYXIS_CUDA_TRY(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return PYXIS_OK;
}

int pyxis_cuda_quantize(pyxis_cuda_ctx *ctx, const void *src, int src_dtype, int src_on_device,
                        size_t n, size_t block_size, int qtype, pyxis_cuda_weights **out) {
    if (!ctx || !out) return fail(PYXIS_EINVAL, "null context or output pointer");
    *out = nullptr;
    if (block_size == 0) return fail(PYXIS_EINVAL, "block_size must be > 0 (assert!, src/weights.rs:95)");
    if (qtype != PYXIS_QTYPE_INT8 && qtype != PYXIS_QTYPE_INT4) return fail(PYXIS_EINVAL, "unknown qtype %d", qtype);
    if (src_dtype != PYXIS_DTYPE_F32 && src_dtype != PYXIS_DTYPE_BF16) return fail(PYXIS_EINVAL, "unknown src dtype %d", src_dtype);
    if (!src && n) return fail(PYXIS_EINVAL, "null source");
    DeviceGuard g(ctx->device);
    if (src_on_device && n) {  // a device source must live on this context's device
        cudaPointerAttributes pa;
        cudaError_t pe = cudaPointerGetAttributes(&pa, src);
        if (pe != cudaSuccess || (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged) ||
            (pa.type == cudaMemoryTypeDevice && pa.device != ctx->device)) {
            cudaGetLastError();
            return fail(PYXIS_EINVAL, "quantize: the device source is not memory of device %d", ctx->device);
        }
    }
    pyxis_cuda_weights *w = nullptr;
    int rc = alloc_weights(ctx, qtype, n, block_size, &w);
    if (rc) return rc;
    const size_t esize = src_dtype == PYXIS_DTYPE_F32 ? 4 : 2;
    const void *dsrc = src;
    void *tmp = nullptr;
    cudaError_t e = cudaSuccess;
    if (!src_on_device && n) {
        e = cudaMalloc(&tmp, n * esize);
        if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, src, n * esize, cudaMemcpyHostToDevice, ctx->stream);
        dsrc = tmp;
    }
    if (e == cudaSuccess)
        e = launch_quantize(dsrc, src_dtype, n, block_size, qtype, w->data, w->scales, ctx->num_sms, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
        pyxis_cuda_weights_free(w);
        return cuda_fail(e, "quantize");
    }
    *out = w;
    return PYXIS_OK;
}

int pyxis_cuda_weights_upload(pyxis_cuda_ctx *ctx, int qtype, const void *data, const float *scales,
                              size_t n, size_t block_size, pyxis_cuda_weights **out) {
    if (!ctx || !out) return fail(PYXIS_EINVAL, "null context or output pointer");
    *out = nullptr;
    if (!is_qtype(qtype)) return fail(PYXIS_EINVAL, "unknown qtype %d", qtype);
    if (!is_dense(qtype) && block_size == 0) return fail(PYXIS_EINVAL, "block_size must be > 0");
    if (n && (!data || (!is_dense(qtype) && !scales))) return fail(PYXIS_EINVAL, "null data or scales");
    DeviceGuard g(ctx->device);
    pyxis_cuda_weights *w = nullptr;
    int rc = alloc_weights(ctx, qtype, n, block_size, &w);
    if (rc) return rc;
    cudaError_t e = cudaSuccess;
    if (w->data_bytes) e = cudaMemcpyAsync(w->data, data, w->data_bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess && w->num_scales)
        e = cudaMemcpyAsync(w->scales, scales, w->num_scales * sizeof(float), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        pyxis_cuda_weights_free(w);
        return cuda_fail(e, "weights upload");
    }
    *out = w;
    return PYXIS_OK;
}

int pyxis_cuda_weights_upload_q8_0(pyxis_cuda_ctx *ctx, const void *blocks, int blocks_on_device, size_t n,
                                   pyxis_cuda_weights **out) {
    if (!ctx || !out) return fail(PYXIS_EINVAL, "null context or output pointer");
    *out = nullptr;
    if (n && !blocks) return fail(PYXIS_EINVAL, "null blocks");
    constexpr size_t kQ8Block = 32, kQ8Bytes = 34;  // src/gguf.rs:246-247
    const size_t nb = div_ceil(n, kQ8Block);
    if (nb > SIZE_MAX / kQ8Bytes) return fail(PYXIS_EINVAL, "tensor too large");  // checked_byte_len
    DeviceGuard g(ctx->device);
    if (blocks_on_device && n) {
        cudaPointerAttributes pa;
        cudaError_t pe = cudaPointerGetAttributes(&pa, blocks);
        if (pe != cudaSuccess || (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged) ||
            (pa.type == cudaMemoryTypeDevice && pa.device != ctx->device)) {
            cudaGetLastError();
            return fail(PYXIS_EINVAL, "upload_q8_0: the blocks are not memory of device %d", ctx->device);
        }
    }
    pyxis_cuda_weights *w = nullptr;
    int rc = alloc_weights(ctx, PYXIS_QTYPE_INT8, n, kQ8Block, &w);
    if (rc) return rc;
    const void *dblocks = blocks;
    void *tmp = nullptr;
    cudaError_t e = cudaSuccess;
    if (!blocks_on_device && n) {
        e = cudaMalloc(&tmp, nb * kQ8Bytes);
        if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, blocks, nb * kQ8Bytes, cudaMemcpyHostToDevice, ctx->stream);
        dblocks = tmp;
    }
    if (e == cudaSuccess && n)
        e = launch_q8_0_unpack(reinterpret_cast<const uint8_t *>(dblocks), n, reinterpret_cast<int8_t *>(w->data),
                               w->scales, ctx->num_sms, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
        pyxis_cuda_weights_free(w);
        return cuda_fail(e, "upload_q8_0");
    }
    *out = w;
    return PYXIS_OK;
}

int pyxis_cuda_weights_info(const pyxis_cuda_weights *w, int *qtype, size_t *n, size_t *bs,
                            size_t *data_bytes, size_t *num_scales) {
    if (!w) return fail(PYXIS_EINVAL, "null weights");
    if (qtype) *qtype = w->qtype;
    if (n) *n = w->num_elements;
    if (bs) *bs = w->block_size;
    if (data_bytes) *data_bytes = w->data_bytes;
    if (num_scales) *num_scales = w->num_scales;
    return PYXIS_OK;
}

int pyxis_cuda_weights_download(const pyxis_cuda_weights *w, void *data, float *scales) {
    if (!w) return fail(PYXIS_EINVAL, "null weights");
    DeviceGuard g(w->device);
    if (data && w->data_bytes) PYXIS_CUDA_TRY(cudaMemcpy(data, w->data, w->data_bytes, cudaMemcpyDeviceToHost), "download data");
    if (scales && w->num_scales)
        PYXIS_CUDA_TRY(cudaMemcpy(scales, w->scales, w->num_scales * sizeof(float), cudaMemcpyDeviceToHost), "download scales");
    return PYXIS_OK;
}

int pyxis_cuda_weights_device_ptrs(const pyxis_cuda_weights *w, const void **data, const float **scales) {
    if (!w) return fail(PYXIS_EINVAL, "null weights");
    if (data) *data = w->data;
    if (scales) *scales = w->scales;
    return PYXIS_OK;
}

int pyxis_cuda_weights_free(pyxis_cuda_weights *w) {
    if (!w) return PYXIS_OK;
    DeviceGuard g(w->device);
    cudaFree(w->data);
    delete w;
    return PYXIS_OK;
}

size_t pyxis_cuda_matmul_workspace_size(size_t M, size_t in_features) {
    size_t need = M >= kTcMinRows ? gemm_tc_workspace_bytes(M, in_features) : 0;
    if (M >= 2 && M <= 64 && in_features % 128 == 0) {  // the weight-streaming matmul's x copies
        QMatrix probe{PYXIS_QTYPE_INT4, nullptr, nullptr, 32, 1, in_features};
        if (gemm_ws_supported(probe, M)) need = std::max(need, gemm_ws_workspace_bytes(M, 1, in_features, 1, 0));
    }
    return need;
}

int pyxis_cuda_reserve_workspace(pyxis_cuda_ctx *ctx, size_t bytes) {
    if (!ctx) return fail(PYXIS_EINVAL, "null context");
    DeviceGuard g(ctx->device);
    PYXIS_CUDA_TRY(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return grow_workspace(ctx, bytes);
}

int pyxis_cuda_check_device_error(pyxis_cuda_ctx *ctx) {
    if (!ctx) return fail(PYXIS_EINVAL, "null context");
    DeviceGuard g(ctx->device);
    PYXIS_CUDA_TRY(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    PYXIS_CUDA_TRY(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    int code = 0;
    PYXIS_CUDA_TRY(cudaMemcpy(&code, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost), "read device error flag");
    if (code == 0) return PYXIS_OK;
    PYXIS_CUDA_TRY(cudaMemset(ctx->d_err, 0, sizeof(int)), "clear device error flag");
    return fail(PYXIS_ETIMEOUT, "a kernel's bounded wait ran out (code 0x%x); its outputs are invalid", code);
}

int pyxis_cuda_matmul_dev(pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, const float *X, size_t M,
                          size_t ldx, size_t out_features, size_t in_features, float *Y, size_t ldy,
                          void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_matmul(ctx, w, out_features, in_features);
    if (rc) return rc;
    if (M == 0 || out_features == 0) return PYXIS_OK;
    if (!X || !Y) return fail(PYXIS_EINVAL, "null X or Y");
    if (M > 1 && (ldx < in_features || ldy < out_features)) return fail(PYXIS_EINVAL, "row stride smaller than the row");
    DeviceGuard g(ctx->device);
    return run_matmul(ctx, w, X, M, ldx, out_features, in_features, Y, ldy, workspace, workspace_bytes,
                      pick_stream(ctx, stream));
}

const char *pyxis_cuda_matmul_kernel(pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, size_t M,
                                     size_t out_features, size_t in_features) {
    if (!ctx || !w || check_matmul(ctx, w, out_features, in_features) || M == 0) return "";
    QMatrix q = qmatrix(w, out_features, in_features);
    // 256-byte aligned, contiguous x: the layout the device-pointer form's callers pass
    const float *x = reinterpret_cast<const float *>(static_cast<uintptr_t>(256));
    if (use_gemm_ws(q, M)) return "gemm_ws_kernel";
    if (use_gemm_tc(q, M, x, in_features)) return "gemm_tc_kernel";
    const size_t b = M < 8 ? M : 8;
    if (use_gemv_tc(ctx, q, b, x, in_features)) return "gemv_tc_i8_kernel";
    return gemv_kernel_name(q, b, ctx->num_sms);
}

// The device address of page-locked host memory that the current device can store to
// (cudaHostAlloc / cudaMallocHost under unified addressing, or cudaHostRegister'ed memory mapped
// for this device); NULL for pageable memory and device memory.
static void *mapped_host(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();  // not a pointer CUDA knows: take the copy path
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

int pyxis_cuda_matmul_batch(pyxis_cuda_ctx *ctx, const float *input, size_t M, const pyxis_cuda_weights *w,
                            size_t out_features, size_t in_features, float *out) {
    int rc = check_matmul(ctx, w, out_features, in_features);
    if (rc) return rc;
    if (M == 0 || out_features == 0) return PYXIS_OK;
    if (!input || !out) return fail(PYXIS_EINVAL, "null input or output");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lock(ctx->host_mu);
    rc = grow(&ctx->dx, &ctx->dx_cap, M * in_features);
    if (rc) return rc;
    // The GEMV kernels store each output element once, with plain stores from whole warps: into a
    // page-locked output they write across PCIe while the kernel runs, instead of in a copy after
    // it (the lm_head at 8 rows: 4.9 MB of results that took a 97 us copy behind a 71 us kernel).
    // The tensor-core products (workspace partial sums, their own epilogues) keep the copy.
    const QMatrix q = qmatrix(w, out_features, in_features);
    float *direct = (use_gemm_ws(q, M) || use_gemm_tc(q, M, ctx->dx, in_features))
                        ? nullptr : static_cast<float *>(mapped_host(out));
    if (!direct) {
        rc = grow(&ctx->dy, &ctx->dy_cap, M * out_features);
        if (rc) return rc;
    }
    PYXIS_CUDA_TRY(cudaMemcpyAsync(ctx->dx, input, M * in_features * sizeof(float), cudaMemcpyHostToDevice, ctx->stream), "copy input");
    rc = pyxis_cuda_matmul_dev(ctx, w, ctx->dx, M, in_features, out_features, in_features, direct ? direct : ctx->dy,
                               out_features, nullptr, 0, nullptr);
    if (rc) return rc;
    if (!direct)
        PYXIS_CUDA_TRY(cudaMemcpyAsync(out, ctx->dy, M * out_features * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream), "copy output");
    PYXIS_CUDA_TRY(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return PYXIS_OK;
}

int pyxis_cuda_matmul(pyxis_cuda_ctx *ctx, const float *input, const pyxis_cuda_weights *w,
                      size_t out_features, size_t in_features, float *out) {
    return pyxis_cuda_matmul_batch(ctx, input, 1, w, out_features, in_features, out);
}

int pyxis_cuda_argmax_dev(pyxis_cuda_ctx *ctx, const float *values, size_t M, size_t n, size_t ld,
                          int64_t index_base, int32_t *idx, float *val, void *stream) {
    if (!ctx) return fail(PYXIS_EINVAL, "null context");
    if (M == 0) return PYXIS_OK;
    if (n == 0) return fail(PYXIS_EINVAL, "argmax of an empty row (assert!, src/output_head.rs:31)");
    if (n > 0xFFFFFFFFull) return fail(PYXIS_EINVAL, "row too long for argmax (%zu)", n);
    if (M > (size_t)kArgmaxMaxRows) return fail(PYXIS_EINVAL, "argmax: %zu rows > %d per call", M, kArgmaxMaxRows);
    if (M > 1 && ld < n) return fail(PYXIS_EINVAL, "row stride smaller than the row");
    if (!values || !idx) return fail(PYXIS_EINVAL, "null values or idx");
    if (index_base < 0 || index_base + (int64_t)n - 1 > (int64_t)INT32_MAX)
        return fail(PYXIS_EINVAL, "argmax: index_base + n - 1 outside [0, 2^31 - 1] (the int32 index)");
    DeviceGuard g(ctx->device);
    cudaError_t e = launch_argmax_scratch(values, M, n, ld, index_base, idx, val, ctx->amax, ctx->num_sms,
                                          pick_stream(ctx, stream));
    if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
    return PYXIS_OK;
}

}  // extern "C"
