/*
 * pyxis_cuda.h -- C ABI of the B200 (sm_100a) backend for pyxis's quantized matmul hot path.
 *
 * This is the boundary a `--cuda` backend binds from Rust (a cuda_matmul.rs binding module and a
 * build.rs that runs the nvcc build), the way src/metal_matmul.rs binds Metal.  It replaces, one
 * for one:
 *
 *   Weights::quantize_int8 / quantize_int4   src/weights.rs:94-118, :120-151  -> pyxis_cuda_quantize
 *   dequantize_weights (bf16 -> f32 arm)     src/model.rs:535-538             -> src_dtype BF16
 *   Weights::to_metal (persistent buffers)   src/weights.rs:65-92             -> pyxis_cuda_weights_upload
 *   read_q8_0_weights (Int8, block 32)       src/gguf.rs:245-271              -> pyxis_cuda_weights_upload_q8_0
 *   Weights::F32 / Weights::Bf16 rows        src/weights.rs:6-8,
 *   (MetalF32 / MetalBf16 buffers)           src/metal_matmul.rs:28-184       -> pyxis_cuda_weights_upload
 *                                                                                (qtype F32 / BF16)
 *   matmul(input, &Weights, out, in)         src/matmul.rs:21-97              -> pyxis_cuda_matmul
 *   MetalMatmul::new / OnceLock singleton    src/metal_matmul.rs:199-219,
 *                                            src/matmul.rs:6-19               -> pyxis_cuda_init
 *   output_head::argmax                      src/output_head.rs:30-44         -> pyxis_cuda_argmax_dev
 *
 * Conventions
 *  - Every function returns PYXIS_OK (0) or a positive pyxis_status; pyxis_cuda_last_error()
 *    returns a message for the calling thread's last failure.  The reference panics on the same
 *    conditions (shape asserts, src/matmul.rs:27-50); a Rust wrapper maps nonzero to panic!.
 *  - Weights live in HBM in the reference's own byte layout: int8 = num_elements i8, int4 =
 *    ceil(num_elements/2) bytes (element i in the low nibble of byte i/2 when i is even, high
 *    nibble when odd, stored as q+8), scales = ceil(num_elements/block_size) f32, blocks running
 *    over the flattened row-major [out_features, in_features] index.
 *  - A context is bound to one device and owns one CUDA stream.  Its kernels share the
 *    context's scratch (the tensor-core GEMV's split-K slots, the GEMM workspace, the argmax
 *    scratch), so its launches must not overlap on the GPU: issue `_dev` calls on one stream or
 *    on streams ordered by events, from one host thread at a time.  The host-pointer entry
 *    points run on the context's stream and return after it drains; pyxis_cuda_matmul and
 *    pyxis_cuda_matmul_batch hold a per-context lock for their staging buffers, so several host
 *    threads may call them at once (the calls run one after another).
 *  - `_dev` entry points take device pointers and a cudaStream_t (NULL = the context's stream;
 *    pass cudaStreamLegacy for the legacy default stream) and do not synchronize.  The host-pointer entry points copy in, compute and copy out, and
 *    return after the result is in host memory (src/metal_matmul.rs:311-354 behaves the same).
 */
#ifndef PYXIS_CUDA_H
#define PYXIS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    PYXIS_OK = 0,
    PYXIS_EINVAL = 1,   /* bad argument or shape mismatch (the reference's assert!s) */
    PYXIS_ENODEV = 2,   /* no CUDA device / not sm_100 (MetalMatmul::new -> None) */
    PYXIS_ECUDA = 3,    /* a CUDA runtime error */
    PYXIS_ENOMEM = 4,   /* device or host allocation failed */
    PYXIS_ETIMEOUT = 5, /* a bounded device-side wait gave up */
    PYXIS_EUNSUPPORTED = 6,
    PYXIS_ENCCL = 7     /* a collective of a multi-GPU communicator failed (pyxis_comm.h) */
} pyxis_status;

/* Weight layouts (enum Weights arms, src/weights.rs:6-21): the two quantized ones and the two
 * unquantized ones (F32: num_elements f32; BF16: num_elements u16 bf16 bit patterns, widened by
 * u32 << 16 in the dot, src/matmul.rs:289-295).  Unquantized weights have no scales. */
typedef enum {
    PYXIS_QTYPE_INT8 = 1,
    PYXIS_QTYPE_INT4 = 2,
    PYXIS_QTYPE_F32 = 3,
    PYXIS_QTYPE_BF16 = 4
} pyxis_qtype;

/* Source element types for quantisation: F32 (Weights::F32), BF16 (Weights::Bf16, widened by
 * u32 << 16 before quantising, src/model.rs:535-538). */
typedef enum { PYXIS_DTYPE_F32 = 1, PYXIS_DTYPE_BF16 = 2 } pyxis_dtype;

typedef struct pyxis_cuda_ctx pyxis_cuda_ctx;
typedef struct pyxis_cuda_weights pyxis_cuda_weights;

/* Message of the calling thread's last failure ("" if none).  Never NULL. */
const char *pyxis_cuda_last_error(void);

/* ABI version (major << 16 | minor). */
uint32_t pyxis_cuda_abi_version(void);

/* Create a context on `device` (MetalMatmul::new, src/metal_matmul.rs:199-219): checks the device
 * is sm_100, creates its stream.  PYXIS_ENODEV when there is no such device. */
int pyxis_cuda_init(int device, pyxis_cuda_ctx **ctx);
int pyxis_cuda_destroy(pyxis_cuda_ctx *ctx);
/* The context's stream, as a cudaStream_t. */
void *pyxis_cuda_stream(pyxis_cuda_ctx *ctx);
int pyxis_cuda_synchronize(pyxis_cuda_ctx *ctx);

/* Quantise and pack on the device, bit-exact with Weights::quantize_int8 (qtype INT8,
 * src/weights.rs:94-118) or Weights::quantize_int4 (qtype INT4, :120-151) applied to the f32
 * values of `src` (num_elements of src_dtype; host memory when src_on_device == 0, else a device
 * pointer on the context's device).  block_size > 0, any value (the model's policy is
 * in_features for int8 and 32 for int4, src/model.rs:20,520-530).  On success *w owns HBM.
 * The call runs on the context's stream, which does not wait for other streams: a device
 * source must be complete when the call is made.  It returns after the packing has finished. */
int pyxis_cuda_quantize(pyxis_cuda_ctx *ctx, const void *src, int src_dtype, int src_on_device,
                        size_t num_elements, size_t block_size, int qtype,
                        pyxis_cuda_weights **w);

/* Upload weights already in one of the layouts from host memory: a pack quantised on the host
 * or downloaded before (int8 -> num_elements bytes, int4 -> ceil(num_elements/2) bytes;
 * scales: ceil(num_elements/block_size) f32), or unquantized rows (qtype F32: num_elements f32,
 * BF16: num_elements u16; `scales` and `block_size` are ignored and may be NULL / 0). */
int pyxis_cuda_weights_upload(pyxis_cuda_ctx *ctx, int qtype, const void *data,
                              const float *scales, size_t num_elements, size_t block_size,
                              pyxis_cuda_weights **w);

/* read_q8_0_weights (src/gguf.rs:245-271) on the device: `blocks` is a GGUF Q8_0 tensor,
 * ceil(num_elements/32) blocks of 34 bytes (f16 scale, little-endian, then 32 int8), in host
 * memory (blocks_on_device == 0) or device memory of the context's device.  The result is INT8
 * weights with block_size 32: the codes truncated to num_elements and each scale widened to f32
 * exactly as half 2.7.1's f16::to_f32 does (a NaN keeps its payload and gets the quiet bit).
 * As for pyxis_cuda_quantize, device blocks must be complete when the call is made. */
int pyxis_cuda_weights_upload_q8_0(pyxis_cuda_ctx *ctx, const void *blocks, int blocks_on_device,
                                   size_t num_elements, pyxis_cuda_weights **w);

/* Layout of a weights handle (Weights::len, src/weights.rs:35-46 = num_elements). */
int pyxis_cuda_weights_info(const pyxis_cuda_weights *w, int *qtype, size_t *num_elements,
                            size_t *block_size, size_t *data_bytes, size_t *num_scales);

/* Copy the packed bytes and scales back to host buffers (sizes as in _upload). */
int pyxis_cuda_weights_download(const pyxis_cuda_weights *w, void *data, float *scales);

/* Device addresses of the packed bytes and scales (valid until pyxis_cuda_weights_free). */
int pyxis_cuda_weights_device_ptrs(const pyxis_cuda_weights *w, const void **data,
                                   const float **scales);

int pyxis_cuda_weights_free(pyxis_cuda_weights *w);

/* matmul(input, &weight, out_features, in_features) -> Vec<f32> (src/matmul.rs:21-97) with host
 * buffers: input [in_features] f32, out [out_features] f32.  Checks the reference's asserts
 * (:27-50): weight length == out_features * in_features.  Returns when out is filled. */
int pyxis_cuda_matmul(pyxis_cuda_ctx *ctx, const float *input, const pyxis_cuda_weights *w,
                      size_t out_features, size_t in_features, float *out);

/* Batched form with host buffers: M independent rows, input [M, in_features] -> out
 * [M, out_features] (the reference's prefill calls matmul once per position,
 * src/attention.rs:74-79).  When `out` is page-locked memory this device can address
 * (cudaHostAlloc / cudaMallocHost, or cudaHostRegister'ed and mapped) and the product runs on a
 * GEMV kernel (every M <= 8, and larger M that the tensor-core products do not take), the kernel
 * stores the results into it directly instead of through a device buffer and a copy; the values
 * are the same either way.  Pageable `out` takes the copy. */
int pyxis_cuda_matmul_batch(pyxis_cuda_ctx *ctx, const float *input, size_t M,
                            const pyxis_cuda_weights *w, size_t out_features, size_t in_features,
                            float *out);

/* Device-pointer form, asynchronous on `stream` (NULL: the context's stream).  X [M, in] f32
 * with row stride ldx (elements), Y [M, out] f32 with row stride ldy.  Kernels by shape:
 *  - M = 1: the decode GEMVs (CUDA cores; int8 one-scale-per-row matrices of >= 16384 rows on
 *    the tensor cores, kind::i8);
 *  - 9..64 rows of int4 / int8 with a scale per 32 values or int8 with one scale per row,
 *    in_features % 128 == 0: the weight-streaming tensor-core matmul;
 *  - other M <= 15: the GEMVs, 8 rows per launch; M >= 16 with int8/int4 weights: the tensor-core
 *    prefill GEMM.
 * The tensor-core products need `workspace` of pyxis_cuda_matmul_workspace_size() bytes (device
 * memory, 256-byte aligned).  A NULL workspace uses the context's, allocated at init and grown
 * when a product needs more (not allowed while the stream is being captured:
 * pyxis_cuda_reserve_workspace grows it beforehand); it also has room for split-K partial sums,
 * which a caller workspace of the minimum size lacks, so matrices with fewer 128-row tiles than
 * SMs run faster on it. */
int pyxis_cuda_matmul_dev(pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, const float *X,
                          size_t M, size_t ldx, size_t out_features, size_t in_features,
                          float *Y, size_t ldy, void *workspace, size_t workspace_bytes,
                          void *stream);

/* Workspace bytes pyxis_cuda_matmul_dev needs for M rows of in_features (0 for the GEMV). */
size_t pyxis_cuda_matmul_workspace_size(size_t M, size_t in_features);

/* Grows the context's own workspace to at least `bytes` (synchronizes the context's stream), so
 * that later pyxis_cuda_matmul_dev calls with a NULL workspace allocate nothing -- e.g. before
 * they are captured into a CUDA graph. */
int pyxis_cuda_reserve_workspace(pyxis_cuda_ctx *ctx, size_t bytes);

/* Synchronizes the context's device and reports whether a kernel's bounded device-side wait ran
 * out since the last check (PYXIS_ETIMEOUT; the outputs of that launch are invalid), clearing the
 * flag.  Kernels never spin without a limit: a stuck pipeline ends the launch instead. */
int pyxis_cuda_check_device_error(pyxis_cuda_ctx *ctx);

/* Diagnostics, no counterpart in the reference: the name of the kernel pyxis_cuda_matmul_dev
 * launches for M rows of a contiguous, 16-byte aligned x (for M > 8 on the GEMV path, the kernel
 * of each 8-row chunk).  "" for invalid arguments. */
const char *pyxis_cuda_matmul_kernel(pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, size_t M,
                                     size_t out_features, size_t in_features);

/* Row-wise argmax (src/output_head.rs:30-44: first index of the maximum under strict >) of
 * M rows of n f32 on the device: idx[M] int32 and val[M] f32 (val may be NULL).  `index_base`
 * is added to every index (a vocab shard's first row); with index_base > 0 the row is a shard
 * that does not hold index 0, so a NaN at its start is skipped like any other NaN (the reference's
 * "values[0] NaN wins" rule belongs to the shard with index_base 0).  index_base >= 0 and
 * index_base + n - 1 <= 2^31 - 1 (the indices are int32), else PYXIS_EINVAL.  Asynchronous on
 * `stream`. */
int pyxis_cuda_argmax_dev(pyxis_cuda_ctx *ctx, const float *values, size_t M, size_t n,
                          size_t ld, int64_t index_base, int32_t *idx, float *val, void *stream);

/* Row-wise argmax that allocates nothing: the same result as pyxis_cuda_argmax_dev, for callers
 * that cannot call cudaMalloc -- code running under an allocator it does not own (a framework's
 * caching allocator, a memory-capped or pre-reserved pool), or code that may not grow its device
 * footprint after start-up.  It has no counterpart in the reference and needs no context.
 *  - Runs on the calling thread's current device, on `stream` (NULL: that device's default
 *    stream); values, idx and val are device pointers, as in pyxis_cuda_argmax_dev.
 *  - Its scratch is a fixed 33 KiB array inside the library's device image (every device that
 *    uses it holds it until the process exits).  Every call looks up that array's device
 *    address on the current device (cudaGetSymbolAddress, which allocates nothing), so a
 *    device reset by the application does not leave a stale address behind; make the first call
 *    on each device before any stream capture (it loads the library's module there).
 *  - index_base >= 0 and index_base + n - 1 <= 2^31 - 1, as for pyxis_cuda_argmax_dev.
 *  - At most 64 rows per call (PYXIS_EINVAL beyond, rows of up to 2^32 - 1 values).
 *  - Every call shares the one array: calls that can overlap on the GPU (different streams
 *    without ordering, several host threads) race and must not be issued that way.
 *  - Allocates no memory: no cudaMalloc/cudaFree or allocating library calls; it clears its
 *    row counters with cudaMemsetAsync on `stream` before each launch. */
int pyxis_cuda_argmax_noalloc(const float *values, size_t M, size_t n, size_t ld, int64_t index_base,
                              int32_t *idx, float *val, void *stream);

#ifdef __cplusplus
}
#endif
#endif
