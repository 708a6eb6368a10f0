// gemv_ring.cu -- batch-1 decode GEMV that streams weight rows through a shared-memory ring.
//
// y[n] = sum_k x[k] * q[n, k] * scale(n, k) (src/matmul.rs:67-96 for one input row), HBM-bound:
// every packed weight byte is read once.  The bytes in flight, not the arithmetic, set the speed,
// so one persistent CTA per SM splits the work:
//   warp 12 (producer)  cp.async.bulk copies of whole row tiles -- RT consecutive rows are one
//                       contiguous block of the reference layout, and their group scales another
//                       -- into an S-stage ring (up to ~144 KB in flight per SM), one mbarrier
//                       with a transaction count per stage;
//   warps 0-11          consumers.  A team of W_t warps covers one row; thread t of a team owns
//                       the 16-byte chunks t, t + 32 W_t, ... of every row, so its slice of x stays
//                       in registers for the whole kernel.  Each stage is read from shared memory
//                       once (consecutive lanes read consecutive chunks: no bank conflicts),
//                       decoded to exact floats, multiplied with paired fp32 FMAs, reduced with
//                       warp shuffles (and a named barrier across a team's warps).
// Tiles go to CTAs round-robin.  Every wait is bounded; a wait that runs out records an error in
// the context's device flag, and the CTA finishes its loop without touching the missing data.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace pyxis {

// Shared with gemv.cu: dot product of one 16-byte chunk with its x values.
template <int QT>
PYXIS_DEVINL float ring_chunk_dot(const uint4 w, const float2 *x) {
    float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    if (QT == kQInt8) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 q01, q23;
            i8x4_to_f32(ws[i], q01, q23);
            a0 = ffma2(x[2 * i], q01, a0);
            a1 = ffma2(x[2 * i + 1], q23, a1);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 e01, e23, e45, e67;
            u4x8_to_f32(ws[i], e01, e23, e45, e67);
            a0 = ffma2(x[4 * i], e01, a0);
            a1 = ffma2(x[4 * i + 1], e23, a1);
            a0 = ffma2(x[4 * i + 2], e45, a0);
            a1 = ffma2(x[4 * i + 3], e67, a1);
        }
    }
    a0 = fadd2(a0, a1);
    return a0.x + a0.y;
}

namespace {

constexpr int kConsumerWarps = 12;
constexpr int kRingThreads = (kConsumerWarps + 1) * 32;  // 416
constexpr int kMaxStages = 8;
constexpr uint32_t kRingBytes = 160 * 1024;
constexpr uint32_t kRingSmem = kRingBytes + 2 * kMaxStages * 8 + kConsumerWarps * 4 + 256;
constexpr uint64_t kRingTimeoutNs = 2000000000ull;
enum { kErrRingProducer = 0x201, kErrRingConsumer = 0x202, kErrRingDrain = 0x203 };

enum { kScaleRow = 0, kScaleChunk = 1 };

struct RingParams {
    const uint8_t *W;
    const float *S;
    const float *x;
    float *y;
    int N, K;
    int row_bytes;
    int team_warps;     // W_t
    int rows_per_pass;  // kConsumerWarps / W_t
    int rt;             // rows per tile, a multiple of rows_per_pass
    int num_tiles;
    int stages;
    uint32_t stage_bytes;
    uint32_t scale_off;  // scales' offset within a stage (kScaleChunk)
    int blocks_per_row;
    int chunks_per_block;
    int *err;
};

PYXIS_DEVINL void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(tc::smem_u32(dst)), "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

PYXIS_DEVINL void named_bar(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <int QT, int CPL, int SMODE>
__global__ void __maxnreg__(152) gemv_ring_kernel(const RingParams p) {
    constexpr int EPC = QT == kQInt8 ? 16 : 32;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kRingBytes);
    uint64_t *empty = full + kMaxStages;
    float *red = reinterpret_cast<float *>(empty + kMaxStages);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(red + kConsumerWarps);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], kConsumerWarps);
        }
        *abort_flag = 0;
        tc::fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            int issued = 0;
            for (int i = 0;; ++i) {
                const int tile = blockIdx.x + i * gridDim.x;
                if (tile >= p.num_tiles) break;
                const int s = i % p.stages;
                if (i >= p.stages &&
                    !tc::mbar_wait_bounded(&empty[s], ((i / p.stages) - 1) & 1, abort_flag, p.err, kErrRingProducer,
                                           kRingTimeoutNs))
                    break;
                const int row0 = tile * p.rt;
                const int rows = min(p.rt, p.N - row0);
                const uint32_t wbytes = (uint32_t)rows * (uint32_t)p.row_bytes;
                const uint32_t sbytes = SMODE == kScaleChunk ? (uint32_t)rows * p.blocks_per_row * 4u : 0u;
                uint8_t *st = ring + (size_t)s * p.stage_bytes;
                tc::mbar_arrive_expect_tx(&full[s], wbytes + sbytes);
                bulk_g2s(st, p.W + (size_t)row0 * p.row_bytes, wbytes, &full[s]);
                if (SMODE == kScaleChunk)
                    bulk_g2s(st + p.scale_off, p.S + (size_t)row0 * p.blocks_per_row, sbytes, &full[s]);
                ++issued;
            }
            if (*abort_flag) {  // let issued copies land before the CTA exits
                volatile int no_abort = 0;
                for (int j = issued > p.stages ? issued - p.stages : 0; j < issued; ++j)
                    tc::mbar_wait_bounded(&full[j % p.stages], (j / p.stages) & 1, &no_abort, p.err, kErrRingDrain,
                                          100000000ull);
            }
        }
    } else {
        // ---------------------------------------------------------------- consumers
        const int Wt = p.team_warps;
        const int team = warp / Wt, wt = warp - team * Wt;
        const int t = wt * 32 + lane;
        const int cstride = 32 * Wt;
        pdl_wait();  // x comes from the previous kernel; the producer's weight copies do not wait
        pdl_trigger();
        float2 xr[CPL][EPC / 2];
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const float4 *xp = reinterpret_cast<const float4 *>(p.x + (size_t)(t + j * cstride) * EPC);
#pragma unroll
            for (int v = 0; v < EPC / 4; ++v) {
                const float4 f = __ldg(xp + v);
                xr[j][2 * v] = f2(f.x, f.y);
                xr[j][2 * v + 1] = f2(f.z, f.w);
            }
        }
        const int passes = p.rt / p.rows_per_pass;
        for (int i = 0;; ++i) {
            const int tile = blockIdx.x + i * gridDim.x;
            if (tile >= p.num_tiles) break;
            const int s = i % p.stages;
            int ok = 1;
            if (lane == 0)
                ok = tc::mbar_wait_bounded(&full[s], (i / p.stages) & 1, abort_flag, p.err, kErrRingConsumer,
                                           kRingTimeoutNs);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            const uint8_t *st = ring + (size_t)s * p.stage_bytes;
            const int row0 = tile * p.rt;
            const int rows = min(p.rt, p.N - row0);
            for (int pass = 0; pass < passes; ++pass) {
                const int rl = pass * p.rows_per_pass + team;
                float acc = 0.f;
                if (ok && rl < rows) {
                    const uint8_t *wrow = st + (size_t)rl * p.row_bytes;
#pragma unroll
                    for (int j = 0; j < CPL; ++j) {
                        const int c = t + j * cstride;
                        const uint4 w = *reinterpret_cast<const uint4 *>(wrow + (size_t)c * 16);
                        const float d = ring_chunk_dot<QT>(w, xr[j]);
                        if (SMODE == kScaleChunk) {
                            const float sc = *reinterpret_cast<const float *>(
                                st + p.scale_off + ((size_t)rl * p.blocks_per_row + c / p.chunks_per_block) * 4);
                            acc = fmaf(sc, d, acc);
                        } else {
                            acc += d;
                        }
                    }
                }
                acc = warp_sum(acc);
                if (Wt == 1) {
                    if (lane == 0 && ok && rl < rows) {
                        const int row = row0 + rl;
                        p.y[row] = SMODE == kScaleRow ? acc * __ldg(p.S + row) : acc;
                    }
                } else {
                    if (lane == 0) red[warp] = acc;
                    named_bar(1 + team, 32 * Wt);
                    if (wt == 0 && lane == 0 && ok && rl < rows) {
                        float sum = 0.f;
                        for (int w = 0; w < Wt; ++w) sum += red[team * Wt + w];
                        const int row = row0 + rl;
                        p.y[row] = SMODE == kScaleRow ? sum * __ldg(p.S + row) : sum;
                    }
                    named_bar(1 + team, 32 * Wt);
                }
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&empty[s]);
        }
    }
    __syncwarp();
    __syncthreads();
}

}  // namespace

// ---------------------------------------------------------------------------------------------
struct RingPlan {
    bool ok = false;
    int smode = 0, cpl = 0, team = 1, rows_per_pass = 0, rt = 0, stages = 0;
    uint32_t stage_bytes = 0, scale_off = 0;
};

static RingPlan ring_plan(const QMatrix &w, int num_sms) {
    RingPlan pl;
    const int epc = w.qtype == kQInt8 ? 16 : 32;
    const size_t K = w.K, bs = w.block_size;
    if (K == 0 || K % epc || K > (1u << 20) || w.N > (size_t)INT32_MAX) return pl;
    if ((reinterpret_cast<uintptr_t>(w.data) & 15) || (reinterpret_cast<uintptr_t>(w.scales) & 15)) return pl;
    int smode;
    size_t bpr = 1;
    if (bs == K) smode = kScaleRow;
    else if (bs % epc == 0 && K % bs == 0 && (K / bs) % 4 == 0) { smode = kScaleChunk; bpr = K / bs; }
    else return pl;
    const int chunks = (int)(K / epc);
    if (chunks % 32) return pl;
    const int max_cpl = w.qtype == kQInt8 ? 4 : 2;  // <= 64 x registers per thread
    int team = 0, cpl = 0;
    for (int wt : {1, 2, 3, 4, 6, 12}) {
        if (chunks % (32 * wt)) continue;
        const int c = chunks / (32 * wt);
        if (c <= max_cpl) { team = wt; cpl = c; break; }
    }
    if (!team) return pl;
    const int row_bytes = (int)(w.qtype == kQInt8 ? K : K / 2);
    const int rpp = kConsumerWarps / team;
    const uint32_t row_total = (uint32_t)row_bytes + (smode == kScaleChunk ? (uint32_t)bpr * 4u : 0u);
    int k = 1;
    for (int kk = 4; kk >= 1; --kk) {
        const uint32_t tb = (uint32_t)(rpp * kk) * row_total;
        const size_t tiles = (w.N + rpp * kk - 1) / (rpp * kk);
        if (tb <= 32 * 1024 && tiles >= (size_t)2 * num_sms) { k = kk; break; }
    }
    const int rt = rpp * k;
    const uint32_t wbytes = (uint32_t)rt * row_bytes;
    const uint32_t sbytes = smode == kScaleChunk ? (uint32_t)rt * (uint32_t)bpr * 4u : 0u;
    const uint32_t stage = ((wbytes + 127) & ~127u) + ((sbytes + 127) & ~127u);
    const int stages = std::min<int>(kMaxStages, (int)(kRingBytes / stage));
    if (stages < 2) return pl;
    pl.ok = true;
    pl.smode = smode;
    pl.cpl = cpl;
    pl.team = team;
    pl.rows_per_pass = rpp;
    pl.rt = rt;
    pl.stages = stages;
    pl.stage_bytes = stage;
    pl.scale_off = (wbytes + 127) & ~127u;
    return pl;
}

bool gemv_ring_supported(const QMatrix &w, int num_sms) { return ring_plan(w, num_sms).ok; }

template <int QT, int CPL, int SMODE>
static cudaError_t run_ring(const RingParams &p, int grid, cudaStream_t st) {
    auto kern = gemv_ring_kernel<QT, CPL, SMODE>;
    static const bool attr =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kRingSmem) == cudaSuccess;
    if (!attr) return cudaErrorInvalidConfiguration;
    return launch_kernel(kern, dim3(grid), dim3(kRingThreads), kRingSmem, st, p);
}

template <int QT, int SMODE>
static cudaError_t dispatch_ring(int cpl, const RingParams &p, int grid, cudaStream_t st) {
    switch (cpl) {
    case 1: return run_ring<QT, 1, SMODE>(p, grid, st);
    case 2: return run_ring<QT, 2, SMODE>(p, grid, st);
    case 3: return QT == kQInt8 ? run_ring<QT, 3, SMODE>(p, grid, st) : cudaErrorInvalidValue;
    default: return QT == kQInt8 ? run_ring<QT, 4, SMODE>(p, grid, st) : cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv_ring(const QMatrix &w, const float *x, float *y, int *err, int num_sms, cudaStream_t st) {
    const RingPlan pl = ring_plan(w, num_sms);
    if (!pl.ok) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(x) & 15) return cudaErrorInvalidValue;
    RingParams p{};
    p.W = w.data;
    p.S = w.scales;
    p.x = x;
    p.y = y;
    p.N = (int)w.N;
    p.K = (int)w.K;
    p.row_bytes = (int)(w.qtype == kQInt8 ? w.K : w.K / 2);
    p.team_warps = pl.team;
    p.rows_per_pass = pl.rows_per_pass;
    p.rt = pl.rt;
    p.num_tiles = (int)((w.N + pl.rt - 1) / pl.rt);
    p.stages = pl.stages;
    p.stage_bytes = pl.stage_bytes;
    p.scale_off = pl.scale_off;
    p.blocks_per_row = pl.smode == kScaleChunk ? (int)(w.K / w.block_size) : 1;
    p.chunks_per_block = pl.smode == kScaleChunk ? (int)(w.block_size / (w.qtype == kQInt8 ? 16 : 32)) : 1;
    p.err = err;
    const int grid = std::max(1, std::min(num_sms, p.num_tiles));
    if (w.qtype == kQInt8)
        return pl.smode == kScaleRow ? dispatch_ring<kQInt8, kScaleRow>(pl.cpl, p, grid, st)
                                     : dispatch_ring<kQInt8, kScaleChunk>(pl.cpl, p, grid, st);
    return pl.smode == kScaleRow ? dispatch_ring<kQInt4, kScaleRow>(pl.cpl, p, grid, st)
                                 : dispatch_ring<kQInt4, kScaleChunk>(pl.cpl, p, grid, st);
}

}  // namespace pyxis
