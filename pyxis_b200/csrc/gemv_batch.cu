// gemv_batch.cu -- matmul for 1-8 input rows on the CUDA cores (int4 groups, int8, and the
// unquantized f32 / bf16 rows), the decode shapes the tensor-core GEMV does not take:
// y[b, n] = sum_k x[b, k] * dequant(W)[n, k] (src/matmul.rs:21-97 for each of the B input rows).
//
// Layout of the work.  A row group is 4 weight rows.  A CTA takes `groups_cta` row groups at a
// time and splits each group's K range over `slices` warps: warp (g, s) streams the 16-byte
// chunks s*32 + lane, s*32 + lane + 32*slices, ... of its 4 rows, one chunk ahead of the math
// (the first chunk is requested before the kernel waits on its predecessor).  Each lane keeps 4
// rows x B tokens of paired accumulators (even / odd k), multiplies every decoded code pair with
// the token's x pair in one fma.f32x2, and the warp reduces its 32 (row, token) sums with halving
// exchanges (31 shuffles) so lane l ends with row l/8, token l%8.  The slices of a group are
// added in fixed order through shared memory: results do not depend on timing.
//
// x [B, K] arrives in shared memory by TMA (one 3-D box per token and 256 rows of 32 floats),
// 128-byte swizzled: the 16-byte unit u of each 128-byte row r sits at u ^ (r % 8), so the eight
// lanes of one shared-memory phase, reading eight consecutive chunks, hit eight different banks.
#include <algorithm>
#include <cstring>

#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace pyxis {
namespace {

constexpr int kRows = 4;        // weight rows per warp
constexpr int kMaxWarps = 12;   // 384 threads: up to 168 registers per thread
// 7-8 input rows need more than 168 registers (4 x 8 paired accumulators, 16 x quads, two
// chunks of codes): at most 8 warps, up to 255 registers
constexpr int max_warps(int B) { return B >= 7 ? 8 : kMaxWarps; }
constexpr int kXBoxRows = 256;  // TMA box limit per dimension (rows of 32 floats)
constexpr int kErrX = 0x401;    // x never arrived
constexpr uint64_t kTimeoutNs = 2000000000ull;
enum { kScaleRow = 0, kScaleChunk = 1, kScaleNone = 2 };  // per row / per block of whole chunks / none

struct BatchParams {
    const uint8_t *W;
    const float *S;
    float *Y;
    int N, K, ldy;
    int row_bytes;         // bytes per weight row
    int chunks;            // 16-byte chunks per row
    int blocks_per_row;    // scale blocks per row (chunk mode)
    int chunks_per_block;  // chunks per scale block (chunk mode)
    int cpb_shift;         // log2(chunks_per_block) when it is a power of two, else -1
    int slices;            // warps per row group
    int groups_cta;        // row groups per CTA item
    int items;             // ceil(row groups / groups_cta)
    int x_boxes;           // TMA boxes per token
    int box_rows;          // rows of 32 floats per box (multiple of 8)
    uint32_t tok_stride;   // bytes per token in shared memory (multiple of 1024)
    int *err;
    GemvPrologue pro;      // batch 1: x computed in every CTA instead of copied (kind != kProNone)
};

template <int QT>
struct Codes;
template <>
struct Codes<kQInt8> {
    static constexpr int EPC = 16;
};
template <>
struct Codes<kQInt4> {
    static constexpr int EPC = 32;
};
template <>
struct Codes<kQF32> {
    static constexpr int EPC = 4;
};
template <>
struct Codes<kQBF16> {
    static constexpr int EPC = 8;
};

constexpr int elems_per_chunk(int qtype) {
    return qtype == kQInt8 ? 16 : qtype == kQInt4 ? 32 : qtype == kQF32 ? 4 : 8;
}
constexpr bool dense_qtype(int qtype) { return qtype == kQF32 || qtype == kQBF16; }

// byte offset of logical offset `off` in a 1024-byte aligned, 128-byte swizzled region
PYXIS_DEVINL uint32_t swz128(uint32_t off) { return off ^ (((off >> 7) & 7u) << 4); }

// x of a batch-1 product computed from the previous step's outputs, written into token 0's
// swizzled tile: residual add + RMSNorm (src/transformer.rs:40-42,54-59, src/rmsnorm.rs:11-20:
// x += delta; h = x * ((1 / sqrt(mean(x^2) + eps)) * w)), CTA 0 storing the new residual, or
// SiLU(gate) * up (src/ffn.rs:39-41,52-54) from the stacked [gate; up] output.
// Each thread handles quads k4 = tid + u * blockDim (u < PQ) at once, every load issued before
// the first use; K <= 4 * PQ * blockDim is one round (the decode shapes).  The norm weight does not
// depend on the previous kernel and is read before griddepcontrol.wait.
template <int PRO>
PYXIS_DEVINL void run_prologue(const GemvPrologue &pr, int K, uint8_t *xs, float *red) {
    constexpr int PQ = 4;
    const int nq = K / 4, nt = blockDim.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(pr.x);
    if constexpr (PRO == kProAddNorm) {
        const float4 *d4 = reinterpret_cast<const float4 *>(pr.delta);
        const float4 *w4 = reinterpret_cast<const float4 *>(pr.w);
        float4 wv[PQ];
#pragma unroll
        for (int u = 0; u < PQ; ++u)
            if (threadIdx.x + u * nt < nq) wv[u] = __ldg(w4 + threadIdx.x + u * nt);
        pdl_wait();
        pdl_trigger();
        float ss = 0.f;
        for (int base = threadIdx.x; base < nq; base += PQ * nt) {
            float4 v[PQ], d[PQ];
#pragma unroll
            for (int u = 0; u < PQ; ++u) {
                const int k4 = base + u * nt;
                if (k4 < nq) {
                    v[u] = __ldg(x4 + k4);
                    if (pr.delta) d[u] = __ldg(d4 + k4);
                }
            }
#pragma unroll
            for (int u = 0; u < PQ; ++u) {
                const int k4 = base + u * nt;
                if (k4 >= nq) break;
                if (pr.delta) {
                    v[u] = make_float4(__fadd_rn(v[u].x, d[u].x), __fadd_rn(v[u].y, d[u].y), __fadd_rn(v[u].z, d[u].z),
                                       __fadd_rn(v[u].w, d[u].w));
                    if (blockIdx.x == 0) reinterpret_cast<float4 *>(pr.xout)[k4] = v[u];
                }
                *reinterpret_cast<float4 *>(xs + swz128((uint32_t)k4 * 16)) = v[u];
                ss = __fadd_rn(ss, __fmul_rn(v[u].x, v[u].x));
                ss = __fadd_rn(ss, __fmul_rn(v[u].y, v[u].y));
                ss = __fadd_rn(ss, __fmul_rn(v[u].z, v[u].z));
                ss = __fadd_rn(ss, __fmul_rn(v[u].w, v[u].w));
            }
        }
        ss = warp_sum(ss);
        const int warp = threadIdx.x >> 5, nw = nt >> 5;
        if ((threadIdx.x & 31) == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
        for (int i = 0; i < nw; ++i) tot = __fadd_rn(tot, red[i]);
        const float factor = rms_factor(tot, K, pr.eps);
        for (int base = threadIdx.x; base < nq; base += PQ * nt) {
#pragma unroll
            for (int u = 0; u < PQ; ++u) {
                const int k4 = base + u * nt;
                if (k4 >= nq) break;
                const float4 w = base == (int)threadIdx.x ? wv[u] : __ldg(w4 + k4);
                float4 *px = reinterpret_cast<float4 *>(xs + swz128((uint32_t)k4 * 16));
                float4 v = *px;
                v = make_float4(rms_scale(v.x, factor, w.x), rms_scale(v.y, factor, w.y), rms_scale(v.z, factor, w.z),
                                rms_scale(v.w, factor, w.w));
                *px = v;
            }
        }
    } else {
        pdl_wait();
        pdl_trigger();
        auto silu_mul = [](float g, float u) { return __fmul_rn(silu_f(g), u); };
        for (int base = threadIdx.x; base < nq; base += PQ * nt) {
            float4 g[PQ], u4[PQ];
#pragma unroll
            for (int u = 0; u < PQ; ++u) {
                const int k4 = base + u * nt;
                if (k4 < nq) {
                    g[u] = __ldg(x4 + k4);
                    u4[u] = __ldg(x4 + nq + k4);
                }
            }
#pragma unroll
            for (int u = 0; u < PQ; ++u) {
                const int k4 = base + u * nt;
                if (k4 >= nq) break;
                *reinterpret_cast<float4 *>(xs + swz128((uint32_t)k4 * 16)) =
                    make_float4(silu_mul(g[u].x, u4[u].x), silu_mul(g[u].y, u4[u].y), silu_mul(g[u].z, u4[u].z),
                                silu_mul(g[u].w, u4[u].w));
            }
        }
    }
    __syncthreads();
}

// acc[r][t] += W[row r, the 16-byte chunk's values] * x[t, the same k] for one chunk: codes
// decoded to exact float pairs (int8 / int4) or unquantized f32 / bf16 (bf16 -> f32 by u32 << 16,
// src/matmul.rs:289-295), x read from its 128-byte swizzled shared-memory tile at byte offset xoff
// (4 * the chunk's first k).  Group scales (chunk mode; a chunk lies inside one group): up to 4
// input rows sum q x over the chunk and multiply by the scale once (one paired FMA per row and
// token instead of a paired multiply per code pair); 5-8 rows, which would need more than 255
// registers for the chunk sums, scale the code pairs (one multiply per pair serves every token).
template <int QT, int B, int SMODE>
PYXIS_DEVINL void fma_chunk(const uint4 (&wc)[kRows], const float2 (&sc)[kRows], const uint8_t *xs,
                            uint32_t tok_stride, uint32_t xoff, float2 (&acc)[kRows][B]) {
    constexpr int EPC = Codes<QT>::EPC;
    if constexpr (SMODE == kScaleChunk && B <= (QT == kQInt4 ? 4 : 3)) {
        float2 part[kRows][B];
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int t = 0; t < B; ++t) part[r][t] = f2(0.f, 0.f);
        float2 one[kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r) one[r] = f2(1.f, 1.f);
        fma_chunk<QT, B, kScaleRow>(wc, one, xs, tok_stride, xoff, part);
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int t = 0; t < B; ++t) acc[r][t] = ffma2(part[r][t], sc[r], acc[r][t]);
        return;
    }
    if constexpr (dense_qtype(QT)) {
        // an f32 chunk is one quad of weights, a bf16 chunk two
#pragma unroll
        for (int qd = 0; qd < EPC / 4; ++qd) {
            float4 xq[B];
#pragma unroll
            for (int t = 0; t < B; ++t)
                xq[t] = *reinterpret_cast<const float4 *>(xs + (size_t)t * tok_stride + swz128(xoff + (uint32_t)qd * 16));
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
                float2 q0, q1;
                if constexpr (QT == kQF32) {
                    q0 = f2(__uint_as_float(wc[r].x), __uint_as_float(wc[r].y));
                    q1 = f2(__uint_as_float(wc[r].z), __uint_as_float(wc[r].w));
                } else {
                    const uint32_t a = qd == 0 ? wc[r].x : wc[r].z, b = qd == 0 ? wc[r].y : wc[r].w;
                    q0 = f2(__uint_as_float(a << 16), __uint_as_float(a & 0xffff0000u));
                    q1 = f2(__uint_as_float(b << 16), __uint_as_float(b & 0xffff0000u));
                }
#pragma unroll
                for (int t = 0; t < B; ++t) {
                    acc[r][t] = ffma2(q0, f2(xq[t].x, xq[t].y), acc[r][t]);
                    acc[r][t] = ffma2(q1, f2(xq[t].z, xq[t].w), acc[r][t]);
                }
            }
        }
    } else {
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            // one 32-bit word of codes per row: int8 4 elements (1 x quad), int4 8 (2 quads)
            constexpr int QPW = EPC / 16;
            float4 xq[QPW][B];
#pragma unroll
            for (int qd = 0; qd < QPW; ++qd)
#pragma unroll
                for (int t = 0; t < B; ++t)
                    xq[qd][t] = *reinterpret_cast<const float4 *>(xs + (size_t)t * tok_stride +
                                                                  swz128(xoff + (uint32_t)(wi * QPW + qd) * 16));
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
                const uint32_t word = wi == 0 ? wc[r].x : wi == 1 ? wc[r].y : wi == 2 ? wc[r].z : wc[r].w;
                float2 q[2 * QPW];
                if constexpr (QT == kQInt8) i8x4_to_f32(word, q[0], q[1]);
                else u4x8_to_f32(word, q[0], q[1], q[2], q[3]);
                if constexpr (SMODE == kScaleChunk) {
#pragma unroll
                    for (int j = 0; j < 2 * QPW; ++j) q[j] = __fmul2_rn(q[j], sc[r]);
                }
#pragma unroll
                for (int qd = 0; qd < QPW; ++qd)
#pragma unroll
                    for (int t = 0; t < B; ++t) {
                        acc[r][t] = ffma2(q[2 * qd], f2(xq[qd][t].x, xq[qd][t].y), acc[r][t]);
                        acc[r][t] = ffma2(q[2 * qd + 1], f2(xq[qd][t].z, xq[qd][t].w), acc[r][t]);
                    }
            }
        }
    }
}

// The warp's 32 (row, token) sums: even + odd partials, then halving exchanges over
// v[r*8 + t] (31 shuffles); lane l ends with row l/8, token l%8.
template <int B>
PYXIS_DEVINL float reduce_rows_tokens(const float2 (&acc)[kRows][B], int lane) {
    float v[32];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int t = 0; t < 8; ++t) v[r * 8 + t] = t < B ? acc[r][t].x + acc[r][t].y : 0.f;
#pragma unroll
    for (int o = 16, n = 32; o >= 1; o >>= 1, n >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = upper ? v[i] : v[i + n / 2];
            const float keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    return v[0];
}

template <int QT, int B, int SMODE, int PRO>
__global__ void __launch_bounds__(max_warps(B) * 32, 1)
    gemv_batch_kernel(const __grid_constant__ CUtensorMap tm_x, const BatchParams p) {
    constexpr int EPC = Codes<QT>::EPC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *xs = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *red = reinterpret_cast<float *>(xs + (size_t)B * p.tok_stride);  // [2][kMaxWarps][32]
    uint64_t *bar = reinterpret_cast<uint64_t *>(red + 2 * kMaxWarps * 32);
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gi = warp / p.slices, s = warp - gi * p.slices;
    const int c0 = s * 32 + lane;
    const int cstep = 32 * p.slices;

    uint4 wn[kRows];
    float sn[kRows];
    auto load = [&](int row0, int c) {
        // the chunk's scale block (a shift for the usual power-of-two groups: a division per chunk
        // was a visible share of the lanes' instructions)
        const int blk = SMODE == kScaleChunk ? (p.cpb_shift >= 0 ? c >> p.cpb_shift : c / p.chunks_per_block) : 0;
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const int row = min(row0 + r, p.N - 1);
            wn[r] = ld_stream_v4(p.W + (size_t)row * p.row_bytes + (size_t)c * 16);
            sn[r] = SMODE == kScaleChunk ? ld_nc_f32(p.S + (size_t)row * p.blocks_per_row + blk) : 1.f;
        }
    };
    auto row0_of = [&](int item) { return (item * p.groups_cta + gi) * kRows; };

    // the weights do not depend on the previous kernel: request them before waiting on it
    int it = blockIdx.x;
    if (it < p.items && row0_of(it) < p.N && c0 < p.chunks) load(row0_of(it), c0);

    if constexpr (PRO != kProNone) {
        run_prologue<PRO>(p.pro, p.K, xs, red);  // waits on the previous kernels itself
    } else {
    if (threadIdx.x == 0) {
        abort_flag = 0;
        tc::mbar_init(bar, 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tm_x);
    }
    __syncthreads();
    pdl_wait();  // x comes from the previous kernel
    pdl_trigger();
    if (threadIdx.x == 0) {
        tc::mbar_arrive_expect_tx(bar, (uint32_t)(B * p.x_boxes * p.box_rows * 128));
        for (int t = 0; t < B; ++t)
            for (int bx = 0; bx < p.x_boxes; ++bx)
                tc::tma_load_3d(xs + (size_t)t * p.tok_stride + (size_t)bx * p.box_rows * 128, &tm_x, 0,
                                bx * p.box_rows, t, bar);
    }
    tc::mbar_wait_bounded(bar, 0, &abort_flag, p.err, kErrX, kTimeoutNs);
    __syncthreads();  // every thread has its verdict; abort_flag is final
    if (abort_flag) {
        // x is still in flight: wait (bounded) for the copy before the CTA's memory goes away
        if (threadIdx.x == 0) {
            int no_abort = 0;
            tc::mbar_wait_bounded(bar, 0, &no_abort, p.err, kErrX, kTimeoutNs);
        }
        return;
    }
    }

    int buf = 0;
    for (; it < p.items; it += gridDim.x, buf ^= 1) {
        const int row0 = row0_of(it);
        const bool active = row0 < p.N;
        float2 acc[kRows][B];
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int t = 0; t < B; ++t) acc[r][t] = f2(0.f, 0.f);
        if (active) {
            for (int c = c0; c < p.chunks; c += cstep) {
                uint4 wc[kRows];
                float2 sc[kRows];
#pragma unroll
                for (int r = 0; r < kRows; ++r) {
                    wc[r] = wn[r];
                    sc[r] = f2(sn[r], sn[r]);
                }
                // next chunk of these rows, or the first chunk of this warp's next item
                if (c + cstep < p.chunks) {
                    load(row0, c + cstep);
                } else {
                    const int nit = it + gridDim.x;
                    if (nit < p.items && row0_of(nit) < p.N) load(row0_of(nit), c0);
                }
                fma_chunk<QT, B, SMODE>(wc, sc, xs, p.tok_stride, (uint32_t)c * (EPC * 4), acc);
            }
        }
        const float v0 = reduce_rows_tokens<B>(acc, lane);
        float *rb = red + buf * (kMaxWarps * 32);
        rb[warp * 32 + lane] = v0;
        __syncthreads();
        if (s == 0 && active) {
            float y = 0.f;
            for (int j = 0; j < p.slices; ++j) y += rb[(gi * p.slices + j) * 32 + lane];
            const int row = row0 + (lane >> 3), t = lane & 7;
            if (t < B && row < p.N) {
                if (SMODE == kScaleRow) y *= ld_nc_f32(p.S + row);
                p.Y[(size_t)t * p.ldy + row] = y;
            }
        }
    }
}

struct Shape {
    bool ok = false;
    int slices = 1, groups_cta = 1, items = 0, x_boxes = 1, box_rows = 8;
    uint32_t tok_stride = 0;
    size_t smem = 0;
};

// 227 KB per block minus room for the kernel's static shared memory (the attribute counts only
// the dynamic part, and a value the device rejects would leave the 48 KB default in place)
constexpr size_t kMaxSmem = 226 * 1024;

Shape shape_for(const QMatrix &w, size_t B, int num_sms) {
    Shape sh;
    if (w.qtype < kQInt8 || w.qtype > kQBF16) return sh;
    const int epc = elems_per_chunk(w.qtype);
    const size_t K = w.K, bs = w.block_size;
    if (B < 1 || B > 8 || K == 0 || K % 32 != 0 || K > (1u << 20) || w.N == 0 || w.N > (size_t)INT32_MAX / 2)
        return sh;
    if (reinterpret_cast<uintptr_t>(w.data) & 15) return sh;
    if (!dense_qtype(w.qtype) && !(bs == K || (bs % epc == 0 && K % bs == 0))) return sh;
    const int chunks = (int)(K / epc);
    const int rows = (int)(K / 32);
    sh.x_boxes = (rows + kXBoxRows - 1) / kXBoxRows;
    sh.box_rows = ((rows + sh.x_boxes - 1) / sh.x_boxes + 7) & ~7;
    sh.tok_stride = (uint32_t)(((size_t)sh.x_boxes * sh.box_rows * 128 + 1023) & ~size_t(1023));
    sh.smem = 1024 + B * (size_t)sh.tok_stride + 2 * kMaxWarps * 32 * sizeof(float) + 64;
    if (sh.smem > kMaxSmem) return sh;
    const int mw = max_warps((int)B);
    sh.slices = std::min(mw, (chunks + 31) / 32);
    const long groups = ((long)w.N + kRows - 1) / kRows;
    const long want = (groups + num_sms - 1) / num_sms;  // groups per CTA that fill every SM once
    sh.groups_cta = (int)std::max<long>(1, std::min<long>(want, mw / sh.slices));
    sh.items = (int)((groups + sh.groups_cta - 1) / sh.groups_cta);
    sh.ok = true;
    return sh;
}

template <int QT, int B, int SMODE, int PRO = kProNone>
cudaError_t run(const CUtensorMap &tm, const BatchParams &p, const Shape &sh, int num_sms, cudaStream_t st) {
    auto kern = gemv_batch_kernel<QT, B, SMODE, PRO>;
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t attr = once_per_device(
        attr_done, [&] { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem); });
    if (attr != cudaSuccess) return attr;
    const int threads = sh.slices * sh.groups_cta * 32;
    const int grid = std::max(1, std::min(sh.items, num_sms));
    return launch_kernel(kern, dim3(grid), dim3(threads), sh.smem, st, tm, p);
}

template <int QT, int SMODE>
cudaError_t dispatch(size_t B, const CUtensorMap &tm, const BatchParams &p, const Shape &sh, int num_sms,
                     cudaStream_t st) {
    switch (B) {
    case 1: return run<QT, 1, SMODE>(tm, p, sh, num_sms, st);
    case 2: return run<QT, 2, SMODE>(tm, p, sh, num_sms, st);
    case 3: return run<QT, 3, SMODE>(tm, p, sh, num_sms, st);
    case 4: return run<QT, 4, SMODE>(tm, p, sh, num_sms, st);
    case 5: return run<QT, 5, SMODE>(tm, p, sh, num_sms, st);
    case 6: return run<QT, 6, SMODE>(tm, p, sh, num_sms, st);
    case 7: return run<QT, 7, SMODE>(tm, p, sh, num_sms, st);
    default: return run<QT, 8, SMODE>(tm, p, sh, num_sms, st);
    }
}

}  // namespace

bool gemv_batch_supported(const QMatrix &w, size_t B, int num_sms) { return shape_for(w, B, num_sms).ok; }

namespace {

BatchParams make_params(const QMatrix &w, const Shape &sh, float *Y, size_t ldy, int *err) {
    const int epc = elems_per_chunk(w.qtype);
    const bool chunk_mode = !dense_qtype(w.qtype) && w.block_size != w.K;
    BatchParams p{};
    p.W = w.data;
    p.S = w.scales;
    p.Y = Y;
    p.N = (int)w.N;
    p.K = (int)w.K;
    p.ldy = (int)ldy;
    p.row_bytes = (int)(w.K / epc * 16);
    p.chunks = (int)(w.K / epc);
    p.blocks_per_row = chunk_mode ? (int)(w.K / w.block_size) : 1;
    p.chunks_per_block = chunk_mode ? (int)(w.block_size / epc) : 1;
    p.cpb_shift = (p.chunks_per_block & (p.chunks_per_block - 1)) == 0 ? __builtin_ctz((unsigned)p.chunks_per_block) : -1;
    p.slices = sh.slices;
    p.groups_cta = sh.groups_cta;
    p.items = sh.items;
    p.x_boxes = sh.x_boxes;
    p.box_rows = sh.box_rows;
    p.tok_stride = sh.tok_stride;
    p.err = err;
    return p;
}

}  // namespace

cudaError_t launch_gemv_batch(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y, size_t ldy,
                              int *err, int num_sms, cudaStream_t st) {
    const Shape sh = shape_for(w, B, num_sms);
    if (!sh.ok) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(X) & 15) || (B > 1 && ldx % 4)) return cudaErrorInvalidValue;
    auto fn = tensor_map_encoder();
    if (!fn) return cudaErrorNotSupported;
    // x as [B][K/32][32] f32: one 128-byte row per 32 values, 128-byte swizzle
    CUtensorMap tm;
    const cuuint64_t rows = w.K / 32;
    cuuint64_t dims[3] = {32, rows, (cuuint64_t)B};
    cuuint64_t strides[2] = {128, (cuuint64_t)(B > 1 ? ldx : w.K) * sizeof(float)};
    cuuint32_t box[3] = {32, (cuuint32_t)sh.box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (fn(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(X), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    const BatchParams p = make_params(w, sh, Y, ldy, err);
    if (w.qtype == kQF32) return dispatch<kQF32, kScaleNone>(B, tm, p, sh, num_sms, st);
    if (w.qtype == kQBF16) return dispatch<kQBF16, kScaleNone>(B, tm, p, sh, num_sms, st);
    const bool chunk_mode = w.block_size != w.K;
    if (w.qtype == kQInt8)
        return chunk_mode ? dispatch<kQInt8, kScaleChunk>(B, tm, p, sh, num_sms, st)
                          : dispatch<kQInt8, kScaleRow>(B, tm, p, sh, num_sms, st);
    return chunk_mode ? dispatch<kQInt4, kScaleChunk>(B, tm, p, sh, num_sms, st)
                      : dispatch<kQInt4, kScaleRow>(B, tm, p, sh, num_sms, st);
}

bool gemv_batch_pro_supported(const QMatrix &w, const GemvPrologue &pro, int num_sms) {
    if (pro.kind != kProAddNorm && pro.kind != kProSiluMul) return false;
    if (w.qtype != kQInt8 && w.qtype != kQInt4) return false;  // the decode model's layouts
    if (!pro.x || (reinterpret_cast<uintptr_t>(pro.x) & 15)) return false;
    if (pro.kind == kProAddNorm) {
        if (!pro.w || (reinterpret_cast<uintptr_t>(pro.w) & 15)) return false;
        if (pro.delta && ((reinterpret_cast<uintptr_t>(pro.delta) & 15) || !pro.xout ||
                          (reinterpret_cast<uintptr_t>(pro.xout) & 15)))
            return false;
    }
    return shape_for(w, 1, num_sms).ok;
}

cudaError_t launch_gemv_batch_pro(const QMatrix &w, const GemvPrologue &pro, float *Y, int *err, int num_sms,
                                  cudaStream_t st) {
    if (!gemv_batch_pro_supported(w, pro, num_sms)) return cudaErrorInvalidValue;
    const bool chunk_mode = w.block_size != w.K;
    CUtensorMap tm;  // not read: the prologue writes x itself
    memset(&tm, 0, sizeof(tm));
    const Shape sh = shape_for(w, 1, num_sms);
    BatchParams p = make_params(w, sh, Y, w.N, err);
    p.pro = pro;
    if (pro.kind == kProAddNorm) {
        if (w.qtype == kQInt8)
            return chunk_mode ? run<kQInt8, 1, kScaleChunk, kProAddNorm>(tm, p, sh, num_sms, st)
                              : run<kQInt8, 1, kScaleRow, kProAddNorm>(tm, p, sh, num_sms, st);
        return chunk_mode ? run<kQInt4, 1, kScaleChunk, kProAddNorm>(tm, p, sh, num_sms, st)
                          : run<kQInt4, 1, kScaleRow, kProAddNorm>(tm, p, sh, num_sms, st);
    }
    if (w.qtype == kQInt8)
        return chunk_mode ? run<kQInt8, 1, kScaleChunk, kProSiluMul>(tm, p, sh, num_sms, st)
                          : run<kQInt8, 1, kScaleRow, kProSiluMul>(tm, p, sh, num_sms, st);
    return chunk_mode ? run<kQInt4, 1, kScaleChunk, kProSiluMul>(tm, p, sh, num_sms, st)
                      : run<kQInt4, 1, kScaleRow, kProSiluMul>(tm, p, sh, num_sms, st);
}

}  // namespace pyxis
