// gemv_mma.cu -- matmul for 1-8 input rows with the dequantised codes handed from registers to the
// tensor cores (mma.sync m16n8k16, fp16 x fp16 -> f32):
//     y[b, n] = sum_k x[b, k] * dequant(W)[n, k]
// (src/matmul.rs:21-97 for each input row; int4 src/matmul.rs:149-173, int8 :297-317) for int4 or
// int8 codes with a scale per group of 32, or one scale per row.
//
// Why this shape of kernel.  At 1-8 tokens the op streams the weights once (0.5-1 byte per code)
// and does 2-16 flops per code.  On the CUDA cores the paired FMAs per code grow with the tokens
// (8 tokens: four f32x2 FMAs and the decode per code, several times the HBM time of the codes);
// tcgen05 would need the converted codes staged in shared memory or TMEM by other warps and every
// scale group's accumulator read back from TMEM.  An m16n8k16 mma.sync instead takes the codes
// straight from the registers of the thread that converted them and returns the 16 x 8 sums of a
// scale group in registers, where the group's scale is applied: per 16 codes a thread spends about
// 35 instructions at any batch up to 4 (about 40 at 8), and the weights' bytes set the time.
//
// Layout of the work.  A CTA takes 128 weight rows (8 warps x 16) over one K part; the parts of a
// row tile form a thread-block cluster.  All weight bytes of the CTA are requested at kernel start
// (before griddepcontrol.wait: they do not depend on the previous kernel), as TMA boxes of 128 rows
// x 128 bytes with 128-byte swizzle (int4: 256 of K = 8 groups; int8: 128 of K = 4 groups), the
// group scales with them (boxes of 128 rows x the box's groups), one mbarrier per box.  Two CTAs
// fit on an SM, so the next launch in a stream can start streaming while this one finishes.
//
// x.  After the wait, warp t splits token t's slice of the part: every value is scaled by the
// power of two 2^e of the (token, part) (max |x| 2^e in [2^14, 2^15)) and written as fp16 hi + lo
// (22 significant bits) in the layout of the MMA's B fragments.  Up to 4 tokens share one n8 tile
// as (token, hi) and (token, lo) columns; 5-8 tokens take two tiles.  A thread (g = lane / 4,
// j = lane % 4) owns 8 consecutive codes of each scale group for rows g and g + 8 of its warp's 16
// (int4: word j of the group's 16 bytes; int8: bytes 8j..8j+7), and the K order inside the group
// is permuted so that those 8 codes are exactly its A fragments of the group's two k16 steps;
// x's fragments follow the same permutation, so the products are the reference's products.
//
// Arithmetic.  Codes are exact in fp16; code x hi and code x lo are exact in the f32 products.
// Each group's two k16 steps go through one fresh accumulator (two MMAs into zero), and the
// thread adds (hi + lo column) x scale into f32 registers with round-to-nearest, in group order.
// The tile's partials times 2^-e go to shared memory; after a cluster barrier CTA c adds rows
// [c 128 / parts, (c + 1) 128 / parts) over the parts in rank order through distributed shared
// memory (row scales are applied here) and writes y: results do not depend on timing.  Every
// mbarrier wait is bounded; a wait that runs out records a code in the context's device flag.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "fp16_codes.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace pyxis {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileRows = kWarps * 16;                // weight rows per CTA
constexpr int kBoxBytes = 128;                        // K bytes per weight box (one swizzle row)
constexpr uint32_t kBoxSmem = kTileRows * kBoxBytes;  // 16 KB
constexpr int kMaxBoxes = 6;                          // boxes per CTA (one K part)
constexpr int kMaxParts = 8;                          // K parts = portable cluster size
constexpr int kMaxTok = 8;
constexpr size_t kMaxSmem = 226 * 1024;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr int kErrWeights = 0x801;  // a weight box never arrived

struct MmaParams {
    const float *X;
    const float *S;  // row scales (read at the end); group scales come by TMA
    float *Y;
    long long ldx, ldy;
    int N, K, B;
    int parts;  // K parts per row tile (cluster size)
    int nb;     // weight boxes per row
    int *err;
};

template <int QT>
struct MmaCodes;
template <>
struct MmaCodes<kQInt4> {
    static constexpr int kBoxK = 256, kGPB = 8;  // K per box, scale groups per box
};
template <>
struct MmaCodes<kQInt8> {
    static constexpr int kBoxK = 128, kGPB = 4;
};

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled box (8-row 1024-byte atoms).
PYXIS_DEVINL uint32_t sw128(uint32_t r, uint32_t c) { return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4); }

// d += A B for one m16n8k16 step (A row-major 16 x 16 fp16, B column-major 16 x 8 fp16, f32 d).
PYXIS_DEVINL void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Cluster barrier halves (every thread of every CTA of the cluster executes each, in turn).
PYXIS_DEVINL void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
PYXIS_DEVINL void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
PYXIS_DEVINL void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Stores v at `local`'s offset in the shared memory of the cluster's CTA `rank`.
PYXIS_DEVINL void st_cluster_f32(float *local, uint32_t rank, float v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(tc::smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// e with max |x| 2^e in [2^14, 2^15) for the largest magnitude m (0 for 0, Inf or NaN), in
// [-64, 64], and 2^e exactly.
PYXIS_DEVINL int x_scale_exp(float m) {
    if (!(m > 0.f) || !(m < 3.0e38f)) return 0;
    const int e = 14 - ((int)((__float_as_uint(m) >> 23) & 0xFFu) - 127);
    return e < -64 ? -64 : (e > 64 ? 64 : e);
}
PYXIS_DEVINL float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

template <int QT, bool GROUP, int NT>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_mma_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                    const MmaParams p) {
    constexpr int GPB = MmaCodes<QT>::kGPB;
    constexpr int KB = MmaCodes<QT>::kBoxK;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *wt = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int nmax = (p.nb + p.parts - 1) / p.parts;
    float *st = reinterpret_cast<float *>(wt + (size_t)nmax * kBoxSmem);           // [box][128][GPB]
    uint8_t *xs = reinterpret_cast<uint8_t *>(st + (GROUP ? nmax * kTileRows * GPB : 0));  // [group][NT][8][4] x 16 B
    float *recv = reinterpret_cast<float *>(xs + (size_t)nmax * GPB * NT * 512);     // [parts][128 / parts][8]
    float *xinv = recv + kTileRows * kMaxTok;                                         // [8]
    uint64_t *bar = reinterpret_cast<uint64_t *>(xinv + kMaxTok);                     // [nmax]
    __shared__ int abort_flag;

    const int part = blockIdx.x, tile = blockIdx.y;  // part = the CTA's rank in its cluster
    const int b0 = part * p.nb / p.parts, nbox = (part + 1) * p.nb / p.parts - b0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // first half of the barrier that tells every CTA of the cluster that the others have started
    // (their shared memory may be written): waited on only before the partials are sent
    if (p.parts > 1) cluster_arrive_relaxed();

    // the weights (and group scales) do not depend on the previous kernel: request them first
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int b = 0; b < nbox; ++b) tc::mbar_init(&bar[b], 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tm_w);
        if constexpr (GROUP) tc::prefetch_tmap(&tm_s);
        for (int b = 0; b < nbox; ++b) {
            tc::mbar_arrive_expect_tx(&bar[b], kBoxSmem + (GROUP ? kTileRows * GPB * 4 : 0));
            tc::tma_load_2d(wt + (size_t)b * kBoxSmem, &tm_w, (b0 + b) * kBoxBytes, tile * kTileRows, &bar[b]);
            if constexpr (GROUP)
                tc::tma_load_2d(st + (size_t)b * kTileRows * GPB, &tm_s, (b0 + b) * GPB, tile * kTileRows, &bar[b]);
        }
    }
    __syncthreads();
    pdl_wait();  // x comes from the previous kernel
    pdl_trigger();

    // ---- x: warp t writes token t's hi / lo fragments of this part (zeros for absent tokens); a
    // lane holds its words (8 values each) in registers between the max and the split
    constexpr int MW = kMaxBoxes * KB / 8 / 32;  // words per lane at most
    const int k0 = b0 * KB, words = nbox * KB / 8;
    if (warp < 4 * NT) {
        const int t = warp, tt = t >> 2, nh = 2 * (t & 3);
        if (t < p.B) {
            const float4 *xr = reinterpret_cast<const float4 *>(p.X + (long long)t * p.ldx + k0);
            float4 xa[MW], xb[MW];
            float m = 0.f;
#pragma unroll
            for (int u = 0; u < MW; ++u) {
                const int q = lane + 32 * u;
                if (q < words) {
                    xa[u] = __ldg(xr + 2 * q);
                    xb[u] = __ldg(xr + 2 * q + 1);
                }
            }
#pragma unroll
            for (int u = 0; u < MW; ++u) {
                if (lane + 32 * u < words) {
                    m = fmaxf(m, fmaxf(fmaxf(fabsf(xa[u].x), fabsf(xa[u].y)), fmaxf(fabsf(xa[u].z), fabsf(xa[u].w))));
                    m = fmaxf(m, fmaxf(fmaxf(fabsf(xb[u].x), fabsf(xb[u].y)), fmaxf(fabsf(xb[u].z), fabsf(xb[u].w))));
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const int e = x_scale_exp(m);
            const float sc = pow2f(e);
            if (lane == 0) xinv[t] = pow2f(-e);
#pragma unroll
            for (int u = 0; u < MW; ++u) {
                const int q = lane + 32 * u;
                if (q >= words) break;
                const float x[8] = {xa[u].x * sc, xa[u].y * sc, xa[u].z * sc, xa[u].w * sc,
                                    xb[u].x * sc, xb[u].y * sc, xb[u].z * sc, xb[u].w * sc};
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    // int4 pairs (x_i, x_i+4) as u4x8_to_h pairs the codes; int8 (x_2i, x_2i+1)
                    const float2 pr = QT == kQInt4 ? make_float2(x[i], x[i + 4]) : make_float2(x[2 * i], x[2 * i + 1]);
                    split_pair_f32(pr, hi[i], lo[i]);
                }
                uint8_t *dst = xs + ((size_t)(((q >> 2) * NT + tt) * 8 + nh) * 4 + (q & 3)) * 16;
                *reinterpret_cast<uint4 *>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4 *>(dst + 64) = make_uint4(lo[0], lo[1], lo[2], lo[3]);  // column nh + 1
            }
        } else {
            for (int q = lane; q < words; q += 32) {
                uint8_t *dst = xs + ((size_t)(((q >> 2) * NT + tt) * 8 + nh) * 4 + (q & 3)) * 16;
                *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4 *>(dst + 64) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
    __syncthreads();

    // ---- the tile: warp w, rows r and r + 8 of its 16, codes of word / byte block j of each group
    const int g = lane >> 2, j = lane & 3;
    const int r = warp * 16 + g;
    float acc[2][NT];
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) acc[0][tt] = acc[1][tt] = 0.f;
    for (int b = 0; b < nbox; ++b) {
        tc::mbar_wait_bounded(&bar[b], 0, &abort_flag, p.err, kErrWeights, kTimeoutNs);
        const uint8_t *wb = wt + (size_t)b * kBoxSmem;
        float s0[GPB], s1[GPB];
        if constexpr (GROUP) {
            const float4 *sp0 = reinterpret_cast<const float4 *>(st + ((size_t)b * kTileRows + r) * GPB);
            const float4 *sp1 = reinterpret_cast<const float4 *>(st + ((size_t)b * kTileRows + r + 8) * GPB);
#pragma unroll
            for (int i = 0; i < GPB / 4; ++i) {
                const float4 u = sp0[i], v = sp1[i];
                s0[4 * i] = u.x, s0[4 * i + 1] = u.y, s0[4 * i + 2] = u.z, s0[4 * i + 3] = u.w;
                s1[4 * i] = v.x, s1[4 * i + 1] = v.y, s1[4 * i + 2] = v.z, s1[4 * i + 3] = v.w;
            }
        }
        // four groups at a time: their loads first, then the first k16 step of all four, then the
        // second, so consecutive MMAs do not depend on each other
#pragma unroll
        for (int g0 = 0; g0 < GPB; g0 += 4) {
            uint32_t a[4][2][4];  // [group][k16 step][fragment]
            uint4 xf[4][NT];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int gb = g0 + q;
                if constexpr (QT == kQInt4) {
                    const uint32_t w0 = *reinterpret_cast<const uint32_t *>(wb + sw128(r, gb) + 4 * j);
                    const uint32_t w1 = *reinterpret_cast<const uint32_t *>(wb + sw128(r + 8, gb) + 4 * j);
                    uint32_t h0[4], h1[4];
                    u4x8_to_h(w0, h0);
                    u4x8_to_h(w1, h1);
#pragma unroll
                    for (int s2 = 0; s2 < 2; ++s2) {
                        a[q][s2][0] = h0[2 * s2];
                        a[q][s2][1] = h1[2 * s2];
                        a[q][s2][2] = h0[2 * s2 + 1];
                        a[q][s2][3] = h1[2 * s2 + 1];
                    }
                } else {
                    const uint32_t off = (uint32_t)(j & 1) * 8;
                    const uint2 v0 = *reinterpret_cast<const uint2 *>(wb + sw128(r, 2 * gb + (j >> 1)) + off);
                    const uint2 v1 = *reinterpret_cast<const uint2 *>(wb + sw128(r + 8, 2 * gb + (j >> 1)) + off);
                    i8x4_to_h(v0.x, a[q][0][0], a[q][0][2]);
                    i8x4_to_h(v1.x, a[q][0][1], a[q][0][3]);
                    i8x4_to_h(v0.y, a[q][1][0], a[q][1][2]);
                    i8x4_to_h(v1.y, a[q][1][1], a[q][1][3]);
                }
                const int G = b * GPB + gb;
#pragma unroll
                for (int tt = 0; tt < NT; ++tt)
                    xf[q][tt] = *reinterpret_cast<const uint4 *>(xs + ((size_t)((G * NT + tt) * 8 + g) * 4 + j) * 16);
            }
            float d[4][NT][4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int tt = 0; tt < NT; ++tt) {
                    d[q][tt][0] = d[q][tt][1] = d[q][tt][2] = d[q][tt][3] = 0.f;
                    mma16816(d[q][tt], a[q][0], xf[q][tt].x, xf[q][tt].y);
                }
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int tt = 0; tt < NT; ++tt) mma16816(d[q][tt], a[q][1], xf[q][tt].z, xf[q][tt].w);
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int tt = 0; tt < NT; ++tt) {
                    const float v0 = d[q][tt][0] + d[q][tt][1], v1 = d[q][tt][2] + d[q][tt][3];  // (hi + lo), rows r, r + 8
                    if constexpr (GROUP) {
                        acc[0][tt] = fmaf(v0, s0[g0 + q], acc[0][tt]);
                        acc[1][tt] = fmaf(v1, s1[g0 + q], acc[1][tt]);
                    } else {
                        acc[0][tt] += v0;
                        acc[1][tt] += v1;
                    }
                }
        }
    }
    // ---- the parts of each row, added in rank order: CTA c of the cluster owns rows
    // [c 128 / parts, (c + 1) 128 / parts) of the tile; every CTA sends it their partials of them
    const int rows_per = kTileRows / p.parts;
    if (p.parts > 1) cluster_wait();  // every CTA of the cluster has started
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
        const int t = 4 * tt + j;
        if (t < p.B) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int rr = r + 8 * h;
                const int owner = rr / rows_per;
                float *slot = recv + ((size_t)part * rows_per + (rr - owner * rows_per)) * kMaxTok + t;
                const float v = acc[h][tt] * xinv[t];
                if (p.parts > 1) st_cluster_f32(slot, (uint32_t)owner, v);
                else *slot = v;
            }
        }
    }
    if (p.parts > 1) {
        cluster_arrive_release();
        cluster_wait();
    } else {
        __syncthreads();
    }
    for (int i = threadIdx.x; i < rows_per * p.B; i += kThreads) {
        const int rl = i / p.B, t = i - rl * p.B;
        const int row = tile * kTileRows + part * rows_per + rl;
        float v = recv[(size_t)rl * kMaxTok + t];
        for (int q = 1; q < p.parts; ++q) v += recv[((size_t)q * rows_per + rl) * kMaxTok + t];
        if (row < p.N) {
            if constexpr (!GROUP) v *= __ldg(p.S + row);
            p.Y[(long long)t * p.ldy + row] = v;
        }
    }
    if (abort_flag && threadIdx.x == 0) {
        // boxes may still be in flight: wait (bounded) before the CTA's memory goes away
        int no_abort = 0;
        for (int b = 0; b < nbox; ++b) tc::mbar_wait_bounded(&bar[b], 0, &no_abort, p.err, kErrWeights, kTimeoutNs);
    }
}

struct MmaShape {
    bool ok = false;
    int parts = 1, nb = 0, nmax = 0, tiles = 0;
    size_t smem = 0;
};

MmaShape mma_shape(const QMatrix &w, size_t B, int num_sms) {
    MmaShape sh;
    if (w.qtype != kQInt4 && w.qtype != kQInt8) return sh;
    if (B < 1 || B > (size_t)kMaxTok || w.N == 0 || w.K == 0) return sh;
    const bool group = w.block_size == 32 && w.K != 32, row = w.block_size == w.K;
    if (!group && !row) return sh;
    const size_t box_k = w.qtype == kQInt4 ? 256 : 128;
    if (w.K % box_k || w.K > (1u << 20) || w.N > (size_t)65535 * kTileRows) return sh;
    if ((reinterpret_cast<uintptr_t>(w.data) & 15) || (reinterpret_cast<uintptr_t>(w.scales) & 15)) return sh;
    sh.nb = (int)(w.K / box_k);
    sh.tiles = (int)((w.N + kTileRows - 1) / kTileRows);
    int best = 0;
    for (int p = 1; p <= kMaxParts && p <= sh.nb; p *= 2) {
        if ((sh.nb + p - 1) / p > kMaxBoxes) continue;
        best = p;
        if ((long)sh.tiles * p >= num_sms) break;  // every SM has a CTA
    }
    if (!best) return sh;
    sh.parts = best;
    sh.nmax = (sh.nb + best - 1) / best;
    const int nt = B > 4 ? 2 : 1;
    const int gpb = w.qtype == kQInt4 ? MmaCodes<kQInt4>::kGPB : MmaCodes<kQInt8>::kGPB;
    sh.smem = 1024 + (size_t)sh.nmax * kBoxSmem + (group ? (size_t)sh.nmax * kTileRows * gpb * 4 : 0) +
              (size_t)sh.nmax * gpb * nt * 512 + kTileRows * kMaxTok * 4 + kMaxTok * 4 + (size_t)sh.nmax * 8;
    sh.ok = sh.smem <= kMaxSmem;
    return sh;
}

template <int QT, bool GROUP, int NT>
cudaError_t run_mma(const CUtensorMap &tw, const CUtensorMap &ts, const MmaParams &p, const MmaShape &sh,
                    cudaStream_t st) {
    auto kern = gemv_mma_kernel<QT, GROUP, NT>;
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t attr = once_per_device(
        attr_done, [&] { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem); });
    if (attr != cudaSuccess) return attr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)sh.parts, (unsigned)sh.tiles);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sh.smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    if (sh.parts > 1) {
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = (unsigned)sh.parts;
        attrs[na].val.clusterDim.y = 1;
        attrs[na].val.clusterDim.z = 1;
        ++na;
    }
    if (pdl_enabled()) {
        attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, tw, ts, p);
}

template <int QT, bool GROUP>
cudaError_t run_mma_nt(size_t B, const CUtensorMap &tw, const CUtensorMap &ts, const MmaParams &p,
                       const MmaShape &sh, cudaStream_t st) {
    return B > 4 ? run_mma<QT, GROUP, 2>(tw, ts, p, sh, st) : run_mma<QT, GROUP, 1>(tw, ts, p, sh, st);
}

}  // namespace

bool gemv_mma_supported(const QMatrix &w, size_t B, int num_sms) { return mma_shape(w, B, num_sms).ok; }

cudaError_t launch_gemv_mma(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y, size_t ldy, int *err,
                            int num_sms, cudaStream_t st) {
    const MmaShape sh = mma_shape(w, B, num_sms);
    if (!sh.ok) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(X) & 15) || (B > 1 && ldx % 4)) return cudaErrorInvalidValue;
    auto fn = tensor_map_encoder();
    if (!fn) return cudaErrorNotSupported;
    const bool group = w.block_size != w.K;
    const bool int4 = w.qtype == kQInt4;
    // codes [N][row_bytes] u8 in 128-row x 128-byte boxes, 128-byte swizzle
    CUtensorMap tw, ts;
    memset(&ts, 0, sizeof(ts));
    const cuuint64_t row_bytes = int4 ? w.K / 2 : w.K;
    {
        cuuint64_t dims[2] = {row_bytes, (cuuint64_t)w.N};
        cuuint64_t strides[1] = {row_bytes};
        cuuint32_t box[2] = {(cuuint32_t)kBoxBytes, (cuuint32_t)kTileRows};
        cuuint32_t es[2] = {1, 1};
        if (fn(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(w.data), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    if (group) {
        // scales [N][K / 32] f32 in 128-row boxes of one weight box's groups
        const cuuint32_t gpb = int4 ? MmaCodes<kQInt4>::kGPB : MmaCodes<kQInt8>::kGPB;
        cuuint64_t dims[2] = {(cuuint64_t)(w.K / 32), (cuuint64_t)w.N};
        cuuint64_t strides[1] = {(cuuint64_t)(w.K / 32) * sizeof(float)};
        cuuint32_t box[2] = {gpb, (cuuint32_t)kTileRows};
        cuuint32_t es[2] = {1, 1};
        if (fn(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(w.scales), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    MmaParams p{};
    p.X = X;
    p.S = w.scales;
    p.Y = Y;
    p.ldx = (long long)(B > 1 ? ldx : w.K);
    p.ldy = (long long)ldy;
    p.N = (int)w.N;
    p.K = (int)w.K;
    p.B = (int)B;
    p.parts = sh.parts;
    p.nb = sh.nb;
    p.err = err;
    if (int4)
        return group ? run_mma_nt<kQInt4, true>(B, tw, ts, p, sh, st) : run_mma_nt<kQInt4, false>(B, tw, ts, p, sh, st);
    return group ? run_mma_nt<kQInt8, true>(B, tw, ts, p, sh, st) : run_mma_nt<kQInt8, false>(B, tw, ts, p, sh, st);
}

}  // namespace pyxis
