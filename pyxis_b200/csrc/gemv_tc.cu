// gemv_tc.cu -- int8 decode GEMV / small-batch matmul on the tensor cores (tcgen05 kind::i8).
//
// y[b, n] = s[n] * sum_k x[b, k] * q[n, k] for int8 weights with one scale per row (the model's
// int8 policy, src/model.rs:527; block == in_features) and B = 1..8 input rows: the decode GEMVs
// and the lm_head of src/matmul.rs:21-97 / src/output_head.rs:21-23.
//
// The weights never touch the CUDA cores.  Each 128-row x 128-byte block of codes goes from HBM
// to shared memory by TMA (128-byte swizzle = the MMA's canonical K-major layout) and from there
// straight into tcgen05.mma.kind::i8 as operand A.  Operand B is x written as four signed 7-bit
// digits per element: with 2^E > max|x_b| (one power of two per input row),
//     t = rint(x * 2^(27 - E)),  t = d0 2^21 + d1 2^14 + d2 2^7 + d3,  |d_i| <= 64,
// so x is carried to 27 bits and every product and sum inside the MMA is exact int32.  B's 16 or
// 32 columns are (row b, digit i) pairs; the epilogue recombines
//     y = s[n] * 2^(E - 27) * (D0 2^21 + D1 2^14 + D2 2^7 + D3)
// in int64 / double and rounds once to f32.  The only error is x's 27-bit representation.
//
// CTA (persistent, one per SM): warp 0 = TMA producer into an S-stage ring (16 KB stages),
// warp 1 = TMEM owner + MMA issuer (M=128, N=16|32, K=32 per instruction, 8 accumulators per
// tile segment so that consecutive stages do not wait on each other, double-buffered in TMEM
// across segments), warps 2-5 = epilogue (tcgen05.ld, one TMEM lane = one weight row), warps
// 6-11 helpers.  x itself arrives by one TMA box straight into the digit operand's shared memory
// (each 512-byte block of 128 values of one token is where that block's four digit rows go),
// issued before the first weight copy (or, under programmatic dependent launch, by a helper warp
// right after the predecessor finishes), so the whole ring streams weights from the start; warps
// 2-11 convert the blocks in place in the order the MMAs take the K-blocks, and the MMA issuer
// waits for each K-block's digits only.  A tile whose stages span several CTAs has its partial int32
// sums added exactly with atomics into a scratch slot, and the CTA that finishes the tile last
// converts it and zeroes the scratch for the next launch.  The schedule is stream-K: every CTA
// gets the same number of (tile, K-block) stages, and works on its (possibly shared) first and
// last tiles before the whole tiles between them.  Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "argmax.h"
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace pyxis {
namespace {

constexpr int TM = 128;    // weight rows per tile
constexpr int TKB = 128;   // K bytes (= int8 codes) per stage
constexpr int kMaxTok = 8;
// warp 0 the TMA producer, warp 1 the MMA issuer, warps 2-5 the epilogue, 6-11 helpers: warps 2-11
// build x's digit operand (with one warp per SM sub-partition the build's dependent chains ran
// at ~1.2 us per pass; more warps hide their latency)
constexpr int kEpiWarps = 4, kHelperWarps = 6;
constexpr int kBuildWarp0 = 2, kBuildWarps = kEpiWarps + kHelperWarps;
constexpr int kXWarp = 2 + kEpiWarps;  // the helper that issues x's copy under programmatic launch
constexpr int kThreads = 32 * (kBuildWarp0 + kBuildWarps);
constexpr int kMaxKb = 48;  // K-blocks of the digit operand (it is at most 96 KB)
constexpr uint32_t kStageBytes = TM * TKB;
constexpr uint32_t kSmemTotal = 222 * 1024;
constexpr int kMaxStages = 12;
constexpr uint64_t kTimeoutNs = 2000000000ull;
// The 4 MMAs of a stage (one per 32-byte K slice) write 4 separate accumulators, and the even and
// odd stages of a tile use two different sets of 4: an MMA depends only on the one issued 8 MMAs
// (two stages) earlier, so consecutive stages do not serialise on the MMA latency.  The epilogue
// adds them (exact int32).  TMEM: 2 buffers x 8 accumulators x NB columns (256 or 512).
constexpr int kAccPerStage = TKB / 32;
constexpr int kAccSets = 2;
constexpr int kAccPerBuf = kAccPerStage * kAccSets;
// x -> digits: t + kDigitBias has the base-128 digits d_i + 64 (all in [0, 128]), so the balanced
// digits come out of shifts and masks; kDigitBias = 64 * (2^21 + 2^14 + 2^7 + 1).
constexpr int kDigitBias = 135274560;
enum { kErrProd = 0x301, kErrMma = 0x302, kErrEpi = 0x303, kErrDrain = 0x304 };

struct Params {
    int N, K, B, NB;
    int num_kb, num_tiles, stages;
    uint32_t tmem_cols;
    int pdl;       // launched with programmatic stream serialization
    long long total_stages;  // num_tiles * num_kb, split evenly over the grid (stream-K)
    uint32_t xd_bytes;
    const float *x;
    long long ldx;
    const float *scales;
    float *y;
    long long ldy;
    int *accum;         // [grid][NB][128] int32 partial tiles, zero between launches
    unsigned *tickets;  // [grid], zero between launches
    int *err;
    // A vocab shard of the greedy head: keys[b] = the max over this launch's logits of row b of
    // argmax_key_global(y, key_base + n) (0 on entry); null otherwise.
    unsigned long long *keys;
    long long key_base;
};

// int8 instruction descriptor: s32 accumulate, signed A and B, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

PYXIS_DEVINL void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

PYXIS_DEVINL void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2^e as a float for -126 <= e <= 127 (exact)
PYXIS_DEVINL float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// max that keeps a NaN once seen (fmaxf drops it): a NaN in x must reach every output
PYXIS_DEVINL float max_nan(float m, float a) { return (a > m || a != a) ? a : m; }

PYXIS_DEVINL void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

PYXIS_DEVINL float combine(const int *D, double xs, double sr) {
    const long long s = (long long)D[0] * 2097152LL + (long long)D[1] * 16384LL + (long long)D[2] * 128LL + D[3];
    return (float)((double)s * xs * sr);
}

// Stream-K schedule: the num_tiles x num_kb stages are cut into gridDim.x equal contiguous
// ranges; a tile whose stages span several CTAs is combined exactly (int32 atomics) in the slot
// of the first CTA that touches it -- each CTA is the first of at most one shared tile.
// A CTA works through its range as tile segments in this order: the first tile's, the last
// tile's (the two that may be shared with the neighbouring CTAs, so that their fix-ups happen
// while the stream is still running), then the whole tiles between them.
struct Sched {
    long long T;
    int G, nkb;
    PYXIS_DEVINL long long begin(int c) const { return (long long)c * T / G; }
    PYXIS_DEVINL int owner(long long s) const { return (int)(((s + 1) * G + T - 1) / T - 1); }
    PYXIS_DEVINL int num_segments(long long b, long long e) const {
        return (int)((e - 1) / nkb - b / nkb) + 1;
    }
    // stages [s0, s1) of segment i of the range [b, e)
    PYXIS_DEVINL void segment(long long b, long long e, int i, long long &s0, long long &s1) const {
        const long long ft = b / nkb, lt = (e - 1) / nkb;
        const long long tile = i == 0 ? ft : (i == 1 ? lt : ft + i - 1);
        s0 = b > tile * nkb ? b : tile * nkb;
        s1 = e < (tile + 1) * nkb ? e : (tile + 1) * nkb;
    }
};

// x [B][K] f32 by one TMA box into the digit operand's own space, block (K-block kb, token b) of
// 128 values at byte (kb NB / 4 + b) 512 -- exactly the four digit rows it becomes -- with the
// token slots past B zero-filled.
PYXIS_DEVINL void issue_x_copy(const CUtensorMap *tm_x, uint8_t *xd, uint32_t bytes, uint64_t *xfull) {
    tc::mbar_arrive_expect_tx(xfull, bytes);
    tc::tma_load_3d(xd, tm_x, 0, 0, 0, xfull);
}

__global__ void __launch_bounds__(kThreads, 1)
    gemv_tc_i8_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                      const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *xd = smem;                    // digit operand: [kb][NB rows][128 B], 128-byte swizzle
    uint8_t *ring = smem + p.xd_bytes;     // stages of 128 rows x 128 B codes
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + (size_t)p.stages * kStageBytes);
    uint64_t *full = bars, *empty = bars + kMaxStages;
    uint64_t *tfull = bars + 2 * kMaxStages, *tempty = tfull + 2, *drain = tempty + 2;
    uint64_t *xfull = drain + 1, *xready = drain + 2;                // xready: [kMaxKb]
    double *xscale = reinterpret_cast<double *>(xready + kMaxKb);    // [kMaxTok]
    float *red = reinterpret_cast<float *>(xscale + kMaxTok);        // [kMaxTok][kBuildWarps]
    int *xexp = reinterpret_cast<int *>(red + kMaxTok * kBuildWarps);  // [kMaxTok]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(xexp + kMaxTok);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *last_flag = abort_flag + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 4);
        }
        tc::mbar_init(drain, 1);
        tc::mbar_init(xfull, 1);
        for (int kb = 0; kb < p.num_kb; ++kb) tc::mbar_init(&xready[kb], p.B);  // one arrival per token block
        *abort_flag = 0;
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, p.tmem_cols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const Sched sc{p.total_stages, (int)gridDim.x, p.num_kb};
    const long long my_sb = sc.begin(blockIdx.x), my_se = sc.begin(blockIdx.x + 1);

    if (warp == 0) {
        // -------------------------------------------------------------------- TMA producer
        if (lane == 0) {
            tc::prefetch_tmap(&tm_w);
            tc::prefetch_tmap(&tm_x);
            // x first, ahead of the weight stream in the memory queues -- unless it comes from a
            // kernel still running (PDL): then a helper warp issues it as soon as
            // griddepcontrol.wait returns, while this thread keeps the weight stages coming
            if (!p.pdl) issue_x_copy(&tm_x, xd, p.xd_bytes, xfull);
            int g = 0;
            const long long sb = my_sb, se = my_se;
            const int nseg = sc.num_segments(sb, se);
            bool ok = true;
            // ring slot s of stage g and its round ph = g / stages, tile and K-block of the stage:
            // all advanced by increments (a division per stage was most of this thread's work)
            int s = 0, ph = 0;
            for (int i = 0; i < nseg && ok; ++i) {
                long long s0, s1;
                sc.segment(sb, se, i, s0, s1);
                int tile = (int)(s0 / p.num_kb), kb = (int)(s0 - (long long)tile * p.num_kb);
                for (long long st = s0; st < s1; ++st, ++g) {
                    if (g >= p.stages && !tc::mbar_wait_bounded(&empty[s], (uint32_t)((ph - 1) & 1), abort_flag, p.err,
                                                                kErrProd, kTimeoutNs)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&full[s], kStageBytes);
                    tc::tma_load_2d(ring + (size_t)s * kStageBytes, &tm_w, kb * TKB, tile * TM, &full[s]);
                    if (++kb == p.num_kb) {
                        kb = 0;
                        ++tile;
                    }
                    if (++s == p.stages) {
                        s = 0;
                        ++ph;
                    }
                }
            }
            if (*abort_flag) {  // let the copies already issued land (x: see the helper below)
                volatile int no_abort = 0;
                if (!p.pdl) tc::mbar_wait_bounded(xfull, 0, &no_abort, p.err, kErrDrain, 100000000ull);
                for (int j = g > p.stages ? g - p.stages : 0; j < g; ++j)
                    tc::mbar_wait_bounded(&full[j % p.stages], (j / p.stages) & 1, &no_abort, p.err, kErrDrain, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // -------------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(TM, p.NB);
            // descriptors advance by constant offsets (start address in 16-byte units), the ring
            // slot and its phase by increments: no per-stage division or descriptor rebuild
            const uint64_t ring_d = tc::desc_sw128(tc::smem_u32(ring)), xd_d = tc::desc_sw128(tc::smem_u32(xd));
            const uint32_t stage_step = kStageBytes >> 4, kb_step = (uint32_t)(p.NB * TKB) >> 4;
            int li = 0, s = 0, ph = 0;
            bool ok = true;
            const int nseg = sc.num_segments(my_sb, my_se);
            for (; li < nseg && ok; ++li) {
                long long s0, s1;
                sc.segment(my_sb, my_se, li, s0, s1);
                const int kb0 = (int)(s0 % p.num_kb), nk = (int)(s1 - s0);
                const int buf = li & 1;
                if (li >= 2) {
                    ok = tc::mbar_wait_bounded(&tempty[buf], ((li >> 1) - 1) & 1, abort_flag, p.err, kErrMma, kTimeoutNs);
                    if (!ok) break;
                }
                tc::tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * kAccPerBuf * p.NB);
                for (int kb = kb0; kb < kb0 + nk; ++kb) {
                    // the K-block's digits (converted in place by the builders) and the stage's codes
                    ok = tc::mbar_wait_bounded(&xready[kb], 0, abort_flag, p.err, kErrMma, kTimeoutNs) &&
                         tc::mbar_wait_bounded(&full[s], (uint32_t)(ph & 1), abort_flag, p.err, kErrMma, kTimeoutNs);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint64_t a0 = ring_d + (uint64_t)(s * stage_step);
                    const uint64_t b0 = xd_d + (uint64_t)(kb * kb_step);
                    const uint32_t dset = d + (uint32_t)(((kb - kb0) & 1) * kAccPerStage * p.NB);
#pragma unroll
                    for (int q = 0; q < kAccPerStage; ++q)
                        mma_i8(dset + (uint32_t)(q * p.NB), a0 + (uint64_t)(2 * q), b0 + (uint64_t)(2 * q), idesc,
                               kb - kb0 >= 2 ? 1u : 0u);
                    tc::mma_commit(&empty[s]);
                    if (++s == p.stages) {
                        s = 0;
                        ++ph;
                    }
                }
                if (ok) tc::mma_commit(&tfull[buf]);
            }
            tc::mma_commit(drain);
            volatile int no_abort = 0;
            tc::mbar_wait_bounded(drain, 0, &no_abort, p.err, kErrDrain, kTimeoutNs);
        }
    } else {
        // -------------------------------------------------------------------- digit operand
        const int bt = threadIdx.x - 32 * kBuildWarp0, nbt = 32 * kBuildWarps;  // warps 2-11
        const int bwarp = warp - kBuildWarp0;
        if (p.pdl && warp == kXWarp && lane == 0) {
            pdl_wait();  // x comes from the previous kernel
            issue_x_copy(&tm_x, xd, p.xd_bytes, xfull);
        }
        pdl_trigger();
        // K-blocks this CTA multiplies: a contiguous run (mod num_kb) from need_lo unless it spans
        // a whole tile; the MMAs take them in that order
        const int need_lo = (int)(my_sb % p.num_kb);
        const int n_need = my_se - my_sb >= p.num_kb ? p.num_kb : (int)(my_se - my_sb);
        const int nbq = p.NB / 4;  // token slots per K-block
        const float4 *xd4 = reinterpret_cast<const float4 *>(xd);
        const bool x_ok = tc::mbar_wait_bounded(xfull, 0, abort_flag, p.err, kErrMma, kTimeoutNs);
        // (x was issued after griddepcontrol.wait, by the producer or the helper warp.  The warps
        // that write global memory -- the epilogue: y, the shared scratch, the keys -- wait on the
        // dependency themselves, before their first write.)
        if (x_ok) {
            // max |x| of every token over all of K, the same in every CTA
            float m[kMaxTok];
#pragma unroll
            for (int b = 0; b < kMaxTok; ++b) m[b] = 0.f;
#pragma unroll 2
            for (int i = bt; i < p.num_kb * 32; i += nbt) {  // (K-block, quad of the block)
                const int kb = i >> 5, q = i & 31;
                float4 v[kMaxTok];
#pragma unroll
                for (int b = 0; b < kMaxTok; ++b)
                    if (b < p.B) v[b] = xd4[(size_t)(kb * nbq + b) * 32 + q];
#pragma unroll
                for (int b = 0; b < kMaxTok; ++b)
                    if (b < p.B)
                        m[b] = max_nan(max_nan(max_nan(max_nan(m[b], fabsf(v[b].x)), fabsf(v[b].y)), fabsf(v[b].z)),
                                       fabsf(v[b].w));
            }
            // the tokens' butterflies interleaved, step by step: independent shuffles (tokens past B
            // reduce zeros and are not stored)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int b = 0; b < kMaxTok; ++b) m[b] = max_nan(m[b], __shfl_xor_sync(0xffffffffu, m[b], o));
            if (lane == 0)
#pragma unroll
                for (int b = 0; b < kMaxTok; ++b)
                    if (b < p.B) red[b * kBuildWarps + bwarp] = m[b];
        }
        named_bar(1, nbt);
        if (bt < p.B) {
            float m = red[bt * kBuildWarps];
            for (int w = 1; w < kBuildWarps; ++w) m = max_nan(m, red[bt * kBuildWarps + w]);
            int E = 0;
            if (m > 0.f && isfinite(m)) frexpf(m, &E);  // m < 2^E
            xexp[bt] = E;
            xscale[bt] = isfinite(m) ? ldexp(1.0, E - 27) : __longlong_as_double(0x7ff8000000000000ll);
        }
        named_bar(1, nbt);
        // digits: t = rint(x 2^(27-E)) as 4 balanced base-128 digits.  A warp converts one (K-block,
        // token) block at a time in place -- its 128 f32 values are read into the lanes, then the
        // block's 512 bytes become the token's four 128-byte-swizzled digit rows -- in the order the
        // MMAs take the K-blocks, and each K-block's digits are handed to the MMA warp as soon as
        // its B blocks are done.  The token slots past B arrived as zeros, i.e. zero digits.
        if (x_ok) {
            for (int blk = bwarp; blk < n_need * p.B; blk += kBuildWarps) {
                const int o = blk / p.B, b = blk - o * p.B;
                const int kb = need_lo + o < p.num_kb ? need_lo + o : need_lo + o - p.num_kb;
                uint8_t *kbase = xd + (size_t)kb * (p.NB * TKB);
                const float4 xv = xd4[(size_t)(kb * nbq + b) * 32 + lane];  // elements 4 lane .. 4 lane + 3
                __syncwarp();  // the whole block is in registers before any digit overwrites it
                // x 2^(27-E) exactly, as two power-of-two products (27 - E lies in [-101, 175])
                const int sh = 27 - xexp[b];
                const int sa = sh < 127 ? sh : 127;
                const float f1 = pow2f(sa), f2 = pow2f(sh - sa);
                const float xe[4] = {xv.x, xv.y, xv.z, xv.w};
                uint32_t word[4] = {0, 0, 0, 0};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float v = (xe[e] * f1) * f2;
                    const int t = isfinite(v) ? __float2int_rn(v) : 0;
                    const uint32_t ub = (uint32_t)(t + kDigitBias);
                    word[0] |= (ub >> 21) << (8 * e);
                    word[1] |= ((ub >> 14) & 127u) << (8 * e);
                    word[2] |= ((ub >> 7) & 127u) << (8 * e);
                    word[3] |= (ub & 127u) << (8 * e);
                }
                const int c = lane >> 2;  // 16-byte chunk of the 128-byte row holding K 4 lane .. 4 lane + 3
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = 4 * b + i;
                    uint8_t *row = kbase + (r >> 3) * 1024 + (r & 7) * 128;
                    *reinterpret_cast<uint32_t *>(row + ((c ^ (r & 7)) << 4) + 4 * (lane & 3)) =
                        __vsub4(word[i], 0x40404040u);  // digit + 64 -> digit, per byte
                }
                tc::fence_proxy_async_smem();  // digit writes -> the MMAs' reads
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&xready[kb]);
            }
        }

        if (warp < 2 + kEpiWarps) {
            // ---------------------------------------------------------------- epilogue
            // All four warps run the same item sequence and the same named barriers; a warp
            // whose wait ran out skips the work but keeps the barrier sequence.
            // y, the shared scratch and the keys are written only after the previous kernel is
            // done with them (it has finished by now: x came after the same wait)
            pdl_wait();
            const int qd = warp & 3;  // TMEM lane quarter of this warp
            const int nseg = sc.num_segments(my_sb, my_se);
            uint64_t kmax[kMaxTok];  // the greedy head's keys of the logits this thread wrote
#pragma unroll
            for (int b = 0; b < kMaxTok; ++b) kmax[b] = 0;
            for (int li = 0; li < nseg; ++li) {
                long long s0, s1;
                sc.segment(my_sb, my_se, li, s0, s1);
                const int tile = (int)(s0 / p.num_kb);
                const int nacc = (s1 - s0 >= 2 ? kAccSets : 1) * kAccPerStage;  // accumulators written
                const int first = sc.owner((long long)tile * p.num_kb);
                const int parts = sc.owner((long long)(tile + 1) * p.num_kb - 1) - first + 1;
                const int buf = li & 1;
                int ok = 1;
                if (lane == 0) ok = tc::mbar_wait_bounded(&tfull[buf], (li >> 1) & 1, abort_flag, p.err, kErrEpi, kTimeoutNs);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                int D[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) D[j] = 0;
                if (ok) {
                    tc::tc_fence_after();
                    const uint32_t taddr = tmem_base + ((uint32_t)(32 * qd) << 16) + (uint32_t)(buf * kAccPerBuf * p.NB);
#pragma unroll
                    for (int a = 0; a < kAccPerBuf; ++a) {
                        if (a >= nacc) break;
                        int T[16];
                        tmem_ld16(taddr + (uint32_t)(a * p.NB), T);
#pragma unroll
                        for (int j = 0; j < 16; ++j) D[j] += T[j];
                        if (p.NB == 32) {
                            tmem_ld16(taddr + (uint32_t)(a * p.NB + 16), T);
#pragma unroll
                            for (int j = 0; j < 16; ++j) D[16 + j] += T[j];
                        }
                    }
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&tempty[buf]);
                }
                const int rl = 32 * qd + lane;
                const int row = tile * TM + rl;
                if (parts == 1) {
                    if (ok && row < p.N) {
                        const double sr = (double)__ldg(p.scales + row);
#pragma unroll
                        for (int b = 0; b < kMaxTok; ++b)
                            if (b < p.B) {
                                const float v = combine(&D[4 * b], xscale[b], sr);
                                p.y[(size_t)b * p.ldy + row] = v;
                                if (p.keys) {
                                    const uint64_t k = argmax_key_global(v, p.key_base + row);
                                    kmax[b] = k > kmax[b] ? k : kmax[b];
                                }
                            }
                    }
                } else {
                    // column j of the slot is 128 contiguous ints: a warp's 32 rows share one line
                    int *acc = p.accum + (size_t)first * 32 * TM + rl;
                    if (ok) {
#pragma unroll
                        for (int j = 0; j < 4 * kMaxTok; ++j)
                            if (j < 4 * p.B) atomicAdd(acc + j * TM, D[j]);
                    }
                    __threadfence();
                    named_bar(2, 128);
                    if (warp == 2 && lane == 0) *last_flag = atomicAdd(&p.tickets[first], 1u) == (unsigned)(parts - 1);
                    named_bar(2, 128);
                    const bool last = *last_flag;
                    if (last) {
                        __threadfence();
                        int S[32];
#pragma unroll
                        for (int j = 0; j < 4 * kMaxTok; ++j) {
                            S[j] = 0;
                            if (j < 4 * p.B) {
                                S[j] = __ldcg(acc + j * TM);
                                acc[j * TM] = 0;  // leave the scratch zeroed for the next launch
                            }
                        }
                        if (row < p.N && !*abort_flag) {
                            const double sr = (double)__ldg(p.scales + row);
#pragma unroll
                            for (int b = 0; b < kMaxTok; ++b)
                                if (b < p.B) {
                                    const float v = combine(&S[4 * b], xscale[b], sr);
                                    p.y[(size_t)b * p.ldy + row] = v;
                                    if (p.keys) {
                                        const uint64_t k = argmax_key_global(v, p.key_base + row);
                                        kmax[b] = k > kmax[b] ? k : kmax[b];
                                    }
                                }
                        }
                    }
                    named_bar(2, 128);
                    if (last && warp == 2 && lane == 0) p.tickets[first] = 0;
                }
            }
            if (p.keys) {
                // one atomic per warp and input row; max is associative, so the order of the
                // CTAs' atomics does not matter
#pragma unroll
                for (int b = 0; b < kMaxTok; ++b)
                    if (b < p.B) {
                        const uint64_t k = warp_max_u64(kmax[b]);
                        if (lane == 0 && k) atomicMax(p.keys + b, (unsigned long long)k);
                    }
            }
        }
    }
    if (p.pdl && warp == kXWarp && lane == 0 && *abort_flag) {  // x's copy must land before the CTA leaves
        volatile int no_abort = 0;
        tc::mbar_wait_bounded(xfull, 0, &no_abort, p.err, kErrDrain, 100000000ull);
    }
    __syncwarp();
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tensor_map_encoder(); }

struct Plan {
    bool ok = false;
    int NB = 16, stages = 0;
    uint32_t xd_bytes = 0;
};

Plan plan_for(const QMatrix &w, size_t B, int num_sms) {
    Plan pl;
    if (w.qtype != kQInt8 || w.block_size != w.K || B < 1 || B > (size_t)kMaxTok) return pl;
    if (w.K == 0 || w.K % TKB || w.K > 65536 || w.N == 0 || w.N > (size_t)INT32_MAX / 2) return pl;
    if (reinterpret_cast<uintptr_t>(w.data) & 15) return pl;
    pl.NB = 4 * (int)B <= 16 ? 16 : 32;
    pl.xd_bytes = (uint32_t)(w.K * pl.NB);
    if (pl.xd_bytes > 96 * 1024) return pl;
    if (w.K / TKB > (size_t)kMaxKb) return pl;
    const uint32_t avail = kSmemTotal - 1024 - 2048 - pl.xd_bytes;  // alignment slack, barriers and scalars
    pl.stages = std::min<int>(kMaxStages, (int)(avail / kStageBytes));
    if (pl.stages < 2) return pl;
    pl.ok = true;
    return pl;
}

}  // namespace

size_t gemv_tc_scratch_bytes(int max_grid) {
    return (size_t)max_grid * TM * 32 * sizeof(int) + (size_t)max_grid * sizeof(unsigned) + 256;
}

bool gemv_tc_supported(const QMatrix &w, size_t B, int num_sms) { return plan_for(w, B, num_sms).ok; }

cudaError_t launch_gemv_tc(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y, size_t ldy,
                           void *scratch, size_t scratch_bytes, int *err, int num_sms, cudaStream_t st,
                           uint64_t *keys, long long key_base) {
    const Plan pl = plan_for(w, B, num_sms);
    if (!pl.ok) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(X) & 15) || (B > 1 && ldx % 4)) return cudaErrorInvalidValue;
    const int num_tiles = (int)((w.N + TM - 1) / TM);
    const long long total = (long long)num_tiles * (long long)(w.K / TKB);
    // Every CTA pays a fixed start-up (TMEM, barriers, the digit operand) and shared tiles pay
    // atomics: give each CTA at least kMinStagesPerCta stages unless that leaves SMs idle.
    constexpr long long kMinStagesPerCta = 4;
    const int grid = (int)std::max<long long>(1, std::min<long long>(num_sms, (total + kMinStagesPerCta - 1) / kMinStagesPerCta));
    if (!scratch || scratch_bytes < gemv_tc_scratch_bytes(grid)) return cudaErrorInvalidValue;
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    CUtensorMap tm;
    cuuint64_t dims[2] = {(cuuint64_t)w.K, (cuuint64_t)w.N};
    cuuint64_t strides[1] = {(cuuint64_t)w.K};
    cuuint32_t box[2] = {TKB, TM};
    cuuint32_t es[2] = {1, 1};
    if (fn(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(w.data), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    // x as (128 values of a K-block, token, K-block) with strides (4 B, ldx * 4, 512 B): one box of
    // (128, NB / 4, K / 128) lands as [K-block][token slot][128] f32, token slots past B zero
    CUtensorMap tx;
    {
        cuuint64_t xdims[3] = {(cuuint64_t)TKB, (cuuint64_t)B, (cuuint64_t)(w.K / TKB)};
        cuuint64_t xstrides[2] = {(cuuint64_t)(B > 1 ? ldx : w.K) * sizeof(float), (cuuint64_t)TKB * sizeof(float)};
        cuuint32_t xbox[3] = {(cuuint32_t)TKB, (cuuint32_t)(pl.NB / 4), (cuuint32_t)(w.K / TKB)};
        cuuint32_t xes[3] = {1, 1, 1};
        if (fn(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(X), xdims, xstrides, xbox, xes,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    Params p{};
    p.N = (int)w.N;
    p.K = (int)w.K;
    p.B = (int)B;
    p.NB = pl.NB;
    p.num_kb = (int)(w.K / TKB);
    p.num_tiles = num_tiles;
    p.total_stages = total;
    p.stages = pl.stages;
    p.tmem_cols = (uint32_t)(2 * kAccPerBuf * pl.NB);  // 256 or 512
    p.pdl = pdl_enabled() ? 1 : 0;
    p.xd_bytes = pl.xd_bytes;
    p.x = X;
    p.ldx = (long long)ldx;
    p.scales = w.scales;
    p.y = Y;
    p.ldy = (long long)ldy;
    {
        uint8_t *sb = reinterpret_cast<uint8_t *>(scratch);
        p.accum = reinterpret_cast<int *>(sb);
        p.tickets = reinterpret_cast<unsigned *>(sb + (size_t)grid * TM * 32 * sizeof(int));
    }
    p.err = err;
    p.keys = reinterpret_cast<unsigned long long *>(keys);
    p.key_base = key_base;
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t attr = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(gemv_tc_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal);
    });
    if (attr != cudaSuccess) return attr;
    return launch_kernel(gemv_tc_i8_kernel, dim3(grid), dim3(kThreads), kSmemTotal, st, tm, tx, p);
}

}  // namespace pyxis
