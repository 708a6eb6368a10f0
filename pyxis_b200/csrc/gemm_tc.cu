// gemm_tc.cu -- prefill (many-token) quantized GEMM on the 5th-generation tensor cores.
//
// Y[m, n] = sum_k X[m, k] * q[n, k] * scale(n, k)   for M tokens x N weight rows, the batched form
// of src/matmul.rs:21-97 (the reference's prefill issues one matmul per position,
// src/attention.rs:74-79), computed as:
//
//   1. split_x: each token row is scaled by a power of two 2^e (max |x| -> [2^14, 2^15)) and split
//      into fp16 hi + lo (x*2^e = hi + lo + O(2^-22 |x*2^e|)): 22 significant bits, as accurate
//      against the reference's f32 sums as exact arithmetic (bf16 hi/lo keeps only 16).
//   2. the tile kernel, one CTA per 128 weight rows x 128 tokens (x gridDim.z K slices when
//      there are fewer tiles than SMs and splitting saves waves), warp-specialised:
//        warp 0      TMA producer: raw int8/int4 codes + fp16 X hi/lo tiles into a ring of 4
//                    stages (one scale per row) or 3 (group scales, whose A_lo tiles take room)
//        warp 1      TMEM owner and MMA issuer: tcgen05.mma kind::f16, M=128, K=16; the token
//                    tiles hi and lo sit back to back, so one N=256 MMA per K-step gives W x_hi in
//                    accumulator columns [0,128) and W x_lo in [128,256) (N=64 pairs for tiles of
//                    <= 64 tokens)
//        warps 2-5   converters (one per weight row): codes -> the weight operand in the
//                    128B-swizzled K-major layout.
//                    One scale per row: the codes themselves, exact fp16 integers.  A scale per
//                    group along K (int4 group 32, GGUF int8 block 32): q * s * 2^e (e per row,
//                    keeping the values normal fp16) as fp16 hi + lo, and a second MMA per K-step
//                    adds W_lo x_hi -- so group scales never force a fold.
//        warps 6-21  epilogue: tcgen05.ld the accumulator (4 lane quarters x 4 column quarters),
//                    fold, apply the row scale (or 2^-e) and the token's 2^-e', store Y
//      Accumulation: each "period" of up to 256 of K goes to one of two TMEM buffers; the
//      epilogue folds it into fp32 registers (round-to-nearest) while the MMA warp fills the
//      other buffer.  Long fp32 sums inside the tensor core drift (measured 1.9e-3 on the
//      floor-relative metric for K = 2048 in one accumulator: 256 accumulations); a period is at
//      most 16 K-steps (16 or 32 accumulations per column).
//      The MMA rate is bounded by the issuing thread's own instruction stream (a few scalar
//      instructions per MMA cost as much as the MMA), so that loop is unrolled over the ring and
//      the fold period: slots, phases, buffers and commit points are compile-time.
//   Weight codes are exact in fp16 and the token power of two is exact, so the only rounding
//   besides the fp32 accumulation is the lo terms' 2^-22 (and, with group scales, q * s in f32).
//
// Every mbarrier wait is bounded (globaltimer); a wait that runs out records an error code in
// the context's device flag and the CTA winds down (drains its MMAs / copies, frees TMEM).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "kernels.h"
#include "split_x.cuh"
#include "fp16_codes.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace pyxis {
namespace {

constexpr int BM = 128;  // weight rows per tile: MMA M, TMEM lanes
constexpr int BN = 128;  // tokens per tile
constexpr int BK = 64;   // K per stage: one 128-byte swizzle row of fp16
constexpr int kConvWarp0 = 2, kNumConvWarps = 4;            // one thread per weight row
constexpr int kConvPerRow = kNumConvWarps * 32 / 128;      // threads per weight row (1 or 2)
constexpr int kEpiWarp0 = kConvWarp0 + kNumConvWarps, kNumEpiWarps = 16;  // 4 lane x 4 column quarters
constexpr int kThreads = (kEpiWarp0 + kNumEpiWarps) * 32;  // 704
constexpr uint32_t kAccCols = 2 * BN;                      // one accumulator: x_hi columns | x_lo columns
constexpr uint32_t kTmemCols = 2 * kAccCols;               // double-buffered: 512
constexpr uint32_t kABytes = BM * BK * 2;                  // one fp16 weight tile
constexpr uint32_t kBBytes = BN * BK * 2;                  // one fp16 token tile (hi or lo)
constexpr uint32_t kRBytes = BM * 64;                      // raw codes of a stage (<= 64 B per row)
constexpr uint64_t kTimeoutNs = 4000000000ull;

// Shared memory: a ring of NA converted weight tiles (A_hi, plus A_lo for grouped weights when LO)
// and a ring of NB TMA stages (x_hi|x_lo token tile and raw codes).  A TMA stage's slot is held
// from its copy's issue to its MMAs' end, so NB sets how much copy latency is hidden; a converted
// tile's slot only spans its conversion and its MMAs, so a shorter A ring suffices when converting
// a stage takes no longer than its MMAs.  Per-row weights (no A_lo): NA = NB = 4.  Grouped weights:
// NA = NB = 3 (their converters are the slower role: NA = 2, NB = 4 measured 7% slower).
template <int NA, int NB, bool LO>
struct Smem {
    static constexpr uint32_t ahi = 0;
    static constexpr uint32_t alo = ahi + NA * kABytes;
    static constexpr uint32_t b = alo + (LO ? NA * kABytes : 0);  // per stage: hi rows 0..127, lo rows 128..255
    static constexpr uint32_t r = b + NB * 2 * kBBytes;
    static constexpr uint32_t bar = r + NB * kRBytes;
    static constexpr uint32_t num_bars = 2 * NB + 2 * NA + 2 + 2 + 1;
    static constexpr uint32_t misc = bar + num_bars * 8;
    static constexpr uint32_t rowinv = misc + 16;  // [BM] per-row 2^-e of grouped weights
    static constexpr uint32_t bytes = rowinv + BM * 4 + 1024;  // + alignment slack
};
constexpr int kTilesGrouped = 3, kStagesGrouped = 3, kStagesRow = 4;
static_assert(Smem<kTilesGrouped, kStagesGrouped, true>::bytes <= 232448 &&
                  Smem<kStagesRow, kStagesRow, false>::bytes <= 232448,
              "227 KB of dynamic shared memory per CTA");

// Device error codes (first one wins): which role's wait ran out.
enum { kErrProducer = 0x101, kErrConverter = 0x102, kErrMma = 0x103, kErrEpilogue = 0x104, kErrDrain = 0x105 };

struct TcParams {
    int M, N, K;
    int qtype;
    int grouped;            // 0: one scale per row (block == K), applied at the end; 1: a scale per group
    int group_k;            // grouped: elements per scale group (a multiple of 32)
    int groups_per_row;     // grouped: K / group_k
    int ksteps_per_period;  // K-steps (16 each) accumulated in TMEM before the epilogue folds them
    const float *scales;
    const float *xinv;      // [M] 2^-e per token
    float *Y;
    long long ldy;
    int *err;
    int kb_per_split;       // K-blocks of one blockIdx.z slice (split-K over gridDim.z)
    float *part;            // split-K: [gridDim.z][M][N] partial products, else nullptr
    const float *rowinv;    // pre-converted weights (PRE): [N] 2^-e per row
};




// A pair of codes q (exact floats) times the scale s (f32, rounded once) as fp16 hi + lo pairs:
// 22 significant bits.  hi is w rounded to 11 bits by Veltkamp's split (c = w (2^13 + 1),
// hi = c - (c - w)), so it converts to fp16 exactly and lo = w - hi is exact in f32: one
// f32 -> f16 conversion per value.  The arithmetic is paired f32x2 (five instructions per pair;
// a - b is fma(b, -1, a), rounded once like the subtraction): the FP32 pipe bounds the converters.
PYXIS_DEVINL void split_pair(float2 q, float2 s, uint32_t &hi, uint32_t &lo) {
    const float2 m1 = make_float2(-1.f, -1.f);
    const float2 w = __fmul2_rn(q, s);
    const float2 c = __fmul2_rn(w, make_float2(8193.0f, 8193.0f));
    const float2 h = __ffma2_rn(__ffma2_rn(w, m1, c), m1, c);  // c - (c - w)
    const float2 l = __ffma2_rn(h, m1, w);                      // w - h
    hi = h2_bits(__floats2half2_rn(h.x, h.y));
    lo = h2_bits(__floats2half2_rn(l.x, l.y));
}

// Eight int4 codes (q + 8 in nibbles, element 2j low / 2j+1 high nibble of byte j) as exact float
// pairs in the converter order (e0,e4) (e1,e5) (e2,e6) (e3,e7).
PYXIS_DEVINL void u4x8_to_f32_pairs(uint32_t w, float2 (&e)[4]) {
    const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;  // even / odd elements
    const float2 m = f2(-kMagicU4, -kMagicU4);
    e[0] = fadd2(f2(byte_to_magic(lo, 0), byte_to_magic(lo, 2)), m);
    e[1] = fadd2(f2(byte_to_magic(hi, 0), byte_to_magic(hi, 2)), m);
    e[2] = fadd2(f2(byte_to_magic(lo, 1), byte_to_magic(lo, 3)), m);
    e[3] = fadd2(f2(byte_to_magic(hi, 1), byte_to_magic(hi, 3)), m);
}

// Byte offset of 16-byte chunk c of row r in a 128B-swizzled K-major tile (8-row 1024 B atoms).
PYXIS_DEVINL uint32_t sw128_off(int r, int c) { return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4); }

PYXIS_DEVINL void bar_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }
PYXIS_DEVINL void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
constexpr int kBarRowInv = 1;  // converters publish rowinv, the epilogue reads it at the end
constexpr int kRowInvThreads = (kNumConvWarps + kNumEpiWarps) * 32;

struct MmaRing {
    uint64_t *full, *conv, *empty, *aempty, *accfull, *accempty;
    volatile int *abort_flag;
    int *err;
};

// The MMA issuer for fold periods of SPP stages.  The issuing thread's own instruction stream
// bounds the tensor pipe: a ring slot, parity or accumulator buffer computed at run time between
// the MMAs measured up to 1.8x slower than the pipe's 128 cycles per 128x256x16 MMA.  So the loop
// is unrolled over lcm(2 NA, 2 NB, 2 SPP) stages, which makes the ring slots, the phase parities, the
// TMEM buffer and the commit points compile-time and advances the descriptors by immediates.
// Returns false when a wait gave up (the error is recorded, the abort flag raised).
__host__ __device__ constexpr int lcm_int(int a, int b) {
    int x = a, y = b;
    while (y) {
        const int t = x % y;
        x = y;
        y = t;
    }
    return a / x * b;
}

template <int NA, int NB, int SPP, bool GROUPED, bool SMALL, bool PRE>
__device__ __forceinline__ bool mma_loop(int num_kb, uint64_t ahi0, uint64_t alo0, uint64_t b0, uint32_t tmem_base,
                                      const MmaRing r) {
    constexpr int U = lcm_int(lcm_int(2 * NA, 2 * NB), 2 * SPP);
    constexpr uint32_t id_hilo = tc::idesc_f16_f32(BM, 2 * BN);  // rows x [x_hi; x_lo]
    constexpr uint32_t id_hi = tc::idesc_f16_f32(BM, BN);
    constexpr uint32_t id_64 = tc::idesc_f16_f32(BM, 64);
    for (int j0 = 0; j0 < num_kb; j0 += U) {
        // j0 is a multiple of U: j0 / NA, j0 / NB and j0 / SPP are even, so the ring parities and the
        // accumulator buffer of stage j0 + jj depend on jj alone
#pragma unroll
        for (int jj = 0; jj < U; ++jj) {
            if (j0 + jj >= num_kb) return true;
            const int a = jj % NA, s = jj % NB, sp = jj % SPP, buf = (jj / SPP) & 1;
            // (pre-converted weights arrive by TMA with the stage: full[s] covers them)
            if ((!PRE &&
                 !tc::mbar_wait_bounded(&r.conv[a], (uint32_t)((jj / NA) & 1), r.abort_flag, r.err, kErrMma, kTimeoutNs)) ||
                !tc::mbar_wait_bounded(&r.full[s], (uint32_t)((jj / NB) & 1), r.abort_flag, r.err, kErrMma, kTimeoutNs))
                return false;
            if (sp == 0) {
                const int period = (j0 + jj) / SPP;
                if (period >= 2 && !tc::mbar_wait_bounded(&r.accempty[buf], (uint32_t)(((period >> 1) - 1) & 1),
                                                          r.abort_flag, r.err, kErrMma, kTimeoutNs))
                    return false;
            }
            tc::tc_fence_after();
            const uint64_t ahi = ahi0 + (uint64_t)(a * (kABytes >> 4));
            const uint64_t alo = alo0 + (uint64_t)(a * (kABytes >> 4));
            const uint64_t bhi = b0 + (uint64_t)(s * (2 * kBBytes >> 4));
            const uint64_t blo = bhi + (uint64_t)(kBBytes >> 4);
            const uint32_t d = tmem_base + (uint32_t)(buf * kAccCols);
#pragma unroll
            for (int ks = 0; ks < BK / 16; ++ks) {
                const uint32_t acc = (ks | sp) ? 1u : 0u;  // a period's first K-step starts the sums
                if (!SMALL) {
                    // columns [0, 128): W x_hi, [128, 256): W x_lo -- one instruction reads A once
                    tc::mma_f16(d, ahi + 2 * ks, bhi + 2 * ks, id_hilo, acc);
                    if (GROUPED) tc::mma_f16(d, alo + 2 * ks, bhi + 2 * ks, id_hi, 1u);
                } else {
                    // <= 64 tokens: the rest of the token tile is TMA zero fill
                    tc::mma_f16(d, ahi + 2 * ks, bhi + 2 * ks, id_64, acc);
                    tc::mma_f16(d + BN, ahi + 2 * ks, blo + 2 * ks, id_64, acc);
                    if (GROUPED) tc::mma_f16(d, alo + 2 * ks, bhi + 2 * ks, id_64, 1u);
                }
            }
            tc::mma_commit(&r.empty[s]);
            if (NA != NB) tc::mma_commit(&r.aempty[a]);  // with NA == NB, empty[s] frees both
            if (sp == SPP - 1) tc::mma_commit(&r.accfull[buf]);
        }
    }
    return true;
}

template <int NA, int NB, bool GROUPED, bool SMALL, bool PRE>
__device__ __forceinline__ bool mma_loop_spp(int spp, int num_kb, uint64_t ahi0, uint64_t alo0, uint64_t b0,
                                             uint32_t tmem_base, const MmaRing &r) {
    if (spp == 4) return mma_loop<NA, NB, 4, GROUPED, SMALL, PRE>(num_kb, ahi0, alo0, b0, tmem_base, r);
    if (spp == 2) return mma_loop<NA, NB, 2, GROUPED, SMALL, PRE>(num_kb, ahi0, alo0, b0, tmem_base, r);
    return mma_loop<NA, NB, 1, GROUPED, SMALL, PRE>(num_kb, ahi0, alo0, b0, tmem_base, r);
}

// PRE: the weights were converted once for the call (pre_convert_grouped_kernel): the producer
// brings the A_hi / A_lo tiles by TMA with each stage and the converter warps only publish the
// rows' 2^-e -- for many token tiles, instead of converting every weight tile once per token tile.
template <int NA, int NB, bool LO, bool PRE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xhi,
                   const __grid_constant__ CUtensorMap tm_xlo, const __grid_constant__ CUtensorMap tm_ahi,
                   const __grid_constant__ CUtensorMap tm_alo, const TcParams p) {
    static_assert(!PRE || (LO && NA == NB), "pre-converted weights: group scales, one ring");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using L = Smem<NA, NB, LO>;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar);
    uint64_t *full = bars, *empty = bars + NB;            // TMA stages
    uint64_t *conv = bars + 2 * NB, *aempty = conv + NA;  // converted weight tiles
    uint64_t *accfull = aempty + NA, *accempty = accfull + 2, *drain = accempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::misc + 4);
    float *rowinv = reinterpret_cast<float *>(smem + L::rowinv);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM, m0 = blockIdx.y * BN;
    // this CTA's K range: K-blocks [kb0, kb0 + num_kb) (the whole of K without split-K)
    const int kb0 = blockIdx.z * p.kb_per_split;
    const int num_kb = min(p.K / BK - kb0, p.kb_per_split);
    // a tile with <= 64 tokens multiplies with N = 64: the rest of the token tile is TMA zero fill
    const bool small = p.M - m0 <= 64;
    const int raw_kb_bytes = p.qtype == kQInt8 ? 64 : 32;
    const uint32_t stage_tx = 2 * kBBytes + (PRE ? 2 * kABytes : (uint32_t)(BM * raw_kb_bytes));

    if (threadIdx.x == 0) {
        for (int s = 0; s < NB; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < NA; ++a) {
            tc::mbar_init(&conv[a], kNumConvWarps);
            tc::mbar_init(&aempty[a], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&accfull[b], 1);
            tc::mbar_init(&accempty[b], kNumEpiWarps);
        }
        tc::mbar_init(drain, 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        if (PRE) {
            tc::prefetch_tmap(&tm_ahi);
            tc::prefetch_tmap(&tm_alo);
        } else {
            tc::prefetch_tmap(&tm_w);
        }
        tc::prefetch_tmap(&tm_xhi);
        tc::prefetch_tmap(&tm_xlo);
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int issued = 0;
            for (int j = 0; j < num_kb; ++j) {
                const int s = j % NB, kb = kb0 + j;
                if (j >= NB &&
                    !tc::mbar_wait_bounded(&empty[s], ((j / NB) - 1) & 1, abort_flag, p.err, kErrProducer, kTimeoutNs))
                    break;
                tc::mbar_arrive_expect_tx(&full[s], stage_tx);
                uint8_t *b = smem + L::b + s * 2 * kBBytes;
                if (PRE) {
                    tc::tma_load_2d(smem + L::ahi + s * kABytes, &tm_ahi, kb * BK, n0, &full[s]);
                    tc::tma_load_2d(smem + L::alo + s * kABytes, &tm_alo, kb * BK, n0, &full[s]);
                } else {
                    tc::tma_load_2d(smem + L::r + s * kRBytes, &tm_w, kb * raw_kb_bytes, n0, &full[s]);
                }
                tc::tma_load_2d(b, &tm_xhi, kb * BK, m0, &full[s]);
                tc::tma_load_2d(b + kBBytes, &tm_xlo, kb * BK, m0, &full[s]);
                ++issued;
            }
            if (*abort_flag) {  // let the copies already issued land before the CTA exits
                volatile int no_abort = 0;
                for (int j = issued > NB ? issued - NB : 0; j < issued; ++j)
                    tc::mbar_wait_bounded(&full[j % NB], (j / NB) & 1, &no_abort, p.err, kErrDrain, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint64_t ahi0 = tc::desc_sw128(tc::smem_u32(smem + L::ahi));
            const uint64_t alo0 = tc::desc_sw128(tc::smem_u32(smem + L::alo));
            const uint64_t b0 = tc::desc_sw128(tc::smem_u32(smem + L::b));
            const MmaRing ring{full, conv, empty, aempty, accfull, accempty, abort_flag, p.err};
            const int spp = p.ksteps_per_period / (BK / 16);  // stages per fold period: 1, 2 or 4
            if (small) mma_loop_spp<NA, NB, LO, true, PRE>(spp, num_kb, ahi0, alo0, b0, tmem_base, ring);
            else mma_loop_spp<NA, NB, LO, false, PRE>(spp, num_kb, ahi0, alo0, b0, tmem_base, ring);
            // wait for every MMA this thread issued before TMEM can be released
            tc::mma_commit(drain);
            volatile int no_abort = 0;
            tc::mbar_wait_bounded(drain, 0, &no_abort, p.err, kErrDrain, kTimeoutNs);
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------------------ converters
        // Thread r owns weight row r of the tile.  Per-row scales: codes become exact fp16 integers
        // (A_hi).  Group scales: every code pair is multiplied by its group's scale times a per-row
        // power of two 2^e (max |q s| 2^e < 2^14, so hi and lo stay normal fp16) and split into
        // A_hi + A_lo; the epilogue multiplies by 2^-e.
        const int ct = threadIdx.x - kConvWarp0 * 32;
        const int r = ct % BM, half = ct / BM;  // row r, part `half` of the stage's K
        const int n = n0 + r;
        const bool nrow = n < p.N;
        if (PRE) {
            if (half == 0) rowinv[r] = nrow ? __ldg(p.rowinv + n) : 1.f;
            bar_arrive(kBarRowInv, kRowInvThreads);
        } else {
        const float *srow = p.scales + (size_t)(nrow ? n : 0) * p.groups_per_row;
        float se = 1.f;
        if (LO) {
            const int g0 = kb0 * BK / p.group_k, g1 = ((kb0 + num_kb) * BK + p.group_k - 1) / p.group_k;
            float smax = 0.f;
            if (nrow) {
                // all loads of a batch in flight before the first use: one memory latency per
                // 32 groups instead of one per few groups (this scan precedes the first stage)
                const float *sg = srow + g0;
                const int ng = g1 - g0;
                int g = 0;
                if ((reinterpret_cast<uintptr_t>(sg) & 15) == 0) {
                    const float4 *s4 = reinterpret_cast<const float4 *>(sg);
                    for (; g + 32 <= ng; g += 32) {
                        float4 v[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u) v[u] = __ldg(s4 + g / 4 + u);
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            smax = fmaxf(smax, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
                    }
                }
#pragma unroll 8
                for (; g < ng; ++g) smax = fmaxf(smax, fabsf(__ldg(sg + g)));
            }
            int e = 0;
            const float bound = (p.qtype == kQInt8 ? 127.f : 8.f) * smax;
            if (bound > 0.f && isfinite(bound)) {
                int ex;
                frexpf(bound, &ex);  // bound < 2^ex
                e = min(100, max(-100, 14 - ex));
            }
            se = ldexpf(1.0f, e);
            if (half == 0) rowinv[r] = ldexpf(1.0f, -e);
        }
        bar_arrive(kBarRowInv, kRowInvThreads);
        const int epc = p.qtype == kQInt8 ? 16 : 32;  // codes per 16-byte raw chunk
        constexpr int kChunks8 = 4 / kConvPerRow, kChunks4 = 2 / kConvPerRow;  // raw chunks per thread
        // scale x 2^e of this thread's raw chunks, read two stages ahead (the converters are the
        // slowest role for group scales: a memory round trip per stage would be exposed)
        // (a shift when the group size is a power of two: a division per chunk measured slower)
        const int gshift = (p.group_k & (p.group_k - 1)) == 0 ? __ffs(p.group_k) - 1 : -1;
        float sc_a[kChunks8] = {}, sc_b[kChunks8] = {};
        auto load_scales = [&](int kb, float (&dst)[kChunks8]) {
            if (!LO || !nrow || kb >= kb0 + num_kb) return;
            const int k0 = kb * BK + half * (BK / kConvPerRow);
#pragma unroll
            for (int cc = 0; cc < kChunks8; ++cc)
                if (cc * epc < BK / kConvPerRow) {
                    const int k = k0 + cc * epc;
                    dst[cc] = __ldg(srow + (gshift >= 0 ? k >> gshift : k / p.group_k)) * se;
                }
        };
        // Converts stage j with the scales sc; false when a wait gave up.
        auto convert = [&](int j, const float (&sc)[kChunks8]) -> bool {
            const int s = j % NB, a = j % NA;
            int ok = 1;
            if (lane == 0) {
                ok = tc::mbar_wait_bounded(&full[s], (j / NB) & 1, abort_flag, p.err, kErrConverter, kTimeoutNs);
                // the tile slot's previous stage must be multiplied out (implied by full[s] when NA == NB)
                if (ok && NA != NB && j >= NA)
                    ok = tc::mbar_wait_bounded(&aempty[a], ((j / NA) - 1) & 1, abort_flag, p.err, kErrConverter, kTimeoutNs);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) return false;
            const uint8_t *raw = smem + L::r + s * kRBytes;
            uint8_t *ahi = smem + L::ahi + a * kABytes;
            uint8_t *alo = smem + L::alo + a * kABytes;
            if (p.qtype == kQInt8) {
#pragma unroll
                for (int cc = 0; cc < kChunks8; ++cc) {  // 64-byte rows, 64-byte TMA swizzle
                    const int c = kChunks8 * half + cc;
                    const uint4 w = *reinterpret_cast<const uint4 *>(raw + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
                    if (!LO) {
                        uint32_t h[8];
                        i8x4_to_h(w.x, h[0], h[1]);
                        i8x4_to_h(w.y, h[2], h[3]);
                        i8x4_to_h(w.z, h[4], h[5]);
                        i8x4_to_h(w.w, h[6], h[7]);
                        *reinterpret_cast<uint4 *>(ahi + sw128_off(r, 2 * c)) = make_uint4(h[0], h[1], h[2], h[3]);
                        *reinterpret_cast<uint4 *>(ahi + sw128_off(r, 2 * c + 1)) = make_uint4(h[4], h[5], h[6], h[7]);
                    } else {
                        float2 f[8];  // the 16 codes as exact floats, natural order
                        i8x4_to_f32(w.x, f[0], f[1]);
                        i8x4_to_f32(w.y, f[2], f[3]);
                        i8x4_to_f32(w.z, f[4], f[5]);
                        i8x4_to_f32(w.w, f[6], f[7]);
                        uint32_t hi[8], lo[8];
                        const float2 s2 = f2(sc[cc], sc[cc]);
#pragma unroll
                        for (int i = 0; i < 8; ++i) split_pair(f[i], s2, hi[i], lo[i]);
                        *reinterpret_cast<uint4 *>(ahi + sw128_off(r, 2 * c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4 *>(ahi + sw128_off(r, 2 * c + 1)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                        *reinterpret_cast<uint4 *>(alo + sw128_off(r, 2 * c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        *reinterpret_cast<uint4 *>(alo + sw128_off(r, 2 * c + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                    }
                }
            } else {
#pragma unroll
                for (int cc = 0; cc < kChunks4; ++cc) {
                    const int c = kChunks4 * half + cc;  // 32-byte rows, 32-byte TMA swizzle
                    const uint4 w = *reinterpret_cast<const uint4 *>(raw + r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
                    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        if (!LO) {
                            uint32_t h[4];
                            u4x8_to_h(ws[jj], h);
                            *reinterpret_cast<uint4 *>(ahi + sw128_off(r, 4 * c + jj)) = make_uint4(h[0], h[1], h[2], h[3]);
                        } else {
                            float2 e[4];
                            u4x8_to_f32_pairs(ws[jj], e);
                            const float2 s2 = f2(sc[cc], sc[cc]);
                            uint32_t hi[4], lo[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) split_pair(e[i], s2, hi[i], lo[i]);
                            *reinterpret_cast<uint4 *>(ahi + sw128_off(r, 4 * c + jj)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                            *reinterpret_cast<uint4 *>(alo + sw128_off(r, 4 * c + jj)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        }
                    }
                }
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&conv[a]);
            return true;
        };
        // Unrolled by two with a scale buffer per parity: each buffer is read two stages after its
        // loads were issued and is never copied while they are in flight (a loop-carried rotation
        // of the buffers moved registers with pending loads and stalled every stage).
        load_scales(kb0, sc_a);
        load_scales(kb0 + 1, sc_b);
        for (int j = 0; j < num_kb; j += 2) {
            float sc[kChunks8];
#pragma unroll
            for (int cc = 0; cc < kChunks8; ++cc) sc[cc] = sc_a[cc];
            load_scales(kb0 + j + 2, sc_a);
            if (!convert(j, sc)) break;
            if (j + 1 >= num_kb) break;
#pragma unroll
            for (int cc = 0; cc < kChunks8; ++cc) sc[cc] = sc_b[cc];
            load_scales(kb0 + j + 3, sc_b);
            if (!convert(j + 1, sc)) break;
        }
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int h = (warp - kEpiWarp0) >> 2;  // column quarter: tokens m0 + 32 h ...
        const int rl = 32 * q + lane;
        const int n = n0 + rl;
        const bool row_ok = n < p.N;
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.f;
        const int num_periods = num_kb * BK / (16 * p.ksteps_per_period);
        bool ok = true;
        for (int pd = 0; pd < num_periods; ++pd) {
            const int b = pd & 1;
            int w_ok = 1;
            if (lane == 0) w_ok = tc::mbar_wait_bounded(&accfull[b], (pd >> 1) & 1, abort_flag, p.err, kErrEpilogue, kTimeoutNs);
            w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
            if (!w_ok) {
                ok = false;
                break;
            }
            tc::tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kAccCols + 32 * h);
#pragma unroll
            for (int part = 0; part < 2; ++part) {  // W x_hi, then W x_lo
                uint32_t v[32];
                tc::tmem_ld32_async(taddr + part * BN, v);
                tc::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] += __uint_as_float(v[j]);
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&accempty[b]);
        }
        bar_sync(kBarRowInv, kRowInvThreads);
        if (ok && row_ok) {
            const float sr = LO ? rowinv[rl] : __ldg(p.scales + n);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int m = m0 + 32 * h + j;
                if (m >= p.M) continue;
                const float y = acc[j] * sr * __ldg(p.xinv + m);
                if (p.part) p.part[((size_t)blockIdx.z * p.M + m) * p.N + n] = y;
                else p.Y[(size_t)m * p.ldy + n] = y;
            }
        }
    }

    __syncwarp();
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, kTmemCols);
    }
}

// The group-scaled weights as the GEMM's A operand, once per call (PRE): row n's codes times
// their group scales times 2^e_n, as fp16 hi + lo in the converters' element order (split_pair),
// and 2^-e_n beside them.  e_n keeps max |q s| 2^e_n below 2^14 over the whole row (the
// converters' choice over a K slice differs only by a power of two, which scales hi and lo
// exactly).  One warp per row; int4: a word of 8 codes per lane step, int8: 16 codes.
template <bool INT4>
__global__ void __launch_bounds__(256)
    pre_convert_grouped_kernel(const uint8_t *__restrict__ W, const float *__restrict__ S, int N, int K, int group_k,
                               __half *__restrict__ ahi, __half *__restrict__ alo, float *__restrict__ rowinv) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + warp;
    if (n >= N) return;
    const int gpr = K / group_k;
    const float *srow = S + (size_t)n * gpr;
    float smax = 0.f;
    for (int g = lane; g < gpr; g += 32) smax = fmaxf(smax, fabsf(__ldg(srow + g)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
    int e = 0;
    const float bound = (INT4 ? 8.f : 127.f) * smax;
    if (bound > 0.f && isfinite(bound)) {
        int ex;
        frexpf(bound, &ex);  // bound < 2^ex
        e = min(100, max(-100, 14 - ex));
    }
    const float se = ldexpf(1.0f, e);
    if (lane == 0) rowinv[n] = ldexpf(1.0f, -e);
    __half *hrow = ahi + (size_t)n * K, *lrow = alo + (size_t)n * K;
    if (INT4) {
        const uint32_t *wrow = reinterpret_cast<const uint32_t *>(W + (size_t)n * (K / 2));
        for (int i = lane; i < K / 8; i += 32) {  // word i: elements 8i .. 8i + 7
            float2 e4[4];
            u4x8_to_f32_pairs(__ldg(wrow + i), e4);
            const float sc = __ldg(srow + (8 * i) / group_k) * se;
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) split_pair(e4[j], f2(sc, sc), hi[j], lo[j]);
            *reinterpret_cast<uint4 *>(hrow + 8 * i) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4 *>(lrow + 8 * i) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    } else {
        const uint4 *wrow = reinterpret_cast<const uint4 *>(W + (size_t)n * K);
        for (int i = lane; i < K / 16; i += 32) {  // codes 16i .. 16i + 15 (one group)
            const uint4 w = __ldg(wrow + i);
            float2 f[8];
            i8x4_to_f32(w.x, f[0], f[1]);
            i8x4_to_f32(w.y, f[2], f[3]);
            i8x4_to_f32(w.z, f[4], f[5]);
            i8x4_to_f32(w.w, f[6], f[7]);
            const float sc = __ldg(srow + (16 * i) / group_k) * se;
            uint32_t hi[8], lo[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) split_pair(f[j], f2(sc, sc), hi[j], lo[j]);
            *reinterpret_cast<uint4 *>(hrow + 16 * i) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4 *>(hrow + 16 * i + 8) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
            *reinterpret_cast<uint4 *>(lrow + 16 * i) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<uint4 *>(lrow + 16 * i + 8) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
        }
    }
}

// Split-K: Y[m][n] = sum over the slices z, in order, of part[z][m][n].
__global__ void splitk_reduce_kernel(const float *__restrict__ part, int ks, int M, int N, float *__restrict__ Y,
                                     long long ldy) {
    const size_t MN = (size_t)M * N;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < MN; i += (size_t)gridDim.x * blockDim.x) {
        float y = part[i];
        for (int z = 1; z < ks; ++z) y += part[(size_t)z * MN + i];
        Y[(i / N) * ldy + i % N] = y;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tensor_map_encoder(); }

bool make_map_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

bool gemm_tc_supported(const QMatrix &w) {
    if (w.qtype != kQInt8 && w.qtype != kQInt4) return false;  // unquantized rows take the GEMV
    const size_t K = w.K, bs = w.block_size;
    if (K == 0 || K % BK != 0 || K > (1u << 20) || w.N > (size_t)INT32_MAX) return false;
    if ((reinterpret_cast<uintptr_t>(w.data) & 15) != 0) return false;
    if (bs == K) return true;
    return bs % 32 == 0 && K % bs == 0;
}

size_t gemm_tc_workspace_bytes(size_t M, size_t K) { return 2 * align256(M * K * 2) + align256(M * 4); }

namespace {
// Token rows from which group-scaled weights are converted once per call (more than two token
// tiles share every weight tile) instead of once per token tile.
constexpr size_t kPreMinM = 2 * BN + 1;
size_t pre_bytes(size_t N, size_t K) { return 2 * align256(N * K * 2) + align256(N * 4); }
}  // namespace

namespace {
// K-steps (16 of K each) accumulated in TMEM before the epilogue folds them into fp32 registers:
// the largest power of two <= 16 dividing K / 16, i.e. chains of at most 256 of K (16 or 32 MMA
// accumulations per column).  One accumulator over K = 2048 (256 accumulations) measured 1.9e-3 on
// the parity metric; group scales live in the A operand, so folds need not follow the groups.
int fold_steps(const QMatrix &w) {
    const int steps = (int)(w.K / 16);
    int kpp = 16;
    while (kpp > 1 && steps % kpp) kpp >>= 1;
    return kpp;
}

int gcd_int(int a, int b) {
    while (b) {
        const int t = a % b;
        a = b;
        b = t;
    }
    return a;
}

// Split-K slices when the output tiles do not fill the SMs: the split that minimises
// waves x (a CTA's fixed cost + its K-blocks), in K-block units -- a CTA's start (ring fill, scale
// scan) and epilogue tail cost about kFixedKb K-blocks, the fixed-order reduction of the partials
// about kReduceKb.  Slices are aligned to the fold periods and the scale groups, >= 4 K-blocks
// (256 of K).  Splitting until every SM has a CTA can double the waves (gate|up at 64 tokens:
// 96 tiles x 2 = 192 CTAs on 148 SMs), which this avoids.
void plan_splitk(const QMatrix &w, size_t M, int num_sms, int &ks, int &kb_per) {
    constexpr int kFixedKb = 10, kReduceKb = 5;
    const int kb_all = (int)(w.K / BK);
    const long long tiles = ((long long)w.N + BM - 1) / BM * (((long long)M + BN - 1) / BN);
    int unit = 16 * fold_steps(w);          // K of a fold period
    unit = unit / gcd_int(unit, BK) * BK;   // lcm with the K-block
    const int gran = unit / BK;
    ks = 1;
    kb_per = kb_all;
    if (tiles >= num_sms) return;
    const int max_split = kb_all / std::max(gran, 4);
    long long best = (long long)((tiles + num_sms - 1) / num_sms) * (kFixedKb + kb_all);
    for (int k = 2; k <= max_split; ++k) {
        int per = (kb_all + k - 1) / k;
        per = (per + gran - 1) / gran * gran;
        const int n = (kb_all + per - 1) / per;
        if (n < 2) continue;
        const long long waves = (tiles * n + num_sms - 1) / num_sms;
        const long long cost = waves * (kFixedKb + per) + kReduceKb;
        if (cost < best) {
            best = cost;
            ks = n;
            kb_per = per;
        }
    }
}
}  // namespace

size_t gemm_tc_workspace_bytes_splitk(size_t M, size_t N, size_t K, int block_size_is_k, size_t block_size,
                                      int num_sms) {
    QMatrix q{kQInt8, nullptr, nullptr, block_size_is_k ? K : block_size, N, K};
    int ks, kb;
    plan_splitk(q, M, num_sms, ks, kb);
    return gemm_tc_workspace_bytes(M, K) + (ks > 1 ? align256((size_t)ks * M * N * 4) : 0) +
           (!block_size_is_k && M >= kPreMinM ? pre_bytes(N, K) : 0);
}

cudaError_t launch_gemm_tc(const QMatrix &w, const float *X, size_t M, size_t ldx, float *Y, size_t ldy, void *ws,
                           size_t ws_bytes, int *err, int num_sms, cudaStream_t st) {
    const int K = (int)w.K, N = (int)w.N;
    uint8_t *wsb = reinterpret_cast<uint8_t *>(ws);
    __half *xhi = reinterpret_cast<__half *>(wsb);
    __half *xlo = reinterpret_cast<__half *>(wsb + align256(M * K * 2));
    float *xinv = reinterpret_cast<float *>(wsb + 2 * align256(M * K * 2));
    const unsigned threads = K >= 4096 ? 512 : 256;  // (X is 16-byte aligned, ldx % 4 == 0 on this path)
    if (w.qtype == kQInt4)
        split_x_rows_kernel<true><<<(unsigned)M, threads, 0, st>>>(X, (long long)ldx, K, xhi, xlo, xinv, 1);
    else
        split_x_rows_kernel<false><<<(unsigned)M, threads, 0, st>>>(X, (long long)ldx, K, xhi, xlo, xinv, 1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    CUtensorMap tw, th, tl;
    const uint32_t raw_box = w.qtype == kQInt8 ? 64 : 32;
    const uint64_t row_bytes = w.qtype == kQInt8 ? (uint64_t)K : (uint64_t)K / 2;
    const bool ok = make_map_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.data, row_bytes, (uint64_t)N, row_bytes,
                                raw_box, BM, w.qtype == kQInt8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B) &&
                    make_map_2d(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xhi, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2,
                                BK, BN, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map_2d(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xlo, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2,
                                BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!ok) return cudaErrorInvalidValue;

    TcParams p{};
    p.M = (int)M;
    p.N = N;
    p.K = K;
    p.qtype = w.qtype;
    p.grouped = w.block_size == w.K ? 0 : 1;
    // TMEM accumulation chains stay short (<= 256 along K); longer sums are folded in fp32
    // registers with round-to-nearest, so the drift of long tensor-core accumulations never builds.
    p.ksteps_per_period = fold_steps(w);
    p.group_k = p.grouped ? (int)w.block_size : K;
    p.groups_per_row = p.grouped ? (int)(w.K / w.block_size) : 1;
    p.scales = w.scales;
    p.xinv = xinv;
    p.Y = Y;
    p.ldy = (long long)ldy;
    p.err = err;
    int ks = 1, kb_per = K / BK;
    plan_splitk(w, M, num_sms, ks, kb_per);
    size_t base = gemm_tc_workspace_bytes(M, (size_t)K);
    if (ks > 1 && ws_bytes >= base + align256((size_t)ks * M * N * 4)) {
        p.part = reinterpret_cast<float *>(wsb + base);
        base += align256((size_t)ks * M * N * 4);
    } else {
        ks = 1;
        kb_per = K / BK;
        p.part = nullptr;
    }
    p.kb_per_split = kb_per;
    // group-scaled weights for many token tiles: converted once, then streamed by TMA
    const bool pre = p.grouped && M >= kPreMinM && ws_bytes >= base + pre_bytes((size_t)N, (size_t)K);
    CUtensorMap tah = tw, tal = tw;
    if (pre) {
        __half *ahi = reinterpret_cast<__half *>(wsb + base);
        __half *alo = reinterpret_cast<__half *>(wsb + base + align256((size_t)N * K * 2));
        float *rinv = reinterpret_cast<float *>(wsb + base + 2 * align256((size_t)N * K * 2));
        p.rowinv = rinv;
        if (!make_map_2d(&tah, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ahi, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, BK, BM,
                         CU_TENSOR_MAP_SWIZZLE_128B) ||
            !make_map_2d(&tal, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, alo, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, BK, BM,
                         CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        const unsigned cg = (unsigned)((N + 7) / 8);
        if (w.qtype == kQInt4)
            pre_convert_grouped_kernel<true><<<cg, 256, 0, st>>>(w.data, w.scales, N, K, p.group_k, ahi, alo, rinv);
        else
            pre_convert_grouped_kernel<false><<<cg, 256, 0, st>>>(w.data, w.scales, N, K, p.group_k, ahi, alo, rinv);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    using LG = Smem<kTilesGrouped, kStagesGrouped, true>;
    using LR = Smem<kStagesRow, kStagesRow, false>;
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t attr = once_per_device(attr_done, [] {
        cudaError_t a = cudaFuncSetAttribute(gemm_tc_kernel<kTilesGrouped, kStagesGrouped, true, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, LG::bytes);
        if (a == cudaSuccess)
            a = cudaFuncSetAttribute(gemm_tc_kernel<kStagesGrouped, kStagesGrouped, true, true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, LG::bytes);
        if (a == cudaSuccess)
            a = cudaFuncSetAttribute(gemm_tc_kernel<kStagesRow, kStagesRow, false, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, LR::bytes);
        return a;
    });
    if (attr != cudaSuccess) return attr;
    dim3 grid((unsigned)((N + BM - 1) / BM), (unsigned)((M + BN - 1) / BN), (unsigned)ks);
    if (pre)
        gemm_tc_kernel<kStagesGrouped, kStagesGrouped, true, true><<<grid, kThreads, LG::bytes, st>>>(tw, th, tl, tah,
                                                                                                     tal, p);
    else if (p.grouped)
        gemm_tc_kernel<kTilesGrouped, kStagesGrouped, true, false><<<grid, kThreads, LG::bytes, st>>>(tw, th, tl, tah,
                                                                                                      tal, p);
    else
        gemm_tc_kernel<kStagesRow, kStagesRow, false, false><<<grid, kThreads, LR::bytes, st>>>(tw, th, tl, tah, tal, p);
    e = cudaGetLastError();
    if (e != cudaSuccess || ks == 1) return e;
    const size_t MN = M * (size_t)N;
    const unsigned rgrid = (unsigned)std::min<size_t>((MN + 255) / 256, (size_t)num_sms * 8);
    splitk_reduce_kernel<<<rgrid, 256, 0, st>>>(p.part, ks, (int)M, N, Y, (long long)ldy);
    return cudaGetLastError();
}

}  // namespace pyxis
