// gemm_ws.cu -- weight-streaming matmul for a few tokens (M = 1..64) on the tcgen05 tensor cores:
// the decode-shaped products of src/matmul.rs:21-97 (the batched decode step's projections and
// lm_head, src/attention.rs:77-79,136, src/ffn.rs:36-48, src/output_head.rs:22, with several
// sequences' rows at once) for weights with a scale per group of 32 (int4 q + 8 nibbles, or int8
// codes) or one scale per row (int8).
//
//   y[t, n] = sum_g s[n, g] * sum_{k in g} q[n, k] x[t, k]            (group scales)
//   y[t, n] = s[n] * sum_k q[n, k] x[t, k]                           (row scales)
//
// With few tokens the weights' bytes set the time, so the kernel is built around streaming them
// once with every SM busy:
//   - x is split once per launch (split_x_rows_kernel) into fp16 hi + lo (x 2^e = hi + lo to 22
//     bits, one power of two 2^e per token) and stacked along K: each MMA K-step multiplies the
//     codes with x_hi and then, into the same accumulator, with x_lo, so one fp32 accumulator per
//     (row, token) carries the 22-bit x.
//   - the codes become exact fp16 integers on the CUDA cores (a mask and a paired subtraction per
//     two codes) and go to the tensor core as operand A; no scale is folded into them.
//   - each group of 32 has its own TMEM accumulator (128 rows x the token columns, fp32); the
//     epilogue warps read it back and add s[n, g] * D into fp32 registers, in group order.  With
//     row scales a stage's 128 of K share one accumulator and the scale is applied at the end.
//   - persistent CTAs, one per SM.  Work unit = (128-row tile, K part); the number of K parts per
//     tile is chosen so that the SMs get equal numbers of stages.  A tile split into several parts
//     is finished by the CTA that completes its last part: it adds the parts' partial sums in part
//     order (reruns are bit-identical) and writes y.
//
// Warp roles: 0 TMA producer of the codes (a deep ring of their own, refilled as soon as the
// converters have read a stage), 1 TMA producer of the x_hi / x_lo tiles (a shorter ring, freed by
// the MMAs), 2-3 TMEM owner and MMA issuers, 4-7 converters (one weight row per thread), then the
// epilogue warps (one row per thread, the warp's TMEM lane quarter).  Every mbarrier wait is
// bounded; a wait that runs out records a code in the context's device flag and the CTA winds down
// (drains its copies and MMAs, frees TMEM).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>

#include "kernels.h"
#include "split_x.cuh"
#include "fp16_codes.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace pyxis {
namespace {

constexpr int WM = 128;       // weight rows per tile: MMA M, TMEM lanes
constexpr int WSK = 128;      // K per stage
constexpr int WG = 32;        // K per scale group (group-scale mode)
constexpr int kGroupsPerStage = WSK / WG;
// Warp roles: 0 TMA producer of the codes; 1 TMA producer of x; 2 and 3 MMA issuers (even and
// odd stages: a tcgen05.mma costs its issuing thread about 70 cycles at any N <= 128, and two
// issuers overlap that, measured 39-48 cycles per MMA); 4-7 converters; then the epilogue warps.
// Warp 2 also owns TMEM.
constexpr int kProdWarp = 0, kXWarp = 1, kMmaWarp = 2, kNumIssuers = 2, kConvWarp0 = 4, kNumConv = 4,
              kEpiWarp0 = 8;
constexpr int kMaxTokens = 64;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr uint32_t kABlock = WM * 128;      // one column block (64 of K) of the fp16 weight tile
constexpr uint32_t kABytes = 2 * kABlock;   // one fp16 weight stage
enum { kErrProd = 0x501, kErrConv = 0x502, kErrMma = 0x503, kErrEpi = 0x504, kErrDrain = 0x505 };

struct WsParams {
    int M, N, K;
    int tiles, parts;    // tiles of 128 rows, K parts per tile
    int stages_k;        // stages per row (K / 128)
    int units;           // tiles * parts
    const float *scales;
    const float *xinv;   // [M] 2^-e per token
    float *Y;
    long long ldy;
    float *partial;      // [units][NBT][128] partial sums of split tiles (parts > 1)
    unsigned *tickets;   // [tiles], zero between launches
    int *err;
};




// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled K-major block (8-row 1024 B atoms).
PYXIS_DEVINL uint32_t sw128_off(int r, int c) { return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4); }

PYXIS_DEVINL void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Unit u = (tile u / parts, part u % parts); part p covers stages [p S / parts, (p + 1) S / parts)
// of the row (S = stages_k).  A CTA takes units blockIdx.x, blockIdx.x + gridDim.x, ...
PYXIS_DEVINL void unit_range(const WsParams &p, int u, int &tile, int &part, int &s0, int &s1) {
    tile = u / p.parts;
    part = u - tile * p.parts;
    s0 = part * p.stages_k / p.parts;
    s1 = (part + 1) * p.stages_k / p.parts;
}

// Epilogue warps: 4 lane quarters x EW column slices of CW = 16 token columns (a warp's
// accumulators and two readback buffers stay within the register budget of up to 704 threads).
template <int NBT>
struct WsRoles {
    static constexpr int CW = 16;
    static constexpr int EW = NBT / CW;
    static constexpr int kEpiWarps = 4 * EW;
    static constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;  // 384, 512 or 768
    // A tcgen05.mma costs about the same at any N up to 256, so the MMA count per stage sets the
    // pace.  Up to 32 token columns x_hi and x_lo sit side by side in N (NSTACK): one N = 2 NBT MMA
    // per K-step of 16 multiplies the codes with both, into columns [0, NBT) and [NBT, 2 NBT) of the
    // group's accumulator -- 8 MMAs per stage, 4 independent chains of 2.  With 64 token columns
    // (N would exceed the TMEM budget) x_lo is stacked along K instead: 16 MMAs per stage.  KS = the
    // NBT-column parts a group's readback adds (hi and lo, or one).  Two stages' accumulators (sets)
    // are in flight: the MMAs of one while the epilogue reads the other.
    static constexpr bool NSTACK = NBT <= 32;
    static constexpr int KS = NSTACK ? 2 : 1;
    static constexpr int kAccPerStage = kGroupsPerStage * KS;
    static constexpr int kSetCols = kAccPerStage * NBT;
    // TA: the converted weight tiles live in TMEM (one lane per weight row, 64 columns of fp16
    // pairs per 128 of K) and the MMAs read operand A from there, when the accumulators leave room:
    // shared memory then carries only the codes and the x tiles (the fp16 tile in shared memory
    // cost 32 KB of stores and 32 KB of tensor-core reads per stage), and a converter thread
    // writes its row with two tcgen05.st instead of sixteen 16-byte stores.
    static constexpr bool TA = 2 * kSetCols + 3 * 64 <= 512;
    static constexpr int kNAT = TA ? 3 : 0;  // converted tiles in TMEM
    static constexpr int kSets = 2;
    static constexpr uint32_t kACol0 = kSets * kSetCols;  // first A column
    static constexpr uint32_t kTmemNeed = kSets * kSetCols + kNAT * 64;
    static constexpr uint32_t kTmemCols = kTmemNeed <= 128 ? 128 : (kTmemNeed <= 256 ? 256 : 512);
    static_assert(kTmemNeed <= 512 && kSets >= 2, "two sets of accumulators fit in TMEM");
};

// Shared memory: NA converted fp16 weight tiles, NX x tiles, and as many stages of codes as fit
// (the weight stream is what sets the time: with HBM latency of a few microseconds under load an
// SM needs tens of KB of codes in flight to draw its share of the bandwidth).
template <int NBT, bool INT4>
struct WsSmem {
    static constexpr bool TA = WsRoles<NBT>::TA;
    static constexpr int NA = TA ? WsRoles<NBT>::kNAT : (NBT <= 32 ? 3 : 2);  // converted weight tiles
    static constexpr uint32_t kASlot = TA ? 0 : kABytes;       // (in TMEM with TA)
    static constexpr int NX = TA ? 8 : (NBT == 16 ? 4 : (NBT == 32 ? 3 : 2));  // x tiles
    static constexpr uint32_t kBBlock = NBT * 128;             // one column block of an x tile
    // per 64-K column block c: x_hi rows, x_lo rows (one 2 NBT-row operand for NSTACK)
    static constexpr uint32_t kXStage = 4 * kBBlock;
    static constexpr uint32_t kRaw = INT4 ? WM * 64 : WM * 128;  // codes of a stage
    static constexpr uint32_t kBudget = 232448 - 1024 - 1024;     // alignment slack, barriers
    static constexpr int NRAW_FIT = (int)((kBudget - NA * kASlot - NX * kXStage) / kRaw);
    static constexpr int NRAW = NRAW_FIT > 16 ? 16 : NRAW_FIT;
    static constexpr uint32_t a = 0;
    static constexpr uint32_t x = a + NA * kASlot;
    static constexpr uint32_t r = x + NX * kXStage;
    static constexpr uint32_t bar = r + NRAW * kRaw;
    static constexpr uint32_t num_bars = 2 * NRAW + 2 * NX + 2 * NA + 2 * WsRoles<NBT>::kSets + 2;
    static constexpr uint32_t misc = bar + num_bars * 8;
    static constexpr uint32_t bytes = misc + 64 + 1024;  // + alignment slack
    static_assert(NRAW >= 4, "a few stages of codes in flight");
    static_assert(num_bars * 8 + 64 <= 1024, "barriers fit their reserve");
};
static_assert(WsSmem<16, true>::bytes <= 232448 && WsSmem<32, true>::bytes <= 232448 &&
                  WsSmem<64, true>::bytes <= 232448 && WsSmem<16, false>::bytes <= 232448 &&
                  WsSmem<32, false>::bytes <= 232448 && WsSmem<64, false>::bytes <= 232448,
              "227 KB of shared memory per CTA");

// CW token columns of this warp's 32 TMEM lanes, without waiting (valid after tmem_wait_regs).
template <int CW>
PYXIS_DEVINL void tmem_ld_cols(uint32_t taddr, float (&v)[CW]) {
    uint32_t *r = reinterpret_cast<uint32_t *>(v);
    if constexpr (CW == 16) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr));
    } else {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
              "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
              "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
              "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
    }
}

// tcgen05.wait::ld, then the registers of v are passed through empty asm statements so that no
// use of them is scheduled before the wait.
template <int CW>
PYXIS_DEVINL void tmem_wait_regs(float (&v)[CW]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < CW; i += 8)
        asm volatile("" : "+f"(v[i]), "+f"(v[i + 1]), "+f"(v[i + 2]), "+f"(v[i + 3]), "+f"(v[i + 4]), "+f"(v[i + 5]),
                     "+f"(v[i + 6]), "+f"(v[i + 7]));
}

template <int NBT, bool INT4, bool GROUPED>
__global__ void __launch_bounds__(WsRoles<NBT>::kThreads, 1)
    gemm_ws_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xhi,
                   const __grid_constant__ CUtensorMap tm_xlo, const WsParams p) {
    using L = WsSmem<NBT, INT4>;
    using R = WsRoles<NBT>;
    constexpr int NRAW = L::NRAW, NX = L::NX, NA = L::NA;
    constexpr uint32_t kRaw = L::kRaw;
    constexpr uint32_t kXTx = L::kXStage;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar);
    // codes: rfull (landed) / rempty (read by the converters); x tiles: xfull / xempty (read by the
    // MMAs); converted weight tiles: conv / aempty; accumulator sets: accfull / accempty
    uint64_t *rfull = bars, *rempty = bars + NRAW, *xfull = bars + 2 * NRAW, *xempty = xfull + NX;
    uint64_t *conv = xempty + NX, *aempty = conv + NA;
    uint64_t *accfull = aempty + NA, *accempty = accfull + R::kSets, *drain = accempty + R::kSets;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::misc + 4);
    volatile int *last_flag = reinterpret_cast<volatile int *>(smem + L::misc + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NRAW; ++s) {
            tc::mbar_init(&rfull[s], 1);
            tc::mbar_init(&rempty[s], kNumConv);
        }
        for (int x = 0; x < NX; ++x) {
            tc::mbar_init(&xfull[x], 1);
            tc::mbar_init(&xempty[x], 1);
        }
        for (int a = 0; a < NA; ++a) {
            tc::mbar_init(&conv[a], kNumConv);
            tc::mbar_init(&aempty[a], 1);
        }
        for (int k = 0; k < R::kSets; ++k) {
            tc::mbar_init(&accfull[k], 1);
            tc::mbar_init(&accempty[k], R::kEpiWarps);
        }
        tc::mbar_init(&drain[0], 1);
        tc::mbar_init(&drain[1], 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
    }
    constexpr uint32_t kTmemCols = R::kTmemCols;
    if (warp == kMmaWarp) tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kProdWarp) {
        // ------------------------------------------------------------------ codes producer
        // The codes do not depend on the previous kernel: they stream from the start, as far
        // ahead as the ring allows, while the previous kernel may still be finishing.
        if (lane == 0) {
            tc::prefetch_tmap(&tm_w);
            int g = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                int tile, part, s0, s1;
                unit_range(p, u, tile, part, s0, s1);
                for (int sk = s0; sk < s1; ++sk, ++g) {
                    const int s = g % NRAW;
                    if (g >= NRAW && !tc::mbar_wait_bounded(&rempty[s], (uint32_t)((g / NRAW - 1) & 1), abort_flag,
                                                            p.err, kErrProd, kTimeoutNs)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&rfull[s], kRaw);
                    tc::tma_load_2d(smem + L::r + s * kRaw, &tm_w, sk * (INT4 ? 64 : 128), tile * WM, &rfull[s]);
                }
            }
            if (*abort_flag) {  // let the copies already issued land before the CTA exits
                volatile int no_abort = 0;
                for (int j = g > NRAW ? g - NRAW : 0; j < g; ++j)
                    tc::mbar_wait_bounded(&rfull[j % NRAW], (j / NRAW) & 1, &no_abort, p.err, kErrDrain, 100000000ull);
            }
        }
    } else if (warp == kXWarp) {
        // ------------------------------------------------------------------ x producer
        if (lane == 0) {
            tc::prefetch_tmap(&tm_xhi);
            tc::prefetch_tmap(&tm_xlo);
            pdl_wait();  // x_hi / x_lo are written by the split kernel just before this one
            pdl_trigger();
            int g = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                int tile, part, s0, s1;
                unit_range(p, u, tile, part, s0, s1);
                for (int sk = s0; sk < s1; ++sk, ++g) {
                    const int x = g % NX;
                    if (g >= NX && !tc::mbar_wait_bounded(&xempty[x], (uint32_t)((g / NX - 1) & 1), abort_flag, p.err,
                                                          kErrProd, kTimeoutNs)) {
                        ok = false;
                        break;
                    }
                    uint8_t *b0 = smem + L::x + x * L::kXStage;  // [hi 0 | lo 0 | hi 1 | lo 1]
                    const int k = sk * WSK;
                    tc::mbar_arrive_expect_tx(&xfull[x], kXTx);
                    tc::tma_load_2d(b0, &tm_xhi, k, 0, &xfull[x]);
                    tc::tma_load_2d(b0 + L::kBBlock, &tm_xlo, k, 0, &xfull[x]);
                    tc::tma_load_2d(b0 + 2 * L::kBBlock, &tm_xhi, k + 64, 0, &xfull[x]);
                    tc::tma_load_2d(b0 + 3 * L::kBBlock, &tm_xlo, k + 64, 0, &xfull[x]);
                }
            }
            if (*abort_flag) {
                volatile int no_abort = 0;
                for (int j = g > NX ? g - NX : 0; j < g; ++j)
                    tc::mbar_wait_bounded(&xfull[j % NX], (j / NX) & 1, &no_abort, p.err, kErrDrain, 100000000ull);
            }
        }
    } else if (warp < kMmaWarp + kNumIssuers) {
        // ------------------------------------------------------------------ MMA issuers
        // Issuer i takes the stages st with st % 2 == i, into accumulator set st % kSets; a set (and a
        // ring slot) is reused only after the stage that last held it has been released.
        const int issuer = warp - kMmaWarp;
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16_f32(WM, R::NSTACK ? 2 * NBT : NBT);
            const uint64_t a_d = tc::desc_sw128(tc::smem_u32(smem + L::a));
            const uint64_t b_d = tc::desc_sw128(tc::smem_u32(smem + L::x));
            int st = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                int tile, part, s0, s1;
                unit_range(p, u, tile, part, s0, s1);
                for (int sk = s0; sk < s1; ++sk, ++st) {
                    if ((st & 1) != issuer) continue;
                    const int set = st % R::kSets, use = st / R::kSets;
                    const int x = st % NX, xph = st / NX, a = st % NA, aph = st / NA;
                    ok = tc::mbar_wait_bounded(&conv[a], (uint32_t)(aph & 1), abort_flag, p.err, kErrMma, kTimeoutNs) &&
                         tc::mbar_wait_bounded(&xfull[x], (uint32_t)(xph & 1), abort_flag, p.err, kErrMma, kTimeoutNs) &&
                         (use == 0 || tc::mbar_wait_bounded(&accempty[set], (uint32_t)((use - 1) & 1), abort_flag,
                                                            p.err, kErrMma, kTimeoutNs));
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint64_t abase = a_d + (uint64_t)(a * (kABytes >> 4));
                    const uint32_t at = tmem_base + R::kACol0 + (uint32_t)(a * 64);
                    const uint64_t bbase = b_d + (uint64_t)(x * (L::kXStage >> 4));
                    const uint32_t dset = tmem_base + (uint32_t)(set * R::kSetCols);
                    // K-step ks of group gi covers K [32 gi + 16 ks, +16) of the stage; the issue order
                    // runs over the groups innermost, so consecutive MMAs use different accumulators
#pragma unroll
                    for (int ks = 0; ks < 2; ++ks)
#pragma unroll
                        for (int hl = 0; hl < (R::NSTACK ? 1 : 2); ++hl)
#pragma unroll
                            for (int gi = 0; gi < kGroupsPerStage; ++gi) {
                                const int k = gi * 32 + ks * 16;
                                const uint64_t koff = (uint64_t)((k & 63) >> 3);  // 16-byte units in the row
                                const uint64_t ad = abase + (uint64_t)((k >> 6) * (kABlock >> 4)) + koff;
                                // block c = k / 64 of x: hi rows at 2c blocks, lo rows right after them
                                const uint64_t bd = bbase + (uint64_t)((2 * (k >> 6) + hl) * (L::kBBlock >> 4)) + koff;
                                const uint32_t d = dset + (uint32_t)(gi * R::KS * NBT);
                                // a group's first K-step (x_hi) starts its accumulator
                                if constexpr (R::TA)
                                    tc::mma_f16_ts(d, at + (uint32_t)(k >> 1), bd, idesc, (uint32_t)(ks | hl));
                                else
                                    tc::mma_f16(d, ad, bd, idesc, (uint32_t)(ks | hl));
                            }
                    tc::mma_commit(&accfull[set]);
                    tc::mma_commit(&xempty[x]);
                    tc::mma_commit(&aempty[a]);
                }
            }
            // every MMA this thread issued must complete before TMEM is released
            tc::mma_commit(&drain[issuer]);
            volatile int no_abort = 0;
            tc::mbar_wait_bounded(&drain[issuer], 0, &no_abort, p.err, kErrDrain, kTimeoutNs);
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------------------ converters
        const int r = threadIdx.x - kConvWarp0 * 32;  // weight row of the tile
        int g = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
            int tile, part, s0, s1;
            unit_range(p, u, tile, part, s0, s1);
            for (int sk = s0; sk < s1; ++sk, ++g) {
                const int s = g % NRAW, sph = g / NRAW, a = g % NA, aph = g / NA;
                int w_ok = 1;
                if (lane == 0) {
                    w_ok = tc::mbar_wait_bounded(&rfull[s], (uint32_t)(sph & 1), abort_flag, p.err, kErrConv, kTimeoutNs);
                    if (w_ok && g >= NA)
                        w_ok = tc::mbar_wait_bounded(&aempty[a], (uint32_t)((aph - 1) & 1), abort_flag, p.err, kErrConv,
                                                     kTimeoutNs);
                }
                w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
                if (!w_ok) {
                    ok = false;
                    break;
                }
                const uint8_t *raw = smem + L::r + s * kRaw;
                // the fp16 row as 64 columns of pairs, in two halves of 32 (K order of the converter:
                // the int4 pairs are (e_i, e_i+4) of each 8-element group, x is split in the same order)
                auto convert_half = [&](int hf, uint32_t (&hw)[32]) {
                    if constexpr (INT4) {
                        // 64-byte rows, 64-byte TMA swizzle: chunk c at ((c ^ ((r >> 1) & 3)) << 4); chunk
                        // c holds K [32c, 32c + 32): one scale group -> columns 16c .. 16c + 15
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            const int c = 2 * hf + cc;
                            const uint4 w = *reinterpret_cast<const uint4 *>(raw + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
                            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                            for (int i = 0; i < 4; ++i) {  // word i: K [32c + 8i, +8) -> columns 16c + 4i ..
                                uint32_t h[4];
                                u4x8_to_h(ws[i], h);
#pragma unroll
                                for (int j = 0; j < 4; ++j) hw[cc * 16 + 4 * i + j] = h[j];
                            }
                        }
                    } else {
                        // 128-byte rows, 128-byte TMA swizzle: chunk c (16 of K) at ((c ^ (r & 7)) << 4)
                        // -> columns 8c .. 8c + 7
#pragma unroll
                        for (int cc = 0; cc < 4; ++cc) {
                            const int c = 4 * hf + cc;
                            const uint4 w = *reinterpret_cast<const uint4 *>(raw + r * 128 + ((c ^ (r & 7)) << 4));
                            uint32_t *h = &hw[cc * 8];
                            i8x4_to_h(w.x, h[0], h[1]);
                            i8x4_to_h(w.y, h[2], h[3]);
                            i8x4_to_h(w.z, h[4], h[5]);
                            i8x4_to_h(w.w, h[6], h[7]);
                        }
                    }
                };
                if constexpr (R::TA) {
                    uint32_t h0[32], h1[32];
                    convert_half(0, h0);
                    convert_half(1, h1);
                    const uint32_t ta = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + R::kACol0 + (uint32_t)(a * 64);
                    tc::tmem_st32(ta, h0);
                    tc::tmem_st32(ta + 32, h1);
                    tc::tmem_wait_st();
                    tc::tc_fence_before();  // the tile -> the MMAs that read it after the barrier
                } else {
                    // the canonical K-major 128-byte-swizzled tile: columns 8j .. 8j + 7 (K 16j .. 16j + 15)
                    // are 16-byte chunks 2 (j % 4) and 2 (j % 4) + 1 of 64-K block j / 4
                    uint8_t *ab = smem + L::a + a * kABytes;
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        uint32_t hw[32];
                        convert_half(hf, hw);
                        uint8_t *blk = ab + hf * kABlock;
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            const uint32_t *h = &hw[jj * 8];
                            *reinterpret_cast<uint4 *>(blk + sw128_off(r, 2 * jj)) = make_uint4(h[0], h[1], h[2], h[3]);
                            *reinterpret_cast<uint4 *>(blk + sw128_off(r, 2 * jj + 1)) = make_uint4(h[4], h[5], h[6], h[7]);
                        }
                    }
                    tc::fence_proxy_async_smem();  // the fp16 tile -> the tensor core's reads
                }
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(&conv[a]);
                    tc::mbar_arrive(&rempty[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        // Warp (q, h): TMEM lane quarter q = warp % 4 (rows 32q..32q+31 of the tile, one per
        // lane), token columns [h CW, h CW + CW).  Every group's readback is one tcgen05.ld issued
        // before the previous group's FMAs, so the TMEM latency overlaps them.  All epilogue warps
        // run the same unit / stage sequence and named barriers; a warp whose wait ran out skips
        // the work but keeps the barrier sequence.
        constexpr int CW = R::CW;
        constexpr int kEpiThreads = R::kEpiWarps * 32;
        const int q = warp & 3, h = (warp - kEpiWarp0) >> 2;
        const int rl = 32 * q + lane, c0 = h * CW;
        const int gpr = p.K / WG;  // scale groups per row
        pdl_wait();                // y and the partial sums are written after the previous kernel
        int st = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.units; u += gridDim.x) {
            int tile, part, s0, s1;
            unit_range(p, u, tile, part, s0, s1);
            const int row = tile * WM + rl;
            const bool rowok = row < p.N;
            float acc[CW];
#pragma unroll
            for (int c = 0; c < CW; ++c) acc[c] = 0.f;
            // A stage's 4 groups are read back in turn into two alternating buffers (4 is even, so
            // group gi of every stage uses buffer gi % 2): the readback of group gi is issued before
            // the FMAs of group gi - 1, so the TMEM latency overlaps them.  With row scales the 4
            // groups' sums are added with scale 1 (exact).
            float DA[R::KS * CW], DB[R::KS * CW];
            float s_pend = 0.f;
            bool pend = false;
            auto fma_group = [&](float sg, const float (&D)[R::KS * CW]) {
#pragma unroll
                for (int c = 0; c < CW; ++c) {
                    const float d = R::KS == 2 ? __fadd_rn(D[c], D[CW + c]) : D[c];
                    acc[c] = fmaf(sg, d, acc[c]);
                }
            };
            for (int sk = s0; sk < s1; ++sk, ++st) {
                const int set = st % R::kSets, use = st / R::kSets;
                float4 sc4 = make_float4(1.f, 1.f, 1.f, 1.f);
                if (GROUPED && rowok) sc4 = __ldg(reinterpret_cast<const float4 *>(p.scales + (size_t)row * gpr + sk * 4));
                const float scs[4] = {sc4.x, sc4.y, sc4.z, sc4.w};
                if (ok) ok = tc::mbar_wait_bounded(&accfull[set], (uint32_t)(use & 1), abort_flag, p.err, kErrEpi,
                                                   kTimeoutNs);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) continue;
                tc::tc_fence_after();
                const uint32_t tset = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(set * R::kSetCols + c0);
#pragma unroll
                for (int gi = 0; gi < kGroupsPerStage; ++gi) {
                    float(&Dn)[R::KS * CW] = (gi & 1) ? DB : DA;
                    float(&Dp)[R::KS * CW] = (gi & 1) ? DA : DB;
#pragma unroll
                    for (int j = 0; j < R::KS; ++j)
                        tmem_ld_cols<CW>(tset + (uint32_t)((gi * R::KS + j) * NBT),
                                         *reinterpret_cast<float(*)[CW]>(Dn + j * CW));
                    if (pend) fma_group(s_pend, Dp);
                    tmem_wait_regs<R::KS * CW>(Dn);
                    s_pend = scs[gi];
                    pend = true;
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&accempty[set]);
            }
            if (pend) fma_group(s_pend, DB);
            const float rs = (!GROUPED && rowok) ? __ldg(p.scales + row) : 1.f;
            float *__restrict__ Y = p.Y;
            if (p.parts == 1) {
                if (ok && rowok) {
#pragma unroll
                    for (int c = 0; c < CW; ++c)
                        if (c0 + c < p.M) Y[(size_t)(c0 + c) * p.ldy + row] = (acc[c] * rs) * __ldg(p.xinv + c0 + c);
                }
            } else {
                float *__restrict__ mine = p.partial + ((size_t)u * NBT + c0) * WM + rl;
#pragma unroll
                for (int c = 0; c < CW; ++c) mine[(size_t)c * WM] = acc[c];
                __threadfence();
                named_bar(1, kEpiThreads);
                if (threadIdx.x == kEpiWarp0 * 32) {
                    const unsigned old = atomicAdd(&p.tickets[tile], 1u);
                    *last_flag = old == (unsigned)(p.parts - 1);
                }
                named_bar(1, kEpiThreads);
                if (*last_flag) {
                    __threadfence();
                    if (ok && rowok) {
                        // the parts' partial sums in part order; two parts' loads in flight at a time
                        const float *__restrict__ base = p.partial + ((size_t)tile * p.parts * NBT + c0) * WM + rl;
                        float y[CW];
#pragma unroll
                        for (int c = 0; c < CW; ++c) y[c] = __ldcg(base + (size_t)c * WM);
                        int pp = 1;
                        for (; pp + 1 < p.parts; pp += 2) {
                            float a[CW], b[CW];
#pragma unroll
                            for (int c = 0; c < CW; ++c) {
                                a[c] = __ldcg(base + ((size_t)pp * NBT + c) * WM);
                                b[c] = __ldcg(base + ((size_t)(pp + 1) * NBT + c) * WM);
                            }
#pragma unroll
                            for (int c = 0; c < CW; ++c) y[c] = (y[c] + a[c]) + b[c];
                        }
                        if (pp < p.parts) {
#pragma unroll
                            for (int c = 0; c < CW; ++c) y[c] += __ldcg(base + ((size_t)pp * NBT + c) * WM);
                        }
#pragma unroll
                        for (int c = 0; c < CW; ++c)
                            if (c0 + c < p.M) Y[(size_t)(c0 + c) * p.ldy + row] = (y[c] * rs) * __ldg(p.xinv + c0 + c);
                    }
                    if (threadIdx.x == kEpiWarp0 * 32) p.tickets[tile] = 0;  // re-armed for the next launch
                }
                named_bar(1, kEpiThreads);  // last_flag is reused by the next unit
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------------------------------------ host side --
int nbt_for(size_t M) { return M <= 16 ? 16 : M <= 32 ? 32 : 64; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// K parts per tile: minimises the busiest CTA's stages, ceil(units / grid) * ceil(S / parts), plus,
// for split tiles, the finishing CTA's reduce (its partial-sum reads: about 2 stages' time per
// pair of parts, more with more token columns), with partial sums no larger than `partial_cap`
// bytes.
int choose_parts(size_t N, size_t K, int nbt, int num_sms, size_t partial_cap) {
    const long T = (long)((N + WM - 1) / WM), S = (long)(K / WSK);
    long best_cost = -1;
    int best = 1;
    for (long P = 1; P <= S && P <= 64; ++P) {
        const long units = T * P;
        if (P > 1 && (size_t)units * nbt * WM * 4 > partial_cap) break;
        const long grid = std::min<long>(num_sms, units);
        const long reduce = P > 1 ? 2 + (2 + nbt / 32) * ((P + 1) / 2) : 0;
        const long cost = (units + grid - 1) / grid * ((S + P - 1) / P) + reduce;
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = (int)P;
        }
    }
    return best;
}

struct WsLayout {
    size_t xhi, xlo, xinv, partial, total;
};
WsLayout ws_layout(size_t M, size_t K, size_t partial_bytes) {
    WsLayout l;
    const size_t xb = align_up(M * K * 2, 1024);
    l.xhi = 0;
    l.xlo = xb;
    l.xinv = 2 * xb;
    l.partial = align_up(l.xinv + M * 4, 1024);
    l.total = l.partial + partial_bytes;
    return l;
}

bool make_map(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NBT, bool INT4, bool GROUPED>
cudaError_t run_ws(const CUtensorMap &tw, const CUtensorMap &th, const CUtensorMap &tl, const WsParams &p, int grid,
                   cudaStream_t st) {
    auto kern = gemm_ws_kernel<NBT, INT4, GROUPED>;
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t e = once_per_device(attr_done, [&] {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)WsSmem<NBT, INT4>::bytes);
    });
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3(grid), dim3(WsRoles<NBT>::kThreads), WsSmem<NBT, INT4>::bytes, st, tw, th, tl, p);
}

template <bool INT4, bool GROUPED>
cudaError_t dispatch_nbt(int nbt, const CUtensorMap &tw, const CUtensorMap &th, const CUtensorMap &tl,
                         const WsParams &p, int grid, cudaStream_t st) {
    switch (nbt) {
    case 16: return run_ws<16, INT4, GROUPED>(tw, th, tl, p, grid, st);
    case 32: return run_ws<32, INT4, GROUPED>(tw, th, tl, p, grid, st);
    default: return run_ws<64, INT4, GROUPED>(tw, th, tl, p, grid, st);
    }
}

}  // namespace

bool gemm_ws_supported(const QMatrix &w, size_t M) {
    if (M < 1 || M > (size_t)kMaxTokens || w.N == 0 || w.N > (size_t)INT32_MAX / 2) return false;
    if (w.K == 0 || w.K % WSK != 0 || w.K > (1u << 20)) return false;
    if (reinterpret_cast<uintptr_t>(w.data) & 15 || reinterpret_cast<uintptr_t>(w.scales) & 15) return false;
    if (w.qtype == kQInt4) return w.block_size == (size_t)WG;
    if (w.qtype == kQInt8) return w.block_size == (size_t)WG || w.block_size == w.K;
    return false;
}

size_t gemm_ws_workspace_bytes(size_t M, size_t N, size_t K, int num_sms, size_t partial_cap) {
    const int nbt = nbt_for(M);
    const int parts = choose_parts(N, K, nbt, num_sms, partial_cap);
    const size_t tiles = (N + WM - 1) / WM;
    const size_t partial = parts > 1 ? tiles * parts * nbt * WM * 4 : 0;
    return ws_layout(M, K, partial).total;
}

cudaError_t launch_gemm_ws(const QMatrix &w, const float *X, size_t M, size_t ldx, float *Y, size_t ldy, void *ws,
                           size_t ws_bytes, unsigned *tickets, size_t num_tickets, int *err, int num_sms,
                           cudaStream_t st) {
    if (!gemm_ws_supported(w, M)) return cudaErrorInvalidValue;
    const int nbt = nbt_for(M);
    const size_t tiles = (w.N + WM - 1) / WM;
    if (tiles > num_tickets) return cudaErrorInvalidValue;
    // the partial sums may use whatever the workspace holds beyond x's fp16 copies
    const WsLayout base = ws_layout(M, w.K, 0);
    if (ws_bytes < base.total || (reinterpret_cast<uintptr_t>(ws) & 255)) return cudaErrorInvalidValue;
    const bool int4 = w.qtype == kQInt4, grouped = w.block_size == (size_t)WG;
    const int parts = choose_parts(w.N, w.K, nbt, num_sms, ws_bytes - base.partial);
    uint8_t *wsb = static_cast<uint8_t *>(ws);
    __half *xhi = reinterpret_cast<__half *>(wsb + base.xhi), *xlo = reinterpret_cast<__half *>(wsb + base.xlo);
    float *xinv = reinterpret_cast<float *>(wsb + base.xinv);

    CUtensorMap tw, th, tl;
    const uint64_t row_bytes = int4 ? w.K / 2 : w.K;
    if (!make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.data, row_bytes, w.N, row_bytes, int4 ? 64 : 128, WM,
                  int4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xhi, w.K, M, w.K * 2, 64, (uint32_t)nbt,
                  CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xlo, w.K, M, w.K * 2, 64, (uint32_t)nbt,
                  CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;

    const int vec = (reinterpret_cast<uintptr_t>(X) & 15) == 0 && (M == 1 || ldx % 4 == 0);
    const unsigned threads = w.K >= 4096 ? 512 : 256;
    cudaError_t e = int4 ? launch_kernel(split_x_rows_kernel<true>, dim3((unsigned)M), dim3(threads), 0, st, X,
                                         (long long)ldx, (int)w.K, xhi, xlo, xinv, vec)
                         : launch_kernel(split_x_rows_kernel<false>, dim3((unsigned)M), dim3(threads), 0, st, X,
                                         (long long)ldx, (int)w.K, xhi, xlo, xinv, vec);
    if (e != cudaSuccess) return e;

    WsParams p{};
    p.M = (int)M;
    p.N = (int)w.N;
    p.K = (int)w.K;
    p.tiles = (int)tiles;
    p.parts = parts;
    p.stages_k = (int)(w.K / WSK);
    p.units = (int)tiles * parts;
    p.scales = w.scales;
    p.xinv = xinv;
    p.Y = Y;
    p.ldy = (long long)ldy;
    p.partial = reinterpret_cast<float *>(wsb + base.partial);
    p.tickets = tickets;
    p.err = err;
    const int grid = std::min(num_sms, p.units);
    if (int4) return dispatch_nbt<true, true>(nbt, tw, th, tl, p, grid, st);
    return grouped ? dispatch_nbt<false, true>(nbt, tw, th, tl, p, grid, st)
                   : dispatch_nbt<false, false>(nbt, tw, th, tl, p, grid, st);
}

const char *gemm_ws_kernel_name() { return "gemm_ws_kernel"; }

}  // namespace pyxis
