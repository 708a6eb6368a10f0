// attn_tc.cu -- the causal prefill attention of the batched decode (src/attention.rs:107-135 for
// every position of a prompt at once) on the tensor cores: tcgen05.mma kind::f16 with fp32
// accumulators in TMEM, operands brought in by TMA.  Operand precision and layout: attn_tc.h.
#include <atomic>

#include "attn_tc.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace pyxis {
namespace {

// CTA = 128 query rows of one head of one sequence (one TMEM lane per row).  Per key tile j of
// 128 keys:
//   S_j = Q K_j^T      24 MMAs (M 128, N 128, K 16) over hi.lo + lo.hi, then hi.hi, into one of
//                      three TMEM score buffers
//   softmax            8 warps, a row per thread and half of the tile's keys per warp: scale,
//                      causal mask, running max (the two halves of a row exchange theirs through
//                      shared memory), p = 2^(s - m), p split into fp16 hi/lo written back over
//                      the scores
//   O_j = P_j V_j      24 MMAs (M 128, N hd, K 16) into a fresh TMEM accumulator: A = the
//                      probabilities straight from TMEM, B = tiles of V^T
//   O += O_j           in fp32 registers of the softmax threads (half of the hd columns each)
// The tensor core's accumulation rounds toward zero, so long chains into one accumulator drift:
// each chain here is one tile's 24 MMAs with the small cross terms first, and the sum over tiles is
// taken with round-to-nearest adds.  Scores are kept in log2 units (s = q.k / sqrt(hd) * log2 e),
// so p = exp2(s - m) is the reference's exp(score - max).  The running maximum m is raised only
// when a tile's maximum exceeds it by more than 11 (so p <= 2^11 stays in fp16 range); then the
// register sum and the row sum are rescaled.  Otherwise the old maximum stays the reference point:
// O / l is the same softmax-weighted sum.
// Warps: 0 TMA producer, 1 MMA issuer (and TMEM owner), 2-9 softmax.  The MMA warp issues
// S_0, S_1, O_0, S_2, O_1, ... so that the scores of tile j+1 are computed while tile j's softmax
// runs; the producer streams K and V in that same order through a ring of 16 KB entries (one
// 64-column block of one operand half each), released as the MMAs finish.
constexpr int kBQ = 128, kBK = 128;
constexpr int kRing = 9;
constexpr uint32_t kEntry = 16384;
constexpr int kProdWarp = 0, kMmaWarp = 1, kSmWarp0 = 2, kSmWarps = 8;
constexpr int kThreads = (kSmWarp0 + kSmWarps) * 32;  // 320
constexpr int kSBufs = 3;
constexpr uint32_t kTmemCols = 512;  // three score buffers of 128 columns, then O_j (hd columns)
constexpr uint32_t kOCol = kSBufs * kBK;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr float kRaise = 11.0f;
constexpr float kLog2e = 1.4426950408889634f;
enum { kErrProd = 0x601, kErrMma = 0x602, kErrSoft = 0x603, kErrDrain = 0x604 };

template <int HD>
struct AtSmem {
    static constexpr int kDB = HD / 64;             // 64-column blocks of a Q or K row
    static constexpr uint32_t kQBlock = kBQ * 128;  // 128 rows x 128 B
    static constexpr uint32_t qh = 0;
    static constexpr uint32_t ql = qh + kDB * kQBlock;
    static constexpr uint32_t ring = ql + kDB * kQBlock;
    static constexpr uint32_t red = ring + kRing * kEntry;  // [2 tiles][2 halves][128 rows] f32
    static constexpr uint32_t bar = red + 2 * 2 * kBQ * 4;
    static constexpr uint32_t num_bars = 2 * kRing + 1 + 3 * kSBufs + 2;
    static constexpr uint32_t misc = bar + num_bars * 8;
    static constexpr uint32_t bytes = misc + 16 + 1024;  // + alignment slack
};
static_assert(AtSmem<128>::bytes <= 232448 && AtSmem<64>::bytes <= 232448, "227 KB of shared memory per CTA");
static_assert(kOCol + 128 <= kTmemCols, "TMEM columns");

struct AtParams {
    int P, Pp, n_q, n_kv;
    long long rows_q, rows_k, rows_v;  // rows of the hi half of each operand (lo rows follow)
    const float *qinv;
    const unsigned *kvmax;
    float *out;
    int *err;
};

PYXIS_DEVINL void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// The MMA schedule: op i of 2T is S_0 (i = 0), O_{T-1} (i = 2T-1), else S_{(i+1)/2} (odd i) or
// O_{i/2-1} (even i).  is_s / tile out.
PYXIS_DEVINL void at_op(int i, int T, bool &is_s, int &tile) {
    if (i == 0) {
        is_s = true, tile = 0;
    } else if (i == 2 * T - 1) {
        is_s = false, tile = T - 1;
    } else if (i & 1) {
        is_s = true, tile = (i + 1) >> 1;
    } else {
        is_s = false, tile = (i >> 1) - 1;
    }
}

// Scores of 32 keys (columns col0.. of this thread's row) in log2 units, with the causal mask of
// the diagonal tile.
PYXIS_DEVINL void score32(const uint32_t (&r)[32], float c2, bool diag, int col0, int row, float (&s)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
        s[i] = (!diag || col0 + i <= row) ? __uint_as_float(r[i]) * c2 : -INFINITY;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attention_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                                const __grid_constant__ CUtensorMap tm_v, const AtParams p) {
    using L = AtSmem<HD>;
    constexpr int kDB = L::kDB;
    constexpr int kOH = HD / 2;                       // O columns per softmax warp
    constexpr uint32_t kVBytes = (uint32_t)HD * 128;  // one 64-key block of V^T: hd rows x 128 B
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar);
    uint64_t *full = bars, *empty = bars + kRing, *qfull = bars + 2 * kRing;
    // per score buffer: sfull (S_j landed), pfull (P_j written), odone (O_j landed, so P_j is read)
    uint64_t *sfull = qfull + 1, *pfull = sfull + kSBufs, *odone = pfull + kSBufs;
    uint64_t *ofree = odone + kSBufs, *drain = ofree + 1;  // ofree: the softmax has read O_j
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::misc + 4);
    float *red = reinterpret_cast<float *>(smem + L::red);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = gridDim.x - 1 - blockIdx.x;  // the query tiles with the most keys start first
    const int head = blockIdx.y, seq = blockIdx.z;
    const int kvh = head / (p.n_q / p.n_kv);
    const int q0 = qt * kBQ, T = qt + 1;  // key tiles 0..qt
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRing; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(qfull, 1);
        for (int b = 0; b < kSBufs; ++b) {
            tc::mbar_init(&sfull[b], 1);
            tc::mbar_init(&pfull[b], kSmWarps);
            tc::mbar_init(&odone[b], 1);
        }
        tc::mbar_init(ofree, kSmWarps);
        tc::mbar_init(drain, 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
    }
    if (warp == kMmaWarp) tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // the operands are written by the kernels before this one
    pdl_trigger();

    if (warp == kProdWarp) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tc::prefetch_tmap(&tm_q);
            tc::prefetch_tmap(&tm_k);
            tc::prefetch_tmap(&tm_v);
            const int qrow = (int)(((long long)seq * p.n_q + head) * p.Pp + q0);
            tc::mbar_arrive_expect_tx(qfull, 2 * kDB * L::kQBlock);
            for (int c = 0; c < kDB; ++c) {
                tc::tma_load_2d(smem + L::qh + c * L::kQBlock, &tm_q, c * 64, qrow, qfull);
                tc::tma_load_2d(smem + L::ql + c * L::kQBlock, &tm_q, c * 64, (int)(qrow + p.rows_q), qfull);
            }
            const int krow = (int)(((long long)seq * p.n_kv + kvh) * p.Pp);
            const int vrow = (int)(((long long)seq * p.n_kv + kvh) * HD);
            int e = 0;
            bool ok = true;
            for (int i = 0; i < 2 * T && ok; ++i) {
                bool is_s;
                int j;
                at_op(i, T, is_s, j);
                const int nblk = is_s ? kDB : 2;
                for (int c = 0; c < nblk && ok; ++c)
                    for (int hl = 0; hl < 2; ++hl, ++e) {
                        const int s = e % kRing;
                        if (e >= kRing && !tc::mbar_wait_bounded(&empty[s], (uint32_t)((e / kRing - 1) & 1), abort_flag,
                                                                 p.err, kErrProd, kTimeoutNs)) {
                            ok = false;
                            break;
                        }
                        uint8_t *dst = smem + L::ring + s * kEntry;
                        if (is_s) {
                            tc::mbar_arrive_expect_tx(&full[s], kBK * 128);
                            tc::tma_load_2d(dst, &tm_k, c * 64, (int)(krow + j * kBK + (hl ? p.rows_k : 0)), &full[s]);
                        } else {
                            tc::mbar_arrive_expect_tx(&full[s], kVBytes);
                            tc::tma_load_2d(dst, &tm_v, j * kBK + c * 64, (int)(vrow + (hl ? p.rows_v : 0)), &full[s]);
                        }
                    }
            }
            if (*abort_flag) {  // let the copies already issued land before the CTA exits
                volatile int no_abort = 0;
                tc::mbar_wait_bounded(qfull, 0, &no_abort, p.err, kErrDrain, 100000000ull);
                for (int x = e > kRing ? e - kRing : 0; x < e; ++x)
                    tc::mbar_wait_bounded(&full[x % kRing], (uint32_t)((x / kRing) & 1), &no_abort, p.err, kErrDrain,
                                          100000000ull);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = tc::idesc_f16_f32(kBQ, kBK);
            constexpr uint32_t idesc_o = tc::idesc_f16_f32(kBQ, HD);
            const uint64_t qh_d = tc::desc_sw128(tc::smem_u32(smem + L::qh));
            const uint64_t ql_d = tc::desc_sw128(tc::smem_u32(smem + L::ql));
            const uint64_t ring_d = tc::desc_sw128(tc::smem_u32(smem + L::ring));
            const uint32_t tO = tmem_base + kOCol;
            bool ok = tc::mbar_wait_bounded(qfull, 0, abort_flag, p.err, kErrMma, kTimeoutNs);
            int e = 0;
            for (int i = 0; i < 2 * T && ok; ++i) {
                bool is_s;
                int j;
                at_op(i, T, is_s, j);
                const int b = j % kSBufs, use = j / kSBufs;
                const uint32_t tS = tmem_base + (uint32_t)(b * kBK);
                if (is_s) {
                    // the buffer's previous probabilities (tile j-3) have been read by O_{j-3}
                    if (use > 0 && !tc::mbar_wait_bounded(&odone[b], (uint32_t)((use - 1) & 1), abort_flag, p.err,
                                                          kErrMma, kTimeoutNs)) {
                        ok = false;
                        break;
                    }
                    // the two small cross terms (hi.lo, lo.hi) of every block first, while the
                    // accumulator is small, then the hi.hi products on top of them
                    const int e0 = e;
                    for (int c = 0; c < kDB && ok; ++c, e += 2) {
                        const int sh = e % kRing, sl = (e + 1) % kRing;
                        ok = tc::mbar_wait_bounded(&full[sh], (uint32_t)((e / kRing) & 1), abort_flag, p.err, kErrMma,
                                                   kTimeoutNs) &&
                             tc::mbar_wait_bounded(&full[sl], (uint32_t)(((e + 1) / kRing) & 1), abort_flag, p.err,
                                                   kErrMma, kTimeoutNs);
                        if (!ok) break;
                        tc::tc_fence_after();
                        const uint64_t kh_d = ring_d + (uint64_t)(sh * (kEntry >> 4));
                        const uint64_t kl_d = ring_d + (uint64_t)(sl * (kEntry >> 4));
                        const uint64_t qo = (uint64_t)(c * (L::kQBlock >> 4));
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint64_t ko = (uint64_t)(kk * 2);  // 16 fp16 = 32 B along the row
                            tc::mma_f16(tS, qh_d + qo + ko, kl_d + ko, idesc_s, (uint32_t)(c | kk));
                            tc::mma_f16(tS, ql_d + qo + ko, kh_d + ko, idesc_s, 1u);
                        }
                        tc::mma_commit(&empty[sl]);
                    }
                    if (!ok) break;
                    for (int c = 0, x = e0; c < kDB; ++c, x += 2) {
                        const int sh = x % kRing;
                        const uint64_t kh_d = ring_d + (uint64_t)(sh * (kEntry >> 4));
                        const uint64_t qo = (uint64_t)(c * (L::kQBlock >> 4));
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc::mma_f16(tS, qh_d + qo + (uint64_t)(kk * 2), kh_d + (uint64_t)(kk * 2), idesc_s, 1u);
                        tc::mma_commit(&empty[sh]);
                    }
                    tc::mma_commit(&sfull[b]);
                } else {
                    // P_j written, and O_{j-1} read out of the single O accumulator
                    ok = tc::mbar_wait_bounded(&pfull[b], (uint32_t)(use & 1), abort_flag, p.err, kErrMma, kTimeoutNs) &&
                         (j == 0 || tc::mbar_wait_bounded(ofree, (uint32_t)((j - 1) & 1), abort_flag, p.err, kErrMma,
                                                          kTimeoutNs));
                    if (!ok) break;
                    tc::tc_fence_after();
                    const int e0 = e;
                    for (int c = 0; c < 2 && ok; ++c, e += 2) {
                        const int sh = e % kRing, sl = (e + 1) % kRing;
                        ok = tc::mbar_wait_bounded(&full[sh], (uint32_t)((e / kRing) & 1), abort_flag, p.err, kErrMma,
                                                   kTimeoutNs) &&
                             tc::mbar_wait_bounded(&full[sl], (uint32_t)(((e + 1) / kRing) & 1), abort_flag, p.err,
                                                   kErrMma, kTimeoutNs);
                        if (!ok) break;
                        tc::tc_fence_after();
                        const uint64_t vh_d = ring_d + (uint64_t)(sh * (kEntry >> 4));
                        const uint64_t vl_d = ring_d + (uint64_t)(sl * (kEntry >> 4));
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint32_t acol = (uint32_t)((c * 4 + kk) * 8);  // 16 keys = 8 columns
                            const uint64_t ko = (uint64_t)(kk * 2);
                            tc::mma_f16_ts(tO, tS + 64 + acol, vh_d + ko, idesc_o, (uint32_t)(c | kk));
                            tc::mma_f16_ts(tO, tS + acol, vl_d + ko, idesc_o, 1u);
                        }
                        tc::mma_commit(&empty[sl]);
                    }
                    if (!ok) break;
                    for (int c = 0, x = e0; c < 2; ++c, x += 2) {
                        const int sh = x % kRing;
                        const uint64_t vh_d = ring_d + (uint64_t)(sh * (kEntry >> 4));
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc::mma_f16_ts(tO, tS + (uint32_t)((c * 4 + kk) * 8), vh_d + (uint64_t)(kk * 2), idesc_o, 1u);
                        tc::mma_commit(&empty[sh]);
                    }
                    tc::mma_commit(&odone[b]);
                }
            }
            // every MMA this thread issued must complete before TMEM is released
            tc::mma_commit(drain);
            volatile int no_abort = 0;
            tc::mbar_wait_bounded(drain, 0, &no_abort, p.err, kErrDrain, kTimeoutNs);
        }
    } else {
        // ------------------------------------------------------------------ softmax
        const int quad = warp & 3;                 // TMEM lanes 32 quad .. 32 quad + 31
        const int half = (warp - kSmWarp0) >> 2;   // keys [64 half, +64) of each tile, O columns [kOH half, +kOH)
        const int row = quad * 32 + lane, qi = q0 + row;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const uint32_t tOh = tmem_base + lane_off + kOCol + (uint32_t)(half * kOH);
        const float kmax = __uint_as_float(__ldg(&p.kvmax[((size_t)seq * p.n_kv + kvh) * 2]));
        const float vmax = __uint_as_float(__ldg(&p.kvmax[((size_t)seq * p.n_kv + kvh) * 2 + 1]));
        const float qinv = __ldg(&p.qinv[((size_t)seq * p.n_q + head) * p.Pp + qi]);
        // score in log2 units: acc * 2^-(eq + ek) / sqrt(hd) * log2 e
        const float c2 = qinv * attn_pow2(-attn_scale_exp(kmax)) * (kLog2e / sqrtf((float)HD));
        float m_run = -INFINITY, l = 0.f;
        float acc[kOH];
#pragma unroll
        for (int i = 0; i < kOH; ++i) acc[i] = 0.f;
        // O_{t} (scale of the maximum at tile t) into acc, then acc *= alpha
        auto fold_o = [&](int t, float alpha) -> bool {
            const bool w = __all_sync(0xffffffffu, tc::mbar_wait_bounded(&odone[t % kSBufs], (uint32_t)((t / kSBufs) & 1),
                                                                         abort_flag, p.err, kErrSoft, kTimeoutNs));
            if (!w) return false;
            tc::tc_fence_after();
#pragma unroll
            for (int c = 0; c < kOH / 32; ++c) {
                uint32_t o[32];
                tc::tmem_ld32_async(tOh + (uint32_t)(c * 32), o);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) acc[c * 32 + i] = (acc[c * 32 + i] + __uint_as_float(o[i])) * alpha;
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(ofree);
            return true;
        };
        bool ok = true;
        for (int j = 0; j < T; ++j) {
            const int b = j % kSBufs, use = j / kSBufs;
            const uint32_t tS = tmem_base + lane_off + (uint32_t)(b * kBK);
            const bool diag = j == qt;  // the diagonal tile: key k0 + col attends query q0 + row iff col <= row
            ok = ok && __all_sync(0xffffffffu, tc::mbar_wait_bounded(&sfull[b], (uint32_t)(use & 1), abort_flag,
                                                                      p.err, kErrSoft, kTimeoutNs));
            float mt = -INFINITY;
            if (ok) {
                tc::tc_fence_after();
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t r[32];
                    float s[32];
                    tc::tmem_ld32_async(tS + half * 64 + c * 32, r);
                    tc::tmem_wait_ld();
                    score32(r, c2, diag, half * 64 + c * 32, row, s);
#pragma unroll
                    for (int i = 0; i < 32; ++i) mt = fmaxf(mt, s[i]);
                }
            }
            float *rd = red + (j & 1) * 2 * kBQ;
            rd[half * kBQ + row] = mt;
            named_bar(1 + quad, 64);  // both halves of these 32 rows
            mt = fmaxf(mt, rd[(1 - half) * kBQ + row]);
            if (!ok) continue;
            const bool raise = mt > m_run + kRaise;
            const float alpha = raise ? exp2f(m_run - mt) : 1.0f;  // 0 on the first tile
            if (raise) {
                l *= alpha;
                m_run = mt;
            }
            uint32_t ph[32], pl[32];
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t r[32];
                float s[32];
                tc::tmem_ld32_async(tS + half * 64 + c * 32, r);
                tc::tmem_wait_ld();
                score32(r, c2, diag, half * 64 + c * 32, row, s);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = exp2f(s[2 * i] - m_run), p1 = exp2f(s[2 * i + 1] - m_run);
                    sum += p0 + p1;
                    const __half2 h = __floats2half2_rn(p0, p1);
                    const float2 hf = __half22float2(h);
                    const __half2 lo = __floats2half2_rn(p0 - hf.x, p1 - hf.y);
                    ph[c * 16 + i] = *reinterpret_cast<const uint32_t *>(&h);
                    pl[c * 16 + i] = *reinterpret_cast<const uint32_t *>(&lo);
                }
            }
            l += sum;
            // keys 2i, 2i+1 of this half -> column half * 32 + i (hi) and 64 + half * 32 + i (lo)
            tc::tmem_st32(tS + half * 32, ph);
            tc::tmem_st32(tS + 64 + half * 32, pl);
            tc::tmem_wait_st();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&pfull[b]);
            // the previous tile's P V, at the previous maximum, then this tile's rescale
            if (j > 0) ok = fold_o(j - 1, alpha);
        }
        ok = ok && fold_o(T - 1, 1.0f);
        // the row sum of both halves, then O / l of this half's columns
        float *rd = red + (T & 1) * 2 * kBQ;
        rd[half * kBQ + row] = l;
        named_bar(1 + quad, 64);
        const float lt = l + rd[(1 - half) * kBQ + row];
        if (ok && qi < p.P) {
            const float sc = __fdiv_rn(attn_pow2(-attn_scale_exp(vmax)), lt);
            const int q_dim = p.n_q * HD;
            float *dst = p.out + ((size_t)seq * p.P + qi) * q_dim + (size_t)head * HD + half * kOH;
#pragma unroll
            for (int i = 0; i < kOH; i += 4)
                *reinterpret_cast<float4 *>(dst + i) =
                    make_float4(acc[i] * sc, acc[i + 1] * sc, acc[i + 2] * sc, acc[i + 3] * sc);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == kMmaWarp) tc::tmem_dealloc(tmem_base, kTmemCols);
}

// K and V of 64 cache rows of one kv head -> scaled fp16 hi/lo: K row-major, V transposed.
// grid (Pp / 64, n_kv, cs), 256 threads.
template <int HD>
__global__ void __launch_bounds__(256)
    attn_prep_kv_kernel(const float *__restrict__ kc, const float *__restrict__ vc, long long cache_stride, int P,
                        int Pp, int n_kv, int cs, __half *__restrict__ k, __half *__restrict__ vt,
                        const unsigned *__restrict__ kvmax) {
    constexpr int LD = HD + 1;
    __shared__ float vs[64 * LD];  // [key][d]
    pdl_wait();
    pdl_trigger();
    const int j0 = blockIdx.x * 64, kvh = blockIdx.y, seq = blockIdx.z;
    const int kv_dim = n_kv * HD;
    const float ksc = attn_pow2(attn_scale_exp(__uint_as_float(kvmax[((size_t)seq * n_kv + kvh) * 2])));
    const float vsc = attn_pow2(attn_scale_exp(__uint_as_float(kvmax[((size_t)seq * n_kv + kvh) * 2 + 1])));
    const size_t k_half = (size_t)cs * n_kv * Pp * HD, v_half = (size_t)cs * n_kv * HD * Pp;
    __half *kh = k + (((size_t)seq * n_kv + kvh) * Pp + j0) * HD;
    const float *kb = kc + seq * cache_stride + (size_t)j0 * kv_dim + (size_t)kvh * HD;
    const float *vb = vc + seq * cache_stride + (size_t)j0 * kv_dim + (size_t)kvh * HD;
    for (int idx = threadIdx.x; idx < 64 * (HD / 4); idx += 256) {
        const int r = idx / (HD / 4), c4 = idx % (HD / 4);
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), v = a;
        if (j0 + r < P) {
            a = *reinterpret_cast<const float4 *>(kb + (size_t)r * kv_dim + c4 * 4);
            v = *reinterpret_cast<const float4 *>(vb + (size_t)r * kv_dim + c4 * 4);
        }
        const float2 x01 = make_float2(a.x * ksc, a.y * ksc), x23 = make_float2(a.z * ksc, a.w * ksc);
        const __half2 h01 = __float22half2_rn(x01), h23 = __float22half2_rn(x23);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const __half2 l01 = __floats2half2_rn(x01.x - f01.x, x01.y - f01.y);
        const __half2 l23 = __floats2half2_rn(x23.x - f23.x, x23.y - f23.y);
        __half2 *dh = reinterpret_cast<__half2 *>(kh + (size_t)r * HD + c4 * 4);
        __half2 *dl = reinterpret_cast<__half2 *>(kh + k_half + (size_t)r * HD + c4 * 4);
        dh[0] = h01, dh[1] = h23, dl[0] = l01, dl[1] = l23;
        float *vr = vs + r * LD + c4 * 4;
        vr[0] = v.x * vsc, vr[1] = v.y * vsc, vr[2] = v.z * vsc, vr[3] = v.w * vsc;
    }
    __syncthreads();
    __half *vh = vt + ((size_t)seq * n_kv + kvh) * HD * Pp + j0;
    for (int idx = threadIdx.x; idx < HD * 8; idx += 256) {  // row d of V^T, keys c8 * 8 .. + 8
        const int d = idx >> 3, c8 = idx & 7;
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float x0 = vs[(c8 * 8 + 2 * t) * LD + d], x1 = vs[(c8 * 8 + 2 * t + 1) * LD + d];
            const __half2 h = __floats2half2_rn(x0, x1);
            const float2 f = __half22float2(h);
            const __half2 lo = __floats2half2_rn(x0 - f.x, x1 - f.y);
            hw[t] = *reinterpret_cast<const uint32_t *>(&h);
            lw[t] = *reinterpret_cast<const uint32_t *>(&lo);
        }
        *reinterpret_cast<uint4 *>(vh + (size_t)d * Pp + c8 * 8) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(vh + v_half + (size_t)d * Pp + c8 * 8) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
}

bool make_map_f16(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint32_t box_outer) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {64, box_outer};
    cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD>
cudaError_t run_attn(const CUtensorMap &q, const CUtensorMap &k, const CUtensorMap &v, const AtParams &p, dim3 grid,
                     cudaStream_t st) {
    auto kern = attention_prefill_tc_kernel<HD>;
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t e = once_per_device(attr_done, [&] {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AtSmem<HD>::bytes);
    });
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, grid, dim3(kThreads), AtSmem<HD>::bytes, st, q, k, v, p);
}

}  // namespace

bool attn_tc_supported(int head_dim) { return head_dim == 64 || head_dim == 128; }

cudaError_t launch_attn_prep_kv(const float *kc, const float *vc, long long cache_stride, int cs, int P, int n_kv,
                                int hd, const AttnTcBuffers &b, cudaStream_t st) {
    const int Pp = attn_tc_padded(P);
    const dim3 grid(Pp / 64, n_kv, cs);
    if (hd == 128)
        return launch_kernel(attn_prep_kv_kernel<128>, grid, dim3(256), 0, st, kc, vc, cache_stride, P, Pp, n_kv, cs,
                             b.k, b.vt, (const unsigned *)b.kvmax);
    if (hd == 64)
        return launch_kernel(attn_prep_kv_kernel<64>, grid, dim3(256), 0, st, kc, vc, cache_stride, P, Pp, n_kv, cs,
                             b.k, b.vt, (const unsigned *)b.kvmax);
    return cudaErrorInvalidValue;
}

cudaError_t launch_attention_prefill_tc(int cs, int P, int n_q, int n_kv, int hd, const AttnTcBuffers &b, float *out,
                                        int *err, cudaStream_t st) {
    if (!attn_tc_supported(hd) || n_kv <= 0 || n_q % n_kv != 0 || P <= 0 || cs <= 0) return cudaErrorInvalidValue;
    const int Pp = attn_tc_padded(P);
    AtParams p;
    p.P = P;
    p.Pp = Pp;
    p.n_q = n_q;
    p.n_kv = n_kv;
    p.rows_q = (long long)cs * n_q * Pp;
    p.rows_k = (long long)cs * n_kv * Pp;
    p.rows_v = (long long)cs * n_kv * hd;
    p.qinv = b.qinv;
    p.kvmax = b.kvmax;
    p.out = out;
    p.err = err;
    if (2 * p.rows_q >= (1ll << 31) || 2 * p.rows_k >= (1ll << 31)) return cudaErrorInvalidValue;
    CUtensorMap tq, tk, tv;
    if (!make_map_f16(&tq, b.q, (uint64_t)hd, (uint64_t)(2 * p.rows_q), kBQ) ||
        !make_map_f16(&tk, b.k, (uint64_t)hd, (uint64_t)(2 * p.rows_k), kBK) ||
        !make_map_f16(&tv, b.vt, (uint64_t)Pp, (uint64_t)(2 * p.rows_v), (uint32_t)hd))
        return cudaErrorInvalidValue;
    const dim3 grid(Pp / kBQ, n_q, cs);
    return hd == 128 ? run_attn<128>(tq, tk, tv, p, grid, st) : run_attn<64>(tq, tk, tv, p, grid, st);
}

}  // namespace pyxis
