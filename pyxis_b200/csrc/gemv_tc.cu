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
// warp 1 = TMEM owner + MMA issuer (M=128, N=16|32, K=32 per instruction, accumulator
// double-buffered in TMEM across tile segments), warps 2-5 = epilogue (tcgen05.ld, one TMEM
// lane = one weight row).  Warps 1-5 build the digit operand while the producer's first copies
// are in flight.  A tile whose stages span several CTAs has its partial int32 sums added exactly
// with atomics into a scratch slot, and the CTA that finishes the tile last
// converts it and zeroes the scratch for the next launch.  The schedule is stream-K: every CTA
// gets the same number of (tile, K-block) stages.  Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace pyxis {
namespace {

constexpr int TM = 128;    // weight rows per tile
constexpr int TKB = 128;   // K bytes (= int8 codes) per stage
constexpr int kMaxTok = 8;
constexpr int kThreads = 192;
constexpr uint32_t kStageBytes = TM * TKB;
constexpr uint32_t kSmemTotal = 222 * 1024;
constexpr int kMaxStages = 12;
constexpr uint64_t kTimeoutNs = 2000000000ull;
// The 4 MMAs of a stage (one per 32-byte K slice) write 4 separate accumulators, so they do not
// wait on each other; the epilogue adds them (exact int32).  2 buffers x 4 x NB(<= 32) columns.
constexpr int kAccPerBuf = TKB / 32;
constexpr uint32_t kTmemCols = 256;
enum { kErrProd = 0x301, kErrMma = 0x302, kErrEpi = 0x303, kErrDrain = 0x304 };

struct Params {
    int N, K, B, NB;
    int num_kb, num_tiles, stages;
    long long total_stages;  // num_tiles * num_kb, split evenly over the grid (stream-K)
    uint32_t xd_bytes;
    const float *x;
    long long ldx;
    const float *scales;
    float *y;
    long long ldy;
    int *accum;         // [grid][128][NB] int32 partial tiles, zero between launches
    unsigned *tickets;  // [grid], zero between launches
    int *err;
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

PYXIS_DEVINL void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

PYXIS_DEVINL float combine(const int *D, double xs, double sr) {
    const long long s = (long long)D[0] * 2097152LL + (long long)D[1] * 16384LL + (long long)D[2] * 128LL + D[3];
    return (float)((double)s * xs * sr);
}

// Stream-K schedule: the num_tiles x num_kb stages are cut into gridDim.x equal contiguous
// ranges; a tile whose stages span several CTAs is combined exactly (int32 atomics) in the slot
// of the first CTA that touches it -- each CTA is the first of at most one shared tile.
struct Sched {
    long long T;
    int G, nkb;
    PYXIS_DEVINL long long begin(int c) const { return (long long)c * T / G; }
    PYXIS_DEVINL int owner(long long s) const { return (int)(((s + 1) * G + T - 1) / T - 1); }
};

__global__ void __launch_bounds__(kThreads, 1)
    gemv_tc_i8_kernel(const __grid_constant__ CUtensorMap tm_w, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *xd = smem;                    // digit operand: [kb][NB rows][128 B], 128-byte swizzle
    uint8_t *ring = smem + p.xd_bytes;     // stages of 128 rows x 128 B codes
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + (size_t)p.stages * kStageBytes);
    uint64_t *full = bars, *empty = bars + kMaxStages;
    uint64_t *tfull = bars + 2 * kMaxStages, *tempty = tfull + 2, *drain = tempty + 2;
    double *xscale = reinterpret_cast<double *>(drain + 1);          // [kMaxTok]
    float *red = reinterpret_cast<float *>(xscale + kMaxTok);        // [kMaxTok][5]
    int *xexp = reinterpret_cast<int *>(red + kMaxTok * 5);          // [kMaxTok]
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
        *abort_flag = 0;
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // -------------------------------------------------------------------- TMA producer
        if (lane == 0) {
            tc::prefetch_tmap(&tm_w);
            int g = 0;
            const Sched sc{p.total_stages, (int)gridDim.x, p.num_kb};
            const long long se = sc.begin(blockIdx.x + 1);
            for (long long st = sc.begin(blockIdx.x); st < se; ++st, ++g) {
                const int s = g % p.stages;
                if (g >= p.stages &&
                    !tc::mbar_wait_bounded(&empty[s], ((g / p.stages) - 1) & 1, abort_flag, p.err, kErrProd, kTimeoutNs))
                    break;
                const int tile = (int)(st / p.num_kb), kb = (int)(st % p.num_kb);
                tc::mbar_arrive_expect_tx(&full[s], kStageBytes);
                tc::tma_load_2d(ring + (size_t)s * kStageBytes, &tm_w, kb * TKB, tile * TM, &full[s]);
            }
            if (*abort_flag) {  // let the copies already issued land
                volatile int no_abort = 0;
                for (int j = g > p.stages ? g - p.stages : 0; j < g; ++j)
                    tc::mbar_wait_bounded(&full[j % p.stages], (j / p.stages) & 1, &no_abort, p.err, kErrDrain, 100000000ull);
            }
        }
    } else {
        // -------------------------------------------------------------------- digit operand
        const int bt = threadIdx.x - 32, nbt = kThreads - 32;  // warps 1-5
        const int bwarp = warp - 1;
        pdl_wait();  // x comes from the previous kernel; the producer's weight copies do not wait
        pdl_trigger();
        const Sched sc{p.total_stages, (int)gridDim.x, p.num_kb};
        const long long my_sb = sc.begin(blockIdx.x), my_se = sc.begin(blockIdx.x + 1);
        // K-blocks this CTA multiplies: a contiguous run (mod num_kb) unless it spans a whole tile
        const int need_lo = (int)(my_sb % p.num_kb);
        const long long need_n = my_se - my_sb;
        auto needed = [&](int kb) { return need_n >= p.num_kb || ((kb - need_lo + p.num_kb) % p.num_kb) < need_n; };
        for (int b = 0; b < p.B; ++b) {
            const float *xb = p.x + (size_t)b * p.ldx;
            float m = 0.f;
            for (int k = bt; k < p.K; k += nbt) m = fmaxf(m, fabsf(xb[k]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) red[b * 5 + bwarp] = m;
        }
        {
            const uint4 z = make_uint4(0, 0, 0, 0);
            const uint32_t per_kb = (uint32_t)p.NB * TKB / 16;
            for (uint32_t i = bt; i < p.xd_bytes / 16; i += nbt)
                if (needed((int)(i / per_kb))) reinterpret_cast<uint4 *>(xd)[i] = z;
        }
        named_bar(1, nbt);
        if (bt < p.B) {
            float m = red[bt * 5];
            for (int w = 1; w < 5; ++w) m = fmaxf(m, red[bt * 5 + w]);
            int E = 0;
            if (m > 0.f && isfinite(m)) frexpf(m, &E);  // m < 2^E
            xexp[bt] = E;
            xscale[bt] = isfinite(m) ? ldexp(1.0, E - 27) : __longlong_as_double(0x7ff8000000000000ll);
        }
        named_bar(1, nbt);
        const int kq = p.K / 4;
        for (int idx = bt; idx < p.B * kq; idx += nbt) {
            const int b = idx / kq, k = (idx - b * kq) * 4;
            if (!needed(k / TKB)) continue;
            const int E = xexp[b];
            const float4 xv = *reinterpret_cast<const float4 *>(p.x + (size_t)b * p.ldx + k);
            const float xs4[4] = {xv.x, xv.y, xv.z, xv.w};
            uint32_t word[4] = {0, 0, 0, 0};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float v = ldexpf(xs4[e], 27 - E);
                int t = isfinite(v) ? (int)rintf(v) : 0;
                int dg[4];
#pragma unroll
                for (int i = 3; i >= 1; --i) {
                    dg[i] = ((t + 64) & 127) - 64;
                    t = (t - dg[i]) >> 7;
                }
                dg[0] = t;
#pragma unroll
                for (int i = 0; i < 4; ++i) word[i] |= ((uint32_t)(dg[i] & 0xff)) << (8 * e);
            }
            const int kb = k / TKB, kk = k % TKB, c = kk >> 4;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = 4 * b + i;
                uint8_t *row = xd + (size_t)kb * (p.NB * TKB) + (r >> 3) * 1024 + (r & 7) * 128;
                *reinterpret_cast<uint32_t *>(row + ((c ^ (r & 7)) << 4) + (kk & 15)) = word[i];
            }
        }
        tc::fence_proxy_async_smem();
        named_bar(1, nbt);

        if (warp == 1) {
            // ---------------------------------------------------------------- MMA issuer
            if (lane == 0) {
                const uint32_t idesc = idesc_i8(TM, p.NB);
                int g = 0, li = 0;
                bool ok = true;
                for (long long st = my_sb; st < my_se && ok; ++li) {
                    const int tile = (int)(st / p.num_kb);
                    const long long tend = my_se < (long long)(tile + 1) * p.num_kb ? my_se : (long long)(tile + 1) * p.num_kb;
                    const int kb0 = (int)(st % p.num_kb), nk = (int)(tend - st);
                    st = tend;
                    const int buf = li & 1;
                    if (li >= 2) {
                        ok = tc::mbar_wait_bounded(&tempty[buf], ((li >> 1) - 1) & 1, abort_flag, p.err, kErrMma, kTimeoutNs);
                        if (!ok) break;
                    }
                    tc::tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(buf * kAccPerBuf * p.NB);
                    for (int kb = kb0; kb < kb0 + nk; ++kb, ++g) {
                        const int s = g % p.stages;
                        ok = tc::mbar_wait_bounded(&full[s], (g / p.stages) & 1, abort_flag, p.err, kErrMma, kTimeoutNs);
                        if (!ok) break;
                        tc::tc_fence_after();
                        const uint64_t a0 = tc::desc_sw128(tc::smem_u32(ring + (size_t)s * kStageBytes));
                        const uint64_t b0 = tc::desc_sw128(tc::smem_u32(xd + (size_t)kb * (p.NB * TKB)));
#pragma unroll
                        for (int q = 0; q < TKB / 32; ++q)
                            mma_i8(d + (uint32_t)(q * p.NB), a0 + (uint64_t)(2 * q), b0 + (uint64_t)(2 * q), idesc,
                                   kb > kb0 ? 1u : 0u);
                        tc::mma_commit(&empty[s]);
                    }
                    if (ok) tc::mma_commit(&tfull[buf]);
                }
                tc::mma_commit(drain);
                volatile int no_abort = 0;
                tc::mbar_wait_bounded(drain, 0, &no_abort, p.err, kErrDrain, kTimeoutNs);
            }
        } else {
            // ---------------------------------------------------------------- epilogue
            // All four warps run the same item sequence and the same named barriers; a warp
            // whose wait ran out skips the work but keeps the barrier sequence.
            const int qd = warp & 3;  // TMEM lane quarter of this warp
            int li = 0;
            for (long long st = my_sb; st < my_se; ++li) {
                const int tile = (int)(st / p.num_kb);
                st = my_se < (long long)(tile + 1) * p.num_kb ? my_se : (long long)(tile + 1) * p.num_kb;
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
                        for (int b = 0; b < p.B; ++b) p.y[(size_t)b * p.ldy + row] = combine(&D[4 * b], xscale[b], sr);
                    }
                } else {
                    int *acc = p.accum + ((size_t)first * TM + rl) * p.NB;
                    if (ok)
                        for (int j = 0; j < 4 * p.B; ++j) atomicAdd(acc + j, D[j]);
                    __threadfence();
                    named_bar(2, 128);
                    if (warp == 2 && lane == 0) *last_flag = atomicAdd(&p.tickets[first], 1u) == (unsigned)(parts - 1);
                    named_bar(2, 128);
                    const bool last = *last_flag;
                    if (last) {
                        __threadfence();
                        int S[32];
                        for (int j = 0; j < 4 * p.B; ++j) {
                            S[j] = __ldcg(acc + j);
                            acc[j] = 0;  // leave the scratch zeroed for the next launch
                        }
                        if (row < p.N && !*abort_flag) {
                            const double sr = (double)__ldg(p.scales + row);
                            for (int b = 0; b < p.B; ++b) p.y[(size_t)b * p.ldy + row] = combine(&S[4 * b], xscale[b], sr);
                        }
                    }
                    named_bar(2, 128);
                    if (last && warp == 2 && lane == 0) p.tickets[first] = 0;
                }
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
    const uint32_t avail = kSmemTotal - 1024 - 1024 - pl.xd_bytes;  // alignment slack, barriers
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
                           void *scratch, size_t scratch_bytes, int *err, int num_sms, cudaStream_t st) {
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
    Params p{};
    p.N = (int)w.N;
    p.K = (int)w.K;
    p.B = (int)B;
    p.NB = pl.NB;
    p.num_kb = (int)(w.K / TKB);
    p.num_tiles = num_tiles;
    p.total_stages = total;
    p.stages = pl.stages;
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
    static const bool attr =
        cudaFuncSetAttribute(gemv_tc_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal) == cudaSuccess;
    if (!attr) return cudaErrorInvalidConfiguration;
    return launch_kernel(gemv_tc_i8_kernel, dim3(grid), dim3(kThreads), kSmemTotal, st, tm, p);
}

}  // namespace pyxis
