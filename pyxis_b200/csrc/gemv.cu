// gemv.cu -- decode GEMV over int8 / int4 weights in the reference layout, fp32 accumulation.
//
// Computes what src/matmul.rs:67-96 computes row by row -- y[n] = sum_i x[i] * q[n,i] *
// scale(n,i) -- for B = 1..8 input rows at once, streaming the packed weights from HBM once.
//
// Kernels (chosen by launch_gemv from the shape):
//   team   B = 1.  A "team" of T threads (a multiple of 32) covers one row: thread t owns the
//          16-byte chunks t, t+T, ... of every row it visits, so its slice of x stays in
//          registers for the whole kernel and x costs no shared-memory or L1 traffic.  Each team
//          loads R rows' chunks before using any (R * CPT 128-bit loads in flight per thread).
//   batch  B = 2..8 (and B = 1 shapes the team kernel does not take): gemv_batch.cu.
//   generic  any shape the two above do not take (K not a multiple of the chunk, blocks that
//          straddle rows, odd K with int4 rows that start mid-byte): one warp per row,
//          element-wise decode with the reference's scales[g / block_size] lookup.
// A 16-byte chunk is 16 int8 or 32 int4 codes.  Codes become exact floats by byte_perm into
// the mantissa of 2^23 and a paired subtraction; products accumulate with paired fp32 FMAs
// (fma.rn.f32x2).  Scales: block == K applies the row scale once after the row sum; blocks that
// are a multiple of the chunk and divide K scale each chunk's partial sum.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace pyxis {

enum { kScaleRow = 0, kScaleChunk = 1 };

template <int QT>
struct QT_ {
    static constexpr int EPC = QT == kQInt8 ? 16 : 32;  // elements per 16-byte chunk
};

// Dot product of one 16-byte chunk with its EPC x values (as EPC/2 float2).
template <int QT>
PYXIS_DEVINL float chunk_dot(const uint4 w, const float2 *x) {
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

struct GemvParams {
    const uint8_t *W;
    const float *S;
    const float *X;
    float *Y;
    int N, K;
    int ldx, ldy;
    int row_bytes;       // bytes per row of W
    int chunks;          // 16-byte chunks per row
    int team;            // team size (threads), multiple of 32
    int teams_per_cta;
    int blocks_per_row;  // kScaleChunk: K / block_size
    int chunks_per_block;
};

// ---------------------------------------------------------------- team kernel (B = 1) --------
template <int QT, int CPT, int R, int SMODE>
__global__ void __launch_bounds__(512) gemv_team_kernel(GemvParams p) {
    constexpr int EPC = QT_<QT>::EPC;
    __shared__ float red[16][R];  // per-warp partial sums (teams wider than one warp)
    const int tid = threadIdx.x;
    const int team_local = tid / p.team;
    const int t = tid - team_local * p.team;
    const int warp = tid >> 5, lane = tid & 31;
    const int warps_per_team = p.team >> 5;

    float2 xr[CPT][EPC / 2];
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
        const float4 *xp = reinterpret_cast<const float4 *>(p.X + (size_t)(t + j * p.team) * EPC);
#pragma unroll
        for (int v = 0; v < EPC / 4; ++v) {
            float4 f = __ldg(xp + v);
            xr[j][2 * v] = f2(f.x, f.y);
            xr[j][2 * v + 1] = f2(f.z, f.w);
        }
    }

    const int rows_per_cta_iter = p.teams_per_cta * R;
    for (int base = blockIdx.x * rows_per_cta_iter; base < p.N; base += gridDim.x * rows_per_cta_iter) {
        const int row0 = base + team_local * R;
        uint4 wv[R][CPT];
        float sv[R][CPT];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = row0 + r;
            const bool ok = row < p.N;
            const uint8_t *wrow = p.W + (size_t)row * p.row_bytes;
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                const int c = t + j * p.team;
                wv[r][j] = ok ? ld_stream_v4(wrow + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
                if (SMODE == kScaleChunk)
                    sv[r][j] = ok ? ld_nc_f32(p.S + (size_t)row * p.blocks_per_row + c / p.chunks_per_block) : 0.f;
            }
            if (SMODE == kScaleRow) sv[r][0] = ok ? ld_nc_f32(p.S + row) : 0.f;
        }
        float part[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                float d = chunk_dot<QT>(wv[r][j], xr[j]);
                if (SMODE == kScaleChunk) acc = fmaf(sv[r][j], d, acc);
                else acc += d;
            }
            part[r] = warp_sum(acc);
        }
        if (warps_per_team == 1) {
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int row = row0 + r;
                    if (row < p.N) p.Y[row] = SMODE == kScaleRow ? part[r] * sv[r][0] : part[r];
                }
            }
        } else {
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; ++r) red[warp][r] = part[r];
            }
            __syncthreads();
            if (t < R) {
                const int row = row0 + t;
                const int w0 = team_local * warps_per_team;
                float s = 0.f;
                for (int w = 0; w < warps_per_team; ++w) s += red[w0 + w][t];
                if (row < p.N) {
                    float sc = 1.f;
                    if (SMODE == kScaleRow) sc = ld_nc_f32(p.S + row);
                    p.Y[row] = SMODE == kScaleRow ? s * sc : s;
                }
            }
            __syncthreads();
        }
    }
}

// ---------------------------------------------------------------- generic kernel --------------
template <int QT>
__global__ void gemv_generic_kernel(const uint8_t *W, const float *S, size_t bs, const float *X,
                                    size_t ldx, float *Y, size_t ldy, size_t N, size_t K, int B) {
    const size_t row = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= N) return;
    for (int b = 0; b < B; ++b) {
        const float *x = X + (size_t)b * ldx;
        float acc = 0.f;
        for (size_t i = lane; i < K; i += 32) {
            const size_t g = row * K + i;  // flattened index: blocks run over it (src/matmul.rs:70)
            float q;
            if (QT == kQInt8) {
                q = (float)(int8_t)W[g];
            } else {
                const uint8_t byte = W[g / 2];
                q = (float)((g & 1) ? (byte >> 4) : (byte & 0x0f)) - 8.0f;
            }
            acc += (x[i] * q) * S[g / bs];
        }
        acc = warp_sum(acc);
        if (lane == 0) Y[(size_t)b * ldy + row] = acc;
    }
}

// ---------------------------------------------------------------- dispatch --------------------
namespace {

struct Plan {
    enum Kind { kTeam, kGeneric } kind;
    int smode;
    int cpt, r;  // team kernel
    int team;
};

Plan make_plan(const QMatrix &w, size_t B, size_t ldx) {
    Plan pl{Plan::kGeneric, kScaleRow, 0, 0, 0};
    const int epc = w.qtype == kQInt8 ? 16 : 32;
    const size_t K = w.K, bs = w.block_size;
    if (K == 0 || K % epc != 0 || K > (1u << 20) || w.N > (size_t)INT32_MAX) return pl;
    if ((reinterpret_cast<uintptr_t>(w.data) & 15) != 0) return pl;
    if (B > 1 && (ldx % 4) != 0) return pl;
    int smode;
    if (bs == K) smode = kScaleRow;
    else if (bs % epc == 0 && K % bs == 0) smode = kScaleChunk;
    else return pl;
    pl.smode = smode;
    const int chunks = (int)(K / epc);
    if (B == 1) {
        const int max_cpt = w.qtype == kQInt8 ? 4 : 2;  // <= 64 x registers per thread
        for (int cpt = max_cpt; cpt >= 1; --cpt) {
            if (chunks % cpt) continue;
            const int team = chunks / cpt;
            if (team % 32 || team > 512) continue;
            pl.kind = Plan::kTeam;
            pl.cpt = cpt;
            pl.team = team;
            pl.r = cpt >= 3 ? 1 : (cpt == 2 ? 2 : 4);
            return pl;
        }
    }
    pl.kind = Plan::kGeneric;
    return pl;
}

template <typename KernelT>
int max_ctas_per_sm(KernelT kern, int threads, size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem) != cudaSuccess || n < 1) n = 1;
    return n;
}

template <int QT, int CPT, int R, int SMODE>
cudaError_t run_team(const GemvParams &p0, int num_sms, cudaStream_t st) {
    GemvParams p = p0;
    p.teams_per_cta = std::max(1, 256 / p.team);
    const int threads = p.teams_per_cta * p.team;
    static const int occ = max_ctas_per_sm(gemv_team_kernel<QT, CPT, R, SMODE>, threads, 0);
    const long rows_per_cta = (long)p.teams_per_cta * R;
    long grid = (p.N + rows_per_cta - 1) / rows_per_cta;
    grid = std::min<long>(grid, (long)occ * num_sms);
    gemv_team_kernel<QT, CPT, R, SMODE><<<(unsigned)std::max<long>(grid, 1), threads, 0, st>>>(p);
    return cudaGetLastError();
}

template <int QT, int SMODE>
cudaError_t dispatch_team(const Plan &pl, const GemvParams &p, int num_sms, cudaStream_t st) {
    if (QT == kQInt8) {  // make_plan caps int8 at 4 chunks per thread, int4 at 2
        switch (pl.cpt) {
        case 4: return run_team<QT, 4, 1, SMODE>(p, num_sms, st);
        case 3: return run_team<QT, 3, 1, SMODE>(p, num_sms, st);
        case 2: return run_team<QT, 2, 2, SMODE>(p, num_sms, st);
        default: return run_team<QT, 1, 4, SMODE>(p, num_sms, st);
        }
    }
    if (pl.cpt == 2) return run_team<QT, 2, 2, SMODE>(p, num_sms, st);
    return run_team<QT, 1, 4, SMODE>(p, num_sms, st);
}

}  // namespace

const char *gemv_kernel_name(const QMatrix &w, size_t B, int num_sms) {
    if (B == 1 && gemv_ring_supported(w, num_sms)) return "gemv_ring_kernel";
    Plan pl = make_plan(w, B, 4);
    if (pl.kind != Plan::kTeam && gemv_batch_supported(w, B, num_sms)) return "gemv_batch_kernel";
    switch (pl.kind) {
    case Plan::kTeam: return "gemv_team_kernel";
    default: return "gemv_generic_kernel";
    }
}

cudaError_t launch_gemv(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y,
                        size_t ldy, int *err, int num_sms, cudaStream_t st) {
    if (w.N == 0 || B == 0) return cudaSuccess;
    if (B == 1 && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && gemv_ring_supported(w, num_sms))
        return launch_gemv_ring(w, X, Y, err, num_sms, st);
    if ((reinterpret_cast<uintptr_t>(X) & 15) != 0) ldx = 1;  // unaligned x: force generic
    Plan pl = make_plan(w, B, ldx);
    if ((reinterpret_cast<uintptr_t>(X) & 15) != 0) pl.kind = Plan::kGeneric;
    if (pl.kind != Plan::kTeam && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && (B == 1 || ldx % 4 == 0) &&
        gemv_batch_supported(w, B, num_sms))
        return launch_gemv_batch(w, X, B, ldx, Y, ldy, err, num_sms, st);
    if (pl.kind != Plan::kGeneric) {
        const int epc = w.qtype == kQInt8 ? 16 : 32;
        GemvParams p{};
        p.W = w.data;
        p.S = w.scales;
        p.X = X;
        p.Y = Y;
        p.N = (int)w.N;
        p.K = (int)w.K;
        p.ldx = (int)ldx;
        p.ldy = (int)ldy;
        p.row_bytes = w.qtype == kQInt8 ? (int)w.K : (int)(w.K / 2);
        p.chunks = (int)(w.K / epc);
        p.team = pl.team;
        p.blocks_per_row = pl.smode == kScaleChunk ? (int)(w.K / w.block_size) : 1;
        p.chunks_per_block = pl.smode == kScaleChunk ? (int)(w.block_size / epc) : 1;
        if (pl.kind == Plan::kTeam) {
            if (w.qtype == kQInt8)
                return pl.smode == kScaleRow ? dispatch_team<kQInt8, kScaleRow>(pl, p, num_sms, st)
                                             : dispatch_team<kQInt8, kScaleChunk>(pl, p, num_sms, st);
            return pl.smode == kScaleRow ? dispatch_team<kQInt4, kScaleRow>(pl, p, num_sms, st)
                                         : dispatch_team<kQInt4, kScaleChunk>(pl, p, num_sms, st);
        }
    }
    const size_t threads = w.N * 32;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    if (w.qtype == kQInt8)
        gemv_generic_kernel<kQInt8><<<grid, 256, 0, st>>>(w.data, w.scales, w.block_size, X, ldx, Y, ldy, w.N, w.K, (int)B);
    else
        gemv_generic_kernel<kQInt4><<<grid, 256, 0, st>>>(w.data, w.scales, w.block_size, X, ldx, Y, ldy, w.N, w.K, (int)B);
    return cudaGetLastError();
}

}  // namespace pyxis
