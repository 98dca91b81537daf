// Pipelined skinny GEMM  y[n, o] = act( sum_k x[n, k] W[o, k] )  for the
// decode projections, on the tensor cores (mma.sync.m16n8k16, fp16 x fp16 ->
// fp32), with weights either in the MLX affine 4-bit group-64 container
// (FMT 0) or dense fp16 (FMT 1).
//
// CTA = 4 warps = 64 weight rows x BN activation rows.  K advances one
// 64-column group per pipeline stage; the weight tile (64 rows x 32 bytes of
// codes, or 64 x 128 bytes of fp16) and the activation tile (BN rows x 64
// fp16) of each stage are copied global -> shared with cp.async, STAGES-1
// groups ahead of the arithmetic.  Scales and biases of the CTA's rows and
// K range are staged once into shared memory.  Warps tile the CTA as
// MW x (4/MW): each warp owns (4/MW) m-tiles of 16 rows and the matching
// n-tiles of 8 activation rows, so B fragments (and the activation group sums
// needed for the bias term) are shared across its m-tiles.
//
// 4-bit codes follow the k permutation of gemv_mma.cuh (nibble pairs (j, j+4)
// of words 2t / 2t+1 at k-step j), so one LOP3 + HSUB2 yields two exact codes.
//
// Split-K: gridDim.z = n-blocks x S.  With S > 1 each CTA writes its fp32
// partial tile to a workspace and the last CTA of a tile (atomic ticket)
// sums the S partials in split order -- deterministic -- and runs the
// epilogue, then re-arms the ticket for the next launch / graph replay.
#pragma once

#include "gemv_mma.cuh"

namespace rwkv {

constexpr int GW_THREADS = 128;
constexpr int GW_BM = 64;

struct GemmArgs {
    GemvJobs jobs;
    int njobs;
    int R;          // activation rows
    int S;          // K splits
    float* ws;      // split-K partials
    int* tickets;   // one per (job, m-block, n-block); zero between launches
};

__device__ __forceinline__ void cp_async16_cg(void* smem, const void* gmem, bool valid) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// One pipeline stage holds GPS consecutive 64-column groups, so every weight
// row is fetched in GPS*32-byte (4-bit) or GPS*128-byte (fp16) runs: with
// GPS = 4 a 4-bit row contributes one full 128-byte line per stage.
template <int FMT, int BN, int STAGES, int GPS>
struct GemmSmem {
    static constexpr int XROW = 64 * GPS + 8;                 // fp16 per activation row (+16 B pad)
    // u32 words (4-bit) or fp16 (dense) per weight row, padded by 32 bytes so
    // the per-lane fragment loads of 8 consecutive rows hit distinct banks
    static constexpr int WROW = FMT == 0 ? 8 * GPS + 8 : 64 * GPS + 8;
    static constexpr int W_BYTES = FMT == 0 ? GW_BM * WROW * 4 : GW_BM * WROW * 2;
    static constexpr int X_BYTES = BN * XROW * 2;
    static constexpr int STAGE = W_BYTES + X_BYTES;
    static constexpr int PIPE = STAGES * STAGE;
};

template <int FMT, int BN, int MW, int STAGES, int GPS>
__global__ void __launch_bounds__(GW_THREADS)
gemm_w4_kernel(const GemmArgs args, int max_groups) {
    using SM = GemmSmem<FMT, BN, STAGES, GPS>;
    constexpr int NW = 4 / MW;           // warps along N
    constexpr int WMT = 4 / MW;          // m-tiles per warp
    constexpr int WNT = BN / 8 / NW;     // n-tiles per warp
    static_assert(WNT >= 1, "BN too small for the warp layout");
    extern __shared__ __align__(16) unsigned char smem[];
    __half* sc_s = reinterpret_cast<__half*>(smem + SM::PIPE);   // [64][max_groups]
    __half* bi_s = sc_s + GW_BM * max_groups;

    const GemvJob& jb = args.jobs.j[blockIdx.y];
    const int m0 = blockIdx.x * GW_BM;
    if (m0 >= jb.OUT) return;
    const int nblk = blockIdx.z / args.S, kz = blockIdx.z % args.S;
    const int n0 = nblk * BN;
    if (n0 >= args.R) return;
    const int NG = (jb.IN + 63) / 64;   // K groups (the last may be partial for FMT 1)
    const int g0 = (int)((int64_t)NG * kz / args.S), g1 = (int)((int64_t)NG * (kz + 1) / args.S);
    const int ngr = g1 - g0;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int wm = warp % MW, wn = warp / MW;

    const int nst = (ngr + GPS - 1) / GPS;  // stages of this CTA
    auto stage_ptr = [&](int s) { return smem + s * SM::STAGE; };
    // weights and activations of groups g0 + GPS*si .. into stage s; the
    // weights do not depend on the previous kernel, the activations do
    auto issue_w = [&](int si, int s) {
        unsigned char* st = stage_ptr(s);
        const int G0 = g0 + GPS * si;
        if (FMT == 0) {
            // 64 rows x GPS*32 bytes
            for (int e = tid; e < GW_BM * 2 * GPS; e += GW_THREADS) {
                const int r = e / (2 * GPS), c = e % (2 * GPS);
                const int o = min(m0 + r, jb.OUT - 1);
                const bool valid = G0 + c / 2 < g1;
                const uint32_t* src = (const uint32_t*)jb.w + (int64_t)o * (jb.IN / 8) + (valid ? 8 * G0 + 4 * c : 0);
                cp_async16_cg(st + r * SM::WROW * 4 + c * 16, src, valid);
            }
        } else {
            for (int e = tid; e < GW_BM * 8 * GPS; e += GW_THREADS) {
                const int r = e / (8 * GPS), c = e % (8 * GPS);
                const int o = min(m0 + r, jb.OUT - 1);
                const int col = 64 * G0 + 8 * c;
                const bool valid = col < jb.IN && G0 + c / 8 < g1;
                const __half* src = (const __half*)jb.w + (int64_t)o * jb.IN + (valid ? col : 0);
                cp_async16_cg(st + (r * SM::WROW + 8 * c) * 2, src, valid);
            }
        }
    };
    auto issue_x = [&](int si, int s) {
        const int G0 = g0 + GPS * si;
        unsigned char* xs = stage_ptr(s) + SM::W_BYTES;
        for (int e = tid; e < BN * 8 * GPS; e += GW_THREADS) {
            const int r = e / (8 * GPS), c = e % (8 * GPS);
            const int n = n0 + r;
            const int col = 64 * G0 + 8 * c;
            const bool valid = n < args.R && col < jb.IN && G0 + c / 8 < g1;
            const __half* src = (const __half*)jb.x + (valid ? (int64_t)n * jb.x_stride + col : 0);
            cp_async16_cg(xs + (r * SM::XROW + 8 * c) * 2, src, valid);
        }
    };

    float acc[WMT][WNT][4];
#pragma unroll
    for (int i = 0; i < WMT; i++)
#pragma unroll
        for (int j = 0; j < WNT; j++) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;

    // first stages' weights, then (under programmatic launch) wait for the
    // previous kernel before its activations: cp.async group s still holds
    // stage s's activations, so the per-stage waits below are unchanged
    if (tid == 0) pdl_trigger();
#pragma unroll
    for (int s = 0; s < STAGES - 1; s++)
        if (s < nst) issue_w(s, s);
    // scales / biases of this CTA's rows and groups -> shared, while the
    // first stages are in flight
    if (FMT == 0) {
        const int NGT = jb.IN / 64;
        for (int e = tid; e < GW_BM * ngr; e += GW_THREADS) {
            const int r = e / ngr, gg = e % ngr;
            const int o = min(m0 + r, jb.OUT - 1);
            sc_s[r * max_groups + gg] = jb.scales[(int64_t)o * NGT + g0 + gg];
            bi_s[r * max_groups + gg] = jb.biases[(int64_t)o * NGT + g0 + gg];
        }
    }
    pdl_wait();
#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (s < nst) issue_x(s, s);
        cp_commit();
    }


    for (int si = 0; si < nst; si++) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        if (si + STAGES - 1 < nst) {
            issue_w(si + STAGES - 1, (si + STAGES - 1) % STAGES);
            issue_x(si + STAGES - 1, (si + STAGES - 1) % STAGES);
        }
        cp_commit();
        const unsigned char* st = stage_ptr(si % STAGES);
#pragma unroll
      for (int q = 0; q < GPS; q++) {
        const int gi = si * GPS + q;
        if (gi >= ngr) break;
        const __half* xs = reinterpret_cast<const __half*>(st + SM::W_BYTES) + 64 * q;

        // B fragments and group sums of this warp's n-tiles
        uint32_t b[WNT][4][2];
        float X0[WNT], X1[WNT];
#pragma unroll
        for (int j = 0; j < WNT; j++) {
            const int nr = (wn * WNT + j) * 8 + g;  // activation row within the tile
            const __half* xr = xs + nr * SM::XROW;
            if (FMT == 0) {
                const uint4 lo = *reinterpret_cast<const uint4*>(xr + 16 * t);
                const uint4 hi = *reinterpret_cast<const uint4*>(xr + 16 * t + 8);
                const uint32_t h[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint32_t sel = (kk & 1) ? 0x7632u : 0x5410u;
                    b[j][kk][0] = __byte_perm(h[kk >> 1], h[(kk >> 1) + 2], sel);
                    b[j][kk][1] = __byte_perm(h[(kk >> 1) + 4], h[(kk >> 1) + 6], sel);
                }
                float s = 0.f;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
                    s += f.x + f.y;
                }
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                X0[j] = __shfl_sync(0xffffffffu, s, 8 * t);
                X1[j] = __shfl_sync(0xffffffffu, s, 8 * t + 4);
            } else {
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    b[j][kk][0] = *reinterpret_cast<const uint32_t*>(xr + 16 * kk + 2 * t);
                    b[j][kk][1] = *reinterpret_cast<const uint32_t*>(xr + 16 * kk + 2 * t + 8);
                }
                X0[j] = X1[j] = 0.f;
            }
        }
#pragma unroll
        for (int i = 0; i < WMT; i++) {
            const int rl = (wm * WMT + i) * 16 + g;  // weight row within the tile
            uint32_t a[4][4];
            if (FMT == 0) {
                const uint32_t* ws0 = reinterpret_cast<const uint32_t*>(st) + rl * SM::WROW + 8 * q + 2 * t;
                const uint32_t* ws1 = ws0 + 8 * SM::WROW;
                const uint2 A0 = *reinterpret_cast<const uint2*>(ws0);
                const uint2 A1 = *reinterpret_cast<const uint2*>(ws1);
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    a[kk][0] = nib_pair(A0.x, kk);
                    a[kk][1] = nib_pair(A1.x, kk);
                    a[kk][2] = nib_pair(A0.y, kk);
                    a[kk][3] = nib_pair(A1.y, kk);
                }
            } else {
                const __half* w0 = reinterpret_cast<const __half*>(st) + rl * SM::WROW + 64 * q + 2 * t;
                const __half* w1 = w0 + 8 * SM::WROW;
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    a[kk][0] = *reinterpret_cast<const uint32_t*>(w0 + 16 * kk);
                    a[kk][1] = *reinterpret_cast<const uint32_t*>(w1 + 16 * kk);
                    a[kk][2] = *reinterpret_cast<const uint32_t*>(w0 + 16 * kk + 8);
                    a[kk][3] = *reinterpret_cast<const uint32_t*>(w1 + 16 * kk + 8);
                }
            }
            if (FMT == 0) {
                const float s0 = __half2float(sc_s[rl * max_groups + gi]);
                const float s1 = __half2float(sc_s[(rl + 8) * max_groups + gi]);
                const float c0 = __half2float(bi_s[rl * max_groups + gi]);
                const float c1 = __half2float(bi_s[(rl + 8) * max_groups + gi]);
#pragma unroll
                for (int j = 0; j < WNT; j++) {
                    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) mma16816(d, a[kk], b[j][kk]);
                    acc[i][j][0] = fmaf(s0, d[0], fmaf(c0, X0[j], acc[i][j][0]));
                    acc[i][j][1] = fmaf(s0, d[1], fmaf(c0, X1[j], acc[i][j][1]));
                    acc[i][j][2] = fmaf(s1, d[2], fmaf(c1, X0[j], acc[i][j][2]));
                    acc[i][j][3] = fmaf(s1, d[3], fmaf(c1, X1[j], acc[i][j][3]));
                }
            } else {
#pragma unroll
                for (int j = 0; j < WNT; j++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) mma16816(acc[i][j], a[kk], b[j][kk]);
            }
        }
      }
    }
    cp_wait<0>();
    __syncthreads();  // the pipeline buffers are free: they hold the output tile now

    // ---- epilogue through a shared [BN][64 + 8] fp32 tile, one compact loop
    constexpr int TS = GW_BM + 8;
    float* tile_s = reinterpret_cast<float*>(smem);
    auto to_tile = [&](float (&v)[WMT][WNT][4]) {
#pragma unroll
        for (int i = 0; i < WMT; i++)
#pragma unroll
            for (int j = 0; j < WNT; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int ol = (wm * WMT + i) * 16 + g + ((e & 2) ? 8 : 0);
                    const int nl = (wn * WNT + j) * 8 + 2 * t + (e & 1);
                    tile_s[nl * TS + ol] = v[i][j][e];
                }
    };
    auto tile_out = [&]() {
        __syncthreads();
        const int nr = min(BN, args.R - n0), orr = min(GW_BM, jb.OUT - m0);
        for (int e = tid; e < BN * GW_BM; e += GW_THREADS) {
            const int nl = e / GW_BM, ol = e % GW_BM;
            if (nl < nr && ol < orr) epilogue(jb, m0 + ol, n0 + nl, tile_s[nl * TS + ol]);
        }
    };
    if (args.S == 1) {
        to_tile(acc);
        tile_out();
        return;
    }
    const int nnb = (args.R + BN - 1) / BN;
    const int tile = (blockIdx.y * gridDim.x + blockIdx.x) * nnb + nblk;
    constexpr int TILE = GW_BM * BN;
    constexpr int PER = WMT * WNT * 4;  // fragment floats per thread (multiple of 4)
    float* part = args.ws + ((size_t)tile * args.S) * TILE;
    // each thread stores its fragments contiguously at a fixed per-thread slot
    float4* mine = reinterpret_cast<float4*>(part + (size_t)kz * TILE + tid * PER);
#pragma unroll
    for (int i = 0; i < WMT; i++)
#pragma unroll
        for (int j = 0; j < WNT; j++)
            mine[i * WNT + j] = make_float4(acc[i][j][0], acc[i][j][1], acc[i][j][2], acc[i][j][3]);
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (tid == 0) last = (atomicAdd(&args.tickets[tile], 1) == args.S - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    // sum the S partials in split order; loads of several splits in flight
    float sum[WMT][WNT][4];
#pragma unroll
    for (int i = 0; i < WMT; i++)
#pragma unroll
        for (int j = 0; j < WNT; j++) sum[i][j][0] = sum[i][j][1] = sum[i][j][2] = sum[i][j][3] = 0.f;
    const float4* slot = reinterpret_cast<const float4*>(part + tid * PER);
    constexpr int TILE4 = TILE / 4;
    int z = 0;
    for (; z + 4 <= args.S; z += 4) {
        float4 v[4][WMT * WNT];
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int q = 0; q < WMT * WNT; q++) v[u][q] = __ldcg(slot + (size_t)(z + u) * TILE4 + q);
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int q = 0; q < WMT * WNT; q++) {
                float* sq = sum[q / WNT][q % WNT];
                sq[0] += v[u][q].x; sq[1] += v[u][q].y; sq[2] += v[u][q].z; sq[3] += v[u][q].w;
            }
    }
    for (; z < args.S; z++) {
#pragma unroll
        for (int q = 0; q < WMT * WNT; q++) {
            const float4 v = __ldcg(slot + (size_t)z * TILE4 + q);
            float* sq = sum[q / WNT][q % WNT];
            sq[0] += v.x; sq[1] += v.y; sq[2] += v.z; sq[3] += v.w;
        }
    }
    to_tile(sum);
    tile_out();
    if (tid == 0) args.tickets[tile] = 0;
}

// Split-K workspace needs for a launch (floats / tickets).
struct GemmPlan {
    int BN, MW, S, nnb, mblocks;
    size_t ws_floats, tickets;
};

inline GemmPlan plan_gemm(const GemvJobs& jobs, int njobs, int R, int sm_count) {
    GemmPlan p{};
    p.BN = R <= 8 ? 8 : R <= 16 ? 16 : R <= 32 ? 32 : 64;
    p.MW = p.BN <= 16 ? 4 : p.BN == 32 ? 2 : 1;
    p.nnb = (R + p.BN - 1) / p.BN;
    int maxo = 0, maxg = 0;
    for (int i = 0; i < njobs; i++) {
        maxo = std::max(maxo, jobs.j[i].OUT);
        maxg = std::max(maxg, (jobs.j[i].IN + 63) / 64);
    }
    p.mblocks = (maxo + GW_BM - 1) / GW_BM;
    const int ctas = p.mblocks * njobs * p.nnb;
    const int target = 2 * sm_count;
    int S = (target + ctas - 1) / ctas;
    S = std::max(1, std::min(S, maxg / 8));  // at least eight groups (two 4-group stages) per split
    p.S = S;
    p.ws_floats = S > 1 ? (size_t)p.mblocks * njobs * p.nnb * S * GW_BM * p.BN : 0;
    p.tickets = S > 1 ? (size_t)p.mblocks * njobs * p.nnb : 0;
    return p;
}

template <int FMT, int BN, int MW, int STAGES, int GPS>
inline cudaError_t launch_gemm_t(const GemmArgs& a, const GemmPlan& p, cudaStream_t st, bool pdl) {
    int maxg = 0;
    for (int i = 0; i < a.njobs; i++) maxg = std::max(maxg, (a.jobs.j[i].IN + 63) / 64);
    const int max_groups = (maxg + a.S - 1) / a.S + 1;
    const size_t smem = GemmSmem<FMT, BN, STAGES, GPS>::PIPE + (FMT == 0 ? 2 * GW_BM * max_groups * 2 : 0);
    auto kern = gemm_w4_kernel<FMT, BN, MW, STAGES, GPS>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid(p.mblocks, a.njobs, p.nnb * a.S);
    if (pdl) return launch_pdl(kern, grid, dim3(GW_THREADS), smem, st, a, max_groups);
    kern<<<grid, GW_THREADS, smem, st>>>(a, max_groups);
    return cudaGetLastError();
}

template <int FMT>
// pdl: launch as a programmatic dependent of the previous kernel in the stream
inline cudaError_t launch_gemm(GemmArgs& a, const GemmPlan& p, cudaStream_t st, bool pdl = false) {
    a.S = p.S;
    switch (p.BN) {
        case 8: return launch_gemm_t<FMT, 8, 4, 3, FMT == 0 ? 4 : 1>(a, p, st, pdl);
        case 16: return launch_gemm_t<FMT, 16, 4, 3, FMT == 0 ? 4 : 1>(a, p, st, pdl);
        case 32: return launch_gemm_t<FMT, 32, 2, 4, FMT == 0 ? 2 : 1>(a, p, st, pdl);
        default: return launch_gemm_t<FMT, 64, 1, 3, FMT == 0 ? 2 : 1>(a, p, st, pdl);
    }
}

}  // namespace rwkv
