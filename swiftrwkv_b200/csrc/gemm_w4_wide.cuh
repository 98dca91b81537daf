// Wide-batch variant of the decode GEMM (activation rows R > 8): the
// quantised weight is dequantised ONCE per CTA and K-step into fp16 fragments,
//   w = half(scale * q + bias)        (one fp16 FMA, as MLX's quantized matmul
//                                      dequantises into the activation type),
// and the tensor core accumulates over the whole K range in fp32.  This keeps
// the dequant cost per weight constant while one A fragment feeds every
// n-tile of the warp (BN/8 of them).
//
// CTA = 4 warps = 64 weight rows x BN activation rows; warp w owns rows
// 16w..16w+15 and all BN columns.  Per 64-column group (pipeline stage):
//   cp.async   codes (64 x 32 B) + activation tile (BN x 64 fp16)
//   permute    the activation tile into per-lane B fragments (the nibble-pair
//              k order of gemv_mma.cuh), one pass shared by the 4 warps
//   mma        4 k-steps x BN/8 n-tiles per warp.
// Dense fp16 weights (FMT 1) take the natural k order and skip the permute.
// Split-K and the shared-memory epilogue follow gemm_w4.cuh.
#pragma once

#include "gemm_w4.cuh"

namespace rwkv {

template <int FMT, int BN, int STAGES>
struct WideSmem {
    static constexpr int XROW = 64 + 8;
    static constexpr int WROW = FMT == 0 ? 8 : 64 + 8;
    static constexpr int W_BYTES = FMT == 0 ? GW_BM * 32 : GW_BM * WROW * 2;
    static constexpr int X_BYTES = BN * XROW * 2;
    static constexpr int STAGE = W_BYTES + X_BYTES;
    static constexpr int PIPE = STAGES * STAGE;
    static constexpr int BFRAG = FMT == 0 ? (BN / 8) * 32 * 32 : 0;  // [nt][lane][4 k-steps] uint2
    static constexpr int TILE = BN * (GW_BM + 8) * 4;
    static constexpr int MAIN = PIPE + BFRAG;
    static constexpr int TOTAL = MAIN > TILE ? MAIN : TILE;
};

template <int FMT, int BN, int STAGES>
__global__ void __launch_bounds__(GW_THREADS)
gemm_w4_wide_kernel(const GemmArgs args, int max_groups) {
    using SM = WideSmem<FMT, BN, STAGES>;
    constexpr int NT = BN / 8;
    extern __shared__ __align__(16) unsigned char smem[];
    uint2* bfr = reinterpret_cast<uint2*>(smem + SM::PIPE);
    __half2* sb_s = reinterpret_cast<__half2*>(smem + SM::TOTAL);  // [64][max_groups] (scale, bias)

    const GemvJob& jb = args.jobs.j[blockIdx.y];
    const int m0 = blockIdx.x * GW_BM;
    if (m0 >= jb.OUT) return;
    const int nblk = blockIdx.z / args.S, kz = blockIdx.z % args.S;
    const int n0 = nblk * BN;
    if (n0 >= args.R) return;
    const int NG = (jb.IN + 63) / 64;
    const int g0 = (int)((int64_t)NG * kz / args.S), g1 = (int)((int64_t)NG * (kz + 1) / args.S);
    const int ngr = g1 - g0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;

    auto stage_ptr = [&](int s) { return smem + s * SM::STAGE; };
    auto issue = [&](int gi, int s) {
        unsigned char* st = stage_ptr(s);
        const int G = g0 + gi;
        if (FMT == 0) {
            const int r = tid >> 1, half = tid & 1;
            const int o = min(m0 + r, jb.OUT - 1);
            const uint32_t* src = (const uint32_t*)jb.w + (int64_t)o * (jb.IN / 8) + 8 * G + 4 * half;
            cp_async16_cg(st + r * 32 + half * 16, src, true);
        } else {
            for (int e = tid; e < GW_BM * 8; e += GW_THREADS) {
                const int r = e >> 3, c = e & 7;
                const int o = min(m0 + r, jb.OUT - 1);
                const int col = 64 * G + 8 * c;
                const bool valid = col < jb.IN;
                const __half* src = (const __half*)jb.w + (int64_t)o * jb.IN + (valid ? col : 0);
                cp_async16_cg(st + (r * SM::WROW + 8 * c) * 2, src, valid);
            }
        }
        unsigned char* xs = st + SM::W_BYTES;
        for (int e = tid; e < BN * 8; e += GW_THREADS) {
            const int r = e >> 3, c = e & 7;
            const int n = n0 + r;
            const int col = 64 * G + 8 * c;
            const bool valid = n < args.R && col < jb.IN;
            const __half* src = (const __half*)jb.x + (valid ? (int64_t)n * jb.x_stride + col : 0);
            cp_async16_cg(xs + (r * SM::XROW + 8 * c) * 2, src, valid);
        }
    };

#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (s < ngr) issue(s, s);
        cp_commit();
    }
    // scales and biases of the CTA's rows and groups, while the first stages fly
    if (FMT == 0) {
        const int NGT = jb.IN / 64;
        for (int e = tid; e < GW_BM * ngr; e += GW_THREADS) {
            const int r = e / ngr, gg = e % ngr;
            const int o = min(m0 + r, jb.OUT - 1);
            sb_s[r * max_groups + gg] = __halves2half2(jb.scales[(int64_t)o * NGT + g0 + gg],
                                                       jb.biases[(int64_t)o * NGT + g0 + gg]);
        }
    }

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const int rl = warp * 16 + g;

    for (int gi = 0; gi < ngr; gi++) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        if (gi + STAGES - 1 < ngr) issue(gi + STAGES - 1, (gi + STAGES - 1) % STAGES);
        cp_commit();
        const unsigned char* st = stage_ptr(gi % STAGES);
        const __half* xs = reinterpret_cast<const __half*>(st + SM::W_BYTES);
        if (FMT == 0) {
            // activation tile -> B fragments in the nibble-pair k order
            for (int e = tid; e < NT * 32; e += GW_THREADS) {
                const int nt = e >> 5, ln = e & 31;
                const int gg = ln >> 2, tt = ln & 3;
                const __half* xr = xs + (nt * 8 + gg) * SM::XROW + 16 * tt;
                const uint4 lo = *reinterpret_cast<const uint4*>(xr);
                const uint4 hi = *reinterpret_cast<const uint4*>(xr + 8);
                const uint32_t h[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                uint2 out[4];
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint32_t sel = (kk & 1) ? 0x7632u : 0x5410u;
                    out[kk].x = __byte_perm(h[kk >> 1], h[(kk >> 1) + 2], sel);
                    out[kk].y = __byte_perm(h[(kk >> 1) + 4], h[(kk >> 1) + 6], sel);
                }
                uint4* dst = reinterpret_cast<uint4*>(bfr + (nt * 32 + ln) * 4);
                dst[0] = make_uint4(out[0].x, out[0].y, out[1].x, out[1].y);
                dst[1] = make_uint4(out[2].x, out[2].y, out[3].x, out[3].y);
            }
            __syncthreads();
        }
        uint32_t a[4][4];
        if (FMT == 0) {
            const uint32_t* ws0 = reinterpret_cast<const uint32_t*>(st) + rl * 8 + 2 * t;
            const uint2 A0 = *reinterpret_cast<const uint2*>(ws0);
            const uint2 A1 = *reinterpret_cast<const uint2*>(ws0 + 64);
            const __half2 sb0 = sb_s[rl * max_groups + gi], sb1 = sb_s[(rl + 8) * max_groups + gi];
            const __half2 s0 = __low2half2(sb0), c0 = __high2half2(sb0);
            const __half2 s1 = __low2half2(sb1), c1 = __high2half2(sb1);
            auto dq = [](uint32_t q2, __half2 s, __half2 c) {
                __half2 w = __hfma2(*reinterpret_cast<__half2*>(&q2), s, c);
                return *reinterpret_cast<uint32_t*>(&w);
            };
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                a[kk][0] = dq(nib_pair(A0.x, kk), s0, c0);
                a[kk][1] = dq(nib_pair(A1.x, kk), s1, c1);
                a[kk][2] = dq(nib_pair(A0.y, kk), s0, c0);
                a[kk][3] = dq(nib_pair(A1.y, kk), s1, c1);
            }
#pragma unroll
            for (int j = 0; j < NT; j++) {
                const uint4* src = reinterpret_cast<const uint4*>(bfr + (j * 32 + lane) * 4);
                const uint4 b01 = src[0], b23 = src[1];
                const uint32_t b[4][2] = {{b01.x, b01.y}, {b01.z, b01.w}, {b23.x, b23.y}, {b23.z, b23.w}};
#pragma unroll
                for (int kk = 0; kk < 4; kk++) mma16816(acc[j], a[kk], b[kk]);
            }
        } else {
            const __half* w0 = reinterpret_cast<const __half*>(st) + rl * SM::WROW + 2 * t;
            const __half* w1 = w0 + 8 * SM::WROW;
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                a[kk][0] = *reinterpret_cast<const uint32_t*>(w0 + 16 * kk);
                a[kk][1] = *reinterpret_cast<const uint32_t*>(w1 + 16 * kk);
                a[kk][2] = *reinterpret_cast<const uint32_t*>(w0 + 16 * kk + 8);
                a[kk][3] = *reinterpret_cast<const uint32_t*>(w1 + 16 * kk + 8);
            }
#pragma unroll
            for (int j = 0; j < NT; j++) {
                const __half* xr = xs + (j * 8 + g) * SM::XROW + 2 * t;
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint32_t b[2] = {*reinterpret_cast<const uint32_t*>(xr + 16 * kk),
                                           *reinterpret_cast<const uint32_t*>(xr + 16 * kk + 8)};
                    mma16816(acc[j], a[kk], b);
                }
            }
        }
    }
    cp_wait<0>();
    __syncthreads();

    constexpr int TS = GW_BM + 8;
    float* tile_s = reinterpret_cast<float*>(smem);
    auto to_tile = [&](float (&v)[NT][4]) {
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int ol = rl + ((e & 2) ? 8 : 0);
                const int nl = j * 8 + 2 * t + (e & 1);
                tile_s[nl * TS + ol] = v[j][e];
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
    constexpr int PER = NT * 4;
    float* part = args.ws + ((size_t)tile * args.S) * TILE;
    float4* mine = reinterpret_cast<float4*>(part + (size_t)kz * TILE + tid * PER);
#pragma unroll
    for (int j = 0; j < NT; j++) mine[j] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (tid == 0) last = (atomicAdd(&args.tickets[tile], 1) == args.S - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    float sum[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) sum[j][0] = sum[j][1] = sum[j][2] = sum[j][3] = 0.f;
    const float4* slot = reinterpret_cast<const float4*>(part + tid * PER);
    constexpr int TILE4 = TILE / 4;
    int z = 0;
    for (; z + 2 <= args.S; z += 2) {
        float4 v[2][NT];
#pragma unroll
        for (int u = 0; u < 2; u++)
#pragma unroll
            for (int q = 0; q < NT; q++) v[u][q] = __ldcg(slot + (size_t)(z + u) * TILE4 + q);
#pragma unroll
        for (int u = 0; u < 2; u++)
#pragma unroll
            for (int q = 0; q < NT; q++) {
                sum[q][0] += v[u][q].x; sum[q][1] += v[u][q].y; sum[q][2] += v[u][q].z; sum[q][3] += v[u][q].w;
            }
    }
    for (; z < args.S; z++) {
#pragma unroll
        for (int q = 0; q < NT; q++) {
            const float4 v = __ldcg(slot + (size_t)z * TILE4 + q);
            sum[q][0] += v.x; sum[q][1] += v.y; sum[q][2] += v.z; sum[q][3] += v.w;
        }
    }
    to_tile(sum);
    tile_out();
    if (tid == 0) args.tickets[tile] = 0;
}

template <int FMT, int BN, int STAGES>
inline cudaError_t launch_wide_t(const GemmArgs& a, const GemmPlan& p, cudaStream_t st) {
    using SM = WideSmem<FMT, BN, STAGES>;
    int maxg = 0;
    for (int i = 0; i < a.njobs; i++) maxg = std::max(maxg, (a.jobs.j[i].IN + 63) / 64);
    const int max_groups = (maxg + a.S - 1) / a.S + 1;
    const size_t smem = SM::TOTAL + (FMT == 0 ? (size_t)GW_BM * max_groups * 4 : 0);
    auto kern = gemm_w4_wide_kernel<FMT, BN, STAGES>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid(p.mblocks, a.njobs, p.nnb * a.S);
    kern<<<grid, GW_THREADS, smem, st>>>(a, max_groups);
    return cudaGetLastError();
}

// R > 8: BN = 16 .. 128.  Split-K only to reach about one wave.
inline GemmPlan plan_wide(const GemvJobs& jobs, int njobs, int R, int sm_count) {
    GemmPlan p{};
    p.BN = R <= 16 ? 16 : R <= 32 ? 32 : R <= 64 ? 64 : 128;
    p.MW = 4;
    p.nnb = (R + p.BN - 1) / p.BN;
    int maxo = 0, maxg = 0;
    for (int i = 0; i < njobs; i++) {
        maxo = std::max(maxo, jobs.j[i].OUT);
        maxg = std::max(maxg, (jobs.j[i].IN + 63) / 64);
    }
    p.mblocks = (maxo + GW_BM - 1) / GW_BM;
    const int ctas = p.mblocks * njobs * p.nnb;
    int S = (sm_count + ctas - 1) / ctas;
    S = std::max(1, std::min(S, maxg / 4));  // at least four groups per split
    p.S = S;
    p.ws_floats = S > 1 ? (size_t)p.mblocks * njobs * p.nnb * S * GW_BM * p.BN : 0;
    p.tickets = S > 1 ? (size_t)p.mblocks * njobs * p.nnb : 0;
    return p;
}

template <int FMT>
inline cudaError_t launch_wide(GemmArgs& a, const GemmPlan& p, cudaStream_t st) {
    a.S = p.S;
    switch (p.BN) {
        case 16: return launch_wide_t<FMT, 16, 4>(a, p, st);
        case 32: return launch_wide_t<FMT, 32, 4>(a, p, st);
        case 64: return launch_wide_t<FMT, 64, 3>(a, p, st);
        default: return launch_wide_t<FMT, 128, 3>(a, p, st);
    }
}

// Dispatcher used by the runtime and rwkv_q_gemm: exact per-group scaling for
// R <= 8 (gemm_w4_kernel), fp16 dequant + K accumulation above.
inline GemmPlan plan_any(const GemvJobs& jobs, int njobs, int R, int sm_count) {
    return R <= 8 ? plan_gemm(jobs, njobs, R, sm_count) : plan_wide(jobs, njobs, R, sm_count);
}

template <int FMT>
inline cudaError_t launch_any(GemmArgs& a, const GemmPlan& p, cudaStream_t st, bool pdl = false) {
    // (the R <= 8 kernel supports programmatic launch; the wide kernel is launched plainly)
    return a.R <= 8 ? launch_gemm<FMT>(a, p, st, pdl) : launch_wide<FMT>(a, p, st);
}

}  // namespace rwkv
