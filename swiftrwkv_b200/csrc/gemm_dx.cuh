// Projection backward through a frozen base on the tcgen05 tensor cores:
//
//     dX[n, i] = bf16( sum_o bf16(dY[n, o]) * Wb[o, i] )        (fp32 accumulation)
//
// with Wb the base weight [OUT, IN] in bf16: a dense bf16 matrix (DX_BF16), or
// the MLX affine 4-bit group-64 container dequantised on the fly (DX_Q4,
// Wb = bf16(q * scale + bias), one rounding).  This is the VJP X070Backbone
// gives its frozen base projections (baseMatmul, X070Backbone.swift:337-356:
// matmul(cotangent.asType(bf16), weight(bf16)), a bf16 result, then cast to
// the primal's type).
//
// Tile = 128 IN columns (the MMA's M: A = Wb^T, read MN-major straight from
// the [OUT, IN] rows) x BN token rows (N: B = dY, K-major), K = OUT in stages
// of 64.  A persistent CTA per SM walks the tiles; the accumulator of tile t
// lives in TMEM half (t & 1), so the epilogue of one tile overlaps the MMAs
// of the next.
//   warp 0       TMA producer: per stage the A tile (DX_BF16: two 64x64 bf16
//                boxes, 128-byte swizzle, IN-major rows; DX_Q4: a 64-row box of
//                packed codes) and one BN x 64 dY box (128-byte swizzle)
//   warp 1       TMEM owner; one thread issues 4 tcgen05.mma (M=128, N=BN,
//                K=16, A MN-major) per stage and commits the stage / tile
//   warps 2-5    epilogue: TMEM lane quadrant (warp & 3) = 32 IN columns;
//                tcgen05.ld 32 token columns at a time, stores coalesced
//                along IN (128 bytes per warp and token)
//   warps 6-13   DX_Q4 only: each thread turns 4 code words per stage into
//                bf16 chunks of the swizzled MN-major A tile (scales and
//                biases for the next stage prefetched into registers), then
//                fences the stores into the async proxy
// Every mbarrier wait is bounded (tc::mbar_wait); a wait that gives up sets
// the shared error flag, every role winds down, the producer waits (bounded)
// for its copies in flight and TMEM is freed after the final MMA commit.
#pragma once

#include "gemm_tc.cuh"

namespace rwkv {

constexpr int DX_BM = 128;  // IN columns per tile
constexpr int DX_BK = 64;   // OUT rows per stage

template <int FMT, int BN>
struct DxCfg {
    static constexpr int A_HALF = DX_BK * 128;                 // 64 K-rows x 64 IN columns of bf16
    static constexpr int A_BYTES = 2 * A_HALF;
    static constexpr int B_BYTES = BN * 128;                   // BN rows x 64 bf16
    static constexpr int C_BYTES = FMT == DX_Q4 ? DX_BK * 64 : 0;  // 64 rows x 16 code words
    static constexpr int STAGE = A_BYTES + B_BYTES + C_BYTES;
    static constexpr int ST = (220 * 1024 / STAGE) < 8 ? (220 * 1024 / STAGE) : 8;
    static constexpr int TX = (FMT == DX_Q4 ? C_BYTES : A_BYTES) + B_BYTES;  // TMA bytes per stage
    static constexpr int DQT = FMT == DX_Q4 ? 256 : 0;         // dequant threads
    static constexpr int THREADS = 64 + 128 + DQT;
    static constexpr int TMC = 2 * BN;                         // two accumulators
    static constexpr int NBAR = 3 * ST + 5;
    static constexpr int B_OFF = ST * STAGE;
    static constexpr int T_OFF = B_OFF + NBAR * 8;
    static constexpr int TOTAL = T_OFF + 16 + 1024;
    static_assert(STAGE % 1024 == 0, "stage bases stay 1024-byte aligned");
    static_assert(ST >= 2, "pipeline depth");
    static_assert(TOTAL <= 227 * 1024, "shared memory per CTA");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "M=128 MMA: N % 16 == 0, <= 256; epilogue in 32s");
    static_assert(TMC == 64 || TMC == 128 || TMC == 256 || TMC == 512, "TMEM allocation is a power of two");
    static_assert(FMT != DX_Q4 || 4 * DQT == DX_BK * 16, "4 code words per dequant thread and stage");
};

struct DxArgs {
    CUtensorMap amap;  // DX_BF16: Wb {IN, OUT} bf16, box {64, 64}, 128-byte swizzle;
                       // DX_Q4: codes {IN/8, OUT} u32, box {16, 64}, no swizzle
    CUtensorMap bmap;  // dY {OUT, rows} bf16, box {64, BN}, 128-byte swizzle
    const __half* scales;  // DX_Q4: [OUT, IN/64]
    const __half* biases;
    void* dx;              // [rows, IN]
    int dx_dtype;          // RWKV_F32 / RWKV_BF16 / RWKV_F16
    int accumulate;        // RWKV_F32 only: dX += result
    int rows, OUT, IN;
    int* err;              // device flag: a wait gave up
    int* err_host;         // mapped host record
};

namespace tc {
// Shared-memory operand descriptor, MN-major with 128-byte swizzle: 64
// MN-elements (128 B) per row, 8-row K groups 1024 B apart (SBO), the second
// 64-element MN half 8192 B on (LBO), descriptor version 1.
__device__ __forceinline__ uint64_t mn_sw128_desc(uint32_t smem_addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
// kind::f16 instruction descriptor: D f32, A and B bf16, A MN-major, B K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_amn(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// Two fp32 values rounded to bf16 (round to nearest even), packed low / high.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}
}  // namespace tc

template <int FMT, int BN>
__global__ void __launch_bounds__(DxCfg<FMT, BN>::THREADS, 1)
gemm_dx_kernel(const __grid_constant__ DxArgs a) {
    using C = DxCfg<FMT, BN>;
    constexpr int ST = C::ST;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::B_OFF);
    uint64_t* dqf = full + ST;      // DX_Q4: the stage's A tile is dequantised
    uint64_t* empty = dqf + ST;     // the stage's MMAs are done
    uint64_t* accf = empty + ST;    // [2] the tile's accumulator is complete
    uint64_t* acce = accf + 2;      // [2] the epilogue has drained it
    uint64_t* done = acce + 2;      // every MMA is done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::T_OFF);
    int* skip_slot = reinterpret_cast<int*>(smem + C::T_OFF + 8);

    const int nib = a.IN / DX_BM, ntb = (a.rows + BN - 1) / BN;
    const int ntiles = nib * ntb, nk = a.OUT / DX_BK;
    const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int* err = a.err;

    if (tid == 0) {
        for (int s = 0; s < ST; s++) {
            tc::mbar_init(full + s, 1);
            tc::mbar_init(dqf + s, C::DQT > 0 ? C::DQT : 1);
            tc::mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(accf + b, 1);
            tc::mbar_init(acce + b, 128);
        }
        tc::mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // an earlier wait gave up and nobody cleared the flag: skip the work
        *skip_slot = *(volatile int*)err;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(tc::saddr(tmem_slot)), "r"(C::TMC));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc::tc_before();
    __syncthreads();
    tc::tc_after();
    const uint32_t tmem = *tmem_slot;
    const bool skip = *skip_slot != 0;
    bool ok = !skip;
    const int nstages = skip ? 0 : my_tiles * nk;  // stages this CTA runs, tile-major

    auto tile_of = [&](int it, int& m0, int& n0) {
        const int t = (int)blockIdx.x + it * (int)gridDim.x;
        m0 = (t % nib) * DX_BM;
        n0 = (t / nib) * BN;
    };

    if (warp == 0) {
        if (lane == 0 && nstages > 0) {  // ---- TMA producer
            int issued = 0;
            for (int g = 0; g < nstages; g++) {
                const int s = g % ST, ks = g % nk;
                int m0, n0;
                tile_of(g / nk, m0, n0);
                if (g >= ST && !tc::mbar_wait(empty + s, ((g / ST) - 1) & 1, err)) {
                    ok = false;
                    break;
                }
                unsigned char* st = smem + s * C::STAGE;
                tc::mbar_expect_tx(full + s, C::TX);
                if constexpr (FMT == DX_Q4) {
                    tc::tma_2d(st + C::A_BYTES + C::B_BYTES, &a.amap, full + s, m0 / 8, ks * DX_BK);
                } else {
                    tc::tma_2d(st, &a.amap, full + s, m0, ks * DX_BK);
                    tc::tma_2d(st + C::A_HALF, &a.amap, full + s, m0 + 64, ks * DX_BK);
                }
                tc::tma_2d(st + C::A_BYTES, &a.bmap, full + s, ks * DX_BK, n0);
                issued = g + 1;
            }
            // the copies issued here land before the CTA may exit
            for (int g = max(0, issued - ST); g < issued; g++)
                if (!tc::mbar_wait_own(full + (g % ST), (g / ST) & 1, err)) ok = false;
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            constexpr uint32_t IDESC = tc::idesc_bf16_amn(DX_BM, BN);
            int g = 0;
            for (int it = 0; it < (skip ? 0 : my_tiles) && ok; it++) {
                const int b = it & 1;
                if (it >= 2 && !tc::mbar_wait(acce + b, ((it >> 1) - 1) & 1, err)) {
                    ok = false;
                    break;
                }
                tc::tc_after();
                const uint32_t d = tmem + b * BN;
                for (int ks = 0; ks < nk; ks++, g++) {
                    const int s = g % ST;
                    if (!tc::mbar_wait(full + s, (g / ST) & 1, err) ||
                        (FMT == DX_Q4 && !tc::mbar_wait(dqf + s, (g / ST) & 1, err))) {
                        ok = false;
                        break;
                    }
                    tc::tc_after();
                    const uint32_t sa = tc::saddr(smem + s * C::STAGE);
                    const uint64_t bd = tc::sw128_desc(sa + C::A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        tc::umma_ss(d, tc::mn_sw128_desc(sa + kk * 2048, C::A_HALF), bd + 2 * kk, IDESC,
                                    (ks | kk) ? 1u : 0u);
                    tc::umma_commit(empty + s);
                }
                if (!ok) break;
                tc::umma_commit(accf + b);
            }
            tc::umma_commit(done);  // also after an early exit: TMEM is freed after the MMAs
            if (!tc::mbar_wait_own(done, 0, err)) ok = false;
        }
    } else if (warp < 6) {
        // ---- epilogue: IN columns m0 + 32q + lane, token rows n0 + j
        const int q = warp & 3;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        for (int it = 0; it < (skip ? 0 : my_tiles); it++) {
            const int b = it & 1;
            if (!tc::mbar_wait(accf + b, (it >> 1) & 1, err)) {
                ok = false;
                break;
            }
            tc::tc_after();
            int m0, n0;
            tile_of(it, m0, n0);
            const int col = m0 + 32 * q + lane;
            for (int j0 = 0; j0 < BN && n0 + j0 < a.rows; j0 += 32) {
                uint32_t r[32];
                tc::tmem_ld32_async(tmem + lane_base + b * BN + j0, r);
                tc::tmem_ld_wait();
                const int nj = min(32, a.rows - n0 - j0);
                const int64_t base = (int64_t)(n0 + j0) * a.IN + col;
                // the sum rounded to bf16 (the reference's matmul result), then stored in dx_dtype
                if (a.dx_dtype == RWKV_F32) {
                    float* o = (float*)a.dx + base;
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        if (i >= nj) break;
                        const float v = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[i])));
                        if (a.accumulate) o[(int64_t)i * a.IN] += v;
                        else o[(int64_t)i * a.IN] = v;
                    }
                } else if (a.dx_dtype == RWKV_BF16) {
                    __nv_bfloat16* o = (__nv_bfloat16*)a.dx + base;
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        if (i >= nj) break;
                        o[(int64_t)i * a.IN] = __float2bfloat16_rn(__uint_as_float(r[i]));
                    }
                } else {
                    __half* o = (__half*)a.dx + base;
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        if (i >= nj) break;
                        o[(int64_t)i * a.IN] =
                            __float2half_rn(__bfloat162float(__float2bfloat16_rn(__uint_as_float(r[i]))));
                    }
                }
            }
            tc::tc_before();
            tc::mbar_arrive(acce + b);
        }
    } else if constexpr (FMT == DX_Q4) {
        // ---- dequant: thread d handles code word wi = d % 16 of rows
        // r = d / 16 + 16 j (j < 4) of each stage; group (m0 / 64) + wi / 8
        const int d = tid - 192;
        const int wi = d & 15, r0 = d >> 4;
        const int NG = a.IN / 64;
        const uint32_t cchunk = (uint32_t)(wi & 7), chalf = (uint32_t)(wi >> 3);
        __half sc[4], bi[4];
        auto fetch = [&](int g) {
            if (g >= nstages) return;
            int m0, n0;
            tile_of(g / nk, m0, n0);
            const int64_t grp = m0 / 64 + (wi >> 3);
            const int k0 = (g % nk) * DX_BK;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int64_t o = (int64_t)(k0 + r0 + 16 * j) * NG + grp;
                sc[j] = a.scales[o];
                bi[j] = a.biases[o];
            }
        };
        fetch(0);
        for (int g = 0; g < nstages; g++) {
            const int s = g % ST;
            float s4[4], b4[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                s4[j] = __half2float(sc[j]);
                b4[j] = __half2float(bi[j]);
            }
            fetch(g + 1);
            if (!tc::mbar_wait(full + s, (g / ST) & 1, err)) {
                ok = false;
                break;
            }
            const unsigned char* cs = smem + s * C::STAGE + C::A_BYTES + C::B_BYTES;
            const uint32_t sa = tc::saddr(smem + s * C::STAGE);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int r = r0 + 16 * j;
                const uint32_t w = *reinterpret_cast<const uint32_t*>(cs + r * 64 + wi * 4);
                uint32_t p[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    // codes 2u, 2u+1 of the word (LSB first) as exact floats
                    const float c0 = __uint_as_float(0x4B000000u | ((w >> (8 * u)) & 15u)) - 8388608.f;
                    const float c1 = __uint_as_float(0x4B000000u | ((w >> (8 * u + 4)) & 15u)) - 8388608.f;
                    p[u] = tc::pack_bf16x2(__fmaf_rn(c0, s4[j], b4[j]), __fmaf_rn(c1, s4[j], b4[j]));
                }
                const uint32_t off = chalf * C::A_HALF + (uint32_t)r * 128 + ((cchunk ^ (uint32_t)(r & 7)) << 4);
                tc::st_shared_v4(sa + off, p[0], p[1], p[2], p[3]);
            }
            tc::fence_async_smem();
            tc::mbar_arrive(dqf + s);
        }
    }
    tc::tc_before();
    const int bad = __syncthreads_or(!ok && (warp >= 2 || lane == 0));
    if (warp == 1) {
        tc::tc_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMC));
    }
    if (tid == 0 && bad) {
        *(volatile int*)a.err_host = 1;
        __threadfence_system();
    }
}

// Host side: tensor maps, grid (one persistent CTA per SM at most), launch.
// Shapes are checked by the caller: IN % 128 == 0, OUT % 64 == 0, rows >= 1,
// dY / W / codes 16-byte aligned.
inline bool encode_dx_maps(int FMT, int BN, DxArgs& a, const void* dy, const void* w, const uint32_t* wq) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint32_t es[2] = {1, 1};
    if (FMT == DX_Q4) {
        cuuint64_t dims[2] = {(cuuint64_t)(a.IN / 8), (cuuint64_t)a.OUT};
        cuuint64_t strides[1] = {(cuuint64_t)a.IN / 2};
        cuuint32_t box[2] = {16, (cuuint32_t)DX_BK};
        if (enc(&a.amap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, (void*)wq, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    } else {
        cuuint64_t dims[2] = {(cuuint64_t)a.IN, (cuuint64_t)a.OUT};
        cuuint64_t strides[1] = {(cuuint64_t)a.IN * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)DX_BK};
        if (enc(&a.amap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)w, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    cuuint64_t dims[2] = {(cuuint64_t)a.OUT, (cuuint64_t)a.rows};
    cuuint64_t strides[1] = {(cuuint64_t)a.OUT * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)BN};
    return enc(&a.bmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)dy, dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int FMT, int BN>
inline cudaError_t launch_dx_t(const DxArgs& a, int sm_count, cudaStream_t st) {
    using C = DxCfg<FMT, BN>;
    auto kern = gemm_dx_kernel<FMT, BN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::TOTAL);
    if (e != cudaSuccess) return e;
    const int ntiles = (a.IN / DX_BM) * ((a.rows + BN - 1) / BN);
    const int grid = ntiles < sm_count ? ntiles : sm_count;
    kern<<<grid, C::THREADS, C::TOTAL, st>>>(a);
    return cudaGetLastError();
}

// BN = 64 token rows per tile up to 64 rows, else 256.
inline cudaError_t launch_gemm_dx(int FMT, DxArgs& a, const void* dy, const void* w, const uint32_t* wq,
                                  int sm_count, cudaStream_t st) {
    const int BN = a.rows <= 64 ? 64 : 256;
    if (!encode_dx_maps(FMT, BN, a, dy, w, wq)) return cudaErrorInvalidValue;
    if (FMT == DX_Q4) return BN == 64 ? launch_dx_t<DX_Q4, 64>(a, sm_count, st) : launch_dx_t<DX_Q4, 256>(a, sm_count, st);
    return BN == 64 ? launch_dx_t<DX_BF16, 64>(a, sm_count, st) : launch_dx_t<DX_BF16, 256>(a, sm_count, st);
}

}  // namespace rwkv
