// Streaming GEMV on the CUDA cores for the MLX affine 4-bit group-64
// container and 1..2 activation rows (fp16):
//   y[n, o] = sum_g scale[o, g] * sum_{k in g} q[o, k] x[n, k] + bias[o, g] * sum_{k in g} x[n, k]
// (MLX's quantized matrix-vector numerics: fp32 sums, codes summed in column
// order, scale and bias applied once per group).
//
// A persistent grid: CTA c owns the row blocks c, c + gridDim.x, ... of its
// job (jobs.j[blockIdx.y]).  All of x and its per-group sums are staged in
// shared memory once per CTA; after that a thread only streams codes, one
// 128-code unit per step (gemv_tile.cuh layout: TPR threads per output row,
// RPC rows per block; TPR 64 for IN a multiple of 8192), the next step's
// unit loaded while this one is summed, so loads stay in flight across row
// blocks; the TPR partials of a row meet in a fixed shuffle tree (and, at
// TPR 64, one add of the row's two warp sums).
//
// Codes become fp16 two at a time: the nibbles at bits 0-3 / 16-19 of a word
// OR'd under the exponent of 1024 read 1024 + q, one HSUB2 takes 1024 off;
// the nibbles at bits 4-7 / 20-23 read 1024 + 16 q, one HFMA2 (x 1/16 - 64)
// gives q -- each step exact for q < 16.  Products use sm_100's mixed-
// precision fma.rn.f32.f16: the f16 x f16 product is exact in fp32 and the
// sum is rounded once, i.e. fmaf(float(q), float(x), acc) on fp16 activations.
//
// Measured against the exact-code mma.sync GEMV (gemm_w4.cuh) on the 1.5B
// projection shapes this kernel is the faster one at 1 and 2 rows; from 3
// rows on the tensor cores' reuse of each unpacked code across rows wins.
#pragma once

#include "gemv_mma.cuh"
#include "gemv_tile.cuh"

namespace rwkv {

constexpr int QS_MAXR = 2;  // activation rows this kernel takes

__device__ __forceinline__ float fma_f16f32(__half a, __half b, float c) {
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(__half_as_ushort(a)), "h"(__half_as_ushort(b)), "f"(c));
    return d;
}
__device__ __forceinline__ __half2 qs_u2h(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// Codes 0..7 of a word (LSB first) as four fp16 pairs: c[0] = (q0, q4),
// c[1] = (q1, q5), c[2] = (q2, q6), c[3] = (q3, q7).
__device__ __forceinline__ void qs_codes8(uint32_t w, __half2 (&c)[4]) {
    const __half2 k1024 = __half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
    const __half2 k16 = __half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));   // 1/16
    const __half2 km64 = __half2(__ushort_as_half(0xD400), __ushort_as_half(0xD400));  // -64
    const uint32_t w8 = w >> 8;
    c[0] = __hsub2(qs_u2h((w & 0x000F000Fu) | 0x64006400u), k1024);
    c[1] = __hfma2(qs_u2h((w & 0x00F000F0u) | 0x64006400u), k16, km64);
    c[2] = __hsub2(qs_u2h((w8 & 0x000F000Fu) | 0x64006400u), k1024);
    c[3] = __hfma2(qs_u2h((w8 & 0x00F000F0u) | 0x64006400u), k16, km64);
}

// Staged activations: fp16, a 128-column unit padded to 136 halves (17
// 16-byte chunks, an odd count, so the 16 threads of a row -- one unit each --
// read two conflict-free wavefronts of 16-byte vectors).
constexpr int QS_HU = 136;

// Threads per output row: 64 when IN / 128 is a multiple of 64 (a row
// spans two warps: one window, 4 rows per CTA, so the 2048 x 8192 shapes
// launch 4x the CTAs and keep a whole matrix in flight), else gemv_tile.cuh's
// choice (<= 16).
__host__ __device__ __forceinline__ int qs_tpr(int IN) { return (IN / TG_UNIT) % 64 == 0 ? 64 : tg_tpr(IN); }

// Shared memory for IN columns and R rows: x, then the group sums (fp32).
__host__ __device__ __forceinline__ size_t qs_gs_off(int IN, int R) {
    return ((size_t)R * (IN / TG_UNIT) * QS_HU * 2 + 15) & ~(size_t)15;
}
__host__ __device__ __forceinline__ size_t q4_stream_smem(int IN, int R) {
    return qs_gs_off(IN, R) + (size_t)R * (IN / 64) * sizeof(float);
}

template <int R>
__global__ void __launch_bounds__(TG_T, R == 1 ? 4 : 3) q4_gemv_stream_kernel(const GemvJobs jobs, int rows) {
    extern __shared__ __align__(16) unsigned char smq[];
    const GemvJob& jb = jobs.j[blockIdx.y];
    const int OUT = jb.OUT, IN = jb.IN;
    const int TPR = qs_tpr(IN), RPC = TG_T / TPR, W = TPR * TG_UNIT, NW = IN / W;
    const int NU = IN / TG_UNIT, RS = NU * QS_HU, NG = IN / 64;
    __shared__ float red[2][TG_T / 32][R];  // TPR 64: the two warps' partials of a row
    __half* xh = reinterpret_cast<__half*>(smq);
    float* gs = reinterpret_cast<float*>(smq + qs_gs_off(IN, R));
    const int tid = threadIdx.x, lr = tid / TPR, u = tid - lr * TPR;
    const int nrb = (OUT + RPC - 1) / RPC;
    const int nblk = (int)blockIdx.x < nrb ? (nrb - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    if (tid == 0) pdl_trigger();
    if (nblk == 0) {  // more CTAs than row blocks in this job
        pdl_wait();
        return;
    }
    const int total = nblk * NW;
    // the load stream: row block lrb, window lwin; soff indexes the unit's
    // first (scale, bias) pair, 8 x soff its first code word
    int lrb = blockIdx.x, lwin = 0, soff = 0;
    auto set_row = [&]() { soff = min(lrb * RPC + lr, OUT - 1) * NG + 2 * u; };
    uint4 cw[4];
    __half2 s2, b2;
    auto load = [&]() {
        const uint4* src = reinterpret_cast<const uint4*>((const uint32_t*)jb.w + 8 * (int64_t)soff);
#pragma unroll
        for (int v = 0; v < 4; v++) cw[v] = __ldg(src + v);
        s2 = __ldg(reinterpret_cast<const __half2*>(jb.scales + soff));
        b2 = __ldg(reinterpret_cast<const __half2*>(jb.biases + soff));
    };
    set_row();
    load();
    pdl_wait();
    {  // stage x (16-byte vectors when aligned) permuted per 8 columns, then the group sums
        const __half* x = (const __half*)jb.x;
        const bool vec = (((uintptr_t)x | (uintptr_t)(jb.x_stride * 2)) & 15) == 0;
        const int nch = NU * 16;  // 16-byte chunks of a row
        for (int e = tid; e < R * nch; e += TG_T) {
            const int n = e / nch, ch = e - n * nch;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (n < rows) {
                const __half* src = x + (int64_t)n * jb.x_stride + ch * 8;
                if (vec) {
                    v = __ldg(reinterpret_cast<const uint4*>(src));
                } else {
                    const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
                    v = make_uint4(s16[0] | (uint32_t)s16[1] << 16, s16[2] | (uint32_t)s16[3] << 16,
                                   s16[4] | (uint32_t)s16[5] << 16, s16[6] | (uint32_t)s16[7] << 16);
                }
            }
            // (x0 x1)(x2 x3)(x4 x5)(x6 x7) -> (x0 x4)(x1 x5)(x2 x6)(x3 x7): pair j matches code pair j
            const uint4 o = make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632),
                                       __byte_perm(v.y, v.w, 0x5410), __byte_perm(v.y, v.w, 0x7632));
            *reinterpret_cast<uint4*>(xh + n * RS + (ch >> 4) * QS_HU + (ch & 15) * 8) = o;
        }
        __syncthreads();
        for (int e = tid; e < R * NG; e += TG_T) {
            const int n = e / NG, g = e - n * NG;
            const __half* p = xh + n * RS + (g >> 1) * QS_HU + (g & 1) * 64;
            float t = 0.f;
            // column order: column c of a piece sits at slot 2 (c % 4) + c / 4
#pragma unroll 16
            for (int c = 0; c < 64; c++) t += __half2float(p[(c & ~7) + 2 * (c & 3) + ((c >> 2) & 1)]);
            gs[e] = t;
        }
        __syncthreads();
    }
    float acc[R];
#pragma unroll
    for (int n = 0; n < R; n++) acc[n] = 0.f;
    int win = 0, crb = blockIdx.x;  // the compute stream's window and row block
    for (int it = 0; it < total; it++) {
        const uint32_t wd[16] = {cw[0].x, cw[0].y, cw[0].z, cw[0].w, cw[1].x, cw[1].y, cw[1].z, cw[1].w,
                                 cw[2].x, cw[2].y, cw[2].z, cw[2].w, cw[3].x, cw[3].y, cw[3].z, cw[3].w};
        const float sg[2] = {__low2float(s2), __high2float(s2)}, bg[2] = {__low2float(b2), __high2float(b2)};
        if (it + 1 < total) {  // the next unit, in flight during this one
            if (++lwin == NW) {
                lwin = 0;
                lrb += gridDim.x;
                set_row();
            } else {
                soff += W / 64;
            }
            load();
        }
        const int unit = win * TPR + u;
        const __half* xu = xh + unit * QS_HU;
#pragma unroll
        for (int gq = 0; gq < 2; gq++) {
            float dv[R];
#pragma unroll
            for (int n = 0; n < R; n++) dv[n] = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                __half2 c[4];
                qs_codes8(wd[8 * gq + i], c);
#pragma unroll
                for (int n = 0; n < R; n++) {
                    const uint4 xv = *reinterpret_cast<const uint4*>(xu + n * RS + gq * 64 + i * 8);
                    const __half2 xp[4] = {qs_u2h(xv.x), qs_u2h(xv.y), qs_u2h(xv.z), qs_u2h(xv.w)};
                    float d = dv[n];
#pragma unroll
                    for (int j = 0; j < 4; j++) d = fma_f16f32(__low2half(c[j]), __low2half(xp[j]), d);
#pragma unroll
                    for (int j = 0; j < 4; j++) d = fma_f16f32(__high2half(c[j]), __high2half(xp[j]), d);
                    dv[n] = d;
                }
            }
            const int g = unit * 2 + gq;
#pragma unroll
            for (int n = 0; n < R; n++) acc[n] = fmaf(sg[gq], dv[n], fmaf(bg[gq], gs[n * NG + g], acc[n]));
        }
        if (win == NW - 1) {  // the row block's last window: reduce the row, store, restart
            const int row = crb * RPC + lr;
            float v[R];
#pragma unroll
            for (int n = 0; n < R; n++) {
                v[n] = acc[n];
                for (int o = min(TPR, 32) / 2; o > 0; o >>= 1) v[n] += __shfl_xor_sync(0xffffffffu, v[n], o);
                acc[n] = 0.f;
            }
            if (TPR == 64) {  // two warps per row: meet in shared memory (double-buffered by row block)
                float(&rb)[TG_T / 32][R] = red[((crb - (int)blockIdx.x) / (int)gridDim.x) & 1];
                if ((tid & 31) == 0) {
#pragma unroll
                    for (int n = 0; n < R; n++) rb[tid >> 5][n] = v[n];
                }
                __syncthreads();
#pragma unroll
                for (int n = 0; n < R; n++) v[n] = rb[2 * lr][n] + rb[2 * lr + 1][n];
            }
            if (u == 0 && row < OUT) {
#pragma unroll
                for (int n = 0; n < R; n++)
                    if (n < rows) epilogue(jb, row, n, v[n]);
            }
            win = 0;
            crb += gridDim.x;
        } else {
            win++;
        }
    }
}

// Shared memory the streaming kernel is set up for (x of up to 2 rows of
// 8192 columns, with room to spare).
constexpr int QS_SMEM_MAX = 96 * 1024;

// Whether jobs[0..nj) can take the streaming kernel at `rows` activation rows:
// 4-bit group-64 affine weights, IN a multiple of 128, 16-byte aligned codes,
// 4-byte aligned scales and biases, staged x within QS_SMEM_MAX.
inline bool q4_stream_eligible(const GemvJobs& jobs, int nj, int rows) {
    if (rows < 1 || rows > QS_MAXR || nj < 1) return false;
    for (int i = 0; i < nj; i++) {
        const GemvJob& j = jobs.j[i];
        if (j.wfmt != WFMT_AFFINE || j.IN % TG_UNIT || j.OUT < 1) return false;
        if ((int64_t)j.OUT * (j.IN / 64) >= (int64_t)1 << 31) return false;  // 32-bit (scale, bias) index
        if (((uintptr_t)j.w & 15) || (((uintptr_t)j.scales | (uintptr_t)j.biases) & 3)) return false;
        if (q4_stream_smem(j.IN, rows) > (size_t)QS_SMEM_MAX) return false;
    }
    return true;
}

// One launch over the jobs (checked by q4_stream_eligible): the persistent
// grid fills the SMs at the kernel's occupancy, shared between the jobs.
inline cudaError_t launch_q4_gemv_stream(const GemvJobs& jobs, int nj, int rows, int sm_count, bool pdl,
                                         cudaStream_t st) {
    int maxin = 0, maxrb = 0;
    for (int i = 0; i < nj; i++) {
        maxin = std::max(maxin, jobs.j[i].IN);
        const int rpc = TG_T / qs_tpr(jobs.j[i].IN);
        maxrb = std::max(maxrb, (jobs.j[i].OUT + rpc - 1) / rpc);
    }
    const int R = rows <= 1 ? 1 : 2;
    const size_t smem = q4_stream_smem(maxin, R);
    auto go = [&](auto kern) {
        // both instances share one function-pointer type, so the opt-in is
        // set per call (a host-side attribute, no device work)
        cudaError_t e = smem > 48 * 1024
                            ? cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, QS_SMEM_MAX)
                            : cudaSuccess;
        if (e != cudaSuccess) return e;
        int occ = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, TG_T, smem);
        if (e != cudaSuccess) return e;
        const int G = std::max(1, std::min(maxrb, std::max(1, occ) * sm_count / nj));
        const dim3 grid(G, nj);
        if (!pdl) {
            kern<<<grid, TG_T, smem, st>>>(jobs, rows);
            return cudaGetLastError();
        }
        return launch_pdl(kern, grid, dim3(TG_T), smem, st, jobs, rows);
    };
    return R == 1 ? go(q4_gemv_stream_kernel<1>) : go(q4_gemv_stream_kernel<2>);
}

// ---- dense fp16 GEMV for 1..2 activation rows (the low-rank branches) ----
//
// y[n, o] = sum_k W[o, k] x[n, k], W fp16 [OUT, IN] (IN a multiple of 32),
// x fp16, fp32 sums (products exact: fma.rn.f32.f16).  FS_TPR threads per
// output row, each a 32-column chunk per step (four 16-byte loads), two
// chunks in flight; the TPR partials of a row meet in a shuffle tree.  The
// down projections (IN = C) put a warp on a row, so the whole matrix is in
// flight in one round trip.  x is staged in shared memory once per CTA,
// a 32-column chunk padded to 40 halves (80 bytes: the 32 lanes of a row read
// conflict-free 16-byte vectors).
constexpr int FS_CH = 40;

// threads per row: the largest power of two <= 32 dividing IN / 32
__host__ __device__ __forceinline__ int fs_tpr(int IN) {
    const int nc = IN / 32;
    int t = 32;
    while (t > 1 && nc % t) t >>= 1;
    return t;
}
__host__ __device__ __forceinline__ size_t f16_small_smem(int IN, int R) { return (size_t)R * (IN / 32) * FS_CH * 2; }

template <int R>
__global__ void __launch_bounds__(TG_T) f16_gemv_small_kernel(const GemvJobs jobs, int rows) {
    extern __shared__ __align__(16) unsigned char smf[];
    const GemvJob& jb = jobs.j[blockIdx.y];
    const int OUT = jb.OUT, IN = jb.IN;
    const int TPR = fs_tpr(IN), RPC = TG_T / TPR, NC = IN / 32, RS = NC * FS_CH;
    __half* xh = reinterpret_cast<__half*>(smf);
    const int tid = threadIdx.x, lr = tid / TPR, u = tid - lr * TPR;
    const int row0 = blockIdx.x * RPC;
    if (tid == 0) pdl_trigger();
    if (row0 >= OUT) {  // a smaller job of the launch: nothing here
        pdl_wait();
        return;
    }
    const __half* wr = (const __half*)jb.w + (int64_t)min(row0 + lr, OUT - 1) * IN;
    uint4 wv[2][4];
    auto ld = [&](int s, int c) {
        const uint4* p = reinterpret_cast<const uint4*>(wr + c * 32);
#pragma unroll
        for (int v = 0; v < 4; v++) wv[s][v] = __ldg(p + v);
    };
    if (u < NC) ld(0, u);
    if (u + TPR < NC) ld(1, u + TPR);
    pdl_wait();
    {  // stage x (16-byte vectors; the launcher checks the alignment)
        const __half* x = (const __half*)jb.x;
        const int nv = NC * 4;  // 16-byte vectors of a row
        for (int e = tid; e < R * nv; e += TG_T) {
            const int n = e / nv, q = e - n * nv;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (n < rows) v = __ldg(reinterpret_cast<const uint4*>(x + (int64_t)n * jb.x_stride) + q);
            *reinterpret_cast<uint4*>(xh + n * RS + (q >> 2) * FS_CH + (q & 3) * 8) = v;
        }
        __syncthreads();
    }
    float acc[R];
#pragma unroll
    for (int n = 0; n < R; n++) acc[n] = 0.f;
    for (int c0 = u; c0 < NC; c0 += 2 * TPR) {
#pragma unroll
        for (int s = 0; s < 2; s++) {
            const int c = c0 + s * TPR;
            if (c < NC) {
#pragma unroll
                for (int v = 0; v < 4; v++) {
                    const __half2 w01 = qs_u2h(wv[s][v].x), w23 = qs_u2h(wv[s][v].y);
                    const __half2 w45 = qs_u2h(wv[s][v].z), w67 = qs_u2h(wv[s][v].w);
#pragma unroll
                    for (int n = 0; n < R; n++) {
                        const uint4 xv = *reinterpret_cast<const uint4*>(xh + n * RS + c * FS_CH + v * 8);
                        const __half2 x01 = qs_u2h(xv.x), x23 = qs_u2h(xv.y), x45 = qs_u2h(xv.z), x67 = qs_u2h(xv.w);
                        float d = acc[n];
                        d = fma_f16f32(__low2half(w01), __low2half(x01), d);
                        d = fma_f16f32(__high2half(w01), __high2half(x01), d);
                        d = fma_f16f32(__low2half(w23), __low2half(x23), d);
                        d = fma_f16f32(__high2half(w23), __high2half(x23), d);
                        d = fma_f16f32(__low2half(w45), __low2half(x45), d);
                        d = fma_f16f32(__high2half(w45), __high2half(x45), d);
                        d = fma_f16f32(__low2half(w67), __low2half(x67), d);
                        d = fma_f16f32(__high2half(w67), __high2half(x67), d);
                        acc[n] = d;
                    }
                }
                if (c + 2 * TPR < NC) ld(s, c + 2 * TPR);  // this slot's next chunk
            }
        }
    }
    const int row = row0 + lr;
#pragma unroll
    for (int n = 0; n < R; n++) {
        float v = acc[n];
        for (int o = TPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (u == 0 && row < OUT && n < rows) epilogue(jb, row, n, v);
    }
}

// Whether jobs[0..nj) (dense fp16 weights) can take f16_gemv_small_kernel at
// `rows` activation rows: IN a multiple of 32 and at least 256, 16-byte
// aligned W rows and x.  (The up projections, whose IN is the rank, stay on
// the mma.sync GEMV: 1-row decode 0.93 ms with them here, 0.89 without.)
inline bool f16_small_eligible(const GemvJobs& jobs, int nj, int rows) {
    if (rows < 1 || rows > QS_MAXR || nj < 1) return false;
    for (int i = 0; i < nj; i++) {
        const GemvJob& j = jobs.j[i];
        if (j.IN % 32 || j.IN < 256 || j.IN > 8192 || j.OUT < 1) return false;
        if (((uintptr_t)j.w | (uintptr_t)j.x | (uintptr_t)(j.x_stride * 2)) & 15) return false;
    }
    return true;
}

inline cudaError_t launch_f16_gemv_small(const GemvJobs& jobs, int nj, int rows, bool pdl, cudaStream_t st) {
    int maxin = 0, maxb = 0;
    for (int i = 0; i < nj; i++) {
        maxin = std::max(maxin, jobs.j[i].IN);
        const int rpc = TG_T / fs_tpr(jobs.j[i].IN);
        maxb = std::max(maxb, (jobs.j[i].OUT + rpc - 1) / rpc);
    }
    const int R = rows <= 1 ? 1 : 2;
    const size_t smem = f16_small_smem(maxin, R);
    const dim3 grid(maxb, nj);
    auto go = [&](auto kern) {
        if (!pdl) {
            kern<<<grid, TG_T, smem, st>>>(jobs, rows);
            return cudaGetLastError();
        }
        return launch_pdl(kern, grid, dim3(TG_T), smem, st, jobs, rows);
    };
    return R == 1 ? go(f16_gemv_small_kernel<1>) : go(f16_gemv_small_kernel<2>);
}

}  // namespace rwkv
