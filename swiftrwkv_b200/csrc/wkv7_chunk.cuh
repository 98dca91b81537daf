// Shared pieces of the chunked (DPLR) WKV-7 kernels: chunk constants, the
// 3xTF32 tensor-core helpers, chunk staging, the cumulative decay, the
// (I - M)^-1 chain and the chunk scan.  Included by the forward
// (wkv7_chunk.cu) and the backward (wkv7_chunk_bwd.cu); everything is in an
// anonymous namespace, so each includes its own copy.
#pragma once

#include "common.cuh"

namespace rwkv {
namespace {

constexpr int CN = 64;      // head size
constexpr int CL = 16;      // chunk length
constexpr int CT = 256;     // threads
// Row strides (floats) chosen for the m16n8k8 fragment patterns: a row-read
// operand X[g][k + t] (g = lane/4, t = lane%4) is conflict free when the
// stride is 4 mod 32 (64-wide: 68; 16-wide: 20), a column-read operand
// X[k + t][n + g] when it is 8 mod 32 (64-wide: 72).
constexpr int CP = CN + 4;   // 68
constexpr int CQ = CN + 8;   // 72
constexpr int LP = CL + 4;   // 20
constexpr float GUARD = 1e-30f;

// A_c in the order the scan loads it: float4 number (k / 2) * 32 + l (k even)
// holds A[k][2l], A[k][2l+1], A[k+1][2l], A[k+1][2l+1]; warp w of the scan
// reads float4s 8w * 32 .. (8w + 8) * 32 - 1 (k = 16w .. 16w + 15).
__device__ __forceinline__ int scan_a_index(int k, int c) {
    return (((k >> 1) * 32 + (c >> 1)) << 2) + ((k & 1) << 1) + (c & 1);
}


// ------------------------------------------------------------ tensor cores

// x = hi + lo, both rounded to TF32 (10 mantissa bits) to nearest by adding
// half a TF32 ulp to the bit pattern and masking: hi*hi + hi*lo + lo*hi then
// carries x to ~2^-22 relative, unbiased.  Integer ops rather than
// cvt.rna.tf32: the conversion made the 3xTF32 k-step ~1.5x slower on this
// GPU (measured); truncating instead of rounding biases the sums.
__device__ __forceinline__ uint32_t tf32_rn(uint32_t bits) { return (bits + 0x1000u) & 0xffffe000u; }
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    hi = tf32_rn(__float_as_uint(x));
    lo = tf32_rn(__float_as_uint(x - __uint_as_float(hi)));
}
// D(16x8) += A(16x8, row) * B(8x8, col), m16n8k8 tf32 fragments:
// a0 = A[g][t], a1 = A[g+8][t], a2 = A[g][t+4], a3 = A[g+8][t+4];
// b0 = B[t][g], b1 = B[t+4][g]; d0..3 = D[g][2t], D[g][2t+1], D[g+8][2t], D[g+8][2t+1]
// (g = lane / 4, t = lane % 4).
__device__ __forceinline__ void mma_tf32(float* d, const uint32_t* a, const uint32_t* b) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// D += A B in 3xTF32 (A as 4 fp32 fragment values, B as 2)
__device__ __forceinline__ void mma3(float* d, const float* af, const float* bf) {
    uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
    for (int q = 0; q < 4; q++) split_tf32(af[q], ah[q], al[q]);
    split_tf32(bf[0], bh[0], bl[0]);
    split_tf32(bf[1], bh[1], bl[1]);
    mma_tf32(d, al, bh);
    mma_tf32(d, ah, bl);
    mma_tf32(d, ah, bh);
}
// The same product into three independent accumulators (hi*hi, hi*lo,
// lo*hi) so that consecutive k-steps do not wait on each other; sum with
// acc3_sum at the end.
__device__ __forceinline__ void mma3x(float (*d)[4], const float* af, const float* bf) {
    uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
    for (int q = 0; q < 4; q++) split_tf32(af[q], ah[q], al[q]);
    split_tf32(bf[0], bh[0], bl[0]);
    split_tf32(bf[1], bh[1], bl[1]);
    mma_tf32(d[0], ah, bh);
    mma_tf32(d[1], ah, bl);
    mma_tf32(d[2], al, bh);
}
__device__ __forceinline__ void acc3_sum(float* out, float (*d)[4]) {
#pragma unroll
    for (int q = 0; q < 4; q++) out[q] += d[2][q] + d[1][q] + d[0][q];
}

// position of fragment value q of a 16x8 tile at (m0, n0)
__device__ __forceinline__ int frag_i(int m0, int lane, int q) { return m0 + (lane >> 2) + 8 * (q >> 1); }
__device__ __forceinline__ int frag_j(int n0, int lane, int q) { return n0 + 2 * (lane & 3) + (q & 1); }

// One warp: C = (Cin ? Cin : 0) + A B for 16 x 16 matrices (C must not alias
// the inputs).
__device__ __forceinline__ void mm16(float (*C)[LP], const float (*A)[LP], const float (*B)[LP],
                                     const float (*Cin)[LP], int lane) {
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int n0 = 0; n0 < CL; n0 += 8) {
        float d[4];
#pragma unroll
        for (int q = 0; q < 4; q++) d[q] = Cin ? Cin[frag_i(0, lane, q)][frag_j(n0, lane, q)] : 0.f;
#pragma unroll
        for (int k0 = 0; k0 < CL; k0 += 8) {
            const float af[4] = {A[g][k0 + t4], A[g + 8][k0 + t4], A[g][k0 + t4 + 4], A[g + 8][k0 + t4 + 4]};
            const float bf[2] = {B[k0 + t4][n0 + g], B[k0 + t4 + 4][n0 + g]};
            mma3(d, af, bf);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) C[frag_i(0, lane, q)][frag_j(n0, lane, q)] = d[q];
    }
}

// ------------------------------------------------------------ chunk staging

// Chunk inputs for all 64 key channels (r optional) and v for rows
// [v0, v0 + nv) (nv * 16 a multiple of 256); padded tokens are identity
// steps.  Every global load is issued before the first shared store, so a
// CTA waits on memory once.
template <typename T, int NV, int NTH = CT>
__device__ __forceinline__ void stage_chunk(float (*rr)[CN], float (*ww)[CN], float (*kk)[CN],
                                            float (*aa)[CN], float (*bb)[CN], float* vv, int vstride,
                                            const T* r, const T* w, const T* k, const T* v,
                                            const T* a, const T* b, int bi, int hi, int H, int T_,
                                            int t0, int v0) {
    constexpr int PER = CL * CN / NTH, VPER = CL * NV / NTH;
    T lr[PER], lw[PER], lk[PER], la[PER], lb[PER], lv[VPER];
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = threadIdx.x + NTH * i, tl = e / CN, c = e % CN, t = t0 + tl;
        const size_t o = (((size_t)bi * T_ + min(t, T_ - 1)) * H + hi) * CN + c;
        if (rr) lr[i] = r[o];
        lw[i] = w[o]; lk[i] = k[o]; la[i] = a[o]; lb[i] = b[o];
    }
#pragma unroll
    for (int i = 0; i < VPER; i++) {
        const int e = threadIdx.x + NTH * i, tl = e / NV, d = e % NV, t = t0 + tl;
        lv[i] = v[(((size_t)bi * T_ + min(t, T_ - 1)) * H + hi) * CN + v0 + d];
    }
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = threadIdx.x + NTH * i, tl = e / CN, c = e % CN;
        const bool in = t0 + tl < T_;
        if (rr) rr[tl][c] = in ? to_f(lr[i]) : 0.f;
        ww[tl][c] = in ? to_f(lw[i]) : 1.f;
        kk[tl][c] = in ? to_f(lk[i]) : 0.f;
        aa[tl][c] = in ? to_f(la[i]) : 0.f;
        bb[tl][c] = in ? to_f(lb[i]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < VPER; i++) {
        const int e = threadIdx.x + NTH * i, tl = e / NV, d = e % NV;
        vv[tl * vstride + d] = t0 + tl < T_ ? to_f(lv[i]) : 0.f;
    }
}

// c_0 .. c_16 per channel (threads 0-63) and the chunk's smallest c_16;
// ends with a barrier.  red: 2 floats of scratch.
__device__ __forceinline__ float chunk_decay(float (*c)[CN], const float (*ww)[CN], float* red) {
    if (threadIdx.x < CN) {
        float cc = 1.f;
        c[0][threadIdx.x] = 1.f;
#pragma unroll
        for (int t = 0; t < CL; t++) {
            cc *= ww[t][threadIdx.x];
            c[t + 1][threadIdx.x] = cc;
        }
        const float m = warp_min(cc);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    }
    __syncthreads();
    return fminf(red[0], red[1]);
}


// Z = (I - Mb)^-1 by doubling; warps 0 (powers of M) and 1 (products), the
// other warps only take the barriers.  Returns the buffer holding Z.
__device__ __forceinline__ int z_chain(float (*Zb)[CL][LP], float (*Pb)[CL][LP], const float (*Mb)[LP]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0) mm16(Pb[1], Mb, Mb, nullptr, lane);                       // P1 = M^2
    if (warp == 1)
        for (int e = lane; e < CL * CL; e += 32) {
            const int i = e / CL, j = e % CL;
            Zb[0][i][j] = (i == j ? 1.f : 0.f) + Mb[i][j];                   // Z0 = I + M
        }
    __syncthreads();
    if (warp == 0) mm16(Pb[0], Pb[1], Pb[1], nullptr, lane);                 // P2 = P1^2
    if (warp == 1) mm16(Zb[1], Zb[0], Pb[1], Zb[0], lane);                   // Z1 = Z0 (I + P1)
    __syncthreads();
    if (warp == 0) mm16(Pb[1], Pb[0], Pb[0], nullptr, lane);                 // P3 = P2^2
    if (warp == 1) mm16(Zb[0], Zb[1], Pb[0], Zb[1], lane);                   // Z2 = Z1 (I + P2)
    __syncthreads();
    if (warp == 1) mm16(Zb[1], Zb[0], Pb[1], Zb[0], lane);                   // Z3 = Z2 (I + P3)
    __syncthreads();
    return 1;
}

// Token-by-token update of `nr` rows of M (row stride CP) with token t of the
// chunk; v_row(d) gives the row's v value (0 for the pure transition).
// Thread = (row, 16 columns): 4 threads per row, 64 rows per pass.
template <typename VF>
__device__ __forceinline__ void step_rows(float (*M)[CP], int nr, const float (*ww)[CN],
                                          const float (*kk)[CN], const float (*aa)[CN],
                                          const float (*bb)[CN], int t, VF v_row) {
    const int q = threadIdx.x & 3, c0 = 16 * q;
    for (int rr = threadIdx.x >> 2; rr < nr; rr += CT / 4) {
        float sa = 0.f;
#pragma unroll
        for (int j = 0; j < 16; j++) sa = fmaf(M[rr][c0 + j], aa[t][c0 + j], sa);
        sa += __shfl_xor_sync(0xffffffffu, sa, 1);
        sa += __shfl_xor_sync(0xffffffffu, sa, 2);
        const float vd = v_row(rr);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int c = c0 + j;
            M[rr][c] = fmaf(ww[t][c], M[rr][c], fmaf(vd, kk[t][c], sa * bb[t][c]));
        }
    }
}


// ------------------------------------------------------------ scan

// The scan is a chain of small products (8 rows x 64 x 64 per CTA and chunk):
// too small for the tensor cores to pay (3xTF32 on mma.sync needs three
// products and the legacy tensor path is slow on sm_100), so it runs in plain
// fp32 FMAs.  CTA = (head, 8 state rows), 4 warps; warp w takes K = 16w ..
// 16w + 15 for all 8 rows, lane l columns 2l and 2l + 1, and the four partial
// products are summed with B_c in shared memory.  A_c and B_c come straight
// from L2 into registers, three chunks ahead.
//
// The same kernel runs the backward's reverse scan of the gradient at the
// chunk boundaries (reverse = 1: chunks NC-1 .. 0, A_c^T stored in the scan
// order).  S0ws[c] receives the state before chunk c is applied (forward: the
// chunk's start state; reverse: the gradient at the chunk's end), ckpt[c]
// (nullable) the state after it, h_out the final state.
constexpr int SR = 8;     // state rows per scan CTA
constexpr int ST = 128;   // scan threads

__global__ void __launch_bounds__(ST)
wkv7_chunk_scan_kernel(const float* __restrict__ h_in, const float* __restrict__ Aws,
                       const float* __restrict__ Bws, float* __restrict__ S0ws,
                       float* __restrict__ h_out, float* __restrict__ ckpt, int NC, int reverse) {
    __shared__ __align__(16) float S[SR][CN];      // state rows (broadcast reads)
    __shared__ __align__(16) float P[4][SR][CN];   // per-warp partial products
    const int bh = blockIdx.x, dv0 = blockIdx.y * SR;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rr = tid >> 4, c4 = (tid & 15) * 4;   // this thread's 4 state entries
    constexpr int CH4 = CN * CN / 4;                // float4 per chunk matrix
    // step i applies chunk chunk_of(i): 0, 1, .. forward; NC - 1, NC - 2, .. in reverse
    auto chunk_of = [&](int i) { return reverse ? NC - 1 - i : i; };
    {
        const float4 s = h_in ? *reinterpret_cast<const float4*>(h_in + ((size_t)bh * CN + dv0 + rr) * CN + c4)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(&S[rr][c4]) = s;
        *reinterpret_cast<float4*>(S0ws + ((size_t)bh * NC + chunk_of(0)) * CN * CN + (size_t)(dv0 + rr) * CN + c4) = s;
    }
    const float4* Ab = reinterpret_cast<const float4*>(Aws + (size_t)bh * NC * CN * CN) + warp * 8 * 32 + lane;
    const float4* Bb = reinterpret_cast<const float4*>(Bws + (size_t)bh * NC * CN * CN + (size_t)(dv0 + rr) * CN + c4);
    float4 a0[8], a1[8], a2[8], b0, b1, b2;
    auto load = [&](float4 (&av)[8], float4& bv, int ch) {
        if (ch < NC) {
#pragma unroll
            for (int i = 0; i < 8; i++) av[i] = __ldcg(Ab + (size_t)chunk_of(ch) * CH4 + i * 32);
            bv = __ldcg(Bb + (size_t)chunk_of(ch) * CH4);
        }
    };
    load(a0, b0, 0);
    load(a1, b1, 1);
    load(a2, b2, 2);
    __syncthreads();
    auto chunk = [&](float4 (&av)[8], float4& bv, int ch) {
        // columns 2l (acc0) and 2l + 1 (acc1) of the 8 rows; the FMAs are
        // ordered so that the 16 accumulators' chains interleave
        float acc0[SR], acc1[SR];
#pragma unroll
        for (int r = 0; r < SR; r++) acc0[r] = acc1[r] = 0.f;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            float4 sv[SR];
#pragma unroll
            for (int r = 0; r < SR; r++) sv[r] = *reinterpret_cast<const float4*>(&S[r][16 * warp + 4 * q]);
            const float4 lo = av[2 * q], hi = av[2 * q + 1];   // k = 16w + 4q .. +3
#pragma unroll
            for (int r = 0; r < SR; r++) { acc0[r] = fmaf(sv[r].x, lo.x, acc0[r]); acc1[r] = fmaf(sv[r].x, lo.y, acc1[r]); }
#pragma unroll
            for (int r = 0; r < SR; r++) { acc0[r] = fmaf(sv[r].y, lo.z, acc0[r]); acc1[r] = fmaf(sv[r].y, lo.w, acc1[r]); }
#pragma unroll
            for (int r = 0; r < SR; r++) { acc0[r] = fmaf(sv[r].z, hi.x, acc0[r]); acc1[r] = fmaf(sv[r].z, hi.y, acc1[r]); }
#pragma unroll
            for (int r = 0; r < SR; r++) { acc0[r] = fmaf(sv[r].w, hi.z, acc0[r]); acc1[r] = fmaf(sv[r].w, hi.w, acc1[r]); }
        }
#pragma unroll
        for (int r = 0; r < SR; r++)
            *reinterpret_cast<float2*>(&P[warp][r][2 * lane]) = make_float2(acc0[r], acc1[r]);
        __syncthreads();   // partial products complete; every warp is done reading S
        float4 n = bv;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const float4 p = *reinterpret_cast<const float4*>(&P[w][rr][c4]);
            n.x += p.x; n.y += p.y; n.z += p.z; n.w += p.w;
        }
        *reinterpret_cast<float4*>(&S[rr][c4]) = n;
        float* dst = (ch + 1 < NC) ? S0ws + ((size_t)bh * NC + chunk_of(ch + 1)) * CN * CN
                                   : (h_out ? h_out + (size_t)bh * CN * CN : nullptr);
        if (dst) *reinterpret_cast<float4*>(dst + (size_t)(dv0 + rr) * CN + c4) = n;
        if (ckpt)
            *reinterpret_cast<float4*>(ckpt + ((size_t)bh * NC + chunk_of(ch)) * CN * CN + (size_t)(dv0 + rr) * CN + c4) = n;
        load(av, bv, ch + 3);
        __syncthreads();   // the new state is visible; P may be overwritten
    };
    for (int ch = 0; ch < NC; ch += 3) {
        chunk(a0, b0, ch);
        if (ch + 1 < NC) chunk(a1, b1, ch + 1);
        if (ch + 2 < NC) chunk(a2, b2, ch + 2);
    }
}


}  // namespace
}  // namespace rwkv
