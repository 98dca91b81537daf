// Chunked (DPLR) WKV-7 forward for prefill.
//
// The recurrence per head (state S[dv, dk], 64 x 64, WKV7Reference.swift:47-74)
//     S_t = S_{t-1} (diag(w_t) + a_t b_t^T) + v_t k_t^T,   y_t = S_t r_t
// is evaluated 16 tokens at a time.  With c_t = w_1 ... w_t (elementwise
// cumulative decay inside the chunk, c_0 = 1) and
//     a~_t = a_t c_{t-1},  r~_t = r_t c_t,  b^_t = b_t / c_t,  k^_t = k_t / c_t,
// the chunk-normalised state S^_t = S_t diag(1/c_t) obeys
//     S^_t = S^_{t-1} + u_t b^_t^T + v_t k^_t^T,   u_t = S_{t-1} a_t,
// so, with M_b[j,t] = b^_j.a~_t, M_k[j,t] = k^_j.a~_t (j < t) and
// N_b[j,t] = b^_j.r~_t, N_k[j,t] = k^_j.r~_t (j <= t), Z = (I - M_b)^-1:
//     U = (S_0 A~ + V M_k) Z                     (u_t = the sequential "sa")
//     Y = S_0 R~ + U N_b + V N_k
//     S_16 = S_0 A_c + B_c,  A_c = diag(c_16) + A~^T Z B-,  B_c = (V M_k Z) B- + V K-,
// where B-_j = b_j c_16 / c_j and K-_j = k_j c_16 / c_j.  Z = (I + M)(I + M^2)
// (I + M^4)(I + M^8) since M_b is strictly triangular.
//
// Three launches:
//   prep  (chunk, head) in parallel: the chunk transition (A_c, B_c)
//   scan  (head, 8 state rows), sequential over chunks: S_{c+1} = S_c A_c + B_c
//         in fp32 FMAs; stores every chunk's start state
//   out   (chunk, head) in parallel: U and Y from the chunk's start state
// so the T-sequential depth is one 8 x 64 x 64 product per chunk.  The
// products of prep and out run on the tensor cores in 3xTF32 (x = hi + lo,
// hi*hi + hi*lo + lo*hi: about fp32 accuracy).  Every factor is bounded except 1/c_t: a chunk whose
// smallest c_16 is below 1e-30 (decays near zero) takes the sequential update
// token by token instead (prep builds A_c, B_c by stepping; out steps the
// state), so no division overflows.  A partial last chunk is padded with
// identity steps (w = 1, a = b = k = v = 0).
//
// Results equal the sequential kernels up to fp32 rounding (~1e-6 relative),
// not bitwise; the sequential entry points keep the reference's bitwise
// identities (step = forward at T = 1, split = contiguous).
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

__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
    const float rest = x - __uint_as_float(hi);
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(rest));
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
template <typename T, int NV>
__device__ __forceinline__ void stage_chunk(float (*rr)[CN], float (*ww)[CN], float (*kk)[CN],
                                            float (*aa)[CN], float (*bb)[CN], float* vv, int vstride,
                                            const T* r, const T* w, const T* k, const T* v,
                                            const T* a, const T* b, int bi, int hi, int H, int T_,
                                            int t0, int v0) {
    constexpr int PER = CL * CN / CT, VPER = CL * NV / CT;
    T lr[PER], lw[PER], lk[PER], la[PER], lb[PER], lv[VPER];
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = threadIdx.x + CT * i, tl = e / CN, c = e % CN, t = t0 + tl;
        const size_t o = (((size_t)bi * T_ + min(t, T_ - 1)) * H + hi) * CN + c;
        if (rr) lr[i] = r[o];
        lw[i] = w[o]; lk[i] = k[o]; la[i] = a[o]; lb[i] = b[o];
    }
#pragma unroll
    for (int i = 0; i < VPER; i++) {
        const int e = threadIdx.x + CT * i, tl = e / NV, d = e % NV, t = t0 + tl;
        lv[i] = v[(((size_t)bi * T_ + min(t, T_ - 1)) * H + hi) * CN + v0 + d];
    }
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = threadIdx.x + CT * i, tl = e / CN, c = e % CN;
        const bool in = t0 + tl < T_;
        if (rr) rr[tl][c] = in ? to_f(lr[i]) : 0.f;
        ww[tl][c] = in ? to_f(lw[i]) : 1.f;
        kk[tl][c] = in ? to_f(lk[i]) : 0.f;
        aa[tl][c] = in ? to_f(la[i]) : 0.f;
        bb[tl][c] = in ? to_f(lb[i]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < VPER; i++) {
        const int e = threadIdx.x + CT * i, tl = e / NV, d = e % NV;
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

// ------------------------------------------------------------ prep

struct PrepSmem {
    float ww[CL][CN], kk[CL][CN], aa[CL][CN], bb[CL][CN];
    float vv[CL * CQ];                                     // [token][dv], row stride CQ
    float c[CL + 1][CN];
    float At[CL][CP], Bh[CL][CP], Kh[CL][CP], Bb[CL][CQ], Kb[CL][CQ];
    float Mb[CL][LP], Mk[CL][LP], W[CL][LP];
    float Zb[2][CL][LP], Pb[2][CL][LP];
    float E[CN][LP], F[CN][LP];                            // [dk][t], [dv][t]
    float SA[CN][CP], SB[CN][CP];                          // token-by-token chunks only
    float red[2];
};

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

template <typename T>
__global__ void __launch_bounds__(CT)
wkv7_chunk_prep_kernel(const T* __restrict__ w, const T* __restrict__ k, const T* __restrict__ v,
                       const T* __restrict__ a, const T* __restrict__ b, float* __restrict__ Aws,
                       float* __restrict__ Bws, int T_, int H, int NC) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrepSmem& sm = *reinterpret_cast<PrepSmem*>(smem_raw);
    const int ch = blockIdx.x, bh = blockIdx.y, bi = bh / H, hi = bh % H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = ch * CL;
    float* Ag = Aws + ((size_t)bh * NC + ch) * CN * CN;
    float* Bg = Bws + ((size_t)bh * NC + ch) * CN * CN;
    stage_chunk<T, CN>(nullptr, sm.ww, sm.kk, sm.aa, sm.bb, sm.vv, CQ, nullptr, w, k, v, a, b, bi, hi,
                       H, T_, t0, 0);
    __syncthreads();
    const float cmin = chunk_decay(sm.c, sm.ww, sm.red);

    if (cmin < GUARD) {
        // step the transition (from I, v = 0) and the input part (from 0)
        for (int e = tid; e < CN * CN; e += CT) {
            const int i = e / CN, j = e % CN;
            sm.SA[i][j] = i == j ? 1.f : 0.f;
            sm.SB[i][j] = 0.f;
        }
        __syncthreads();
        for (int t = 0; t < CL; t++) {
            step_rows(sm.SA, CN, sm.ww, sm.kk, sm.aa, sm.bb, t, [](int) { return 0.f; });
            step_rows(sm.SB, CN, sm.ww, sm.kk, sm.aa, sm.bb, t, [&](int d) { return sm.vv[t * CQ + d]; });
            __syncthreads();
        }
        for (int e = tid; e < CN * CN; e += CT) {
            Ag[scan_a_index(e / CN, e % CN)] = sm.SA[e / CN][e % CN];
            Bg[e] = sm.SB[e / CN][e % CN];
        }
        return;
    }

    // normalised vectors
    for (int e = tid; e < CL * CN; e += CT) {
        const int t = e / CN, c = e % CN;
        const float ct = sm.c[t + 1][c], cl = sm.c[CL][c];
        const float kh = sm.kk[t][c] / ct, bhh = sm.bb[t][c] / ct;
        sm.At[t][c] = sm.aa[t][c] * sm.c[t][c];
        sm.Kh[t][c] = kh;
        sm.Bh[t][c] = bhh;
        sm.Kb[t][c] = kh * cl;
        sm.Bb[t][c] = bhh * cl;
    }
    __syncthreads();
    // Mb, Mk = [Bh; Kh] A~^T (strictly upper): 2 x 2 tiles, warps 0-3
    if (warp < 4) {
        const int mt = warp >> 1, n0 = (warp & 1) * 8, g = lane >> 2, t4 = lane & 3;
        const float (*Am)[CP] = mt == 0 ? sm.Bh : sm.Kh;
        float d[4] = {0.f, 0.f, 0.f, 0.f}, d3[3][4] = {};
#pragma unroll
        for (int k0 = 0; k0 < CN; k0 += 8) {
            const float af[4] = {Am[g][k0 + t4], Am[g + 8][k0 + t4], Am[g][k0 + t4 + 4], Am[g + 8][k0 + t4 + 4]};
            const float bf[2] = {sm.At[n0 + g][k0 + t4], sm.At[n0 + g][k0 + t4 + 4]};
            mma3x(d3, af, bf);
        }
        acc3_sum(d, d3);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int i = frag_i(0, lane, q), j = frag_j(n0, lane, q);
            (mt == 0 ? sm.Mb : sm.Mk)[i][j] = i < j ? d[q] : 0.f;
        }
    }
    __syncthreads();
    const int zb = z_chain(sm.Zb, sm.Pb, sm.Mb);
    const float (*Z)[LP] = sm.Zb[zb];
    if (warp == 0) mm16(sm.W, sm.Mk, Z, nullptr, lane);  // W = Mk Z
    // E = A~^T Z (64 x 16): 4 x 2 tiles, warps 0-7 (A[dk][j] = At[j][dk])
    {
        const int m0 = (warp >> 1) * 16, n0 = (warp & 1) * 8, g = lane >> 2, t4 = lane & 3;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k0 = 0; k0 < CL; k0 += 8) {
            const float af[4] = {sm.At[k0 + t4][m0 + g], sm.At[k0 + t4][m0 + g + 8],
                                 sm.At[k0 + t4 + 4][m0 + g], sm.At[k0 + t4 + 4][m0 + g + 8]};
            const float bf[2] = {Z[k0 + t4][n0 + g], Z[k0 + t4 + 4][n0 + g]};
            mma3(d, af, bf);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) sm.E[frag_i(m0, lane, q)][frag_j(n0, lane, q)] = d[q];
    }
    __syncthreads();
    // F = V W (64 x 16; V[dv][m] = vv[m][dv])
    {
        const int m0 = (warp >> 1) * 16, n0 = (warp & 1) * 8, g = lane >> 2, t4 = lane & 3;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k0 = 0; k0 < CL; k0 += 8) {
            const float af[4] = {sm.vv[(k0 + t4) * CQ + m0 + g], sm.vv[(k0 + t4) * CQ + m0 + g + 8],
                                 sm.vv[(k0 + t4 + 4) * CQ + m0 + g], sm.vv[(k0 + t4 + 4) * CQ + m0 + g + 8]};
            const float bf[2] = {sm.W[k0 + t4][n0 + g], sm.W[k0 + t4 + 4][n0 + g]};
            mma3(d, af, bf);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) sm.F[frag_i(m0, lane, q)][frag_j(n0, lane, q)] = d[q];
    }
    __syncthreads();
    // A_c = diag(c_16) + E B- ;  B_c = F B- + V K-   (64 x 64 each: 32 tiles each, 8 per warp)
    for (int tile = warp; tile < 64; tile += CT / 32) {
        const bool isA = tile < 32;
        const int tt = tile & 31, m0 = (tt >> 3) * 16, n0 = (tt & 7) * 8;
        const int g = lane >> 2, t4 = lane & 3;
        float d[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int i = frag_i(m0, lane, q), j = frag_j(n0, lane, q);
            d[q] = (isA && i == j) ? sm.c[CL][i] : 0.f;
        }
#pragma unroll
        for (int k0 = 0; k0 < 2 * CL; k0 += 8) {
            if (isA && k0 >= CL) break;
            float af[4], bf[2];
            if (k0 < CL) {
                const float (*Lm)[LP] = isA ? sm.E : sm.F;
                af[0] = Lm[m0 + g][k0 + t4]; af[1] = Lm[m0 + g + 8][k0 + t4];
                af[2] = Lm[m0 + g][k0 + t4 + 4]; af[3] = Lm[m0 + g + 8][k0 + t4 + 4];
                bf[0] = sm.Bb[k0 + t4][n0 + g]; bf[1] = sm.Bb[k0 + t4 + 4][n0 + g];
            } else {
                const int kk0 = k0 - CL;
                af[0] = sm.vv[(kk0 + t4) * CQ + m0 + g]; af[1] = sm.vv[(kk0 + t4) * CQ + m0 + g + 8];
                af[2] = sm.vv[(kk0 + t4 + 4) * CQ + m0 + g]; af[3] = sm.vv[(kk0 + t4 + 4) * CQ + m0 + g + 8];
                bf[0] = sm.Kb[kk0 + t4][n0 + g]; bf[1] = sm.Kb[kk0 + t4 + 4][n0 + g];
            }
            mma3(d, af, bf);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int i = frag_i(m0, lane, q), j = frag_j(n0, lane, q);
            if (isA) Ag[scan_a_index(i, j)] = d[q];
            else Bg[i * CN + j] = d[q];
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
constexpr int SR = 8;     // state rows per scan CTA
constexpr int ST = 128;   // scan threads

__global__ void __launch_bounds__(ST)
wkv7_chunk_scan_kernel(const float* __restrict__ h_in, const float* __restrict__ Aws,
                       const float* __restrict__ Bws, float* __restrict__ S0ws,
                       float* __restrict__ h_out, int NC) {
    __shared__ __align__(16) float S[SR][CN];      // state rows (broadcast reads)
    __shared__ __align__(16) float P[4][SR][CN];   // per-warp partial products
    const int bh = blockIdx.x, dv0 = blockIdx.y * SR;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rr = tid >> 4, c4 = (tid & 15) * 4;   // this thread's 4 state entries
    constexpr int CH4 = CN * CN / 4;                // float4 per chunk matrix
    {
        const float4 s = h_in ? *reinterpret_cast<const float4*>(h_in + ((size_t)bh * CN + dv0 + rr) * CN + c4)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(&S[rr][c4]) = s;
        *reinterpret_cast<float4*>(S0ws + (size_t)bh * NC * CN * CN + (size_t)(dv0 + rr) * CN + c4) = s;
    }
    const float4* Ab = reinterpret_cast<const float4*>(Aws + (size_t)bh * NC * CN * CN) + warp * 8 * 32 + lane;
    const float4* Bb = reinterpret_cast<const float4*>(Bws + (size_t)bh * NC * CN * CN + (size_t)(dv0 + rr) * CN + c4);
    float4 a0[8], a1[8], a2[8], b0, b1, b2;
    auto load = [&](float4 (&av)[8], float4& bv, int ch) {
        if (ch < NC) {
#pragma unroll
            for (int i = 0; i < 8; i++) av[i] = __ldcg(Ab + (size_t)ch * CH4 + i * 32);
            bv = __ldcg(Bb + (size_t)ch * CH4);
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
        float* dst = (ch + 1 < NC) ? S0ws + ((size_t)bh * NC + ch + 1) * CN * CN
                                   : (h_out ? h_out + (size_t)bh * CN * CN : nullptr);
        if (dst) *reinterpret_cast<float4*>(dst + (size_t)(dv0 + rr) * CN + c4) = n;
        load(av, bv, ch + 3);
        __syncthreads();   // the new state is visible; P may be overwritten
    };
    for (int ch = 0; ch < NC; ch += 3) {
        chunk(a0, b0, ch);
        if (ch + 1 < NC) chunk(a1, b1, ch + 1);
        if (ch + 2 < NC) chunk(a2, b2, ch + 2);
    }
}

// ------------------------------------------------------------ out

struct OutSmem {
    float rr[CL][CN], ww[CL][CN], kk[CL][CN], aa[CL][CN], bb[CL][CN];
    float vv[CL * CQ];                                     // [token][dv] (column-read)
    float c[CL + 1][CN];
    float At[CL][CP], Rt[CL][CP], Bh[CL][CP], Kh[CL][CP];  // row-read operands
    float Mb[CL][LP], Mk[CL][LP], Nb[CL][LP], Nk[CL][LP];
    float Zb[2][CL][LP], Pb[2][CL][LP];
    float S[CN][CP];                                       // chunk start state, all 64 rows
    float X[CN][LP], Y[CN][LP], X2[CN][LP], U[CN][LP];     // [dv][token]
    float red[2];
};

// Y (64 x 16 slice at (m0, n0)) of C = Cin + A B with A [64][LP] row-read and
// B [16][LP] column-read, K = 16 (one 16 x 8 tile per call).
__device__ __forceinline__ void tile_64x16(float (*C)[LP], const float (*A)[LP], const float (*B)[LP],
                                           const float (*Cin)[LP], int m0, int n0, int lane) {
    const int g = lane >> 2, t4 = lane & 3;
    float d[4];
#pragma unroll
    for (int q = 0; q < 4; q++) d[q] = Cin ? Cin[frag_i(m0, lane, q)][frag_j(n0, lane, q)] : 0.f;
#pragma unroll
    for (int k0 = 0; k0 < CL; k0 += 8) {
        const float af[4] = {A[m0 + g][k0 + t4], A[m0 + g + 8][k0 + t4], A[m0 + g][k0 + t4 + 4], A[m0 + g + 8][k0 + t4 + 4]};
        const float bf[2] = {B[k0 + t4][n0 + g], B[k0 + t4 + 4][n0 + g]};
        mma3(d, af, bf);
    }
#pragma unroll
    for (int q = 0; q < 4; q++) C[frag_i(m0, lane, q)][frag_j(n0, lane, q)] = d[q];
}

// The chunk's outputs from its start state: CTA = (chunk, head), all 64 rows.
template <typename T>
__global__ void __launch_bounds__(CT)
wkv7_chunk_out_kernel(const T* __restrict__ r, const T* __restrict__ w, const T* __restrict__ k,
                      const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                      const float* __restrict__ S0ws, T* __restrict__ y, float* __restrict__ sa_out,
                      int T_, int H, int NC) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    OutSmem& sm = *reinterpret_cast<OutSmem*>(smem_raw);
    const int ch = blockIdx.x, bh = blockIdx.y, bi = bh / H, hi = bh % H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int t0 = ch * CL;
    {
        // start state (16 floats per thread) with the chunk inputs: one wait on memory
        const float4* S0g = reinterpret_cast<const float4*>(S0ws + ((size_t)bh * NC + ch) * CN * CN);
        float4 s4[4];
#pragma unroll
        for (int i = 0; i < 4; i++) s4[i] = S0g[tid + CT * i];
        stage_chunk<T, CN>(sm.rr, sm.ww, sm.kk, sm.aa, sm.bb, sm.vv, CQ, r, w, k, v, a, b, bi, hi, H, T_, t0, 0);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int p = tid + CT * i, rr = p >> 4, c4 = (p & 15) * 4;
            sm.S[rr][c4] = s4[i].x; sm.S[rr][c4 + 1] = s4[i].y; sm.S[rr][c4 + 2] = s4[i].z; sm.S[rr][c4 + 3] = s4[i].w;
        }
    }
    __syncthreads();
    const float cmin = chunk_decay(sm.c, sm.ww, sm.red);
    auto out_index = [&](int t, int row) { return (((size_t)bi * T_ + t0 + t) * H + hi) * CN + row; };

    if (cmin < GUARD) {
        // token by token on all 64 rows: thread = (row, 16 columns), 4 threads per row
        const int rr = tid >> 2, c0 = 16 * (tid & 3);
        for (int t = 0; t < CL; t++) {
            float sa = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) sa = fmaf(sm.S[rr][c0 + j], sm.aa[t][c0 + j], sa);
            sa = group_sum<4>(sa);
            const float vd = sm.vv[t * CQ + rr];
            float yy = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int c = c0 + j;
                const float sn = fmaf(sm.ww[t][c], sm.S[rr][c], fmaf(vd, sm.kk[t][c], sa * sm.bb[t][c]));
                sm.S[rr][c] = sn;
                yy = fmaf(sn, sm.rr[t][c], yy);
            }
            yy = group_sum<4>(yy);
            if ((tid & 3) == 0 && t0 + t < T_) {
                y[out_index(t, rr)] = from_f<T>(yy);
                if (sa_out) sa_out[out_index(t, rr)] = sa;
            }
        }
        return;
    }

    for (int e = tid; e < CL * CN; e += CT) {
        const int t = e / CN, c = e % CN;
        const float ct = sm.c[t + 1][c];
        sm.At[t][c] = sm.aa[t][c] * sm.c[t][c];
        sm.Rt[t][c] = sm.rr[t][c] * ct;
        sm.Kh[t][c] = sm.kk[t][c] / ct;
        sm.Bh[t][c] = sm.bb[t][c] / ct;
    }
    __syncthreads();
    // [Bh; Kh; S] (96 x 64) x [A~; R~]^T (64 x 32): 6 x 4 = 24 tiles, 3 per warp
    for (int tile = warp; tile < 24; tile += CT / 32) {
        const int mt = tile >> 2, nt = tile & 3;
        const float (*Am)[CP] = mt == 0 ? sm.Bh : mt == 1 ? sm.Kh : sm.S + 16 * (mt - 2);
        const float (*Bm)[CP] = nt < 2 ? sm.At : sm.Rt;
        const int n0 = (nt & 1) * 8;
        float d[4] = {0.f, 0.f, 0.f, 0.f}, d3[3][4] = {};
#pragma unroll
        for (int k0 = 0; k0 < CN; k0 += 8) {
            const float af[4] = {Am[g][k0 + t4], Am[g + 8][k0 + t4], Am[g][k0 + t4 + 4], Am[g + 8][k0 + t4 + 4]};
            const float bf[2] = {Bm[n0 + g][k0 + t4], Bm[n0 + g][k0 + t4 + 4]};
            mma3x(d3, af, bf);
        }
        acc3_sum(d, d3);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int i = frag_i(0, lane, q), j = frag_j(n0, lane, q);
            if (mt >= 2) (nt < 2 ? sm.X : sm.Y)[16 * (mt - 2) + i][j] = d[q];
            else if (nt < 2) (mt == 0 ? sm.Mb : sm.Mk)[i][j] = i < j ? d[q] : 0.f;
            else (mt == 0 ? sm.Nb : sm.Nk)[i][j] = i <= j ? d[q] : 0.f;
        }
    }
    __syncthreads();
    // warps 2-7, beside the Z chain of warps 0-1: X2 = X + V Mk, Y += V Nk
    // (V[dv][m] = vv[m][dv]: 16 tiles of 16 x 8)
    if (warp >= 2)
        for (int tile = warp - 2; tile < 16; tile += 6) {
            const bool isX = tile < 8;
            const int tt = tile & 7, m0 = (tt >> 1) * 16, n0 = (tt & 1) * 8;
            const float (*Bm)[LP] = isX ? sm.Mk : sm.Nk;
            float (*Cm)[LP] = isX ? sm.X : sm.Y;
            float d[4];
#pragma unroll
            for (int q = 0; q < 4; q++) d[q] = Cm[frag_i(m0, lane, q)][frag_j(n0, lane, q)];
#pragma unroll
            for (int k0 = 0; k0 < CL; k0 += 8) {
                const float af[4] = {sm.vv[(k0 + t4) * CQ + m0 + g], sm.vv[(k0 + t4) * CQ + m0 + g + 8],
                                     sm.vv[(k0 + t4 + 4) * CQ + m0 + g], sm.vv[(k0 + t4 + 4) * CQ + m0 + g + 8]};
                const float bf[2] = {Bm[k0 + t4][n0 + g], Bm[k0 + t4 + 4][n0 + g]};
                mma3(d, af, bf);
            }
#pragma unroll
            for (int q = 0; q < 4; q++) (isX ? sm.X2 : sm.Y)[frag_i(m0, lane, q)][frag_j(n0, lane, q)] = d[q];
        }
    const int zb = z_chain(sm.Zb, sm.Pb, sm.Mb);
    // U = X2 Z: 8 tiles, one per warp
    tile_64x16(sm.U, sm.X2, sm.Zb[zb], nullptr, (warp >> 1) * 16, (warp & 1) * 8, lane);
    __syncthreads();
    // Y += U Nb -> y (and sa = U): 8 tiles, one per warp
    {
        const int m0 = (warp >> 1) * 16, n0 = (warp & 1) * 8;
        float d[4];
#pragma unroll
        for (int q = 0; q < 4; q++) d[q] = sm.Y[frag_i(m0, lane, q)][frag_j(n0, lane, q)];
#pragma unroll
        for (int k0 = 0; k0 < CL; k0 += 8) {
            const float af[4] = {sm.U[m0 + g][k0 + t4], sm.U[m0 + g + 8][k0 + t4], sm.U[m0 + g][k0 + t4 + 4],
                                 sm.U[m0 + g + 8][k0 + t4 + 4]};
            const float bf[2] = {sm.Nb[k0 + t4][n0 + g], sm.Nb[k0 + t4 + 4][n0 + g]};
            mma3(d, af, bf);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int i = frag_i(m0, lane, q), j = frag_j(n0, lane, q);
            if (t0 + j < T_) {
                y[out_index(j, i)] = from_f<T>(d[q]);
                if (sa_out) sa_out[out_index(j, i)] = sm.U[i][j];
            }
        }
    }
}

}  // namespace

int64_t wkv7_chunk_workspace(int B, int T_, int H) {
    const int64_t NC = (T_ + CL - 1) / CL;
    return 3 * (int64_t)B * H * NC * CN * CN * (int64_t)sizeof(float);
}

// y, h_out (nullable) and sa (nullable, fp32 [B,T,H,64]) from the chunked form;
// workspace of wkv7_chunk_workspace bytes.
int launch_wkv7_chunk_fwd(int dtype, const void* r, const void* w, const void* k, const void* v,
                          const void* a, const void* b, const float* h_in, void* y, float* h_out,
                          float* sa, int B, int T_, int H, void* workspace, cudaStream_t st) {
    const int NC = (T_ + CL - 1) / CL;
    const size_t per = (size_t)B * H * NC * CN * CN;
    float* Aws = static_cast<float*>(workspace);
    float* Bws = Aws + per;
    float* S0ws = Bws + per;
    return dispatch_dtype(dtype, [&]<typename T>() {
        auto prep = wkv7_chunk_prep_kernel<T>;
        auto out = wkv7_chunk_out_kernel<T>;
        cudaError_t e = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PrepSmem));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(out, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(OutSmem));
        if (e != cudaSuccess) return fail(RWKV_E_CUDA, "wkv7 chunked: %s", cudaGetErrorString(e));
        prep<<<dim3(NC, B * H), CT, sizeof(PrepSmem), st>>>((const T*)w, (const T*)k, (const T*)v,
                                                            (const T*)a, (const T*)b, Aws, Bws, T_, H, NC);
        if (int rc = check_launch("wkv7_chunk_prep_kernel")) return rc;
        wkv7_chunk_scan_kernel<<<dim3(B * H, CN / SR), ST, 0, st>>>(h_in, Aws, Bws, S0ws, h_out, NC);
        if (int rc = check_launch("wkv7_chunk_scan_kernel")) return rc;
        out<<<dim3(NC, B * H), CT, sizeof(OutSmem), st>>>(
            (const T*)r, (const T*)w, (const T*)k, (const T*)v, (const T*)a, (const T*)b, S0ws, (T*)y, sa,
            T_, H, NC);
        return check_launch("wkv7_chunk_out_kernel");
    });
}

}  // namespace rwkv
