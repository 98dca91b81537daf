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
#include "wkv7_chunk.cuh"

namespace rwkv {

namespace {

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


// ------------------------------------------------------------ out

constexpr int FT = 512;   // threads of the out kernel (two CTAs per SM)

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
__global__ void __launch_bounds__(FT, 2)
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
        float4 s4[CN * CN / 4 / FT];
#pragma unroll
        for (int i = 0; i < CN * CN / 4 / FT; i++) s4[i] = S0g[tid + FT * i];
        stage_chunk<T, CN, FT>(sm.rr, sm.ww, sm.kk, sm.aa, sm.bb, sm.vv, CQ, r, w, k, v, a, b, bi, hi, H, T_, t0, 0);
#pragma unroll
        for (int i = 0; i < CN * CN / 4 / FT; i++) {
            const int p = tid + FT * i, rr = p >> 4, c4 = (p & 15) * 4;
            sm.S[rr][c4] = s4[i].x; sm.S[rr][c4 + 1] = s4[i].y; sm.S[rr][c4 + 2] = s4[i].z; sm.S[rr][c4 + 3] = s4[i].w;
        }
    }
    __syncthreads();
    const float cmin = chunk_decay(sm.c, sm.ww, sm.red);
    auto out_index = [&](int t, int row) { return (((size_t)bi * T_ + t0 + t) * H + hi) * CN + row; };

    if (cmin < GUARD) {
        // token by token on all 64 rows: thread = (row, 16 columns), 4 threads per row
        // (threads 0-255; no barrier follows)
        if (tid >= 4 * CN) return;
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

    for (int e = tid; e < CL * CN; e += FT) {
        const int t = e / CN, c = e % CN;
        const float ct = sm.c[t + 1][c];
        sm.At[t][c] = sm.aa[t][c] * sm.c[t][c];
        sm.Rt[t][c] = sm.rr[t][c] * ct;
        sm.Kh[t][c] = sm.kk[t][c] / ct;
        sm.Bh[t][c] = sm.bb[t][c] / ct;
    }
    __syncthreads();
    // [Bh; Kh; S] (96 x 64) x [A~; R~]^T (64 x 32): 6 x 4 = 24 tiles, 3 per warp
    for (int tile = warp; tile < 24; tile += FT / 32) {
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
        for (int tile = warp - 2; tile < 16; tile += FT / 32 - 2) {
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
    // U = X2 Z: 8 tiles, one per warp of warps 0-7
    if (warp < 8) tile_64x16(sm.U, sm.X2, sm.Zb[zb], nullptr, (warp >> 1) * 16, (warp & 1) * 8, lane);
    __syncthreads();
    // Y += U Nb -> y (and sa = U): 8 tiles, one per warp of warps 0-7
    if (warp < 8) {
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

// y, h_out (nullable), sa (nullable, fp32 [B,T,H,64]) and ckpt (nullable, the
// state after every chunk, [B,H,NC,64,64]) from the chunked form; workspace of
// wkv7_chunk_workspace bytes.
int launch_wkv7_chunk_fwd(int dtype, const void* r, const void* w, const void* k, const void* v,
                          const void* a, const void* b, const float* h_in, void* y, float* h_out,
                          float* sa, float* ckpt, int B, int T_, int H, void* workspace, cudaStream_t st) {
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
        wkv7_chunk_scan_kernel<<<dim3(B * H, CN / SR), ST, 0, st>>>(h_in, Aws, Bws, S0ws, h_out, ckpt, NC, 0);
        if (int rc = check_launch("wkv7_chunk_scan_kernel")) return rc;
        out<<<dim3(NC, B * H), FT, sizeof(OutSmem), st>>>(
            (const T*)r, (const T*)w, (const T*)k, (const T*)v, (const T*)a, (const T*)b, S0ws, (T*)y, sa,
            T_, H, NC);
        return check_launch("wkv7_chunk_out_kernel");
    });
}

}  // namespace rwkv
