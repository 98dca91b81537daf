// Chunked (DPLR) WKV-7 backward.
//
// With D_t = dL/dS_t (rows dv, columns dk), the reverse recurrence is
//     D_{t-1} = D_t G_t^T + dy_{t-1} r_{t-1}^T,   G_t = diag(w_t) + a_t b_t^T,
// the same diagonal-plus-low-rank form as the forward run backwards in time.
// Per 16-token chunk, in the forward's chunk-normalised notation (c_t the
// cumulative decay, a~ = a c_{t-1}, r~ = r c_t, b^ = b / c_t, k^ = k / c_t,
// M_b, M_k strict and N_b, N_k inclusive dot matrices, Z = (I - M_b)^-1,
// B- = b^ c_16, K- = k^ c_16), and Q the gradient reaching the chunk's end
// state from later chunks:
//     the gradient into the chunk's start state   Q' = Q A_c^T + DY B'
//         with B' = R~ + (Z N_b)^T A~   (depends on r, w, a, b only)
//     e_t = D_t b_t:                   E  = (Q B-^T + DY N_b^T) Z^T
//     u_t = S_{t-1} a_t (forward):     U  = (S_0 A~^T + V M_k) Z
//     dv_t = D_t k_t:                  dV = Q K-^T + DY N_k^T + E M_k^T
//     dr_t = S_t^T dy_t    = c_t     (S_0^T dy_t + sum_{j<=t} b^_j (u_j.dy_t) + k^_j (v_j.dy_t))
//     da_t = S_{t-1}^T e_t = c_{t-1} (S_0^T e_t  + sum_{j<t}  b^_j (u_j.e_t)  + k^_j (v_j.e_t))
//     dk_t = D_t^T v_t     = (c_16 Q^T v_t + sum_{m>=t} r~_m (dy_m.v_t) + sum_{m>t} a~_m (e_m.v_t)) / c_t
//     db_t = D_t^T u_t     = (c_16 Q^T u_t + sum_{m>=t} r~_m (dy_m.u_t) + sum_{m>t} a~_m (e_m.u_t)) / c_t
//     dw_t = diag(S_{t-1}^T D_t), expanded into the same products (below)
// so a chunk's gradients need only its start state S_0 (the forward's
// checkpoint) and Q.  Three launches:
//   prep  (chunk, head): A_c^T (in the scan's order) and C_c = DY B'
//   scan  the forward's scan kernel in reverse: Q_{c-1} = Q_c A_c^T + C_c from
//         d_h_out, storing every chunk's Q; the last one is d_h_in
//   out   (chunk, head): every gradient of the chunk's 16 tokens
// Products run in 3xTF32 on the tensor cores.  A chunk whose smallest c_16 is
// below 1e-30 is done token by token (states recomputed from S_0), as in the
// forward.  T % 16 == 0 (the training path's condition).
//
// Matches the sequential backward (recompute from checkpoints, no division by
// w: WKV7Train.swift:234-339 semantics) to fp32 rounding; deterministic (no
// atomics, fixed reduction orders).
#include "wkv7_chunk.cuh"

namespace rwkv {
namespace {

// ------------------------------------------------------------ generic tiles

// d (the 16 x 8 tile of C at (m0, n0), fragment order) += A B over k < K, with
// A(i, k) = A[i * ai + k * ak] and B(k, j) = B[k * bk + j * bj]; 3xTF32.
template <int K>
__device__ __forceinline__ void gtile(float* d, const float* A, int ai, int ak, const float* B, int bk,
                                      int bj, int m0, int n0, int lane) {
    const int g = lane >> 2, t4 = lane & 3;
    float d3[3][4] = {};
#pragma unroll
    for (int k0 = 0; k0 < K; k0 += 8) {
        const float af[4] = {A[(m0 + g) * ai + (k0 + t4) * ak], A[(m0 + g + 8) * ai + (k0 + t4) * ak],
                             A[(m0 + g) * ai + (k0 + t4 + 4) * ak], A[(m0 + g + 8) * ai + (k0 + t4 + 4) * ak]};
        const float bf[2] = {B[(k0 + t4) * bk + (n0 + g) * bj], B[(k0 + t4 + 4) * bk + (n0 + g) * bj]};
        mma3x(d3, af, bf);
    }
    acc3_sum(d, d3);
}

// One product C (M x N) = [Cin +] A B, element (i, j) of C at C[i * ci + j * cj]
// (Cin the same layout, may be C itself or NULL).
struct MM {
    const float* A;
    int ai, ak;
    const float* B;
    int bk, bj;
    float* C;
    const float* Cin;
    int ci, cj, M, N;
};

// Several products with the same K, their 16 x 8 tiles spread over the CTA's
// warps (the products must not write each other's inputs).  No barrier.
template <int K, int NJ>
__device__ __forceinline__ void run_mm(const MM (&jobs)[NJ]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    int base = 0;
#pragma unroll
    for (int jb = 0; jb < NJ; jb++) {
        const MM m = jobs[jb];
        const int tn = m.N >> 3, tiles = (m.M >> 4) * tn;
        for (int tile = ((warp - base) % nw + nw) % nw; tile < tiles; tile += nw) {
            const int m0 = (tile / tn) * 16, n0 = (tile % tn) * 8;
            float d[4];
#pragma unroll
            for (int q = 0; q < 4; q++)
                d[q] = m.Cin ? m.Cin[frag_i(m0, lane, q) * m.ci + frag_j(n0, lane, q) * m.cj] : 0.f;
            gtile<K>(d, m.A, m.ai, m.ak, m.B, m.bk, m.bj, m0, n0, lane);
#pragma unroll
            for (int q = 0; q < 4; q++) m.C[frag_i(m0, lane, q) * m.ci + frag_j(n0, lane, q) * m.cj] = d[q];
        }
        base += tiles;
    }
}

// Stage the listed token tensors of the chunk ([t][channel], row stride
// CP; NULL pointers are skipped), every load before the first store.
template <typename T, int NT, int NTH = CT>
__device__ __forceinline__ void stage_tokens(float* const (&dst)[NT], const T* const (&src)[NT], int bi,
                                             int hi, int H, int T_, int t0) {
    constexpr int PER = CL * CN / NTH;
    T l[NT][PER];
#pragma unroll
    for (int n = 0; n < NT; n++)
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int e = threadIdx.x + NTH * i, tl = e / CN, c = e % CN;
            if (src[n]) l[n][i] = src[n][(((size_t)bi * T_ + t0 + tl) * H + hi) * CN + c];
        }
#pragma unroll
    for (int n = 0; n < NT; n++)
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int e = threadIdx.x + NTH * i, tl = e / CN, c = e % CN;
            if (src[n]) dst[n][tl * CP + c] = to_f(l[n][i]);
        }
}

// Suffix decay d_t = w_{t+1} ... w_15 (d_15 = 1) for threads 0-63; no barrier.
__device__ __forceinline__ void suffix_decay(float (*dsuf)[CN], const float (*ww)[CP]) {
    if (threadIdx.x < CN) {
        const int i = threadIdx.x;
        float d = 1.f;
        dsuf[CL - 1][i] = 1.f;
        for (int t = CL - 2; t >= 0; t--) {
            d *= ww[t + 1][i];
            dsuf[t][i] = d;
        }
    }
}

// c_0 .. c_16 (chunk_decay's layout, from a CP-strided w) and the smallest
// c_16; ends with a barrier.
__device__ __forceinline__ float chunk_decay_p(float (*c)[CN], const float (*ww)[CP], float* red) {
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

struct BPrepSmem {
    float rr[CL][CP], ww[CL][CP], aa[CL][CP], bb[CL][CP], dd[CL][CP];   // dd: dy [t][dv]
    float c[CL + 1][CN];
    float At[CL][CP], Rt[CL][CP], Bh[CL][CP], Bb[CL][CP];
    float Mb[CL][LP], Nb[CL][LP], ZN[CL][LP];
    float Zb[2][CL][LP], Pb[2][CL][LP];
    float ZB[CL][CP], Bp[CL][CP];
    float SA[CN][CP], SC[CN][CP];                                        // token-by-token chunks
    float red[2];
};

template <typename T>
__global__ void __launch_bounds__(CT)
wkv7_chunk_bwd_prep_kernel(const T* __restrict__ r, const T* __restrict__ w, const T* __restrict__ a,
                           const T* __restrict__ b, const T* __restrict__ dy, float* __restrict__ Aws,
                           float* __restrict__ Cws, int T_, int H, int NC) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    BPrepSmem& sm = *reinterpret_cast<BPrepSmem*>(smem_raw);
    const int ch = blockIdx.x, bh = blockIdx.y, bi = bh / H, hi = bh % H, tid = threadIdx.x;
    const int t0 = ch * CL;
    float* Ag = Aws + ((size_t)bh * NC + ch) * CN * CN;
    float* Cg = Cws + ((size_t)bh * NC + ch) * CN * CN;
    {
        float* const dst[5] = {&sm.rr[0][0], &sm.ww[0][0], &sm.aa[0][0], &sm.bb[0][0], &sm.dd[0][0]};
        const T* const src[5] = {r, w, a, b, dy};
        stage_tokens<T, 5>(dst, src, bi, hi, H, T_, t0);
    }
    __syncthreads();
    const float cmin = chunk_decay_p(sm.c, sm.ww, sm.red);

    if (cmin < GUARD) {
        // A_c by stepping from I; C_c = sum_t dy_t r_t^T G_t^T .. G_1^T by the
        // reverse steps C <- (C + dy_t r_t^T) G_t^T from 0.  Thread = (row, 16 cols).
        for (int e = tid; e < CN * CN; e += CT) {
            const int i = e / CN, j = e % CN;
            sm.SA[i][j] = i == j ? 1.f : 0.f;
        }
        __syncthreads();
        const int rr = tid >> 2, c0 = 16 * (tid & 3);
        for (int t = 0; t < CL; t++) {
            float sa = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) sa = fmaf(sm.SA[rr][c0 + j], sm.aa[t][c0 + j], sa);
            sa = group_sum<4>(sa);
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int c = c0 + j;
                sm.SA[rr][c] = fmaf(sm.ww[t][c], sm.SA[rr][c], sa * sm.bb[t][c]);
            }
        }
        float C[16];
#pragma unroll
        for (int j = 0; j < 16; j++) C[j] = 0.f;
        for (int t = CL - 1; t >= 0; t--) {
            const float dv = sm.dd[t][rr];
            float e = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                C[j] = fmaf(dv, sm.rr[t][c0 + j], C[j]);
                e = fmaf(C[j], sm.bb[t][c0 + j], e);
            }
            e = group_sum<4>(e);
#pragma unroll
            for (int j = 0; j < 16; j++) C[j] = fmaf(sm.ww[t][c0 + j], C[j], e * sm.aa[t][c0 + j]);
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
            sm.SC[rr][c0 + j] = C[j];
        }
        __syncthreads();
        for (int e = tid; e < CN * CN; e += CT) {
            const int i = e / CN, j = e % CN;
            Ag[scan_a_index(j, i)] = sm.SA[i][j];
            Cg[e] = sm.SC[i][j];
        }
        return;
    }

    for (int e = tid; e < CL * CN; e += CT) {
        const int t = e / CN, c = e % CN;
        const float ct = sm.c[t + 1][c];
        sm.At[t][c] = sm.aa[t][c] * sm.c[t][c];
        sm.Rt[t][c] = sm.rr[t][c] * ct;
        const float bh = sm.bb[t][c] / ct;
        sm.Bh[t][c] = bh;
        sm.Bb[t][c] = bh * sm.c[CL][c];
    }
    __syncthreads();
    {
        const MM jobs[2] = {
            {&sm.Bh[0][0], CP, 1, &sm.At[0][0], 1, CP, &sm.Mb[0][0], nullptr, LP, 1, CL, CL},
            {&sm.Bh[0][0], CP, 1, &sm.Rt[0][0], 1, CP, &sm.Nb[0][0], nullptr, LP, 1, CL, CL}};
        run_mm<CN>(jobs);
    }
    __syncthreads();
    for (int e = tid; e < CL * CL; e += CT) {
        const int j = e / CL, t = e % CL;
        if (j >= t) sm.Mb[j][t] = 0.f;
        if (j > t) sm.Nb[j][t] = 0.f;
    }
    __syncthreads();
    const int zb = z_chain(sm.Zb, sm.Pb, sm.Mb);
    const float* Z = &sm.Zb[zb][0][0];
    {
        // ZB = Z B- (16 x 64), ZN = Z N_b (16 x 16)
        const MM jobs[2] = {{Z, LP, 1, &sm.Bb[0][0], CP, 1, &sm.ZB[0][0], nullptr, CP, 1, CL, CN},
                            {Z, LP, 1, &sm.Nb[0][0], LP, 1, &sm.ZN[0][0], nullptr, LP, 1, CL, CL}};
        run_mm<CL>(jobs);
    }
    __syncthreads();
    {
        // B' = R~ + ZN^T A~ (16 x 64)
        const MM jobs[1] = {{&sm.ZN[0][0], 1, LP, &sm.At[0][0], CP, 1, &sm.Bp[0][0], &sm.Rt[0][0], CP, 1, CL, CN}};
        run_mm<CL>(jobs);
    }
    // A_c = diag(c_16) + A~^T ZB, stored transposed in the scan's order (32 tiles)
    {
        const int warp = tid >> 5, lane = tid & 31;
        for (int tile = warp; tile < 32; tile += CT / 32) {
            const int m0 = (tile >> 3) * 16, n0 = (tile & 7) * 8;
            float d[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int i = frag_i(m0, lane, q), j = frag_j(n0, lane, q);
                d[q] = i == j ? sm.c[CL][i] : 0.f;
            }
            gtile<CL>(d, &sm.At[0][0], 1, CP, &sm.ZB[0][0], CP, 1, m0, n0, lane);
#pragma unroll
            for (int q = 0; q < 4; q++) Ag[scan_a_index(frag_j(n0, lane, q), frag_i(m0, lane, q))] = d[q];
        }
    }
    __syncthreads();
    // C_c = DY B' (64 x 64; DY(dv, m) = dd[m][dv])
    {
        const int warp = tid >> 5, lane = tid & 31;
        for (int tile = warp; tile < 32; tile += CT / 32) {
            const int m0 = (tile >> 3) * 16, n0 = (tile & 7) * 8;
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            gtile<CL>(d, &sm.dd[0][0], 1, CP, &sm.Bp[0][0], CP, 1, m0, n0, lane);
#pragma unroll
            for (int q = 0; q < 4; q++) Cg[frag_i(m0, lane, q) * CN + frag_j(n0, lane, q)] = d[q];
        }
    }
}

// ------------------------------------------------------------ out

constexpr int BT = 512;   // threads of the out kernel (16 warps: its products are latency bound)

struct BOutSmem {
    float rr[CL][CP], ww[CL][CP], kk[CL][CP], vv[CL][CP], aa[CL][CP], bb[CL][CP], dd[CL][CP];
    float c[CL + 1][CN], dsuf[CL][CN];
    float At[CL][CP], Rt[CL][CP], Kh[CL][CP], Bh[CL][CP], Kb[CL][CP], Bb[CL][CP];
    float S[CN][CP], Q[CN][CP];
    float Mb[CL][LP], Mk[CL][LP], Nb[CL][LP], Nk[CL][LP];
    float Zb[2][CL][LP], Pb[2][CL][LP];
    float Pudy[CL][LP], Pvdy[CL][LP], Pue[CL][LP], Pve[CL][LP];
    float Lm[8][CL][LP];                          // masked / transposed dot matrices
    // [64][16] products ([dv][t] or [dk][t])
    float X[CN][LP], U[CN][LP], F[CN][LP], E[CN][LP], G2[CN][LP];
    float SDY[CN][LP], SE[CN][LP], QU[CN][LP], QV[CN][LP];
    float dR[CN][LP], dA[CN][LP], Xk[CN][LP], Xb[CN][LP];
    float q0[CN];
    float red[2];
};

// Token-by-token backward of one chunk from S_0 (sm.S) and Q (sm.Q): D runs
// backwards from Q; S_{t-1} is recomputed from S_0 for every t.  Thread =
// (row, 16 columns); the sums over rows go through `buf` in a fixed order.
template <typename T>
__device__ void chunk_bwd_tokens(BOutSmem& sm, float (*buf)[CN + 1], T* dr, T* dw, T* dk, T* dv, T* da,
                                 T* db, size_t base, int H) {
    // threads 0-255 work (row, 16 columns); the others only take the barriers
    const int tid = threadIdx.x, rr = (tid >> 2) & (CN - 1), c0 = 16 * (tid & 3);
    const bool act = tid < 4 * CN;
    float D[16], Sp[16], Sn[16];
#pragma unroll
    for (int j = 0; j < 16; j++) D[j] = sm.Q[rr][c0 + j];
    auto out = [&](int t, int c) { return base + ((size_t)t * H) * CN + c; };
    for (int t = CL - 1; t >= 0; t--) {
        const float dyr = sm.dd[t][rr], vr = sm.vv[t][rr];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            D[j] = fmaf(dyr, sm.rr[t][c0 + j], D[j]);
            Sp[j] = sm.S[rr][c0 + j];
        }
        for (int s = 0; s < t; s++) {
            float sa = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) sa = fmaf(Sp[j], sm.aa[s][c0 + j], sa);
            sa = group_sum<4>(sa);
            const float vs = sm.vv[s][rr];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int c = c0 + j;
                Sp[j] = fmaf(sm.ww[s][c], Sp[j], fmaf(vs, sm.kk[s][c], sa * sm.bb[s][c]));
            }
        }
        float sa = 0.f, e = 0.f, dvr = 0.f;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            sa = fmaf(Sp[j], sm.aa[t][c0 + j], sa);
            e = fmaf(D[j], sm.bb[t][c0 + j], e);
            dvr = fmaf(D[j], sm.kk[t][c0 + j], dvr);
        }
        sa = group_sum<4>(sa);
        e = group_sum<4>(e);
        dvr = group_sum<4>(dvr);
        if (act && (tid & 3) == 0) dv[out(t, rr)] = from_f<T>(dvr);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int c = c0 + j;
            Sn[j] = fmaf(sm.ww[t][c], Sp[j], fmaf(vr, sm.kk[t][c], sa * sm.bb[t][c]));
        }
        // the five sums over rows: dr = sum S_t dy, dk = sum D v, da = sum S_{t-1} e,
        // db = sum D sa, dw = sum S_{t-1} o D
        for (int q = 0; q < 5; q++) {
#pragma unroll
            for (int j = 0; j < 16; j++) {
                float x;
                if (q == 0) x = Sn[j] * dyr;
                else if (q == 1) x = D[j] * vr;
                else if (q == 2) x = Sp[j] * e;
                else if (q == 3) x = D[j] * sa;
                else x = Sp[j] * D[j];
                if (act) buf[rr][c0 + j] = x;
            }
            __syncthreads();
            if (tid < CN) {
                float s = 0.f;
                for (int i = 0; i < CN; i++) s += buf[i][tid];
                T* dst = q == 0 ? dr : q == 1 ? dk : q == 2 ? da : q == 3 ? db : dw;
                dst[out(t, tid)] = from_f<T>(s);
            }
            __syncthreads();
        }
#pragma unroll
        for (int j = 0; j < 16; j++) D[j] = fmaf(sm.ww[t][c0 + j], D[j], e * sm.aa[t][c0 + j]);
    }
}

template <typename T>
__global__ void __launch_bounds__(BT)
wkv7_chunk_bwd_out_kernel(const T* __restrict__ r, const T* __restrict__ w, const T* __restrict__ k,
                          const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                          const T* __restrict__ dy, const float* __restrict__ h_in,
                          const float* __restrict__ h_ckpt, const float* __restrict__ Qws,
                          T* __restrict__ dr, T* __restrict__ dw, T* __restrict__ dk, T* __restrict__ dv,
                          T* __restrict__ da, T* __restrict__ db, int T_, int H, int NC) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    BOutSmem& sm = *reinterpret_cast<BOutSmem*>(smem_raw);
    const int ch = blockIdx.x, bh = blockIdx.y, bi = bh / H, hi = bh % H, tid = threadIdx.x;
    const int t0 = ch * CL;
    {
        // S_0 (the previous chunk's checkpoint, or h_in) and Q, with the chunk inputs
        const float* S0g = ch > 0 ? h_ckpt + ((size_t)bh * NC + ch - 1) * CN * CN
                                  : (h_in ? h_in + (size_t)bh * CN * CN : nullptr);
        const float4* Qg = reinterpret_cast<const float4*>(Qws + ((size_t)bh * NC + ch) * CN * CN);
        float4 s4[CN * CN / 4 / BT], q4[CN * CN / 4 / BT];
#pragma unroll
        for (int i = 0; i < CN * CN / 4 / BT; i++) {
            s4[i] = S0g ? reinterpret_cast<const float4*>(S0g)[tid + BT * i] : make_float4(0.f, 0.f, 0.f, 0.f);
            q4[i] = Qg[tid + BT * i];
        }
        float* const dst[7] = {&sm.rr[0][0], &sm.ww[0][0], &sm.kk[0][0], &sm.vv[0][0],
                               &sm.aa[0][0], &sm.bb[0][0], &sm.dd[0][0]};
        const T* const src[7] = {r, w, k, v, a, b, dy};
        stage_tokens<T, 7, BT>(dst, src, bi, hi, H, T_, t0);
#pragma unroll
        for (int i = 0; i < CN * CN / 4 / BT; i++) {
            const int p = tid + BT * i, row = p >> 4, c4 = (p & 15) * 4;
            *reinterpret_cast<float4*>(&sm.S[row][c4]) = s4[i];
            *reinterpret_cast<float4*>(&sm.Q[row][c4]) = q4[i];
        }
    }
    __syncthreads();
    const float cmin = chunk_decay_p(sm.c, sm.ww, sm.red);
    const size_t base = (((size_t)bi * T_ + t0) * H + hi) * CN;   // token 0, channel 0 of this chunk
    auto out = [&](int t, int c) { return base + ((size_t)t * H) * CN + c; };

    if (cmin < GUARD) {
        chunk_bwd_tokens<T>(sm, reinterpret_cast<float (*)[CN + 1]>(&sm.X[0][0]), dr, dw, dk, dv, da, db,
                            base, H);
        return;
    }

    suffix_decay(sm.dsuf, sm.ww);
    for (int e = tid; e < CL * CN; e += BT) {
        const int t = e / CN, c = e % CN;
        const float ct = sm.c[t + 1][c], c16 = sm.c[CL][c];
        sm.At[t][c] = sm.aa[t][c] * sm.c[t][c];
        sm.Rt[t][c] = sm.rr[t][c] * ct;
        const float kh = sm.kk[t][c] / ct, bh = sm.bb[t][c] / ct;
        sm.Kh[t][c] = kh;
        sm.Bh[t][c] = bh;
        sm.Kb[t][c] = kh * c16;
        sm.Bb[t][c] = bh * c16;
    }
    if (tid < CN) {
        float s = 0.f;
        for (int i = 0; i < CN; i++) s = fmaf(sm.S[i][tid], sm.Q[i][tid], s);
        sm.q0[tid] = s;
    }
    __syncthreads();
    {
        // K = 64: the dot matrices, S_0 A~^T, Q B-^T, Q K-^T, S_0^T DY, Q^T V, V^T DY
        const MM jobs[10] = {
            {&sm.Bh[0][0], CP, 1, &sm.At[0][0], 1, CP, &sm.Mb[0][0], nullptr, LP, 1, CL, CL},
            {&sm.Kh[0][0], CP, 1, &sm.At[0][0], 1, CP, &sm.Mk[0][0], nullptr, LP, 1, CL, CL},
            {&sm.Bh[0][0], CP, 1, &sm.Rt[0][0], 1, CP, &sm.Nb[0][0], nullptr, LP, 1, CL, CL},
            {&sm.Kh[0][0], CP, 1, &sm.Rt[0][0], 1, CP, &sm.Nk[0][0], nullptr, LP, 1, CL, CL},
            {&sm.S[0][0], CP, 1, &sm.At[0][0], 1, CP, &sm.X[0][0], nullptr, LP, 1, CN, CL},
            {&sm.Q[0][0], CP, 1, &sm.Bb[0][0], 1, CP, &sm.F[0][0], nullptr, LP, 1, CN, CL},
            {&sm.Q[0][0], CP, 1, &sm.Kb[0][0], 1, CP, &sm.G2[0][0], nullptr, LP, 1, CN, CL},
            {&sm.S[0][0], 1, CP, &sm.dd[0][0], 1, CP, &sm.SDY[0][0], nullptr, LP, 1, CN, CL},
            {&sm.Q[0][0], 1, CP, &sm.vv[0][0], 1, CP, &sm.QV[0][0], nullptr, LP, 1, CN, CL},
            {&sm.vv[0][0], CP, 1, &sm.dd[0][0], 1, CP, &sm.Pvdy[0][0], nullptr, LP, 1, CL, CL}};
        run_mm<CN>(jobs);
    }
    __syncthreads();
    for (int e = tid; e < CL * CL; e += BT) {
        const int j = e / CL, t = e % CL;
        if (j >= t) { sm.Mb[j][t] = 0.f; sm.Mk[j][t] = 0.f; }
        if (j > t) { sm.Nb[j][t] = 0.f; sm.Nk[j][t] = 0.f; }
    }
    __syncthreads();
    // warps 2.. beside the Z chain: X += V M_k, F += DY N_b^T, G2 += DY N_k^T (K = 16)
    if ((tid >> 5) >= 2) {
        const int warp = (tid >> 5) - 2, lane = tid & 31;
        for (int tile = warp; tile < 24; tile += BT / 32 - 2) {
            const int p = tile >> 3, tt = tile & 7, m0 = (tt >> 1) * 16, n0 = (tt & 1) * 8;
            float (*C)[LP] = p == 0 ? sm.X : p == 1 ? sm.F : sm.G2;
            float d[4];
#pragma unroll
            for (int q = 0; q < 4; q++) d[q] = C[frag_i(m0, lane, q)][frag_j(n0, lane, q)];
            if (p == 0) gtile<CL>(d, &sm.vv[0][0], 1, CP, &sm.Mk[0][0], LP, 1, m0, n0, lane);
            else gtile<CL>(d, &sm.dd[0][0], 1, CP, p == 1 ? &sm.Nb[0][0] : &sm.Nk[0][0], 1, LP, m0, n0, lane);
#pragma unroll
            for (int q = 0; q < 4; q++) C[frag_i(m0, lane, q)][frag_j(n0, lane, q)] = d[q];
        }
    }
    const int zb = z_chain(sm.Zb, sm.Pb, sm.Mb);
    const float* Z = &sm.Zb[zb][0][0];
    {
        // U = X Z, E = F Z^T
        const MM jobs[2] = {{&sm.X[0][0], LP, 1, Z, LP, 1, &sm.U[0][0], nullptr, LP, 1, CN, CL},
                            {&sm.F[0][0], LP, 1, Z, 1, LP, &sm.E[0][0], nullptr, LP, 1, CN, CL}};
        run_mm<CL>(jobs);
    }
    __syncthreads();
    {
        // K = 64: Q^T U, S_0^T E, U^T DY, U^T E, V^T E
        const MM jobs[5] = {
            {&sm.Q[0][0], 1, CP, &sm.U[0][0], LP, 1, &sm.QU[0][0], nullptr, LP, 1, CN, CL},
            {&sm.S[0][0], 1, CP, &sm.E[0][0], LP, 1, &sm.SE[0][0], nullptr, LP, 1, CN, CL},
            {&sm.U[0][0], 1, LP, &sm.dd[0][0], 1, CP, &sm.Pudy[0][0], nullptr, LP, 1, CL, CL},
            {&sm.U[0][0], 1, LP, &sm.E[0][0], LP, 1, &sm.Pue[0][0], nullptr, LP, 1, CL, CL},
            {&sm.vv[0][0], CP, 1, &sm.E[0][0], LP, 1, &sm.Pve[0][0], nullptr, LP, 1, CL, CL}};
        run_mm<CN>(jobs);
    }
    __syncthreads();
    // masked copies: Lm[0..3] [j][t] for j <= t (udy, vdy) / j < t (ue, ve);
    // Lm[4..7] [m][t] = P[t][m] for m >= t (vdy, udy) / m > t (ve, ue)
    for (int e = tid; e < CL * CL; e += BT) {
        const int x = e / CL, t = e % CL;
        sm.Lm[0][x][t] = x <= t ? sm.Pudy[x][t] : 0.f;
        sm.Lm[1][x][t] = x <= t ? sm.Pvdy[x][t] : 0.f;
        sm.Lm[2][x][t] = x < t ? sm.Pue[x][t] : 0.f;
        sm.Lm[3][x][t] = x < t ? sm.Pve[x][t] : 0.f;
        sm.Lm[4][x][t] = x >= t ? sm.Pvdy[t][x] : 0.f;
        sm.Lm[5][x][t] = x > t ? sm.Pve[t][x] : 0.f;
        sm.Lm[6][x][t] = x >= t ? sm.Pudy[t][x] : 0.f;
        sm.Lm[7][x][t] = x > t ? sm.Pue[t][x] : 0.f;
    }
    __syncthreads();
    {
        // dV = G2 + E M_k^T; dR = SDY + B^^T Lm0; dA = SE + B^^T Lm2; Xk = R~^T Lm4; Xb = R~^T Lm6
        const MM jobs[5] = {
            {&sm.E[0][0], LP, 1, &sm.Mk[0][0], 1, LP, &sm.G2[0][0], &sm.G2[0][0], LP, 1, CN, CL},
            {&sm.Bh[0][0], 1, CP, &sm.Lm[0][0][0], LP, 1, &sm.dR[0][0], &sm.SDY[0][0], LP, 1, CN, CL},
            {&sm.Bh[0][0], 1, CP, &sm.Lm[2][0][0], LP, 1, &sm.dA[0][0], &sm.SE[0][0], LP, 1, CN, CL},
            {&sm.Rt[0][0], 1, CP, &sm.Lm[4][0][0], LP, 1, &sm.Xk[0][0], nullptr, LP, 1, CN, CL},
            {&sm.Rt[0][0], 1, CP, &sm.Lm[6][0][0], LP, 1, &sm.Xb[0][0], nullptr, LP, 1, CN, CL}};
        run_mm<CL>(jobs);
    }
    __syncthreads();
    {
        // dR += K^^T Lm1; dA += K^^T Lm3; Xk += A~^T Lm5; Xb += A~^T Lm7
        const MM jobs[4] = {
            {&sm.Kh[0][0], 1, CP, &sm.Lm[1][0][0], LP, 1, &sm.dR[0][0], &sm.dR[0][0], LP, 1, CN, CL},
            {&sm.Kh[0][0], 1, CP, &sm.Lm[3][0][0], LP, 1, &sm.dA[0][0], &sm.dA[0][0], LP, 1, CN, CL},
            {&sm.At[0][0], 1, CP, &sm.Lm[5][0][0], LP, 1, &sm.Xk[0][0], &sm.Xk[0][0], LP, 1, CN, CL},
            {&sm.At[0][0], 1, CP, &sm.Lm[7][0][0], LP, 1, &sm.Xb[0][0], &sm.Xb[0][0], LP, 1, CN, CL}};
        run_mm<CL>(jobs);
    }
    __syncthreads();
    // outputs but dw; thread = (channel, CL / (BT / 64) tokens)
    {
        constexpr int TG = BT / CN;   // token groups
        const int i = tid & (CN - 1), tq = tid / CN;
        const float c16 = sm.c[CL][i];
#pragma unroll
        for (int u = 0; u < CL / TG; u++) {
            const int t = tq + TG * u;
            const float ct = sm.c[t + 1][i];
            dr[out(t, i)] = from_f<T>(ct * sm.dR[i][t]);
            da[out(t, i)] = from_f<T>(sm.c[t][i] * sm.dA[i][t]);
            dk[out(t, i)] = from_f<T>((c16 * sm.QV[i][t] + sm.Xk[i][t]) / ct);
            db[out(t, i)] = from_f<T>((c16 * sm.QU[i][t] + sm.Xb[i][t]) / ct);
            dv[out(t, i)] = from_f<T>(sm.G2[i][t]);
        }
    }
    // dw_t = c_{t-1} d_t (q0 + sum_{j<t} b^_j Q^T u_j + k^_j Q^T v_j)
    //      + (1 / w_t) (sum_{m>=t} r~_m S_0^T dy_m + sum_{m>t} a~_m S_0^T e_m
    //        + sum_{j<t} [b^_j (sum_{m>=t} (u_j.dy_m) r~_m + sum_{m>t} (u_j.e_m) a~_m)
    //                   + k^_j (sum_{m>=t} (v_j.dy_m) r~_m + sum_{m>t} (v_j.e_m) a~_m)])
    // Thread = (channel i, rows j = 2g, 2g + 1 of the dot matrices), 8 per
    // channel in one warp; t runs down so that the inner sums over m are
    // running suffix sums; the 8 partial j-sums meet by shuffles.
    {
        static_assert(BT == 8 * CN, "eight threads per channel");
        const int i = 4 * (tid >> 5) + ((tid & 31) >> 3), jg = tid & 7, j0 = 2 * jg, j1 = j0 + 1;
        const float bh0 = sm.Bh[j0][i], bh1 = sm.Bh[j1][i], kh0 = sm.Kh[j0][i], kh1 = sm.Kh[j1][i];
        float s1[CL];   // prefix sums over j (the lane with jg == 0 uses them)
        s1[0] = sm.q0[i];
#pragma unroll
        for (int t = 0; t + 1 < CL; t++) s1[t + 1] = fmaf(sm.Bh[t][i], sm.QU[i][t], fmaf(sm.Kh[t][i], sm.QV[i][t], s1[t]));
        float sb0 = 0.f, sb1 = 0.f, sk0 = 0.f, sk1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int t = CL - 1; t >= 0; t--) {
            const float rt = sm.Rt[t][i];
            sb0 = fmaf(sm.Pudy[j0][t], rt, sb0);
            sk0 = fmaf(sm.Pvdy[j0][t], rt, sk0);
            sb1 = fmaf(sm.Pudy[j1][t], rt, sb1);
            sk1 = fmaf(sm.Pvdy[j1][t], rt, sk1);
            if (t + 1 < CL) {
                const float at = sm.At[t + 1][i];
                sb0 = fmaf(sm.Pue[j0][t + 1], at, sb0);
                sk0 = fmaf(sm.Pve[j0][t + 1], at, sk0);
                sb1 = fmaf(sm.Pue[j1][t + 1], at, sb1);
                sk1 = fmaf(sm.Pve[j1][t + 1], at, sk1);
            }
            float x = 0.f;
            if (j0 < t) x = fmaf(bh0, sb0, fmaf(kh0, sk0, x));
            if (j1 < t) x = fmaf(bh1, sb1, fmaf(kh1, sk1, x));
            x += __shfl_xor_sync(0xffffffffu, x, 1);
            x += __shfl_xor_sync(0xffffffffu, x, 2);
            x += __shfl_xor_sync(0xffffffffu, x, 4);
            if (jg == 0) {
                s2 = fmaf(rt, sm.SDY[i][t], s2);
                if (t + 1 < CL) s2 = fmaf(sm.At[t + 1][i], sm.SE[i][t + 1], s2);
                dw[out(t, i)] = from_f<T>(sm.c[t][i] * sm.dsuf[t][i] * s1[t] + (s2 + x) / sm.ww[t][i]);
            }
        }
    }
}

}  // namespace

int64_t wkv7_chunk_bwd_workspace(int B, int T_, int H) {
    const int64_t NC = T_ / CL;
    return 3 * (int64_t)B * H * NC * CN * CN * (int64_t)sizeof(float);
}

// Gradients of the chunked form; T % 16 == 0; workspace of
// wkv7_chunk_bwd_workspace bytes (A_c^T, C_c and Q per chunk and head).
int launch_wkv7_chunk_bwd(int dtype, const void* r, const void* w, const void* k, const void* v,
                          const void* a, const void* b, const float* h_in, const float* h_ckpt,
                          const void* dy, const float* dh_out, void* dr, void* dw, void* dk, void* dv,
                          void* da, void* db, float* dh_in, int B, int T_, int H, void* workspace,
                          cudaStream_t st) {
    const int NC = T_ / CL;
    const size_t per = (size_t)B * H * NC * CN * CN;
    float* Aws = static_cast<float*>(workspace);
    float* Cws = Aws + per;
    float* Qws = Cws + per;
    return dispatch_dtype(dtype, [&]<typename T>() {
        auto prep = wkv7_chunk_bwd_prep_kernel<T>;
        auto out = wkv7_chunk_bwd_out_kernel<T>;
        cudaError_t e = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(BPrepSmem));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(out, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(BOutSmem));
        if (e != cudaSuccess) return fail(RWKV_E_CUDA, "wkv7 chunked backward: %s", cudaGetErrorString(e));
        prep<<<dim3(NC, B * H), CT, sizeof(BPrepSmem), st>>>((const T*)r, (const T*)w, (const T*)a,
                                                             (const T*)b, (const T*)dy, Aws, Cws, T_, H, NC);
        if (int rc = check_launch("wkv7_chunk_bwd_prep_kernel")) return rc;
        wkv7_chunk_scan_kernel<<<dim3(B * H, CN / SR), ST, 0, st>>>(dh_out, Aws, Cws, Qws, dh_in, nullptr, NC, 1);
        if (int rc = check_launch("wkv7_chunk_scan_kernel")) return rc;
        out<<<dim3(NC, B * H), BT, sizeof(BOutSmem), st>>>(
            (const T*)r, (const T*)w, (const T*)k, (const T*)v, (const T*)a, (const T*)b, (const T*)dy, h_in,
            h_ckpt, Qws, (T*)dr, (T*)dw, (T*)dk, (T*)dv, (T*)da, (T*)db, T_, H, NC);
        return check_launch("wkv7_chunk_bwd_out_kernel");
    });
}

}  // namespace rwkv
