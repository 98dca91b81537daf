// WKV-7 recurrence, sequential-in-T kernels (sm_100a).
//
// The recurrence per (batch b, head h) with state S[dv, dk] (fp32):
//   sa = S a;   S <- S diag(w) + v k^T + sa b^T;   y = S r
// (Sources/RWKVKernel/WKV7Reference.swift:47-74).  Rows of S evolve
// independently given the step's (w, k, a, b), so a head's 64 rows are split
// over CTAs: each CTA owns 16 rows, 4 lanes per row, 16 key columns per lane,
// the state slice living in registers for the whole sequence.  The step's
// shared vectors (r, w, k, a, b) and the CTA's v entries for 16 steps are
// streamed into shared memory with cp.async, double-buffered, so the global
// loads of step chunk c+1 overlap the arithmetic of chunk c.
//
// These kernels serve the forward (wkv7SequenceForward), the training forward
// with its sa / 16-step checkpoint outputs (wkv7TrainWithState), and the
// one-token decode step with its fused tail (wkv7StepForward + wkvTail).
#include "common.cuh"

namespace rwkv {

constexpr int HN = 64;       // head size (WKV7_HEAD_SIZE)
constexpr int CHUNK = 16;    // checkpoint cadence (WKV7_CHUNK)
constexpr int RPC = 16;      // state rows per CTA
constexpr int LPR = 4;       // lanes per row
constexpr int CPL = HN / LPR;  // key columns per lane (16)
constexpr int SEQ_THREADS = RPC * LPR;  // 64

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    int n = valid ? 16 : 0;  // zero-fill past the end of the sequence
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Shared staging of one 16-step chunk, raw element type T.
template <typename T>
struct SeqStage {
    T vec[5][CHUNK][HN];  // r, w, k, a, b
    T v[CHUNK][RPC];      // this CTA's rows of v
};

template <typename T>
__device__ __forceinline__ void stage_chunk(SeqStage<T>& st, const T* const* src, const T* v,
                                            int bi, int hi, int t0, int T_, int H, int dv0) {
    constexpr int EPG = 16 / sizeof(T);        // elements per 16-byte granule
    constexpr int GPV = HN / EPG;              // granules per 64-vector
    constexpr int NG = 5 * CHUNK * GPV;        // granules for r,w,k,a,b
    for (int gi = threadIdx.x; gi < NG; gi += SEQ_THREADS) {
        int which = gi / (CHUNK * GPV);
        int rem = gi % (CHUNK * GPV);
        int t = rem / GPV, g = rem % GPV;
        int tt = t0 + t;
        bool valid = tt < T_;
        size_t base = (((size_t)bi * T_ + (valid ? tt : 0)) * H + hi) * HN + g * EPG;
        cp_async16(&st.vec[which][t][g * EPG], src[which] + base, valid);
    }
    constexpr int GPR = RPC / EPG;  // granules per 16-row slice of v
    for (int gi = threadIdx.x; gi < CHUNK * GPR; gi += SEQ_THREADS) {
        int t = gi / GPR, g = gi % GPR;
        int tt = t0 + t;
        bool valid = tt < T_;
        size_t base = (((size_t)bi * T_ + (valid ? tt : 0)) * H + hi) * HN + dv0 + g * EPG;
        cp_async16(&st.v[t][g * EPG], v + base, valid);
    }
}

// Sequence forward.  grid (B*H, HN/RPC), block 64.
template <typename T>
__global__ void __launch_bounds__(SEQ_THREADS)
wkv7_seq_fwd_kernel(const T* __restrict__ r, const T* __restrict__ w, const T* __restrict__ k,
                    const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                    const float* __restrict__ h_in, T* __restrict__ y, float* __restrict__ h_out,
                    float* __restrict__ sa_out, float* __restrict__ h_ckpt, int T_, int H) {
    __shared__ __align__(16) SeqStage<T> st[2];
    const int bh = blockIdx.x, bi = bh / H, hi = bh % H;
    const int dv0 = blockIdx.y * RPC;
    const int rl = threadIdx.x / LPR, q = threadIdx.x % LPR;
    const int dv = dv0 + rl;
    const int c0 = q * CPL;

    float s[CPL];
    const size_t hb = (size_t)bh * HN * HN + (size_t)dv * HN + c0;
    if (h_in) {
#pragma unroll
        for (int j = 0; j < CPL; j += 4) {
            float4 t4 = *reinterpret_cast<const float4*>(h_in + hb + j);
            s[j] = t4.x; s[j + 1] = t4.y; s[j + 2] = t4.z; s[j + 3] = t4.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < CPL; j++) s[j] = 0.f;
    }

    const T* src[5] = {r, w, k, a, b};
    const int nch = (T_ + CHUNK - 1) / CHUNK;
    const int NC = T_ / CHUNK;
    stage_chunk(st[0], src, v, bi, hi, 0, T_, H, dv0);
    cp_async_commit();
    for (int c = 0; c < nch; c++) {
        if (c + 1 < nch) stage_chunk(st[(c + 1) & 1], src, v, bi, hi, (c + 1) * CHUNK, T_, H, dv0);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const SeqStage<T>& cs = st[c & 1];
        const int steps = min(CHUNK, T_ - c * CHUNK);
        for (int t = 0; t < steps; t++) {
            const T* rr = cs.vec[0][t] + c0;
            const T* ww = cs.vec[1][t] + c0;
            const T* kk = cs.vec[2][t] + c0;
            const T* aa = cs.vec[3][t] + c0;
            const T* bb = cs.vec[4][t] + c0;
            float sa0 = 0.f, sa1 = 0.f;
#pragma unroll
            for (int j = 0; j < CPL; j += 2) {
                sa0 = fmaf(s[j], to_f(aa[j]), sa0);
                sa1 = fmaf(s[j + 1], to_f(aa[j + 1]), sa1);
            }
            float sa = group_sum<LPR>(sa0 + sa1);
            const float vv = to_f(cs.v[t][rl]);
            float y0 = 0.f, y1 = 0.f;
#pragma unroll
            for (int j = 0; j < CPL; j++) {
                s[j] = fmaf(to_f(ww[j]), s[j], fmaf(vv, to_f(kk[j]), sa * to_f(bb[j])));
                if (j & 1) y1 = fmaf(s[j], to_f(rr[j]), y1);
                else y0 = fmaf(s[j], to_f(rr[j]), y0);
            }
            float yy = group_sum<LPR>(y0 + y1);
            const int tt = c * CHUNK + t;
            if (q == 0) {
                size_t o = (((size_t)bi * T_ + tt) * H + hi) * HN + dv;
                y[o] = from_f<T>(yy);
                if (sa_out) sa_out[o] = sa;
            }
            if (h_ckpt && ((tt + 1) % CHUNK) == 0) {
                const int cc = (tt + 1) / CHUNK - 1;
                float* dst = h_ckpt + (((size_t)bh * NC + cc) * HN + dv) * HN + c0;
#pragma unroll
                for (int j = 0; j < CPL; j += 4)
                    *reinterpret_cast<float4*>(dst + j) = make_float4(s[j], s[j + 1], s[j + 2], s[j + 3]);
            }
        }
        __syncthreads();  // the buffer just read is refilled by the next iteration
    }
    cp_async_wait<0>();
    if (h_out) {
#pragma unroll
        for (int j = 0; j < CPL; j += 4)
            *reinterpret_cast<float4*>(h_out + hb + j) = make_float4(s[j], s[j + 1], s[j + 2], s[j + 3]);
    }
}

// One decode step for `rows` independent rows, optionally with the fused tmix
// tail.  grid (rows*H), block 256: 4 lanes per state row (16 key columns
// each), 64 rows -- the lane layout and summation order of the sequence
// kernel, so a step equals the forward at T = 1 bit for bit.  The head's
// vectors are staged in shared memory with 4 floats of padding after every
// 32, so the four 16-column segments of a row (q = 0..3) fall in distinct
// bank groups and a lane reads its columns with 16-byte loads.
__device__ __forceinline__ int vpad(int c) { return c + ((c >> 5) << 2); }

template <typename T, bool TAIL>
__global__ void __launch_bounds__(256)
wkv7_step_kernel(const T* __restrict__ r, const T* __restrict__ w, const T* __restrict__ k,
                 const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                 float* __restrict__ h, T* __restrict__ y, const float* __restrict__ rk,
                 const float* __restrict__ lnw, const float* __restrict__ lnb,
                 const float* __restrict__ g, float* __restrict__ out, int H, float eps) {
    constexpr int VP = HN + 8;
    __shared__ __align__(16) float r_s[VP], w_s[VP], k_s[VP], a_s[VP], b_s[VP];
    __shared__ __align__(16) float v_s[HN], ysh[HN], rk_s[HN], lw_s[HN], lb_s[HN], g_s[HN];
    const int rh = blockIdx.x;  // row*H + head
    const int hi = rh % H;
    const int dv = threadIdx.x / LPR, q = threadIdx.x % LPR, c0 = q * CPL;
    float* hp = h + (size_t)rh * HN * HN + (size_t)dv * HN + c0;
    const size_t vb = (size_t)rh * HN, hb = (size_t)hi * HN;

    // state loads first; meanwhile the head's vectors (and the tail's
    // parameters) go to shared memory, one column per thread
    float s[CPL];
#pragma unroll
    for (int j = 0; j < CPL; j += 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(hp + j);
        s[j] = t4.x; s[j + 1] = t4.y; s[j + 2] = t4.z; s[j + 3] = t4.w;
    }
    {
        const int c = threadIdx.x & (HN - 1), cp = vpad(c);
        switch (threadIdx.x >> 6) {
            case 0: r_s[cp] = to_f(r[vb + c]); w_s[cp] = to_f(w[vb + c]); break;
            case 1: k_s[cp] = to_f(k[vb + c]); v_s[c] = to_f(v[vb + c]); break;
            case 2: a_s[cp] = to_f(a[vb + c]); b_s[cp] = to_f(b[vb + c]); break;
            default:
                if (TAIL) { rk_s[c] = rk[hb + c]; lw_s[c] = lnw[hb + c]; lb_s[c] = lnb[hb + c]; g_s[c] = g[vb + c]; }
        }
    }
    __syncthreads();
    const int cb = vpad(c0);  // a lane's 16 columns are contiguous after padding
    float sa0 = 0.f, sa1 = 0.f;
#pragma unroll
    for (int j = 0; j < CPL; j += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(a_s + cb + j);
        sa0 = fmaf(s[j], a4.x, sa0);
        sa1 = fmaf(s[j + 1], a4.y, sa1);
        sa0 = fmaf(s[j + 2], a4.z, sa0);
        sa1 = fmaf(s[j + 3], a4.w, sa1);
    }
    const float sa = group_sum<LPR>(sa0 + sa1);
    const float vv = v_s[dv];
    float y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int j = 0; j < CPL; j += 4) {
        const float4 w4 = *reinterpret_cast<const float4*>(w_s + cb + j);
        const float4 k4 = *reinterpret_cast<const float4*>(k_s + cb + j);
        const float4 b4 = *reinterpret_cast<const float4*>(b_s + cb + j);
        const float4 r4 = *reinterpret_cast<const float4*>(r_s + cb + j);
        s[j] = fmaf(w4.x, s[j], fmaf(vv, k4.x, sa * b4.x));
        y0 = fmaf(s[j], r4.x, y0);
        s[j + 1] = fmaf(w4.y, s[j + 1], fmaf(vv, k4.y, sa * b4.y));
        y1 = fmaf(s[j + 1], r4.y, y1);
        s[j + 2] = fmaf(w4.z, s[j + 2], fmaf(vv, k4.z, sa * b4.z));
        y0 = fmaf(s[j + 2], r4.z, y0);
        s[j + 3] = fmaf(w4.w, s[j + 3], fmaf(vv, k4.w, sa * b4.w));
        y1 = fmaf(s[j + 3], r4.w, y1);
    }
    const float yy = group_sum<LPR>(y0 + y1);
#pragma unroll
    for (int j = 0; j < CPL; j += 4)
        *reinterpret_cast<float4*>(hp + j) = make_float4(s[j], s[j + 1], s[j + 2], s[j + 3]);
    if (!TAIL) {
        if (q == 0) y[vb + dv] = from_f<T>(yy);
        return;
    }
    if (q == 0) ysh[dv] = yy;
    __syncthreads();
    if (threadIdx.x >= 32) return;
    // Tail on one warp: two values per lane (WKV7DecodeKernels.swift:123-157).
    const int l = threadIdx.x, lp = vpad(l), lp2 = vpad(l + 32);
    const float x0 = ysh[l], x1 = ysh[l + 32];
    const float mean = warp_sum(x0 + x1) * (1.0f / HN);
    const float d0 = x0 - mean, d1 = x1 - mean;
    const float var = warp_sum(d0 * d0 + d1 * d1) * (1.0f / HN);
    const float inv = 1.0f / sqrtf(var + eps);
    const float dp = warp_sum(r_s[lp] * k_s[lp] * rk_s[l] + r_s[lp2] * k_s[lp2] * rk_s[l + 32]);
    out[vb + l] = (d0 * inv * lw_s[l] + lb_s[l] + dp * v_s[l]) * g_s[l];
    out[vb + l + 32] = (d1 * inv * lw_s[l + 32] + lb_s[l + 32] + dp * v_s[l + 32]) * g_s[l + 32];
}

// Standalone tail: one warp per (row, head), S % 32 == 0, S <= 256.
template <int PER>
__global__ void wkv_tail_kernel(const float* __restrict__ wkv, const float* __restrict__ r,
                                const float* __restrict__ k, const float* __restrict__ v,
                                const float* __restrict__ rk, const float* __restrict__ lnw,
                                const float* __restrict__ lnb, const float* __restrict__ g,
                                float* __restrict__ out, int nrh, int H, int S, float eps) {
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int l = threadIdx.x & 31;
    if (wid >= nrh) return;
    const int hi = wid % H;
    const size_t base = (size_t)wid * S, hb = (size_t)hi * S;
    float x[PER];
    float s1 = 0.f;
#pragma unroll
    for (int p = 0; p < PER; p++) {
        x[p] = wkv[base + l + 32 * p];
        s1 += x[p];
    }
    const float mean = warp_sum(s1) / (float)S;
    float s2 = 0.f, dp = 0.f;
#pragma unroll
    for (int p = 0; p < PER; p++) {
        const int i = l + 32 * p;
        const float d = x[p] - mean;
        s2 += d * d;
        dp += r[base + i] * k[base + i] * rk[hb + i];
    }
    const float inv = 1.0f / sqrtf(warp_sum(s2) / (float)S + eps);
    dp = warp_sum(dp);
#pragma unroll
    for (int p = 0; p < PER; p++) {
        const int i = l + 32 * p;
        out[base + i] = ((x[p] - mean) * inv * lnw[hb + i] + lnb[hb + i] + dp * v[base + i]) * g[base + i];
    }
}

// ---------------------------------------------------------------- backward
//
// One CTA per (b, h), 64 threads; thread i holds row i and column i of dS
// (the column-held scheme of WKV7Train.swift:247-330).  Instead of
// rebuilding earlier states by dividing by w, each 16-step chunk's states are
// recomputed from the chunk's starting state (h_in or the previous
// checkpoint) into a per-head scratch area of 17 states, read back
// column-wise during the reverse sweep.
constexpr int BWD_SLOTS = CHUNK + 1;

template <typename T>
__global__ void __launch_bounds__(HN)
wkv7_bwd_seq_kernel(const T* __restrict__ r, const T* __restrict__ w, const T* __restrict__ k,
                    const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                    const float* __restrict__ h_in, const float* __restrict__ h_ckpt,
                    const T* __restrict__ dy, const float* __restrict__ dh_out, T* __restrict__ dr,
                    T* __restrict__ dw, T* __restrict__ dk, T* __restrict__ dv,
                    T* __restrict__ da, T* __restrict__ db, float* __restrict__ dh_in, int T_,
                    int H, float* __restrict__ scratch) {
    __shared__ float sr[CHUNK][HN], sw[CHUNK][HN], sk[CHUNK][HN], sv[CHUNK][HN];
    __shared__ float sa_[CHUNK][HN], sb[CHUNK][HN], sdy[CHUNK][HN], ssa[CHUNK][HN];
    __shared__ float dsb_sh[HN];
    const int bh = blockIdx.x, bi = bh / H, hi = bh % H;
    const int i = threadIdx.x;
    const int NC = T_ / CHUNK;
    const size_t NN = (size_t)HN * HN;
    const size_t hb = (size_t)bh * NN;
    float* S = scratch + (size_t)bh * BWD_SLOTS * NN;

    float dst[HN], dstT[HN];
#pragma unroll
    for (int j = 0; j < HN; j++) {
        dst[j] = dh_out ? dh_out[hb + (size_t)i * HN + j] : 0.f;
        dstT[j] = dh_out ? dh_out[hb + (size_t)j * HN + i] : 0.f;
    }

    for (int c = NC - 1; c >= 0; c--) {
        for (int t = 0; t < CHUNK; t++) {
            const size_t base = (((size_t)bi * T_ + c * CHUNK + t) * H + hi) * HN + i;
            sr[t][i] = to_f(r[base]);
            sw[t][i] = to_f(w[base]);
            sk[t][i] = to_f(k[base]);
            sv[t][i] = to_f(v[base]);
            sa_[t][i] = to_f(a[base]);
            sb[t][i] = to_f(b[base]);
            sdy[t][i] = to_f(dy[base]);
        }
        // Recompute the chunk's states; thread i holds row i.
        {
            float row[HN];
            const float* s0 = (c == 0) ? (h_in ? h_in + hb : nullptr)
                                       : (h_ckpt + ((size_t)bh * NC + (c - 1)) * NN);
#pragma unroll
            for (int j = 0; j < HN; j++) row[j] = s0 ? s0[(size_t)i * HN + j] : 0.f;
            __syncthreads();
            float* d0 = S + (size_t)i * HN;
#pragma unroll
            for (int j = 0; j < HN; j += 4)
                *reinterpret_cast<float4*>(d0 + j) = make_float4(row[j], row[j + 1], row[j + 2], row[j + 3]);
            for (int t = 0; t < CHUNK; t++) {
                float s0a = 0.f, s1a = 0.f;
#pragma unroll
                for (int j = 0; j < HN; j += 2) {
                    s0a = fmaf(row[j], sa_[t][j], s0a);
                    s1a = fmaf(row[j + 1], sa_[t][j + 1], s1a);
                }
                const float sav = s0a + s1a;
                ssa[t][i] = sav;
                const float vi = sv[t][i];
#pragma unroll
                for (int j = 0; j < HN; j++)
                    row[j] = fmaf(sw[t][j], row[j], fmaf(vi, sk[t][j], sav * sb[t][j]));
                float* d = S + (size_t)(t + 1) * NN + (size_t)i * HN;
#pragma unroll
                for (int j = 0; j < HN; j += 4)
                    *reinterpret_cast<float4*>(d + j) = make_float4(row[j], row[j + 1], row[j + 2], row[j + 3]);
            }
        }
        __syncthreads();
        for (int t = CHUNK - 1; t >= 0; t--) {
            const float* Sn = S + (size_t)(t + 1) * NN;
            const float* Sp = S + (size_t)t * NN;
            const float dyi = sdy[t][i], ri = sr[t][i], wi = sw[t][i], ai = sa_[t][i];
            float drv = 0.f;
#pragma unroll
            for (int j = 0; j < HN; j++) drv = fmaf(Sn[(size_t)j * HN + i], sdy[t][j], drv);
#pragma unroll
            for (int j = 0; j < HN; j++) {
                dst[j] = fmaf(dyi, sr[t][j], dst[j]);
                dstT[j] = fmaf(ri, sdy[t][j], dstT[j]);
            }
            float dvv = 0.f, dsb = 0.f, dwv = 0.f, dkv = 0.f, dbv = 0.f;
#pragma unroll
            for (int j = 0; j < HN; j++) {
                dvv = fmaf(dst[j], sk[t][j], dvv);
                dsb = fmaf(dst[j], sb[t][j], dsb);
                dwv = fmaf(dstT[j], Sp[(size_t)j * HN + i], dwv);
                dkv = fmaf(dstT[j], sv[t][j], dkv);
                dbv = fmaf(dstT[j], ssa[t][j], dbv);
            }
            dsb_sh[i] = dsb;
            __syncthreads();
            float dav = 0.f;
#pragma unroll
            for (int j = 0; j < HN; j++) dav = fmaf(Sp[(size_t)j * HN + i], dsb_sh[j], dav);
#pragma unroll
            for (int j = 0; j < HN; j++) {
                dst[j] = fmaf(dst[j], sw[t][j], dsb * sa_[t][j]);
                dstT[j] = fmaf(dstT[j], wi, ai * dsb_sh[j]);
            }
            const size_t o = (((size_t)bi * T_ + c * CHUNK + t) * H + hi) * HN + i;
            dr[o] = from_f<T>(drv);
            dw[o] = from_f<T>(dwv);
            dk[o] = from_f<T>(dkv);
            dv[o] = from_f<T>(dvv);
            da[o] = from_f<T>(dav);
            db[o] = from_f<T>(dbv);
            __syncthreads();
        }
    }
    if (dh_in) {
#pragma unroll
        for (int j = 0; j < HN; j++) dh_in[hb + (size_t)i * HN + j] = dst[j];
    }
}

// ------------------------------------------------------------------ launchers

int launch_wkv7_seq(int dtype, const void* r, const void* w, const void* k, const void* v,
                    const void* a, const void* b, const float* h_in, void* y, float* h_out,
                    float* sa, float* h_ckpt, int B, int T_, int H, cudaStream_t st) {
    dim3 grid(B * H, HN / RPC);
    return dispatch_dtype(dtype, [&]<typename T>() {
        wkv7_seq_fwd_kernel<T><<<grid, SEQ_THREADS, 0, st>>>(
            (const T*)r, (const T*)w, (const T*)k, (const T*)v, (const T*)a, (const T*)b, h_in,
            (T*)y, h_out, sa, h_ckpt, T_, H);
        return check_launch("wkv7_seq_fwd_kernel");
    });
}

int launch_wkv7_step(int dtype, const void* r, const void* w, const void* k, const void* v,
                     const void* a, const void* b, float* h, void* y, int rows, int H,
                     cudaStream_t st) {
    return dispatch_dtype(dtype, [&]<typename T>() {
        wkv7_step_kernel<T, false><<<rows * H, 256, 0, st>>>(
            (const T*)r, (const T*)w, (const T*)k, (const T*)v, (const T*)a, (const T*)b, h,
            (T*)y, nullptr, nullptr, nullptr, nullptr, nullptr, H, 0.f);
        return check_launch("wkv7_step_kernel");
    });
}

int launch_wkv7_step_tail(const float* r, const float* w, const float* k, const float* v,
                          const float* a, const float* b, float* h, const float* rk,
                          const float* lnw, const float* lnb, const float* g, float* out,
                          int rows, int H, float eps, cudaStream_t st) {
    wkv7_step_kernel<float, true><<<rows * H, 256, 0, st>>>(r, w, k, v, a, b, h, nullptr, rk, lnw,
                                                           lnb, g, out, H, eps);
    return check_launch("wkv7_step_tail_kernel");
}

int launch_wkv_tail(const float* wkv, const float* r, const float* k, const float* v,
                    const float* rk, const float* lnw, const float* lnb, const float* g,
                    float* out, int rows, int H, int S, float eps, cudaStream_t st) {
    const int nrh = rows * H;
    const int threads = 256, blocks = ceil_div((int64_t)nrh * 32, threads);
    switch (S / 32) {
#define TAIL_CASE(P)                                                                       \
    case P:                                                                                \
        wkv_tail_kernel<P><<<blocks, threads, 0, st>>>(wkv, r, k, v, rk, lnw, lnb, g, out, \
                                                       nrh, H, S, eps);                    \
        break;
        TAIL_CASE(1) TAIL_CASE(2) TAIL_CASE(3) TAIL_CASE(4) TAIL_CASE(5) TAIL_CASE(6)
        TAIL_CASE(7) TAIL_CASE(8)
#undef TAIL_CASE
        default: return fail(RWKV_E_UNSUPPORTED, "wkv_tail: head size %d not in 32..256", S);
    }
    return check_launch("wkv_tail_kernel");
}

int64_t wkv7_bwd_seq_workspace(int B, int H) {
    return (int64_t)B * H * BWD_SLOTS * HN * HN * (int64_t)sizeof(float);
}

int launch_wkv7_bwd_seq(int dtype, const void* r, const void* w, const void* k, const void* v,
                        const void* a, const void* b, const float* h_in, const float* h_ckpt,
                        const void* dy, const float* dh_out, void* dr, void* dw, void* dk,
                        void* dv, void* da, void* db, float* dh_in, int B, int T_, int H,
                        float* scratch, cudaStream_t st) {
    return dispatch_dtype(dtype, [&]<typename T>() {
        wkv7_bwd_seq_kernel<T><<<B * H, HN, 0, st>>>(
            (const T*)r, (const T*)w, (const T*)k, (const T*)v, (const T*)a, (const T*)b, h_in,
            h_ckpt, (const T*)dy, dh_out, (T*)dr, (T*)dw, (T*)dk, (T*)dv, (T*)da, (T*)db, dh_in,
            T_, H, scratch);
        return check_launch("wkv7_bwd_seq_kernel");
    });
}

}  // namespace rwkv
