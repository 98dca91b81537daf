// Glue kernels of the x070 recurrent decode step (one token per row), the
// elementwise and reduction work between the projections:
//   embedding row (4-bit) + LayerNorm ln0        (X070Generation.swift:483-486)
//   ln1 + token shift + six lerps                (tmixStep, :201-230)
//   kk / k / v prep + WKV step + tail            (:258-291, fused)
//   ln2 + token shift + lerp                     (cmixStep, :310-316)
//   ln_out and greedy argmax                     (:496-497, GPUSampler.swift:90)
// One CTA per row (or per (row, head) for the WKV part); LayerNorm is the
// reference's manual fp32 formula (two passes: mean, then mean of squares of
// the deviations; eps 1e-5).
#pragma once

#include "common.cuh"

namespace rwkv {

constexpr int GLUE_T = 256;
constexpr int GLUE_PER = 16;  // values per thread: C <= 4096

__device__ __forceinline__ float block_sum256(float v, float* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    v = (threadIdx.x < GLUE_T / 32) ? sh[threadIdx.x] : 0.f;
    if (warp == 0) v = warp_sum(v);
    if (threadIdx.x == 0) sh[32] = v;
    __syncthreads();
    v = sh[32];
    __syncthreads();
    return v;
}

template <typename A>
__device__ __forceinline__ void st_act(A* p, float v) { *p = from_f<A>(v); }

// Row LayerNorm of v[] (thread holds columns tid + 256*i), in place.
__device__ __forceinline__ void ln_regs(float v[GLUE_PER], int C, const float* __restrict__ w,
                                        const float* __restrict__ b, float* sh) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < GLUE_PER; i++) {
        const int c = threadIdx.x + GLUE_T * i;
        if (c < C) s += v[i];
    }
    const float mean = block_sum256(s, sh) / (float)C;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < GLUE_PER; i++) {
        const int c = threadIdx.x + GLUE_T * i;
        if (c < C) {
            const float d = v[i] - mean;
            q += d * d;
        }
    }
    const float den = sqrtf(block_sum256(q, sh) / (float)C + 1e-5f);
#pragma unroll
    for (int i = 0; i < GLUE_PER; i++) {
        const int c = threadIdx.x + GLUE_T * i;
        if (c < C) v[i] = (v[i] - mean) / den * w[c] + b[c];
    }
}

// ids -> x = ln0(emb[id]).  Embedding in the 4-bit group-64 container
// (emb_wq != NULL) or dense bf16.
__global__ void __launch_bounds__(GLUE_T)
x070_embed_kernel(const int32_t* __restrict__ ids, const uint32_t* __restrict__ emb_wq,
                  const __half* __restrict__ emb_sc, const __half* __restrict__ emb_bi,
                  const __nv_bfloat16* __restrict__ emb_dense, const float* __restrict__ lnw,
                  const float* __restrict__ lnb, float* __restrict__ x, int C, int vocab) {
    pdl_wait();  // launched as a programmatic dependent: predecessor outputs first
    pdl_trigger();
    __shared__ float sh[33];
    const int n = blockIdx.x;
    int id = ids[n];
    id = min(max(id, 0), vocab - 1);
    float v[GLUE_PER];
#pragma unroll
    for (int i = 0; i < GLUE_PER; i++) {
        const int c = threadIdx.x + GLUE_T * i;
        v[i] = 0.f;
        if (c < C) {
            if (emb_wq) {
                const uint32_t word = emb_wq[(int64_t)id * (C / 8) + c / 8];
                const float q = (float)((word >> (4 * (c & 7))) & 15u);
                const int64_t gi = (int64_t)id * (C / 64) + c / 64;
                v[i] = q * __half2float(emb_sc[gi]) + __half2float(emb_bi[gi]);
            } else {
                v[i] = __bfloat162float(emb_dense[(int64_t)id * C + c]);
            }
        }
    }
    ln_regs(v, C, lnw, lnb, sh);
#pragma unroll
    for (int i = 0; i < GLUE_PER; i++) {
        const int c = threadIdx.x + GLUE_T * i;
        if (c < C) x[(int64_t)n * C + c] = v[i];
    }
}

// Row kernels over C channels with 16-byte accesses: thread t holds columns
// 4(t + 256 i) .. +3 for i < GV (C % 4 == 0, C <= 1024 GV).
template <int GV>
__device__ __forceinline__ void ld_row4(float4* d, const float* __restrict__ p, int C) {
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (threadIdx.x + GLUE_T * i);
        d[i] = c < C ? *reinterpret_cast<const float4*>(p + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Two-pass LayerNorm (eps 1e-5) of the row in v[], in place.
template <int GV>
__device__ __forceinline__ void ln_row4(float4* v, const float4* w, const float4* b, int C, float* sh) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < GV; i++)
        if (4 * (threadIdx.x + GLUE_T * i) < C) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = block_sum256(s, sh) / (float)C;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < GV; i++)
        if (4 * (threadIdx.x + GLUE_T * i) < C) {
            const float dx = v[i].x - mean, dy = v[i].y - mean, dz = v[i].z - mean, dw = v[i].w - mean;
            q += (dx * dx + dy * dy) + (dz * dz + dw * dw);
        }
    const float den = sqrtf(block_sum256(q, sh) / (float)C + 1e-5f);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        v[i].x = (v[i].x - mean) / den * w[i].x + b[i].x;
        v[i].y = (v[i].y - mean) / den * w[i].y + b[i].y;
        v[i].z = (v[i].z - mean) / den * w[i].z + b[i].z;
        v[i].w = (v[i].w - mean) / den * w[i].w + b[i].w;
    }
}

template <typename A>
__device__ __forceinline__ void st_act4(A* p, float4 v) {
    p[0] = from_f<A>(v.x); p[1] = from_f<A>(v.y); p[2] = from_f<A>(v.z); p[3] = from_f<A>(v.w);
}
__device__ __forceinline__ float4 lerp4(float4 xl, float4 xx, float4 c) {
    return make_float4(xl.x + xx.x * c.x, xl.y + xx.y * c.y, xl.z + xx.z * c.z, xl.w + xx.w * c.w);
}
__device__ __forceinline__ float4 sub4(float4 a, float4 b) {
    return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
}

// tmix input: xl = ln1(x); xx = shift - xl; shift = xl;
// mix[m] = xl + xx * coef[m] for m = r, w, k, v, a, g  ([6][R][C], act type).
// The weights (never written during a step) are loaded before the
// programmatic-launch wait; x and the shift row after it, in one round trip.
template <typename A, int GV>
__global__ void __launch_bounds__(GLUE_T)
x070_tmix_in_kernel(const float* __restrict__ x, const float* __restrict__ lnw,
                    const float* __restrict__ lnb, float* __restrict__ shift,
                    const float* __restrict__ coef, A* __restrict__ mix, int R, int C) {
    __shared__ float sh[33];
    const int n = blockIdx.x;
    float4 sv[GV], cf[6][GV], w4[GV], b4[GV], v[GV];
#pragma unroll
    for (int m = 0; m < 6; m++) ld_row4<GV>(cf[m], coef + m * C, C);
    ld_row4<GV>(w4, lnw, C);
    ld_row4<GV>(b4, lnb, C);
    // the shift row was last written by this kernel one step earlier
    ld_row4<GV>(sv, shift + (int64_t)n * C, C);
    pdl_wait();  // x: the previous kernel's output
    pdl_trigger();
    ld_row4<GV>(v, x + (int64_t)n * C, C);
    ln_row4<GV>(v, w4, b4, C, sh);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (threadIdx.x + GLUE_T * i);
        if (c >= C) continue;
        const int64_t o = (int64_t)n * C + c;
        const float4 xx = sub4(sv[i], v[i]);
        *reinterpret_cast<float4*>(shift + o) = v[i];
#pragma unroll
        for (int m = 0; m < 6; m++) st_act4(mix + (int64_t)m * R * C + o, lerp4(v[i], xx, cf[m][i]));
    }
}

// cmix input: xl = ln2(x); xx = shift - xl; shift = xl; out = xl + xx * coef.
template <typename A, int GV>
__global__ void __launch_bounds__(GLUE_T)
x070_cmix_in_kernel(const float* __restrict__ x, const float* __restrict__ lnw,
                    const float* __restrict__ lnb, float* __restrict__ shift,
                    const float* __restrict__ coef, A* __restrict__ out, int C) {
    __shared__ float sh[33];
    const int n = blockIdx.x;
    float4 sv[GV], cf[GV], w4[GV], b4[GV], v[GV];
    ld_row4<GV>(cf, coef, C);
    ld_row4<GV>(w4, lnw, C);
    ld_row4<GV>(b4, lnb, C);
    // the shift row was last written by this kernel one step earlier
    ld_row4<GV>(sv, shift + (int64_t)n * C, C);
    pdl_wait();  // x: written by earlier kernels of the step
    pdl_trigger();
    ld_row4<GV>(v, x + (int64_t)n * C, C);
    ln_row4<GV>(v, w4, b4, C, sh);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (threadIdx.x + GLUE_T * i);
        if (c >= C) continue;
        const int64_t o = (int64_t)n * C + c;
        const float4 xx = sub4(sv[i], v[i]);
        *reinterpret_cast<float4*>(shift + o) = v[i];
        st_act4(out + o, lerp4(v[i], xx, cf[i]));
    }
}

template <typename A, int GV>
__global__ void __launch_bounds__(GLUE_T)
x070_ln_out_kernel(const float* __restrict__ x, const float* __restrict__ lnw,
                   const float* __restrict__ lnb, A* __restrict__ out, int C) {
    __shared__ float sh[33];
    const int n = blockIdx.x;
    float4 w4[GV], b4[GV], v[GV];
    ld_row4<GV>(w4, lnw, C);
    ld_row4<GV>(b4, lnb, C);
    pdl_wait();  // x: the previous kernel's output
    pdl_trigger();
    ld_row4<GV>(v, x + (int64_t)n * C, C);
    ln_row4<GV>(v, w4, b4, C, sh);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (threadIdx.x + GLUE_T * i);
        if (c < C) st_act4(out + (int64_t)n * C + c, v[i]);
    }
}

// WKV part of tmixStep for one (row, head):
//   kk = l2norm(k * k_k);  k' = k * (1 + (a - 1) * k_a)
//   v' = v (layer 0, also stored as v_first) or v + (v_first - v) * vv
//   step with (r, w, k', v', -kk, kk * a); tail -> out (act type).
// 128 threads = 4 warps x 16 state rows.  A warp updates two rows per pass:
// lanes 0-15 row dv, lanes 16-31 row dv+1, lane l holding key columns
// 4(l%16) .. 4(l%16)+3 (one 16-byte load per row, a warp load covers 512
// contiguous bytes).  Row reductions (S a, S r) are 16-lane shuffles.  All of
// a warp's 16 rows are loaded before the first is used; two warps meanwhile
// build the head's vectors, and the tail's per-head parameters are fetched
// in the prologue, so a CTA waits on global memory about once.
template <typename A>
__global__ void __launch_bounds__(128)
x070_wkv_kernel(const float* __restrict__ r, const float* __restrict__ wdec,
                const float* __restrict__ kraw, const float* __restrict__ vraw,
                const float* __restrict__ a, const float* __restrict__ vv,
                float* __restrict__ vfirst, const float* __restrict__ kkw,
                const float* __restrict__ kaw, const float* __restrict__ rkw,
                const float* __restrict__ lnxw, const float* __restrict__ lnxb,
                const float* __restrict__ g, float* __restrict__ state, A* __restrict__ out,
                int H, int layer0) {
    constexpr int N = 64, RPW = 16;  // rows per warp
    __shared__ __align__(16) float r_s[N], w_s[N], kp_s[N], aw_s[N], bw_s[N], v_s[N], y_s[N];
    __shared__ __align__(16) float rk_s[N], lw_s[N], lb_s[N], g_s[N];
    __shared__ float red[2];
    const int rh = blockIdx.x;
    const int hi = rh % H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = lane >> 4, c0 = 4 * (lane & 15);
    const size_t vb = (size_t)rh * N;   // [R, H, N] element base of this (row, head)
    const size_t hb = (size_t)hi * N;   // [H, N] parameter base
    // The state and the per-head parameters are read before the wait on the
    // predecessor: no kernel of the step before this one writes them (the
    // state was last written by this kernel one step earlier, and the row
    // kernels in between wait for completion before letting successors
    // start), so their loads overlap the predecessor's tail.
    float* hp = state + (size_t)rh * N * N + (size_t)(RPW * warp + half) * N + c0;
    float4 s[RPW / 2];
#pragma unroll
    for (int p = 0; p < RPW / 2; p++) s[p] = *reinterpret_cast<const float4*>(hp + (size_t)2 * p * N);
    const int pc = threadIdx.x & (N - 1);
    const float par0 = threadIdx.x < N ? kkw[hb + pc] : rkw[hb + pc];
    const float par1 = threadIdx.x < N ? kaw[hb + pc] : lnxw[hb + pc];
    const float par2 = threadIdx.x < N ? 0.f : lnxb[hb + pc];
    pdl_wait();  // launched as a programmatic dependent: predecessor outputs first
    pdl_trigger();
    if (threadIdx.x < N) {  // warps 0-1: per-column vectors; column c = threadIdx.x
        const int c = threadIdx.x;
        const float kr = kraw[vb + c], aa = a[vb + c];
        const float kk = kr * par0;
        float ss = warp_sum(kk * kk);
        if ((c & 31) == 0) red[c >> 5] = ss;
        r_s[c] = r[vb + c];
        w_s[c] = wdec[vb + c];
        const float kp = kr * (1.0f + (aa - 1.0f) * par1);
        kp_s[c] = kp;
        // value row c
        float vd = vraw[vb + c];
        if (layer0) {
            vfirst[vb + c] = vd;
        } else {
            const float f = vfirst[vb + c];
            vd = vd + (f - vd) * vv[vb + c];
        }
        v_s[c] = vd;
        asm volatile("bar.sync 1, 64;");  // the two warps: both halves of the norm are in red[]
        const float inv = 1.0f / sqrtf(red[0] + red[1] + 1e-12f);
        const float kn = kk * inv;
        aw_s[c] = -kn;
        bw_s[c] = kn * aa;
    } else {  // warps 2-3: the tail's per-head parameters and the gate
        const int c = threadIdx.x - N;
        rk_s[c] = par0;
        lw_s[c] = par1;
        lb_s[c] = par2;
        g_s[c] = g[vb + c];
    }
    __syncthreads();
    const float4 aw = *reinterpret_cast<const float4*>(aw_s + c0);
    const float4 bw = *reinterpret_cast<const float4*>(bw_s + c0);
    const float4 ww = *reinterpret_cast<const float4*>(w_s + c0);
    const float4 kp = *reinterpret_cast<const float4*>(kp_s + c0);
    const float4 rr = *reinterpret_cast<const float4*>(r_s + c0);
#pragma unroll
    for (int p = 0; p < RPW / 2; p++) {
        const int dv = RPW * warp + 2 * p + half;
        float4 t = s[p];
        const float sa = group_sum<16>(fmaf(t.x, aw.x, fmaf(t.y, aw.y, fmaf(t.z, aw.z, t.w * aw.w))));
        const float vd = v_s[dv];
        t.x = fmaf(ww.x, t.x, fmaf(vd, kp.x, sa * bw.x));
        t.y = fmaf(ww.y, t.y, fmaf(vd, kp.y, sa * bw.y));
        t.z = fmaf(ww.z, t.z, fmaf(vd, kp.z, sa * bw.z));
        t.w = fmaf(ww.w, t.w, fmaf(vd, kp.w, sa * bw.w));
        *reinterpret_cast<float4*>(hp + (size_t)2 * p * N) = t;
        const float yy = group_sum<16>(fmaf(t.x, rr.x, fmaf(t.y, rr.y, fmaf(t.z, rr.z, t.w * rr.w))));
        if ((lane & 15) == 0) y_s[dv] = yy;
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    // tail on one warp: GroupNorm(64e-5) of y, bonus (sum r*k'*r_k) * v', gate
    const int l = threadIdx.x;
    float dp = r_s[l] * kp_s[l] * rk_s[l] + r_s[l + 32] * kp_s[l + 32] * rk_s[l + 32];
    dp = warp_sum(dp);
    const float x0 = y_s[l], x1 = y_s[l + 32];
    const float mean = warp_sum(x0 + x1) * (1.0f / N);
    const float d0 = x0 - mean, d1 = x1 - mean;
    const float var = warp_sum(d0 * d0 + d1 * d1) * (1.0f / N);
    const float invs = 1.0f / sqrtf(var + 64e-5f);
    const float o0 = (d0 * invs * lw_s[l] + lb_s[l] + dp * v_s[l]) * g_s[l];
    const float o1 = (d1 * invs * lw_s[l + 32] + lb_s[l + 32] + dp * v_s[l + 32]) * g_s[l + 32];
    st_act(out + vb + l, o0);
    st_act(out + vb + l + 32, o1);
}

// ---------------------------------------------------------------- prefill
// Parallel prefill over a block of `Ts` positions of every row (the
// reference's bodyWithState, X070Backbone.swift:1011-1048, over right-padded
// prompts, BatchGenerate.swift:36-51): token n = row * Ts + t sits at prompt
// position p0 + t; it is a real token when p0 + t < len[row], else padding.
// Buffers of these kernels are [rows * Ts, C] (= [rows, Ts, H, 64]).

// The block's token ids from the right-padded [rows, T] prompt matrix.
__global__ void x070_pf_ids_kernel(const int32_t* __restrict__ ids, int T, int p0, int Ts, int rows,
                                   int32_t* __restrict__ out) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= rows * Ts) return;
    const int row = n / Ts, p = p0 + n % Ts;
    out[n] = p < T ? ids[(int64_t)row * T + p] : 0;
}

// tmix input over a block (rwkvTmixForward's token shift and lerps,
// RWKVBlock.swift:171-178): xl = ln1(x) (given), prev = the row's shift row
// at t = 0 else xl of token n - 1; mix[m] = xl + (prev - xl) * coef[m].
template <typename A, int GV>
__global__ void __launch_bounds__(GLUE_T)
x070_pf_tmix_mix_kernel(const float* __restrict__ ln, const float* __restrict__ shift,
                        const float* __restrict__ coef, A* __restrict__ mix, int N, int Ts, int C) {
    const int n = blockIdx.x, t = n % Ts, row = n / Ts;
    float4 cf[6][GV], v[GV], pv[GV];
#pragma unroll
    for (int m = 0; m < 6; m++) ld_row4<GV>(cf[m], coef + m * C, C);
    ld_row4<GV>(v, ln + (int64_t)n * C, C);
    ld_row4<GV>(pv, t == 0 ? shift + (int64_t)row * C : ln + (int64_t)(n - 1) * C, C);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (threadIdx.x + GLUE_T * i);
        if (c >= C) continue;
        const int64_t o = (int64_t)n * C + c;
        const float4 xx = sub4(pv[i], v[i]);
#pragma unroll
        for (int m = 0; m < 6; m++) st_act4(mix + (int64_t)m * N * C + o, lerp4(v[i], xx, cf[m][i]));
    }
}

// cmix input over a block (rwkvCmixForward, RWKVBlock.swift:297-300).
template <typename A, int GV>
__global__ void __launch_bounds__(GLUE_T)
x070_pf_cmix_mix_kernel(const float* __restrict__ ln, const float* __restrict__ shift,
                        const float* __restrict__ coef, A* __restrict__ out, int Ts, int C) {
    const int n = blockIdx.x, t = n % Ts, row = n / Ts;
    float4 cf[GV], v[GV], pv[GV];
    ld_row4<GV>(cf, coef, C);
    ld_row4<GV>(v, ln + (int64_t)n * C, C);
    ld_row4<GV>(pv, t == 0 ? shift + (int64_t)row * C : ln + (int64_t)(n - 1) * C, C);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (threadIdx.x + GLUE_T * i);
        if (c < C) st_act4(out + (int64_t)n * C + c, lerp4(v[i], sub4(pv[i], v[i]), cf[i]));
    }
}

// The WKV inputs of a block (the caller math of RWKVBlock.swift:207-237),
// one warp per (token, head), lanes on channels c and c + 32:
//   kk = l2norm(k * k_k);  k' = k * (1 + (a - 1) * k_a)
//   v' = v (layer 0, also stored as v_first) or v + (v_first - v) * vv
//   a_wkv = -kk;  b_wkv = kk * a
//   padding (p0 + t >= len): w = 1, k' = 0, b_wkv = 0, so the step is the
//   identity on the state (RWKVBlock.swift:221-237).
// w, k, v are rewritten in place; a_wkv / b_wkv go to aw / bw.
__global__ void __launch_bounds__(256)
x070_pf_prep_kernel(float* __restrict__ w, float* __restrict__ k, float* __restrict__ v,
                    const float* __restrict__ a, const float* __restrict__ vv,
                    float* __restrict__ vfirst, float* __restrict__ aw, float* __restrict__ bw,
                    const float* __restrict__ kkw, const float* __restrict__ kaw,
                    const int32_t* __restrict__ len, int p0, int Ts, int H, int layer0) {
    constexpr int N = 64;
    const int n = blockIdx.x, head = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (head >= H) return;
    const bool real = p0 + n % Ts < len[n / Ts];
    const int64_t base = ((int64_t)n * H + head) * N;
    float kk[2], kr[2], aa[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int c = lane + 32 * j;
        kr[j] = k[base + c];
        aa[j] = a[base + c];
        kk[j] = kr[j] * kkw[head * N + c];
    }
    const float inv = 1.0f / sqrtf(warp_sum(kk[0] * kk[0] + kk[1] * kk[1]) + 1e-12f);
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int c = lane + 32 * j;
        const int64_t o = base + c;
        const float kn = kk[j] * inv;
        const float kp = kr[j] * (1.0f + (aa[j] - 1.0f) * kaw[head * N + c]);
        float vd = v[o];
        if (layer0) {
            vfirst[o] = vd;
        } else {
            const float f = vfirst[o];
            vd = vd + (f - vd) * vv[o];
        }
        v[o] = vd;
        aw[o] = -kn;
        if (real) {
            k[o] = kp;
            bw[o] = kn * aa[j];
        } else {
            w[o] = 1.0f;
            k[o] = 0.0f;
            bw[o] = 0.0f;
        }
    }
}

// tmix tail of a block, one warp per (token, head): GroupNorm(64e-5) of the
// WKV output y, bonus (sum r*k'*r_k) * v', gate -> out (activation type);
// the same arithmetic as the decode kernel's tail.
template <typename A>
__global__ void __launch_bounds__(256)
x070_pf_tail_kernel(const float* __restrict__ y, const float* __restrict__ r, const float* __restrict__ kp,
                    const float* __restrict__ v, const float* __restrict__ rkw, const float* __restrict__ lnxw,
                    const float* __restrict__ lnxb, const float* __restrict__ g, A* __restrict__ out, int H) {
    constexpr int N = 64;
    const int n = blockIdx.x, head = blockIdx.y * 8 + (threadIdx.x >> 5), l = threadIdx.x & 31;
    if (head >= H) return;
    const int64_t base = ((int64_t)n * H + head) * N;
    const int hb = head * N;
    float dp = r[base + l] * kp[base + l] * rkw[hb + l] + r[base + l + 32] * kp[base + l + 32] * rkw[hb + l + 32];
    dp = warp_sum(dp);
    const float x0 = y[base + l], x1 = y[base + l + 32];
    const float mean = warp_sum(x0 + x1) * (1.0f / N);
    const float d0 = x0 - mean, d1 = x1 - mean;
    const float var = warp_sum(d0 * d0 + d1 * d1) * (1.0f / N);
    const float invs = 1.0f / sqrtf(var + 64e-5f);
    const float o0 = (d0 * invs * lnxw[hb + l] + lnxb[hb + l] + dp * v[base + l]) * g[base + l];
    const float o1 = (d1 * invs * lnxw[hb + l + 32] + lnxb[hb + l + 32] + dp * v[base + l + 32]) * g[base + l + 32];
    st_act(out + base + l, o0);
    st_act(out + base + l + 32, o1);
}

// End of a block for one layer: each row's token-shift state becomes the
// normalised input at its last real token inside the block (gatherLast at
// lastRealIndex, RWKVBatchState.swift:159-175); rows without a real token
// in the block keep theirs.
__global__ void __launch_bounds__(256)
x070_pf_commit_kernel(const float* __restrict__ ln1, const float* __restrict__ ln2, float* __restrict__ tshift,
                      float* __restrict__ cshift, const int32_t* __restrict__ len, int p0, int Ts, int C) {
    const int row = blockIdx.x;
    const int last = min(len[row] - 1, p0 + Ts - 1) - p0;
    if (last < 0) return;
    const int64_t src = ((int64_t)row * Ts + last) * C, dst = (int64_t)row * C;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        tshift[dst + c] = ln1[src + c];
        cshift[dst + c] = ln2[src + c];
    }
}

// ln_out of each row's last real token, when it lies in this block -> out
// [rows, C] (activation type): the hidden state the head reads.
template <typename A, int GV>
__global__ void __launch_bounds__(GLUE_T)
x070_pf_lnout_kernel(const float* __restrict__ x, const float* __restrict__ lnw, const float* __restrict__ lnb,
                     A* __restrict__ out, const int32_t* __restrict__ len, int p0, int Ts, int C) {
    __shared__ float sh[33];
    const int row = blockIdx.x;
    const int last = len[row] - 1 - p0;
    if (last < 0 || last >= Ts) return;
    float4 w4[GV], b4[GV], v[GV];
    ld_row4<GV>(w4, lnw, C);
    ld_row4<GV>(b4, lnb, C);
    ld_row4<GV>(v, x + ((int64_t)row * Ts + last) * C, C);
    ln_row4<GV>(v, w4, b4, C, sh);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (threadIdx.x + GLUE_T * i);
        if (c < C) st_act4(out + (int64_t)row * C + c, v[i]);
    }
}

// generateBatch's row drop (RWKVBatchState.gather, BatchGenerate.swift:
// 105-108): rows keep[i] -> i of one layer's [rows, E] float block, through
// `tmp` (keep is increasing, but a destination may still be a later source).
__global__ void x070_gather_rows_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                        const int32_t* __restrict__ keep, int nkeep, int64_t E) {
    const int64_t total = (int64_t)nkeep * E;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / E, e = i - r * E;
        dst[i] = src[(int64_t)keep[r] * E + e];
    }
}

// Greedy sampler: first index of the maximum logit per row.  Each CTA scans
// a slice of one row and folds (value, index) into a 64-bit key with
// atomicMax: the high word is the float mapped to an order-preserving
// unsigned, the low word ~index, so the maximum key is the largest logit and,
// among equal logits, the lowest index -- independent of CTA order.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned)(0xFFFFFFFFu - (unsigned)idx);
}

constexpr int ARGMAX_SLICE = 4096;

__global__ void __launch_bounds__(GLUE_T)
x070_argmax_kernel(const float* __restrict__ logits, int V, unsigned long long* __restrict__ keys) {
    pdl_wait();  // launched as a programmatic dependent: predecessor outputs first
    pdl_trigger();
    __shared__ unsigned long long sk[GLUE_T / 32];
    const int n = blockIdx.y;
    const int c0 = blockIdx.x * ARGMAX_SLICE;
    const float* p = logits + (int64_t)n * V;
    unsigned long long best = 0ull;
    const int cend = min(V, c0 + ARGMAX_SLICE);
    if ((V & 3) == 0) {
#pragma unroll 4
        for (int c = c0 + 4 * threadIdx.x; c < cend; c += 4 * GLUE_T) {
            const float4 v4 = *reinterpret_cast<const float4*>(p + c);
            best = max(best, argmax_key(v4.x, c));
            best = max(best, argmax_key(v4.y, c + 1));
            best = max(best, argmax_key(v4.z, c + 2));
            best = max(best, argmax_key(v4.w, c + 3));
        }
    } else {
        for (int c = c0 + threadIdx.x; c < cend; c += GLUE_T) best = max(best, argmax_key(p[c], c));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < GLUE_T / 32; w++) best = max(best, sk[w]);
        atomicMax(keys + n, best);
    }
}

// keys -> ids, and re-arm the keys for the next step.
__global__ void x070_argmax_finish_kernel(unsigned long long* __restrict__ keys,
                                          int32_t* __restrict__ ids, int R) {
    pdl_wait();  // launched as a programmatic dependent: predecessor outputs first
    pdl_trigger();
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= R) return;
    ids[n] = (int32_t)(0xFFFFFFFFu - (unsigned)(keys[n] & 0xFFFFFFFFull));
    keys[n] = 0ull;
}

// CUDA-core GEMV for fp32 activations (the fp32 parity mode): one warp per
// output row, lanes strided over k, up to 8 input rows per launch tile.
template <int FMT>
__global__ void __launch_bounds__(256)
gemv_cc_kernel(const GemvJobs jobs, int R) {
    pdl_wait();  // launched as a programmatic dependent: predecessor outputs first
    pdl_trigger();
    const GemvJob& jb = jobs.j[blockIdx.y];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o = blockIdx.x * 8 + warp;
    if (o >= jb.OUT) return;
    const int n0 = blockIdx.z * 8;
    const int Rz = min(R - n0, 8);
    const float* x = (const float*)jb.x + (int64_t)n0 * jb.x_stride;
    float acc[8];
#pragma unroll
    for (int n = 0; n < 8; n++) acc[n] = 0.f;
    if (FMT == 0) {
        const uint32_t* W = (const uint32_t*)jb.w + (int64_t)o * (jb.IN / 8);
        const int NG = jb.IN / 64;
        for (int c = lane; c < jb.IN; c += 32) {
            const float q = (float)((W[c / 8] >> (4 * (c & 7))) & 15u);
            const int gi = o * NG + c / 64;
            const float wv = q * __half2float(jb.scales[gi]) + __half2float(jb.biases[gi]);
#pragma unroll
            for (int n = 0; n < 8; n++)
                if (n < Rz) acc[n] = fmaf(wv, x[(int64_t)n * jb.x_stride + c], acc[n]);
        }
    } else if (FMT == 1) {
        const __half* W = (const __half*)jb.w + (int64_t)o * jb.IN;
        for (int c = lane; c < jb.IN; c += 32) {
            const float wv = __half2float(W[c]);
#pragma unroll
            for (int n = 0; n < 8; n++)
                if (n < Rz) acc[n] = fmaf(wv, x[(int64_t)n * jb.x_stride + c], acc[n]);
        }
    } else {
        const __nv_bfloat16* W = (const __nv_bfloat16*)jb.w + (int64_t)o * jb.IN;
        for (int c = lane; c < jb.IN; c += 32) {
            const float wv = __bfloat162float(W[c]);
#pragma unroll
            for (int n = 0; n < 8; n++)
                if (n < Rz) acc[n] = fmaf(wv, x[(int64_t)n * jb.x_stride + c], acc[n]);
        }
    }
#pragma unroll
    for (int n = 0; n < 8; n++) {
        const float v = warp_sum(acc[n]);
        if (lane == 0 && n < Rz) epilogue(jb, o, n0 + n, v);
    }
}

// relu(h)^2 into the activation type: the cmix key output when a LoRA
// adapter is added before the activation (n = rows * ffn).
template <typename A>
__global__ void __launch_bounds__(256) x070_relu2_cast_kernel(const float* __restrict__ h, A* __restrict__ out,
                                                              int n) {
    pdl_trigger();
    pdl_wait();
    for (int i = blockIdx.x * 256 + threadIdx.x; i < n; i += gridDim.x * 256) {
        const float v = fmaxf(h[i], 0.f);
        out[i] = from_f<A>(v * v);
    }
}

}  // namespace rwkv
