// Persistent x070 decode step: the whole step (embedding, 24 layers of
// tmix / projections / WKV / cmix, ln_out, head, greedy argmax) in ONE
// cooperative launch of one CTA per SM, for 9..64 rows with fp16 activations
// on the 4-bit group-64 base (X070Generation.swift:449-498 over
// BatchGenerate.swift:54-116's batch).
//
// Why: launched one kernel at a time, each projection GEMM of the step pays a
// launch, a TMEM allocation, a cold TMA pipeline that fills from HBM and a
// split-K cluster exchange -- 10-20 us per GEMM for 2-10 MB of weights (under
// 1 TB/s), while its CTAs hold their SMs.  Here the CTAs stay resident and
// the step is a program of phases separated by grid-wide barriers:
//
//   EMBED | per layer: TMIX, GEMM{r,k,v, low-rank down}, GEMM{low-rank up},
//   WKV, GEMM{o}, CMIX, GEMM{key}, GEMM{value} | LNOUT, GEMM{head}, ARGMAX,
//   ARGFIN
//
// Weights do not depend on the activations, so the TMA producer of each CTA
// streams the weight tiles of its GEMM work items into a 6-slot ring ahead of
// the phase they belong to -- across barriers, glue phases and layers -- and
// issues a tile's activation loads only once its phase has begun.  Only the
// activation loads, the dequantisation of weights already in shared memory,
// the MMAs and the split-K reduction remain on each phase's critical path.
//
// CTA = 320 threads: warp 0 TMA producer, warp 1 MMA issuer (tcgen05, M=128,
// N = BN activation rows, K=16; A from TMEM for 4-bit tiles, from shared
// memory for the fp16 low-rank matrices), warps 2-9 workers: dequantise 4-bit
// stages into TMEM (half(scale * q + bias), the tcgen05 decode GEMM's
// arithmetic), drain accumulators, run the split-K reductions and epilogues,
// the glue phases (the decode glue kernels' arithmetic) and the grid barriers.
//
// A GEMM phase is a list of work items (job = matrix, 128-row m-block,
// K-range); a tile whose K is split over nz items is reduced by the item that
// finishes last (a ticket per tile), which sums the nz partials in split
// order (deterministic) and applies the epilogue -- no clusters, no second
// launch.  Every wait is bounded in time and watches a device error flag;
// once it is set every role skips the rest of the program, so a failing launch
// ends within one wait limit.
#pragma once

#include "gemm_tc.cuh"
#include "x070_kernels.cuh"

namespace rwkv {
namespace pk {

constexpr int WORKERS = 8;                    // worker warps 2..9
constexpr int THREADS = 64 + 32 * WORKERS;    // 320
constexpr int WT = 32 * WORKERS;              // 256 worker threads
constexpr int WST = 6;                        // weight ring slots
constexpr int WCODE = 128 * 128;              // 4-bit stage: 128 rows x 256 codes; fp16 stage: 128 rows x 64
constexpr int WSB = 128 * 16;                 // 4-bit stage: per row 4 x (scale, bias) fp16
constexpr int WSLOT = WCODE + WSB;            // 18 KB (multiple of 1024)
constexpr int XST = 3;                        // activation ring slots
constexpr int XSLOT = 4 * 64 * 128;           // 4 boxes of 64 rows x 64 fp16 (128-byte rows)
constexpr int TMEM_COLS = 512;                // acc b: [64 b, 64 b + 64); A stage a: [256 + 128 a, +128)
constexpr int A_COL = 256;
constexpr int NACC = 2, NA = 2;
constexpr int GLUE_SMEM = 2 * 12 * 64 * 4 + 64;  // two WKV half-groups' vectors + reduction scratch
constexpr int MAX_PHASES = 256;               // phase table copied into shared memory
constexpr int W_OFF = 0;
constexpr int X_OFF = W_OFF + WST * WSLOT;
constexpr int G_OFF = X_OFF + XST * XSLOT;
constexpr int P_OFF = G_OFF + GLUE_SMEM;
constexpr int B_OFF = P_OFF + MAX_PHASES * 16;
constexpr int NBAR = 2 * WST + 2 * XST + 2 * NA + 2 * NACC + 1;
constexpr int T_OFF = B_OFF + NBAR * 8;
constexpr int SMEM = T_OFF + 32 + 1024;       // + slack for 1024-byte alignment
static_assert(WSLOT % 1024 == 0 && XSLOT % 1024 == 0 && G_OFF % 1024 == 0, "swizzled stage bases");
static_assert(SMEM <= 227 * 1024, "shared memory per CTA");

enum : int { FMT_Q4 = 0, FMT_F16 = 1 };
enum : int { PH_EMBED = 0, PH_TMIX, PH_GEMM, PH_WKV, PH_CMIX, PH_LNOUT, PH_ARGMAX, PH_ARGFIN };

// One matrix of a GEMM phase.
struct alignas(128) Job {
    CUtensorMap wmap;  // Q4: codes {IN/8, OUT} u32, box {32, 128}; F16: {IN, OUT} fp16, box {64, 128}; 128-byte swizzle
    CUtensorMap xmap;  // activations {IN, R} fp16, box {64, BN}, 128-byte swizzle
    const unsigned char* sb;  // Q4: scales / biases repacked [OUT/128][IN/256][128][4 x (scale, bias)]
    GemvJob g;         // OUT, IN and the epilogue (act, out, y, y_stride, bias)
    int fmt;
    int sb_stages;     // IN / 256
};

// A work item: job, m-block, K stages [s0, s0 + nst) (256 codes per 4-bit
// stage, 64 per fp16 stage), split z of nz of tile `tile` (numbered across the
// whole program: one ticket per tile per step); its partial (if nz > 1) is
// workspace slot `slot` of the phase (the tile's splits are slots slot - z ..).
struct alignas(16) Item {
    int job, m0, s0, nst, tile, z, nz, slot;
    int fmt, pad;
    const unsigned char* sb;  // 4-bit: the m-block's repacked (scale, bias) stages
};

struct Phase {
    int type, i0, i1, layer;
};

struct Layer {
    const float *ln1w, *ln1b, *ln2w, *ln2b, *coef6, *kkw, *kaw, *rkw, *lnxw, *lnxb, *cxk;
    float *state, *tshift, *cshift;
};

struct Args {
    const Job* jobs;
    const Item* items;
    const Phase* phases;
    const Layer* layers;
    int nphases, R, C, H, V;
    // activations / step buffers (the runtime's, row-major over the R rows)
    float *x, *r, *k, *v, *wdec, *a, *g, *vv, *vfirst, *logits, *ws;
    __half *mix, *tail, *xk, *lnout;
    int32_t* ids;
    unsigned long long* amax_keys;
    const uint32_t* emb_wq;
    const __half *emb_sc, *emb_bi;
    const float *ln0w, *ln0b, *lnow, *lnob;
    int* tickets;       // one per split tile of the program (zeroed before each launch)
    unsigned int* bar;  // grid barrier counter (zeroed before each launch)
    int* err;
    int* err_host;
    // nullable (step profiler): %globaltimer of CTA 0 at the start and after
    // each phase's barrier [0, 1024); per pipeline stage j < 2048 of CTA 0:
    // weight copy issued [T_W + j], activation copy issued [T_X + j], MMA
    // inputs ready [T_M + j], dequantised into TMEM [T_D + j]
    unsigned long long* trace;
};
// per work item k < 512 of CTA 0: [T_E + 4 k + 0] accumulator ready, +1 drained,
// +2 output or partial written (and counted), +3 its split tile reduced
// per phase p < 256 and CTA c < 160: [T_C + 160 p + c] the CTA's workers done
constexpr int T_W = 1024, T_X = T_W + 2048, T_M = T_X + 2048, T_D = T_M + 2048, T_E = T_D + 2048,
              T_C = T_E + 4 * 512, T_END = T_C + 160 * 256;

// ------------------------------------------------------------------ helpers

__device__ __forceinline__ void wbar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Sum over the 256 worker threads (named barrier 1); sh: 9 floats.
__device__ __forceinline__ float wsum(float v, float* sh, int wt) {
    v = warp_sum(v);
    if ((wt & 31) == 0) sh[wt >> 5] = v;
    wbar(1, WT);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < WORKERS; i++) s += sh[i];
    wbar(1, WT);
    return s;
}

// Grid barrier over the launch's CTAs (the 256 workers of each take part):
// the workers meet, one of them releases (the fence covers its CTA's writes
// ordered before the meeting), counts itself in and spins with acquire loads
// until every CTA has; the workers meet again.  Returns false (to every
// worker, through *flag) when the error flag is set or the wait expires.
__device__ __forceinline__ bool grid_barrier(unsigned int* bar, unsigned int gen, int* err, int wt, int* flag) {
    wbar(1, WT);
    if (wt == 0) {
        // acq_rel: releases this CTA's writes (ordered before it by the
        // meeting), and the polling acquire takes every other CTA's
        bool ok = true;
        const unsigned int target = gen * gridDim.x;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        const uint64_t t0 = tc::gtime();
        for (uint32_t it = 0;; it++) {
            unsigned int v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
            if (v >= target) break;
            if ((it & 15) == 15) {
                if (*(volatile int*)err) { ok = false; break; }
                if (tc::gtime() - t0 > tc::WAIT_LIMIT_NS) {
                    atomicExch(err, 1);
                    ok = false;
                    break;
                }
            }
        }
        *flag = ok;
    }
    wbar(1, WT);
    return *flag != 0;
}

template <int GV>
__device__ __forceinline__ void ld4(float4* d, const float* __restrict__ p, int C, int wt) {
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (wt + WT * i);
        d[i] = c < C ? *reinterpret_cast<const float4*>(p + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Two-pass LayerNorm (eps 1e-5) over the worker threads, in place; w4 / b4:
// the weight and bias columns, loaded by the caller with everything else.
template <int GV>
__device__ __forceinline__ void ln4(float4* v, const float4* w4, const float4* b4, int C, float* sh, int wt) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < GV; i++)
        if (4 * (wt + WT * i) < C) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = wsum(s, sh, wt) / (float)C;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < GV; i++)
        if (4 * (wt + WT * i) < C) {
            const float dx = v[i].x - mean, dy = v[i].y - mean, dz = v[i].z - mean, dw = v[i].w - mean;
            q += (dx * dx + dy * dy) + (dz * dz + dw * dw);
        }
    const float den = sqrtf(wsum(q, sh, wt) / (float)C + 1e-5f);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        v[i].x = (v[i].x - mean) / den * w4[i].x + b4[i].x;
        v[i].y = (v[i].y - mean) / den * w4[i].y + b4[i].y;
        v[i].z = (v[i].z - mean) / den * w4[i].z + b4[i].z;
        v[i].w = (v[i].w - mean) / den * w4[i].w + b4[i].w;
    }
}

// ---------------------------------------------------------------- glue

// x[n] = ln0(emb[ids[n]]) (x070_embed_kernel's arithmetic).
template <int GV>
__device__ void do_embed(const Args& A, int n, float* sh, int wt) {
    const int C = A.C;
    int id = A.ids[n];
    id = min(max(id, 0), A.V - 1);
    float4 v[GV];
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (wt + WT * i);
        float e[4] = {0.f, 0.f, 0.f, 0.f};
        if (c < C) {
            const uint32_t word = A.emb_wq[(int64_t)id * (C / 8) + c / 8];
            const int64_t gi = (int64_t)id * (C / 64) + c / 64;
            const float s = __half2float(A.emb_sc[gi]), b = __half2float(A.emb_bi[gi]);
#pragma unroll
            for (int j = 0; j < 4; j++) e[j] = (float)((word >> (4 * ((c + j) & 7))) & 15u) * s + b;
        }
        v[i] = make_float4(e[0], e[1], e[2], e[3]);
    }
    float4 w4[GV], b4[GV];
    ld4<GV>(w4, A.ln0w, C, wt);
    ld4<GV>(b4, A.ln0b, C, wt);
    ln4<GV>(v, w4, b4, C, sh, wt);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (wt + WT * i);
        if (c < C) *reinterpret_cast<float4*>(A.x + (int64_t)n * C + c) = v[i];
    }
}

// tmix input of row n (x070_tmix_in_kernel's arithmetic).
template <int GV>
__device__ void do_tmix(const Args& A, const Layer& L, int n, float* sh, int wt) {
    const int C = A.C, R = A.R;
    // every load first: one round trip
    float4 v[GV], sv[GV], w4[GV], b4[GV], cf[6][GV];
    ld4<GV>(v, A.x + (int64_t)n * C, C, wt);
    ld4<GV>(sv, L.tshift + (int64_t)n * C, C, wt);
    ld4<GV>(w4, L.ln1w, C, wt);
    ld4<GV>(b4, L.ln1b, C, wt);
#pragma unroll
    for (int m = 0; m < 6; m++) ld4<GV>(cf[m], L.coef6 + m * C, C, wt);
    ln4<GV>(v, w4, b4, C, sh, wt);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (wt + WT * i);
        if (c >= C) continue;
        const int64_t o = (int64_t)n * C + c;
        const float4 xx = sub4(sv[i], v[i]);
        *reinterpret_cast<float4*>(L.tshift + o) = v[i];
#pragma unroll
        for (int m = 0; m < 6; m++) st_act4(A.mix + (int64_t)m * R * C + o, lerp4(v[i], xx, cf[m][i]));
    }
}

// cmix input of row n (x070_cmix_in_kernel's arithmetic).
template <int GV>
__device__ void do_cmix(const Args& A, const Layer& L, int n, float* sh, int wt) {
    const int C = A.C;
    float4 v[GV], sv[GV], w4[GV], b4[GV], cf[GV];
    ld4<GV>(v, A.x + (int64_t)n * C, C, wt);
    ld4<GV>(sv, L.cshift + (int64_t)n * C, C, wt);
    ld4<GV>(w4, L.ln2w, C, wt);
    ld4<GV>(b4, L.ln2b, C, wt);
    ld4<GV>(cf, L.cxk, C, wt);
    ln4<GV>(v, w4, b4, C, sh, wt);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (wt + WT * i);
        if (c >= C) continue;
        const int64_t o = (int64_t)n * C + c;
        *reinterpret_cast<float4*>(L.cshift + o) = v[i];
        st_act4(A.xk + o, lerp4(v[i], sub4(sv[i], v[i]), cf[i]));
    }
}

template <int GV>
__device__ void do_lnout(const Args& A, int n, float* sh, int wt) {
    const int C = A.C;
    float4 v[GV], w4[GV], b4[GV];
    ld4<GV>(v, A.x + (int64_t)n * C, C, wt);
    ld4<GV>(w4, A.lnow, C, wt);
    ld4<GV>(b4, A.lnob, C, wt);
    ln4<GV>(v, w4, b4, C, sh, wt);
#pragma unroll
    for (int i = 0; i < GV; i++) {
        const int c = 4 * (wt + WT * i);
        if (c < C) st_act4(A.lnout + (int64_t)n * C + c, v[i]);
    }
}

// This thread's 16 state rows x 4 columns of (row, head) rh (t = 0..127).
__device__ __forceinline__ void wkv_load(const Layer& L, int rh, int t, float4* s) {
    constexpr int N = 64, RPW = 16;
    const int warp = t >> 5, lane = t & 31;
    const float* hp = L.state + (size_t)rh * N * N + (size_t)(RPW * warp + (lane >> 4)) * N + 4 * (lane & 15);
#pragma unroll
    for (int p = 0; p < RPW / 2; p++) s[p] = __ldcg(reinterpret_cast<const float4*>(hp + (size_t)2 * p * N));
}

// The per-column vectors of (row, head) rh this thread needs (t < 64: column
// t of k, a, r, w, k_k, k_a, v, v_first, v-gate; t >= 64: column t - 64 of
// r_k, ln_x weight / bias, gate), loaded one item ahead.
__device__ __forceinline__ void wkv_vec_load(const Args& A, const Layer& L, int rh, int layer0, int t, float* f) {
    constexpr int N = 64;
    const size_t vb = (size_t)rh * N, hb = (size_t)(rh % A.H) * N;
    if (t < N) {
        f[0] = A.k[vb + t];
        f[1] = A.a[vb + t];
        f[2] = A.r[vb + t];
        f[3] = A.wdec[vb + t];
        f[4] = L.kkw[hb + t];
        f[5] = L.kaw[hb + t];
        f[6] = A.v[vb + t];
        f[7] = layer0 ? 0.f : A.vfirst[vb + t];
        f[8] = layer0 ? 0.f : A.vv[vb + t];
    } else {
        const int c = t - N;
        f[0] = L.rkw[hb + c];
        f[1] = L.lnxw[hb + c];
        f[2] = L.lnxb[hb + c];
        f[3] = A.g[vb + c];
    }
}

// WKV step + tail of (row, head) rh by a half-group of 4 warps (t = 0..127),
// x070_wkv_kernel's arithmetic, from the state rows s (wkv_load) and the
// vectors f (wkv_vec_load); sv: this half-group's 11 x 64 floats + 2.
__device__ void do_wkv(const Args& A, const Layer& L, int rh, int layer0, float* sv, int t, int half, float4* s,
                       const float* f) {
    constexpr int N = 64, RPW = 16;
    float *r_s = sv, *w_s = sv + 64, *kp_s = sv + 128, *aw_s = sv + 192, *bw_s = sv + 256, *v_s = sv + 320;
    float *y_s = sv + 384, *rk_s = sv + 448, *lw_s = sv + 512, *lb_s = sv + 576, *g_s = sv + 640, *red = sv + 704;
    const int H = A.H;
    const int hi = rh % H;
    const int warp = t >> 5, lane = t & 31;
    const int hlf = lane >> 4, c0 = 4 * (lane & 15);
    const size_t vb = (size_t)rh * N, hb = (size_t)hi * N;
    float* hp = L.state + (size_t)rh * N * N + (size_t)(RPW * warp + hlf) * N + c0;
    if (t < N) {
        const int c = t;
        const float kr = f[0], aa = f[1];
        const float kk = kr * f[4];
        const float ss = warp_sum(kk * kk);
        if ((c & 31) == 0) red[c >> 5] = ss;
        r_s[c] = f[2];
        w_s[c] = f[3];
        const float kp = kr * (1.0f + (aa - 1.0f) * f[5]);
        kp_s[c] = kp;
        float vd = f[6];
        if (layer0) {
            A.vfirst[vb + c] = vd;
        } else {
            vd = vd + (f[7] - vd) * f[8];
        }
        v_s[c] = vd;
        wbar(4 + half, 64);
        const float inv = 1.0f / sqrtf(red[0] + red[1] + 1e-12f);
        const float kn = kk * inv;
        aw_s[c] = -kn;
        bw_s[c] = kn * aa;
    } else {
        const int c = t - N;
        rk_s[c] = f[0];
        lw_s[c] = f[1];
        lb_s[c] = f[2];
        g_s[c] = f[3];
    }
    wbar(2 + half, 128);
    const float4 aw = *reinterpret_cast<const float4*>(aw_s + c0);
    const float4 bw = *reinterpret_cast<const float4*>(bw_s + c0);
    const float4 ww = *reinterpret_cast<const float4*>(w_s + c0);
    const float4 kp = *reinterpret_cast<const float4*>(kp_s + c0);
    const float4 rr = *reinterpret_cast<const float4*>(r_s + c0);
#pragma unroll
    for (int p = 0; p < RPW / 2; p++) {
        const int dv = RPW * warp + 2 * p + hlf;
        float4 q = s[p];
        const float sa = group_sum<16>(fmaf(q.x, aw.x, fmaf(q.y, aw.y, fmaf(q.z, aw.z, q.w * aw.w))));
        const float vd = v_s[dv];
        q.x = fmaf(ww.x, q.x, fmaf(vd, kp.x, sa * bw.x));
        q.y = fmaf(ww.y, q.y, fmaf(vd, kp.y, sa * bw.y));
        q.z = fmaf(ww.z, q.z, fmaf(vd, kp.z, sa * bw.z));
        q.w = fmaf(ww.w, q.w, fmaf(vd, kp.w, sa * bw.w));
        *reinterpret_cast<float4*>(hp + (size_t)2 * p * N) = q;
        const float yy = group_sum<16>(fmaf(q.x, rr.x, fmaf(q.y, rr.y, fmaf(q.z, rr.z, q.w * rr.w))));
        if ((lane & 15) == 0) y_s[dv] = yy;
    }
    wbar(2 + half, 128);
    if (t < 32) {
        const int l = t;
        float dp = r_s[l] * kp_s[l] * rk_s[l] + r_s[l + 32] * kp_s[l + 32] * rk_s[l + 32];
        dp = warp_sum(dp);
        const float x0 = y_s[l], x1 = y_s[l + 32];
        const float mean = warp_sum(x0 + x1) * (1.0f / N);
        const float d0 = x0 - mean, d1 = x1 - mean;
        const float var = warp_sum(d0 * d0 + d1 * d1) * (1.0f / N);
        const float invs = 1.0f / sqrtf(var + 64e-5f);
        const float o0 = (d0 * invs * lw_s[l] + lb_s[l] + dp * v_s[l]) * g_s[l];
        const float o1 = (d1 * invs * lw_s[l + 32] + lb_s[l + 32] + dp * v_s[l + 32]) * g_s[l + 32];
        A.tail[vb + l] = __float2half_rn(o0);
        A.tail[vb + l + 32] = __float2half_rn(o1);
    }
    wbar(2 + half, 128);  // the vectors may be overwritten by the next item
}

// ---------------------------------------------------------------- kernel

template <int BN>
__global__ void __launch_bounds__(THREADS, 1) x070_persist_kernel(const __grid_constant__ Args A) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + B_OFF);
    uint64_t* wempty = wfull + WST;
    uint64_t* xfull = wempty + WST;
    uint64_t* xempty = xfull + XST;
    uint64_t* afull = xempty + XST;
    uint64_t* aempty = afull + NA;
    uint64_t* accfull = aempty + NA;
    uint64_t* accempty = accfull + NACC;
    uint64_t* mdone = accempty + NACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + T_OFF);
    Phase* phs = reinterpret_cast<Phase*>(smem + P_OFF);
    int* last_flag = reinterpret_cast<int*>(smem + T_OFF + 16);
    float* glue = reinterpret_cast<float*>(smem + G_OFF);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    int* err = A.err;

    for (int p = tid; p < A.nphases; p += THREADS) phs[p] = A.phases[p];
    if (tid == 0) {
        for (int s = 0; s < WST; s++) {
            tc::mbar_init(wfull + s, 1);
            tc::mbar_init(wempty + s, 1);
        }
        for (int s = 0; s < XST; s++) {
            tc::mbar_init(xfull + s, 1);
            tc::mbar_init(xempty + s, 1);
        }
        for (int s = 0; s < NA; s++) {
            tc::mbar_init(afull + s, WT);
            tc::mbar_init(aempty + s, 1);
        }
        for (int s = 0; s < NACC; s++) {
            tc::mbar_init(accfull + s, 1);
            tc::mbar_init(accempty + s, WT);
        }
        tc::mbar_init(mdone, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::saddr(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc::tc_before();
    __syncthreads();
    tc::tc_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer: weights run ahead, activations wait for their phase
            int pw = 0, iw = -1, sw = 0, nw = 0;  // weight cursor: phase, item, stage within it; stages issued
            int px = 0, ix = -1, sx = 0, nx = 0;  // activation cursor
            bool wdone = false, xdone = false;
            int started = 0;                      // phases known to have begun (phase 0 at launch)
            // next GEMM item of this CTA after (p, i): false at the end
            auto next_item = [&](int& p, int& i) {
                for (;;) {
                    if (p >= A.nphases) return false;
                    const Phase ph = phs[p];
                    if (ph.type == PH_GEMM) {
                        const int ni = i < 0 ? ph.i0 + cta : i + G;
                        if (ni < ph.i1) {
                            i = ni;
                            return true;
                        }
                    }
                    p++;
                    i = -1;
                }
            };
            Item wi{}, xi{};  // the cursors' items, read once each
            wdone = !next_item(pw, iw);
            if (!wdone) wi = A.items[iw];
            xdone = !next_item(px, ix);
            if (!xdone) xi = A.items[ix];
            uint64_t t_last = tc::gtime();
            for (uint32_t spin = 0; (!wdone || !xdone) && ok; spin++) {
                bool prog = false;
                if (!wdone && (nw < WST || tc::mbar_try(wempty + (nw % WST), ((nw / WST) - 1) & 1))) {
                    const CUtensorMap* wm = &A.jobs[wi.job].wmap;
                    const int s = nw % WST;
                    unsigned char* dst = smem + W_OFF + s * WSLOT;
                    const int st = wi.s0 + sw;
                    if (wi.fmt == FMT_Q4) {
                        tc::mbar_expect_tx(wfull + s, WCODE + WSB);
                        tc::tma_2d(dst, wm, wfull + s, 32 * st, wi.m0);
                        asm volatile(
                            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                                tc::saddr(dst + WCODE)),
                            "l"(wi.sb + (size_t)st * WSB), "r"(WSB), "r"(tc::saddr(wfull + s))
                            : "memory");
                    } else {
                        tc::mbar_expect_tx(wfull + s, WCODE);
                        tc::tma_2d(dst, wm, wfull + s, 64 * st, wi.m0);
                    }
                    if (A.trace && cta == 0 && nw < 2048) A.trace[T_W + nw] = tc::gtime();
                    nw++;
                    if (++sw == wi.nst) {
                        sw = 0;
                        wdone = !next_item(pw, iw);
                        if (!wdone) wi = A.items[iw];
                    }
                    prog = true;
                }
                if (!xdone && px > started) {
                    // has phase px begun?  (every CTA has passed the barrier ending
                    // px - 1; the acquire orders the other CTAs' writes of px's inputs
                    // before the loads)
                    unsigned int v;
                    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(A.bar) : "memory");
                    if ((int)(v / (unsigned)G) > started) {
                        started = (int)(v / (unsigned)G);
                        asm volatile("fence.proxy.async.global;" ::: "memory");  // generic writes -> TMA reads
                    }
                }
                if (!xdone && px <= started && (nx < XST || tc::mbar_try(xempty + (nx % XST), ((nx / XST) - 1) & 1))) {
                    const CUtensorMap* xm = &A.jobs[xi.job].xmap;
                    const int s = nx % XST;
                    unsigned char* dst = smem + X_OFF + s * XSLOT;
                    const int st = xi.s0 + sx;
                    if (xi.fmt == FMT_Q4) {
                        tc::mbar_expect_tx(xfull + s, 4 * BN * 128);
#pragma unroll
                        for (int q = 0; q < 4; q++) tc::tma_2d(dst + q * BN * 128, xm, xfull + s, 256 * st + 64 * q, 0);
                    } else {
                        tc::mbar_expect_tx(xfull + s, BN * 128);
                        tc::tma_2d(dst, xm, xfull + s, 64 * st, 0);
                    }
                    if (A.trace && cta == 0 && nx < 2048) A.trace[T_X + nx] = tc::gtime();
                    nx++;
                    if (++sx == xi.nst) {
                        sx = 0;
                        xdone = !next_item(px, ix);
                        if (!xdone) xi = A.items[ix];
                    }
                    prog = true;
                }
                if (prog) {
                    t_last = tc::gtime();
                } else if ((spin & 63) == 63) {
                    if (*(volatile int*)err) ok = false;
                    else if (tc::gtime() - t_last > tc::WAIT_LIMIT_NS) {
                        atomicExch(err, 1);
                        ok = false;
                    }
                }
            }
            // copies in flight land before the CTA moves on
            for (int j = max(0, nw - WST); j < nw; j++)
                if (!tc::mbar_wait_own(wfull + (j % WST), (j / WST) & 1, err)) ok = false;
            for (int j = max(0, nx - XST); j < nx; j++)
                if (!tc::mbar_wait_own(xfull + (j % XST), (j / XST) & 1, err)) ok = false;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            constexpr uint32_t IDESC = tc::idesc_f16(128, BN);
            int nw = 0, na = 0, nacc = 0;
            for (int p = 0; p < A.nphases && ok; p++) {
                const Phase ph = phs[p];
                if (ph.type != PH_GEMM) continue;
                for (int i = ph.i0 + cta; i < ph.i1 && ok; i += G) {
                    const Item it = A.items[i];
                    const int fmt = it.fmt;
                    const int b = nacc % NACC;
                    if (nacc >= NACC && !tc::mbar_wait(accempty + b, ((nacc / NACC) - 1) & 1, err)) { ok = false; break; }
                    const uint32_t dacc = tmem + 64 * b;
                    for (int s = 0; s < it.nst; s++, nw++) {
                        const int ws = nw % WST, xs = nw % XST;
                        if (!tc::mbar_wait(wfull + ws, (nw / WST) & 1, err) || !tc::mbar_wait(xfull + xs, (nw / XST) & 1, err)) {
                            ok = false;
                            break;
                        }
                        const int as = na % NA;
                        if (fmt == FMT_Q4 && !tc::mbar_wait(afull + as, (na / NA) & 1, err)) { ok = false; break; }
                        if (A.trace && cta == 0 && nw < 2048) A.trace[T_M + nw] = tc::gtime();
                        tc::tc_after();
                        const uint32_t xsa = tc::saddr(smem + X_OFF + xs * XSLOT);
                        if (fmt == FMT_Q4) {
                            const uint32_t ta = tmem + A_COL + 128 * as;
#pragma unroll
                            for (int q = 0; q < 4; q++) {
                                const uint64_t bd = tc::sw128_desc(xsa + q * BN * 128);
#pragma unroll
                                for (int kk = 0; kk < 4; kk++)
                                    tc::umma_ts(dacc, ta + q * 32 + kk * 8, bd + 2 * kk, IDESC, (s | q | kk) ? 1u : 0u);
                            }
                            tc::umma_commit(aempty + as);
                            na++;
                        } else {
                            const uint64_t ad = tc::sw128_desc(tc::saddr(smem + W_OFF + ws * WSLOT));
                            const uint64_t bd = tc::sw128_desc(xsa);
#pragma unroll
                            for (int kk = 0; kk < 4; kk++) tc::umma_ss(dacc, ad + 2 * kk, bd + 2 * kk, IDESC, (s | kk) ? 1u : 0u);
                        }
                        tc::umma_commit(wempty + ws);
                        tc::umma_commit(xempty + xs);
                    }
                    if (!ok) break;
                    tc::umma_commit(accfull + b);
                    nacc++;
                }
            }
            tc::umma_commit(mdone);  // after an early exit too: TMEM is freed only after the MMAs finish
        }
    } else {
        // ---- workers
        const int wt = tid - 64;                    // 0..255
        const int q4 = warp & 3, h = (warp - 2) >> 2;
        const int rl = 32 * q4 + lane;              // this thread's tile row (TMEM lane)
        const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
        constexpr int CW = BN / 2;
        float* sh = glue + 2 * 12 * 64;             // reduction scratch
        const int R = A.R;
        constexpr int GV = 2;                       // C <= 2048: two 16-byte column groups per thread
        int nw = 0, na = 0, nacc = 0;
        if (A.trace && cta == 0 && wt == 0) A.trace[0] = tc::gtime();
        for (int p = 0; p < A.nphases; p++) {
            const Phase ph = phs[p];
            if (ok) {
                const Layer* L = ph.layer >= 0 ? A.layers + ph.layer : nullptr;
                switch (ph.type) {
                    case PH_EMBED:
                        for (int n = cta; n < R; n += G) do_embed<GV>(A, n, sh, wt);
                        break;
                    case PH_TMIX:
                        for (int n = cta; n < R; n += G) do_tmix<GV>(A, *L, n, sh, wt);
                        break;
                    case PH_CMIX:
                        for (int n = cta; n < R; n += G) do_cmix<GV>(A, *L, n, sh, wt);
                        break;
                    case PH_LNOUT:
                        for (int n = cta; n < R; n += G) do_lnout<GV>(A, n, sh, wt);
                        break;
                    case PH_WKV: {
                        // two (row, head) items at a time; the next item's state is
                        // loaded while the current one is updated
                        const int half = wt >> 7, t = wt & 127, RH = R * A.H, l0 = ph.layer == 0;
                        float4 s[8], sn[8];
                        float f[9], fn[9];
                        int rh = 2 * cta + half;
                        if (rh < RH) {
                            wkv_load(*L, rh, t, s);
                            wkv_vec_load(A, *L, rh, l0, t, f);
                        }
                        for (; rh < RH; rh += 2 * G) {
                            if (rh + 2 * G < RH) {
                                wkv_load(*L, rh + 2 * G, t, sn);
                                wkv_vec_load(A, *L, rh + 2 * G, l0, t, fn);
                            }
                            do_wkv(A, *L, rh, l0, glue + half * 12 * 64, t, half, s, f);
#pragma unroll
                            for (int q = 0; q < 8; q++) s[q] = sn[q];
#pragma unroll
                            for (int q = 0; q < 9; q++) f[q] = fn[q];
                        }
                        break;
                    }
                    case PH_ARGMAX: {
                        const int V = A.V, ns = (V + ARGMAX_SLICE - 1) / ARGMAX_SLICE;
                        for (int it = cta; it < R * ns; it += G) {
                            const int n = it / ns, c0 = (it % ns) * ARGMAX_SLICE, cend = min(V, c0 + ARGMAX_SLICE);
                            const float* lp = A.logits + (int64_t)n * V;
                            unsigned long long best = 0ull;
                            for (int c = c0 + wt; c < cend; c += WT) best = max(best, argmax_key(lp[c], c));
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
                            if (lane == 0) atomicMax(A.amax_keys + n, best);
                        }
                        break;
                    }
                    case PH_ARGFIN:
                        for (int n = cta * WT + wt; n < R; n += G * WT) {
                            A.ids[n] = (int32_t)(0xFFFFFFFFu - (unsigned)(A.amax_keys[n] & 0xFFFFFFFFull));
                            A.amax_keys[n] = 0ull;
                        }
                        break;
                    case PH_GEMM: {
                        const int nacc0 = nacc;
                        for (int i = ph.i0 + cta; i < ph.i1 && ok; i += G) {
                            const Item it = A.items[i];
                            const Job& jb = A.jobs[it.job];
                            if (it.fmt == FMT_Q4) {
                                // dequantise each stage into a TMEM A stage
                                for (int s = 0; s < it.nst; s++, nw++, na++) {
                                    const int ws = nw % WST, as = na % NA;
                                    if (!tc::mbar_wait(wfull + ws, (nw / WST) & 1, err)) { ok = false; break; }
                                    if (na >= NA && !tc::mbar_wait(aempty + as, ((na / NA) - 1) & 1, err)) { ok = false; break; }
                                    tc::tc_after();
                                    const unsigned char* cs = smem + W_OFF + ws * WSLOT;
                                    const uint4 sbv = *reinterpret_cast<const uint4*>(cs + WCODE + rl * 16);
                                    const uint32_t sbw[4] = {sbv.x, sbv.y, sbv.z, sbv.w};  // group j: (scale, bias)
#pragma unroll
                                    for (int cc = 0; cc < 4; cc++) {
                                        const int ch = 4 * h + cc, gidx = ch >> 1;
                                        const __half2 sb2 = *reinterpret_cast<const __half2*>(&sbw[gidx]);
                                        const __half2 s2 = __half2half2(__low2half(sb2)), b2 = __half2half2(__high2half(sb2));
                                        const uint4 cw = *reinterpret_cast<const uint4*>(cs + swz(rl, ch, 128));
                                        uint32_t vv[16];
                                        tc::dq_word(cw.x, s2, b2, vv);
                                        tc::dq_word(cw.y, s2, b2, vv + 4);
                                        tc::dq_word(cw.z, s2, b2, vv + 8);
                                        tc::dq_word(cw.w, s2, b2, vv + 12);
                                        tc::tmem_st16(tmem + lane_base + A_COL + 128 * as + ch * 16, vv);
                                    }
                                    tc::tmem_st_wait();
                                    tc::tc_before();
                                    tc::mbar_arrive(afull + as);
                                    if (A.trace && cta == 0 && wt == 0 && nw < 2048) A.trace[T_D + nw] = tc::gtime();
                                }
                            } else {
                                nw += it.nst;
                            }
                            if (!ok) break;
                            // drain the accumulator: row rl, columns [h CW, (h+1) CW)
                            const int b = nacc % NACC;
                            if (!tc::mbar_wait(accfull + b, (nacc / NACC) & 1, err)) { ok = false; break; }
                            const bool tr = A.trace && cta == 0 && wt == 0 && nacc < 512;
                            if (tr) A.trace[T_E + 4 * nacc] = tc::gtime();
                            tc::tc_after();
                            uint32_t acc[CW];
#pragma unroll
                            for (int c = 0; c < CW; c += 4) tc::tmem_ld4_async(tmem + lane_base + 64 * b + h * CW + c, acc + c);
                            tc::tmem_ld_wait();
                            tc::tc_before();
                            tc::mbar_arrive(accempty + b);
                            if (tr) A.trace[T_E + 4 * nacc + 1] = tc::gtime();
                            const int item_no = nacc;
                            nacc++;
                            const GemvJob g = jb.g;
                            const int o = it.m0 + rl;
                            if (it.nz == 1) {
                                if (o < g.OUT) {
#pragma unroll
                                    for (int c = 0; c < CW; c++) {
                                        const int n = h * CW + c;
                                        if (n < R) epilogue(g, o, n, __uint_as_float(acc[c]));
                                    }
                                }
                            } else {
                                // split-K: publish this item's partial (release by one thread
                                // after the workers meet), then count it in the tile's ticket
                                float* part = A.ws + (size_t)it.slot * BN * 128;
#pragma unroll
                                for (int c = 0; c < CW; c++) part[(h * CW + c) * 128 + rl] = __uint_as_float(acc[c]);
                                wbar(1, WT);
                                if (wt == 0)
                                    asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(A.tickets + it.tile) : "memory");
                            }
                            if (tr) A.trace[T_E + 4 * item_no + 2] = tc::gtime();
                        }
                        // split tiles: once all of a tile's partials are in, item z sums
                        // rows [128 z / nz, 128 (z + 1) / nz) of it over the splits, in
                        // split order.  Every item of every CTA has published its partial
                        // before any CTA waits here, so the waits cannot form a cycle.
                        for (int i = ph.i0 + cta; i < ph.i1 && ok; i += G) {
                            const Item it = A.items[i];
                            if (it.nz == 1) continue;
                            if (wt == 0) {
                                int complete = 0;
                                const uint64_t t0 = tc::gtime();
                                for (uint32_t sp = 0;; sp++) {
                                    int v;
                                    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(A.tickets + it.tile) : "memory");
                                    if (v >= it.nz) { complete = 1; break; }
                                    if ((sp & 15) == 15) {
                                        if (*(volatile int*)err) break;
                                        if (tc::gtime() - t0 > tc::WAIT_LIMIT_NS) {
                                            atomicExch(err, 1);
                                            break;
                                        }
                                    }
                                }
                                *last_flag = complete;
                            }
                            wbar(1, WT);
                            if (!*last_flag) { ok = false; break; }
                            const GemvJob g = A.jobs[it.job].g;
                            const int q0 = 32 * it.z / it.nz, q1 = 32 * (it.z + 1) / it.nz;  // row quads
                            const int nq = q1 - q0;
                            const float* base = A.ws + (size_t)(it.slot - it.z) * BN * 128;
                            for (int task = wt; task < R * nq; task += WT) {
                                const int n = task / nq, rq = 4 * (q0 + task % nq);
                                float4 v = __ldcg(reinterpret_cast<const float4*>(base + (size_t)n * 128 + rq));
                                for (int z = 1; z < it.nz; z++) {
                                    const float4 u = __ldcg(reinterpret_cast<const float4*>(base + ((size_t)z * BN + n) * 128 + rq));
                                    v.x += u.x;
                                    v.y += u.y;
                                    v.z += u.z;
                                    v.w += u.w;
                                }
                                const float vv4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                                for (int j = 0; j < 4; j++)
                                    if (it.m0 + rq + j < g.OUT) epilogue(g, it.m0 + rq + j, n, vv4[j]);
                            }
                            const int k = nacc0 + (i - ph.i0 - cta) / G;
                            if (A.trace && cta == 0 && wt == 0 && k < 512) A.trace[T_E + 4 * k + 3] = tc::gtime();
                        }
                        break;
                    }
                }
            }
            // phase boundary
            if (A.trace && wt == 0 && cta < 160 && p < 256) A.trace[T_C + 160 * p + cta] = tc::gtime();
            if (!grid_barrier(A.bar, (unsigned int)(p + 1), err, wt, last_flag + 1)) ok = false;
            if (A.trace && cta == 0 && wt == 0) A.trace[p + 1] = tc::gtime();
        }
    }

    // wind down: every MMA has finished before TMEM is freed
    if (warp == 1 && lane == 0) tc::mbar_wait_own(mdone, 0, err);
    tc::tc_before();
    const int bad = __syncthreads_or(!ok && (warp >= 2 || lane == 0));
    if (warp == 1) {
        tc::tc_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
    if (tid == 0 && bad) {
        *(volatile int*)A.err_host = 1;
        __threadfence_system();
    }
}

}  // namespace pk
}  // namespace rwkv
