/*
 * rwkv_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, CPU restatement of the arithmetic of SwiftRWKV's two hot paths
 * (the WKV-7 recurrence and the quantised-weight dequant/GEMV), used as the
 * checker for the CUDA library and as the timed CPU baseline in bench.py.
 * Nothing in the product links or calls this file: only tests/, the smoke()
 * check in __graft_entry__.py and bench.py's CPU-baseline leg may load it.
 *
 * Compiled with -ffp-contract=off so that every a*b+c below is two roundings,
 * exactly as written, and every sum runs in the order written.  The reference
 * kernels are Metal source strings run by MLX (Swift), which cannot run here;
 * each function names the reference lines whose order it follows.
 *
 * Parity pins: the WKV forward/backward are checked against a torch-CPU
 * autograd restatement of the unrolled recurrence (WKV7Reference.swift:31-76)
 * and against the reference's own known-answer tests restated in
 * tests/golden; the sym/sb6 unpackers against the hand-computed cases of
 * RwkvqFileTests.swift:237-262 and RwkvqModelTests.swift:455-486.  The MLX
 * affine quantiser is restated from MLX's published algorithm and is
 * parity-unpinned (the reference holds no fixture for it).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define WKV_CHUNK 16 /* WKV7_CHUNK, WKV7.swift:8 */

/* ------------------------------------------------------------------ */
/* fp16 / bf16 conversions (round to nearest even)                     */
/* ------------------------------------------------------------------ */

float orc_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF, x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: m * 2^-24 */
            float f = (float)m * 5.9604644775390625e-08f;
            memcpy(&x, &f, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7F800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

uint16_t orc_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t mant = x & 0x007FFFFF;
    int32_t ex = (int32_t)((x >> 23) & 0xFF);
    if (ex == 0xFF) return (uint16_t)(sign | 0x7C00 | (mant ? 0x200 : 0));
    int32_t e = ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x00800000;
        int shift = 14 - e;
        uint32_t hm = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = mant >> 13, rem = mant & 0x1FFF;
    uint32_t h = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000 || (rem == 0x1000 && (hm & 1))) h++;
    return (uint16_t)h;
}

float orc_bf2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t orc_f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFF) > 0x7F800000) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFF + ((u >> 16) & 1);
    return (uint16_t)(u >> 16);
}

static inline float rh(float f) { return orc_h2f(orc_f2h(f)); } /* round through half */

void orc_f32_to_f16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_f2h(x[i]);
}
void orc_f16_to_f32(const uint16_t* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_h2f(x[i]);
}
void orc_f32_to_bf16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_f2bf(x[i]);
}
void orc_bf16_to_f32(const uint16_t* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_bf2f(x[i]);
}

/* ------------------------------------------------------------------ */
/* WKV-7                                                               */
/* ------------------------------------------------------------------ */

/*
 * Forward over [B,T,H,N] inputs, state S[b,h,dv,dk] (fp32).
 * Per step, for each value row dv (WKV7.swift:213-220, WKV7Train.swift:69-79):
 *   sa = sum_dk S[dv,dk]*a[dk]        (sequential in dk)
 *   S[dv,dk] = w[dk]*S[dv,dk] + v[dv]*k[dk] + sa*b[dk]
 *   y[dv] = sum_dk S[dv,dk]*r[dk]     (on the updated S)
 * h_in may be NULL (zeros).  sa_out / h_ckpt may be NULL; h_ckpt receives the
 * state after every `ckpt_every` steps, [B,H,T/ckpt_every,N,N]
 * (WKV7Train.swift:84-85).
 */
void orc_wkv7_forward(const float* r, const float* w, const float* k, const float* v,
                      const float* a, const float* b, const float* h_in, float* y,
                      float* h_out, float* sa_out, float* h_ckpt, int ckpt_every, int B,
                      int T, int H, int N) {
    int NC = (ckpt_every > 0) ? T / ckpt_every : 0;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int bi = 0; bi < B; bi++) {
        for (int hi = 0; hi < H; hi++) {
            float* S = (float*)malloc(sizeof(float) * N * N);
            size_t hb = ((size_t)bi * H + hi) * N * N;
            for (int i = 0; i < N * N; i++) S[i] = h_in ? h_in[hb + i] : 0.0f;
            for (int t = 0; t < T; t++) {
                size_t base = (((size_t)bi * T + t) * H + hi) * N;
                for (int dv = 0; dv < N; dv++) {
                    float* row = S + (size_t)dv * N;
                    float sa = 0.0f;
                    for (int dk = 0; dk < N; dk++) sa += row[dk] * a[base + dk];
                    if (sa_out) sa_out[base + dv] = sa;
                    float vv = v[base + dv];
                    for (int dk = 0; dk < N; dk++)
                        row[dk] = w[base + dk] * row[dk] + vv * k[base + dk] + sa * b[base + dk];
                    float yy = 0.0f;
                    for (int dk = 0; dk < N; dk++) yy += row[dk] * r[base + dk];
                    y[base + dv] = yy;
                }
                if (h_ckpt && ckpt_every > 0 && (t + 1) % ckpt_every == 0) {
                    int c = (t + 1) / ckpt_every - 1;
                    memcpy(h_ckpt + (((size_t)bi * H + hi) * NC + c) * N * N, S,
                           sizeof(float) * N * N);
                }
            }
            if (h_out) memcpy(h_out + hb, S, sizeof(float) * N * N);
            free(S);
        }
    }
}

/*
 * Backward, v2 scheme (WKV7Train.swift:247-330): column-held state rebuilt
 * backwards by dividing by w, starting from the end-of-chunk checkpoints;
 * four-accumulator dot products for dr/da (dot4, :211-218) and two
 * accumulators for dw/dk/dv/db/dSb (:296-309).  d_h_out may be NULL (zeros).
 * Requires T % 16 == 0 (WKV7Train.swift:380-381).
 */
void orc_wkv7_backward_v2(const float* r, const float* w, const float* k, const float* v,
                          const float* a, const float* b, const float* h_ckpt,
                          const float* sa_fwd, const float* d_out, const float* d_h_out,
                          float* dr_out, float* dw_out, float* dk_out, float* dv_out,
                          float* da_out, float* db_out, float* dh_in, int B, int T, int H,
                          int N) {
    int NC = T / WKV_CHUNK;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int bidx = 0; bidx < B; bidx++) {
        for (int hi = 0; hi < H; hi++) {
            size_t NN = (size_t)N * N;
            float* stT = (float*)malloc(sizeof(float) * NN);  /* stT[i*N+j] = S[j][i] */
            float* dst = (float*)malloc(sizeof(float) * NN);  /* dst[i*N+j] = dS[i][j] */
            float* dstT = (float*)malloc(sizeof(float) * NN); /* dstT[i*N+j] = dS[j][i] */
            float* dsb = (float*)malloc(sizeof(float) * N);
            float* dsbv = (float*)malloc(sizeof(float) * N);
            size_t hbase = ((size_t)bidx * H + hi) * NN;
            for (int i = 0; i < N; i++)
                for (int j = 0; j < N; j++) {
                    dst[i * N + j] = d_h_out ? d_h_out[hbase + (size_t)i * N + j] : 0.0f;
                    dstT[i * N + j] = d_h_out ? d_h_out[hbase + (size_t)j * N + i] : 0.0f;
                }
            for (int c = NC - 1; c >= 0; c--) {
                size_t ckb = (((size_t)bidx * H + hi) * NC + c) * NN;
                for (int i = 0; i < N; i++)
                    for (int j = 0; j < N; j++) stT[i * N + j] = h_ckpt[ckb + (size_t)j * N + i];
                for (int t = WKV_CHUNK - 1; t >= 0; t--) {
                    size_t base = (((size_t)bidx * T + (size_t)c * WKV_CHUNK + t) * H + hi) * N;
                    const float *rs = r + base, *ws = w + base, *ks = k + base, *vs = v + base;
                    const float *as = a + base, *bs = b + base, *dys = d_out + base;
                    const float* sas = sa_fwd + base;
                    for (int i = 0; i < N; i++) {
                        float* st = stT + (size_t)i * N;
                        float* u = dst + (size_t)i * N;
                        float* tt = dstT + (size_t)i * N;
                        float ri = rs[i], wi = ws[i], ki = ks[i], bb = bs[i], dyi = dys[i];
                        /* dr[i] = sum_j S[j][i]*dy[j] on the post-update state */
                        float d0 = 0, d1 = 0, d2 = 0, d3 = 0;
                        for (int j = 0; j < N; j += 4) {
                            d0 += st[j] * dys[j];
                            d1 += st[j + 1] * dys[j + 1];
                            d2 += st[j + 2] * dys[j + 2];
                            d3 += st[j + 3] * dys[j + 3];
                        }
                        dr_out[base + i] = (d0 + d1) + (d2 + d3);
                        float iwi = 1.0f / wi;
                        for (int j = 0; j < N; j++) {
                            st[j] = (st[j] - vs[j] * ki - sas[j] * bb) * iwi;
                            u[j] += dyi * rs[j];
                            tt[j] += ri * dys[j];
                        }
                        float dw0 = 0, dw1 = 0, dkv0 = 0, dkv1 = 0, dvv0 = 0, dvv1 = 0;
                        float db0 = 0, db1 = 0, dsb0 = 0, dsb1 = 0;
                        for (int j = 0; j < N; j += 2) {
                            float tA = tt[j], tB = tt[j + 1];
                            float sA = st[j], sB = st[j + 1];
                            float uA = u[j], uB = u[j + 1];
                            dw0 += tA * sA;
                            dw1 += tB * sB;
                            dkv0 += tA * vs[j];
                            dkv1 += tB * vs[j + 1];
                            db0 += tA * sas[j];
                            db1 += tB * sas[j + 1];
                            dvv0 += uA * ks[j];
                            dvv1 += uB * ks[j + 1];
                            dsb0 += uA * bs[j];
                            dsb1 += uB * bs[j + 1];
                        }
                        dw_out[base + i] = dw0 + dw1;
                        dk_out[base + i] = dkv0 + dkv1;
                        dv_out[base + i] = dvv0 + dvv1;
                        db_out[base + i] = db0 + db1;
                        dsb[i] = dsb0 + dsb1;
                    }
                    for (int i = 0; i < N; i++) dsbv[i] = dsb[i];
                    for (int i = 0; i < N; i++) {
                        float* st = stT + (size_t)i * N;
                        float d0 = 0, d1 = 0, d2 = 0, d3 = 0;
                        for (int j = 0; j < N; j += 4) {
                            d0 += st[j] * dsbv[j];
                            d1 += st[j + 1] * dsbv[j + 1];
                            d2 += st[j + 2] * dsbv[j + 2];
                            d3 += st[j + 3] * dsbv[j + 3];
                        }
                        da_out[base + i] = (d0 + d1) + (d2 + d3);
                    }
                    for (int i = 0; i < N; i++) {
                        float* u = dst + (size_t)i * N;
                        float* tt = dstT + (size_t)i * N;
                        float wi = ws[i], ai = as[i], dsbi = dsb[i];
                        for (int j = 0; j < N; j++) {
                            u[j] = u[j] * ws[j] + dsbi * as[j];
                            tt[j] = tt[j] * wi + ai * dsbv[j];
                        }
                    }
                }
            }
            for (int i = 0; i < N; i++)
                for (int j = 0; j < N; j++) dh_in[hbase + (size_t)i * N + j] = dst[i * N + j];
            free(stT);
            free(dst);
            free(dstT);
            free(dsb);
            free(dsbv);
        }
    }
}

/*
 * Exact (double-precision) forward + backward of the same recurrence, the
 * semantics of the autograd reference (WKV7Reference.swift:31-76): states are
 * stored for every step, so nothing is rebuilt by division.  Used to put
 * error bars on both the fp32 oracle above and the GPU kernels.
 * Any of h_in / d_h_out may be NULL.  Outputs in fp32 after a double
 * computation.  Memory: B*H*(T+1)*N*N doubles per (b,h) in flight.
 */
void orc_wkv7_exact(const float* r, const float* w, const float* k, const float* v,
                    const float* a, const float* b, const float* h_in, const float* d_out,
                    const float* d_h_out, float* y, float* h_out, float* dr, float* dw,
                    float* dk, float* dv, float* da, float* db, float* dh_in, int B, int T,
                    int H, int N) {
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int bi = 0; bi < B; bi++) {
        for (int hi = 0; hi < H; hi++) {
            size_t NN = (size_t)N * N;
            double* S = (double*)malloc(sizeof(double) * NN * (T + 1));
            double* sa = (double*)malloc(sizeof(double) * (size_t)N * T);
            double* dS = (double*)malloc(sizeof(double) * NN);
            double* dsa = (double*)malloc(sizeof(double) * N);
            size_t hb = ((size_t)bi * H + hi) * NN;
            for (size_t i = 0; i < NN; i++) S[i] = h_in ? (double)h_in[hb + i] : 0.0;
            for (int t = 0; t < T; t++) {
                size_t base = (((size_t)bi * T + t) * H + hi) * N;
                double* P = S + (size_t)t * NN;
                double* Q = S + (size_t)(t + 1) * NN;
                for (int dv_ = 0; dv_ < N; dv_++) {
                    double s = 0;
                    for (int dk_ = 0; dk_ < N; dk_++) s += P[dv_ * N + dk_] * (double)a[base + dk_];
                    sa[(size_t)t * N + dv_] = s;
                    double yy = 0;
                    for (int dk_ = 0; dk_ < N; dk_++) {
                        double q = (double)w[base + dk_] * P[dv_ * N + dk_] +
                                   (double)v[base + dv_] * (double)k[base + dk_] +
                                   s * (double)b[base + dk_];
                        Q[dv_ * N + dk_] = q;
                        yy += q * (double)r[base + dk_];
                    }
                    if (y) y[base + dv_] = (float)yy;
                }
            }
            if (h_out)
                for (size_t i = 0; i < NN; i++) h_out[hb + i] = (float)S[(size_t)T * NN + i];
            if (dr) {
                for (size_t i = 0; i < NN; i++) dS[i] = d_h_out ? (double)d_h_out[hb + i] : 0.0;
                for (int t = T - 1; t >= 0; t--) {
                    size_t base = (((size_t)bi * T + t) * H + hi) * N;
                    double* P = S + (size_t)t * NN;
                    double* Q = S + (size_t)(t + 1) * NN;
                    const float *rs = r + base, *ws = w + base, *ks = k + base, *vs = v + base;
                    const float *as = a + base, *bs = b + base, *dys = d_out + base;
                    for (int i = 0; i < N; i++) { /* dr_i = sum_j Q[j][i] dy_j */
                        double s = 0;
                        for (int j = 0; j < N; j++) s += Q[j * N + i] * (double)dys[j];
                        dr[base + i] = (float)s;
                    }
                    for (int j = 0; j < N; j++)
                        for (int i = 0; i < N; i++) dS[j * N + i] += (double)dys[j] * (double)rs[i];
                    for (int j = 0; j < N; j++) {
                        double sv = 0, sb = 0;
                        for (int i = 0; i < N; i++) {
                            sv += dS[j * N + i] * (double)ks[i];
                            sb += dS[j * N + i] * (double)bs[i];
                        }
                        dv[base + j] = (float)sv;
                        dsa[j] = sb;
                    }
                    for (int i = 0; i < N; i++) {
                        double sw = 0, sk = 0, sbb = 0, saa = 0;
                        for (int j = 0; j < N; j++) {
                            sw += dS[j * N + i] * P[j * N + i];
                            sk += dS[j * N + i] * (double)vs[j];
                            sbb += dS[j * N + i] * sa[(size_t)t * N + j];
                            saa += P[j * N + i] * dsa[j];
                        }
                        dw[base + i] = (float)sw;
                        dk[base + i] = (float)sk;
                        db[base + i] = (float)sbb;
                        da[base + i] = (float)saa;
                    }
                    for (int j = 0; j < N; j++)
                        for (int i = 0; i < N; i++)
                            dS[j * N + i] = dS[j * N + i] * (double)ws[i] + dsa[j] * (double)as[i];
                }
                for (size_t i = 0; i < NN; i++) dh_in[hb + i] = (float)dS[i];
            }
            free(S);
            free(sa);
            free(dS);
            free(dsa);
        }
    }
}

/*
 * wkvTail (WKV7DecodeKernels.swift:123-157), per (row, head):
 *   GroupNorm over the head's S values, two passes, eps; bonus dp = sum r*k*r_k;
 *   out = ((norm*lnw + lnb) + dp*v) * g.
 * wkv/r/k/v/g are [rows, H*S]; rk/lnw/lnb are [H*S].
 */
void orc_wkv_tail(const float* wkv, const float* r, const float* k, const float* v,
                  const float* rk, const float* lnw, const float* lnb, const float* g,
                  float* out, int rows, int H, int S, float eps) {
    for (int tg = 0; tg < rows * H; tg++) {
        int h = tg % H;
        size_t base = (size_t)tg * S, hb = (size_t)h * S;
        float s1 = 0;
        for (int i = 0; i < S; i++) s1 += wkv[base + i];
        float mean = s1 / (float)S;
        float s2 = 0;
        for (int i = 0; i < S; i++) {
            float d = wkv[base + i] - mean;
            s2 += d * d;
        }
        float inv = 1.0f / sqrtf(s2 / (float)S + eps);
        float dp = 0;
        for (int i = 0; i < S; i++) dp += r[base + i] * k[base + i] * rk[hb + i];
        for (int i = 0; i < S; i++) {
            float nrm = (wkv[base + i] - mean) * inv;
            float yy = nrm * lnw[hb + i] + lnb[hb + i] + dp * v[base + i];
            out[base + i] = yy * g[base + i];
        }
    }
}

/* ------------------------------------------------------------------ */
/* MLX affine container (QLoRA base): w = scale*q + bias per group      */
/* ------------------------------------------------------------------ */

/* Field p of a row is the LSB-first bit field starting at global bit p*bits
 * of the row's u32 words (RwkvqNative.swift:28-31,161-175). */
static inline uint32_t get_code(const uint32_t* row, int64_t p, int bits) {
    int64_t bit = p * bits;
    int64_t w0 = bit >> 5;
    int off = (int)(bit & 31);
    uint64_t word = (uint64_t)row[w0];
    if (off + bits > 32) word |= (uint64_t)row[w0 + 1] << 32;
    return (uint32_t)((word >> off) & ((1u << bits) - 1));
}

static inline void put_code(uint32_t* row, int64_t p, int bits, uint32_t q) {
    int64_t bit = p * bits;
    int64_t w0 = bit >> 5;
    int off = (int)(bit & 31);
    row[w0] |= q << off;
    if (off + bits > 32) row[w0 + 1] |= q >> (32 - off);
}

/*
 * Affine quantiser writing MLX's container: restated from MLX's published
 * affine_quantize (mlx core as shipped with mlx-swift 0.31.4, called at
 * LoRA.swift:68): per group, scale = max((wmax-wmin)/(2^bits-1), 1e-7) signed
 * toward the larger-magnitude edge, the edge snapped onto the integer grid
 * (scale = edge/round(edge/scale)), bias = edge (0 when that rounds to 0),
 * q = clip(round((w - bias)/scale), 0, 2^bits-1); scale and bias stored in the
 * weight's dtype (fp16 here).  W is [OUT, IN] fp32 values (already fp16-exact).
 * PARITY-UNPINNED: no fixture of MLX's quantiser exists in the reference.
 */
void orc_affine_quantize(const float* W, int OUT, int IN, int group, int bits, uint32_t* wq,
                         uint16_t* scales, uint16_t* biases) {
    int64_t wpr = (int64_t)IN * bits / 32;
    int NG = IN / group;
    float n_bins = (float)((1 << bits) - 1);
#pragma omp parallel for schedule(static)
    for (int o = 0; o < OUT; o++) {
        uint32_t* row = wq + (int64_t)o * wpr;
        memset(row, 0, sizeof(uint32_t) * wpr);
        for (int g = 0; g < NG; g++) {
            const float* x = W + (int64_t)o * IN + (int64_t)g * group;
            float wmax = x[0], wmin = x[0];
            for (int i = 1; i < group; i++) {
                if (x[i] > wmax) wmax = x[i];
                if (x[i] < wmin) wmin = x[i];
            }
            int mask = fabsf(wmin) > fabsf(wmax);
            float scale = (wmax - wmin) / n_bins;
            if (scale < 1e-7f) scale = 1e-7f;
            if (!mask) scale = -scale;
            float edge = mask ? wmin : wmax;
            float q0 = rintf(edge / scale);
            if (q0 != 0.0f) scale = edge / q0;
            float bias = (q0 == 0.0f) ? 0.0f : edge;
            for (int i = 0; i < group; i++) {
                float q = rintf((x[i] - bias) / scale);
                if (q < 0) q = 0;
                if (q > n_bins) q = n_bins;
                put_code(row, (int64_t)g * group + i, bits, (uint32_t)q);
            }
            scales[(int64_t)o * NG + g] = orc_f2h(scale);
            biases[(int64_t)o * NG + g] = orc_f2h(bias);
        }
    }
}

/* Unpacker: w = float(q)*float(scale) + float(bias), one rounding (the product
 * of a <=8-bit code and an fp16 scale is exact in fp32).  scales/biases are
 * fp16 (sdtype 2) or fp32 (sdtype 0). */
static inline float sb_get(const void* p, int64_t i, int sdtype) {
    if (sdtype == 0) return ((const float*)p)[i];
    if (sdtype == 1) return orc_bf2f(((const uint16_t*)p)[i]);
    return orc_h2f(((const uint16_t*)p)[i]);
}

void orc_affine_dequant(const uint32_t* wq, const void* scales, const void* biases, int sdtype,
                        float* out, int OUT, int IN, int group, int bits) {
    int64_t wpr = (int64_t)IN * bits / 32;
    int NG = IN / group;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < OUT; o++) {
        const uint32_t* row = wq + (int64_t)o * wpr;
        for (int i = 0; i < IN; i++) {
            float s = sb_get(scales, (int64_t)o * NG + i / group, sdtype);
            float bb = sb_get(biases, (int64_t)o * NG + i / group, sdtype);
            out[(int64_t)o * IN + i] = (float)get_code(row, i, bits) * s + bb;
        }
    }
}

/* y[n,o] = sum_i x[n,i]*w[o,i] with w the fp32 dequantised weight, the sum in
 * double: the "exact fp32 matmul of the GEMV's own dequant" that
 * RwkvqSb6GEMVTests.swift:53-77 compares against.  x is fp32 [rows, IN]. */
void orc_affine_gemv_exact(const float* x, const uint32_t* wq, const void* scales,
                           const void* biases, int sdtype, float* y, int rows, int OUT, int IN,
                           int group, int bits) {
    int64_t wpr = (int64_t)IN * bits / 32;
    int NG = IN / group;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < OUT; o++) {
        const uint32_t* row = wq + (int64_t)o * wpr;
        for (int n = 0; n < rows; n++) {
            double acc = 0;
            for (int i = 0; i < IN; i++) {
                float s = sb_get(scales, (int64_t)o * NG + i / group, sdtype);
                float bb = sb_get(biases, (int64_t)o * NG + i / group, sdtype);
                float wv = (float)get_code(row, i, bits) * s + bb;
                acc += (double)x[(int64_t)n * IN + i] * (double)wv;
            }
            y[(int64_t)n * OUT + o] = (float)acc;
        }
    }
}

/* The same product as quantizedMM computes it (MLX's qdot, accumulation in
 * fp32): per group  scale * sum(q*x) + bias * sum(x).  This is also the CPU
 * baseline's GEMV.  x fp32 [rows, IN]. */
void orc_affine_gemv(const float* x, const uint32_t* wq, const void* scales, const void* biases,
                     int sdtype, float* y, int rows, int OUT, int IN, int group, int bits) {
    int64_t wpr = (int64_t)IN * bits / 32;
    int NG = IN / group;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < OUT; o++) {
        const uint32_t* row = wq + (int64_t)o * wpr;
        for (int n = 0; n < rows; n++) {
            const float* xn = x + (int64_t)n * IN;
            float acc = 0;
            for (int g = 0; g < NG; g++) {
                float s = sb_get(scales, (int64_t)o * NG + g, sdtype);
                float bb = sb_get(biases, (int64_t)o * NG + g, sdtype);
                float dq = 0, xs = 0;
                if (bits == 4) {
                    const uint32_t* wp = row + (int64_t)g * group / 8;
                    for (int j = 0; j < group / 8; j++) {
                        uint32_t word = wp[j];
                        const float* xx = xn + (int64_t)g * group + j * 8;
                        for (int u = 0; u < 8; u++) {
                            dq += (float)((word >> (4 * u)) & 15u) * xx[u];
                            xs += xx[u];
                        }
                    }
                } else {
                    for (int i = 0; i < group; i++) {
                        int64_t col = (int64_t)g * group + i;
                        dq += (float)get_code(row, col, bits) * xn[col];
                        xs += xn[col];
                    }
                }
                acc += s * dq + bb * xs;
            }
            y[(int64_t)n * OUT + o] = acc;
        }
    }
}

/* ------------------------------------------------------------------ */
/* .rwkvq sb6 (K3 interleave): w = code*half(qs*d) + half(qm*dm)       */
/* ------------------------------------------------------------------ */

/* Codes of one 32-column block (RwkvqDequant.swift:116-127): 16 nibble
 * bytes, byte j -> column j (low) and j+16 (high); optional bit-planes qh
 * (bit 4) and qh2 (bit 5) as u32 masks, bit c -> column c. */
static inline void sb6_codes(const uint8_t* blk, int xbits, uint8_t nib[32]) {
    for (int j = 0; j < 16; j++) {
        nib[j] = blk[j] & 0xF;
        nib[j + 16] = (blk[j] >> 4) & 0xF;
    }
    if (xbits >= 1) {
        uint32_t hb;
        memcpy(&hb, blk + 16, 4);
        for (int c = 0; c < 32; c++) nib[c] |= (uint8_t)(((hb >> c) & 1u) << 4);
    }
    if (xbits >= 2) {
        uint32_t hb2;
        memcpy(&hb2, blk + 20, 4);
        for (int c = 0; c < 32; c++) nib[c] |= (uint8_t)(((hb2 >> c) & 1u) << 5);
    }
}

static inline void sb6_scales(const uint8_t* qsqm, const uint16_t* ddm, int64_t row, int NB,
                              int NSB, int blk, float* s, float* m) {
    uint8_t qs = qsqm[2 * (row * NB + blk)];
    int8_t qm = (int8_t)qsqm[2 * (row * NB + blk) + 1];
    int64_t sb = row * NSB + blk / 8;
    float d = orc_h2f(ddm[2 * sb]), dm = orc_h2f(ddm[2 * sb + 1]);
    *s = rh((float)qs * d);
    *m = rh((float)qm * dm);
}

/* Dense [OUT, IN] fp32 (RwkvqDequant.swift:110-141; combine in float). */
void orc_sb6_dequant(const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm, float* out,
                     int OUT, int IN, int xbits) {
    int NB = IN / 32, NSB = NB / 8, BB = 16 + 4 * xbits;
#pragma omp parallel for schedule(static)
    for (int row = 0; row < OUT; row++) {
        for (int blk = 0; blk < NB; blk++) {
            uint8_t nib[32];
            sb6_codes(qblk + ((int64_t)row * NB + blk) * BB, xbits, nib);
            float s, m;
            sb6_scales(qsqm, ddm, row, NB, NSB, blk, &s, &m);
            float* o = out + (int64_t)row * IN + blk * 32;
            for (int c = 0; c < 32; c++) o[c] = (float)nib[c] * s + m;
        }
    }
}

/* One input row (RwkvqSb6GEMV.swift:118-144): per 32-block s*sum(q*x) + m*xbsum,
 * xbsum = sum of x over the block.  x fp32 [IN]. */
void orc_sb6_gemv(const float* x, const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm,
                  float* y, int OUT, int IN, int xbits) {
    int NB = IN / 32, NSB = NB / 8, BB = 16 + 4 * xbits;
#pragma omp parallel for schedule(static)
    for (int row = 0; row < OUT; row++) {
        float acc = 0;
        for (int blk = 0; blk < NB; blk++) {
            uint8_t nib[32];
            sb6_codes(qblk + ((int64_t)row * NB + blk) * BB, xbits, nib);
            float s, m;
            sb6_scales(qsqm, ddm, row, NB, NSB, blk, &s, &m);
            float dv = 0, xbs = 0;
            for (int c = 0; c < 32; c++) {
                dv += x[blk * 32 + c] * (float)nib[c];
                xbs += x[blk * 32 + c];
            }
            acc += s * dv + m * xbs;
        }
        y[row] = acc;
    }
}

/*
 * sb6 -> MLX affine container, lossless (RwkvqNative.swift:87-196): codes of
 * 4+xbits bits re-packed as an LSB-first bit stream per 32-column group;
 * scale = max(float(half(qs*d)), 1e-8), bias = float(half(qm*dm)).  Scales
 * and biases are written as fp32 here; *fp16_ok is set to 1 when storing them
 * as fp16 would change no dequantised weight (the exactScales rule).
 */
void orc_sb6_to_affine(const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm,
                       uint32_t* wq, float* scales, float* biases, int OUT, int IN, int xbits,
                       int* fp16_ok) {
    int NB = IN / 32, NSB = NB / 8, BB = 16 + 4 * xbits, bits = 4 + xbits;
    int64_t wpr = (int64_t)NB * bits;
    int ok = 1;
    for (int row = 0; row < OUT; row++) {
        uint32_t* wr = wq + (int64_t)row * wpr;
        memset(wr, 0, sizeof(uint32_t) * wpr);
        for (int blk = 0; blk < NB; blk++) {
            uint8_t nib[32];
            sb6_codes(qblk + ((int64_t)row * NB + blk) * BB, xbits, nib);
            float s, m;
            sb6_scales(qsqm, ddm, row, NB, NSB, blk, &s, &m);
            float s32 = s < 1e-8f ? 1e-8f : s;
            if (rh(s32) != s32) {
                for (int c = 0; c < 32; c++)
                    if ((float)nib[c] * rh(s32) + m != (float)nib[c] * s32 + m) ok = 0;
            }
            scales[(int64_t)row * NB + blk] = s32;
            biases[(int64_t)row * NB + blk] = m;
            for (int c = 0; c < 32; c++) put_code(wr, (int64_t)blk * 32 + c, bits, nib[c]);
        }
    }
    *fp16_ok = ok;
}

/* ------------------------------------------------------------------ */
/* .rwkvq sym (blocks of 16, int8 block scale x fp16 d per 256)         */
/* ------------------------------------------------------------------ */

/* Codes of one 32-column pair of 16-blocks at 6 bits (RwkvqDequant.swift:
 * 363-388): 16 nibble bytes, byte j of block q carries column j (low) and j+8
 * (high); 2 bit-planes (bit c -> column c of the pair); stored +32. */
static inline void sym6_codes(const uint8_t* pb, int code[32]) {
    for (int blk = 0; blk < 2; blk++)
        for (int j = 0; j < 8; j++) {
            uint8_t byte = pb[blk * 8 + j];
            code[blk * 16 + j] = byte & 0xF;
            code[blk * 16 + j + 8] = (byte >> 4) & 0xF;
        }
    uint32_t hb, hb2;
    memcpy(&hb, pb + 16, 4);
    memcpy(&hb2, pb + 20, 4);
    for (int c = 0; c < 32; c++) {
        code[c] |= (int)(((hb >> c) & 1u) << 4);
        code[c] |= (int)(((hb2 >> c) & 1u) << 5);
        code[c] -= 32;
    }
}

/* Dense [OUT, IN]; odtype 0 f32 (float product, codec.dequant_sym), 1 bf16
 * (float product, one rounding), 2 f16 (product in half).  out is a float
 * array for f32 and a uint16 array otherwise (RwkvqDequant.swift:320-400,
 * the :442-466 chain for IN % 256 != 0 at 8 bits). */
void orc_sym_dequant(const uint8_t* qblk, const uint8_t* qs, const uint16_t* d, void* out,
                     int odtype, int OUT, int IN, int bits) {
    int NB = IN / 16, NSB = (IN + 255) / 256;
#pragma omp parallel for schedule(static)
    for (int row = 0; row < OUT; row++) {
        for (int c = 0; c < IN; c++) {
            int blk = c / 16;
            float dsb = orc_h2f(d[(int64_t)row * NSB + blk / 16]);
            float s = rh((float)(int8_t)qs[(int64_t)row * NB + blk] * dsb);
            int code;
            if (bits == 8) {
                code = (int8_t)qblk[(int64_t)row * IN + c];
            } else {
                int cc[32];
                sym6_codes(qblk + ((int64_t)row * (IN / 32) + c / 32) * 24, cc);
                code = cc[c % 32];
            }
            float val = (float)code * s;
            int64_t idx = (int64_t)row * IN + c;
            if (odtype == 0)
                ((float*)out)[idx] = val;
            else if (odtype == 1)
                ((uint16_t*)out)[idx] = orc_f2bf(val);
            else
                ((uint16_t*)out)[idx] = orc_f2h(val);
        }
    }
}

/* sym GEMV (RwkvqSymGEMV.swift:126-199): x fp32 [NN*NK, IN] where the K
 * fused matrices of out_per rows each take their own input row
 * (xi = row / out_per); y [NN, OUT]. */
void orc_sym_gemv(const float* x, const uint8_t* qblk, const uint8_t* qs, const uint16_t* d,
                  float* y, int NN, int OUT, int IN, int bits, int out_per) {
    int NB = IN / 16, NSB = IN / 256, NK = OUT / out_per;
#pragma omp parallel for schedule(static)
    for (int row = 0; row < OUT; row++) {
        int xi = row / out_per;
        for (int n = 0; n < NN; n++) {
            const float* xn = x + ((int64_t)n * NK + xi) * IN;
            float acc = 0;
            if (bits == 8) {
                for (int p = 0; p < NB; p++) {
                    float s = rh((float)(int8_t)qs[(int64_t)row * NB + p] *
                                 orc_h2f(d[(int64_t)row * NSB + p / 16]));
                    float dv = 0;
                    for (int c = 0; c < 16; c++)
                        dv += xn[p * 16 + c] * (float)(int8_t)qblk[(int64_t)row * IN + p * 16 + c];
                    acc += s * dv;
                }
            } else {
                for (int p = 0; p < IN / 32; p++) {
                    int cc[32];
                    sym6_codes(qblk + ((int64_t)row * (IN / 32) + p) * 24, cc);
                    float dsb = orc_h2f(d[(int64_t)row * NSB + p / 8]);
                    float s0 = rh((float)(int8_t)qs[(int64_t)row * NB + 2 * p] * dsb);
                    float s1 = rh((float)(int8_t)qs[(int64_t)row * NB + 2 * p + 1] * dsb);
                    float dv0 = 0, dv1 = 0, b0 = 0, b1 = 0;
                    for (int c = 0; c < 16; c++) {
                        dv0 += xn[p * 32 + c] * (float)(cc[c] + 32);
                        b0 += xn[p * 32 + c];
                        dv1 += xn[p * 32 + 16 + c] * (float)(cc[16 + c] + 32);
                        b1 += xn[p * 32 + 16 + c];
                    }
                    acc += s0 * (dv0 - 32.0f * b0) + s1 * (dv1 - 32.0f * b1);
                }
            }
            y[(int64_t)n * OUT + row] = acc;
        }
    }
}

/* Embedding rows from an 8-bit sym table (RwkvqSymRows.swift:402-411):
 * out[n, c] = half(code * half(qs*d)), fp16 bits. */
void orc_sym_rows(const int32_t* ids, int n_ids, const uint8_t* codes, const uint8_t* qs,
                  const uint16_t* d, uint16_t* out, int IN) {
    int NB = IN / 16, NSB = (IN + 255) / 256;
    for (int n = 0; n < n_ids; n++) {
        int64_t row = ids[n];
        for (int c = 0; c < IN; c++) {
            float s = rh((float)(int8_t)qs[row * NB + c / 16] * orc_h2f(d[row * NSB + c / 256]));
            out[(int64_t)n * IN + c] = orc_f2h((float)(int8_t)codes[row * IN + c] * s);
        }
    }
}
