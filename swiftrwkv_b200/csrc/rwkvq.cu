// .rwkvq base formats (Sources/RWKVQuant): sb6 (K3 interleave, blocks of 32,
// 4-6 bit codes with an fp16-rounded scale and min per block) and sym
// (blocks of 16, 6/8-bit symmetric codes, int8 block scale x fp16 d per 256).
//
// sb6 block (RwkvqDequant.swift:30-35): 16 bytes of nibbles -- byte j gives
// column j (low) and j+16 (high) -- then optional bit-plane words qh (bit 4)
// and qh2 (bit 5), bit c -> column c.  s = half(qs*d), m = half(qm*dm),
// w = code*s + m combined in fp32.
// sym 6-bit pair of 16-blocks (RwkvqDequant.swift:363-388): 16 nibble bytes,
// byte j of block q -> column j (low) and j+8 (high) of that block, two
// bit-planes over the pair's 32 columns; codes stored +32.
//
// GEMVs: one warp per output row, lanes strided over blocks, fp32
// accumulation of s*sum(q*x) + m*sum(x) per block (sb6) or
// s*(sum(q*x) - 32*sum(x)) per 16-block (sym 6-bit), warp shuffle reduction.
#include "common.cuh"
#include "gemv_mma.cuh"

namespace rwkv {

__device__ __forceinline__ float rnd_half(float f) { return __half2float(__float2half_rn(f)); }

// Blocks are 16 + 4*xbits bytes (20 or 24 at xbits 1/2), so only 4-byte
// alignment holds: the block is read as u32 words, never as a 16-byte vector.
__device__ __forceinline__ void sb6_block_codes(const uint8_t* blk, int xbits, uint8_t nib[32]) {
    const uint32_t* bw = reinterpret_cast<const uint32_t*>(blk);
    const uint32_t wds[4] = {bw[0], bw[1], bw[2], bw[3]};
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const uint8_t byte = (uint8_t)(wds[j >> 2] >> (8 * (j & 3)));
        nib[j] = byte & 0xF;
        nib[j + 16] = byte >> 4;
    }
    if (xbits >= 1) {
        const uint32_t hb = *reinterpret_cast<const uint32_t*>(blk + 16);
#pragma unroll
        for (int c = 0; c < 32; c++) nib[c] |= (uint8_t)(((hb >> c) & 1u) << 4);
    }
    if (xbits >= 2) {
        const uint32_t hb2 = *reinterpret_cast<const uint32_t*>(blk + 20);
#pragma unroll
        for (int c = 0; c < 32; c++) nib[c] |= (uint8_t)(((hb2 >> c) & 1u) << 5);
    }
}

__device__ __forceinline__ void sb6_block_scales(const uint8_t* qsqm, const __half* ddm, int64_t row,
                                                 int NB, int NSB, int blk, float& s, float& m) {
    const uint8_t qs = qsqm[2 * (row * NB + blk)];
    const int8_t qm = (int8_t)qsqm[2 * (row * NB + blk) + 1];
    const int64_t sb = row * NSB + blk / 8;
    s = rnd_half((float)qs * __half2float(ddm[2 * sb]));
    m = rnd_half((float)qm * __half2float(ddm[2 * sb + 1]));
}

template <typename TO>
__global__ void sb6_dequant_kernel(const uint8_t* __restrict__ qblk, const uint8_t* __restrict__ qsqm,
                                   const __half* __restrict__ ddm, TO* __restrict__ out, int OUT,
                                   int IN, int xbits) {
    const int NB = IN / 32, NSB = NB / 8, BB = 16 + 4 * xbits;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)OUT * NB) return;
    const int64_t row = idx / NB;
    const int blk = (int)(idx % NB);
    uint8_t nib[32];
    sb6_block_codes(qblk + (row * NB + blk) * BB, xbits, nib);
    float s, m;
    sb6_block_scales(qsqm, ddm, row, NB, NSB, blk, s, m);
    TO* o = out + row * IN + blk * 32;
#pragma unroll
    for (int c = 0; c < 32; c++) o[c] = from_f<TO>((float)nib[c] * s + m);
}

template <typename TX, int R, bool EP = false>
__global__ void __launch_bounds__(256)
sb6_gemv_kernel(const TX* __restrict__ x, const uint8_t* __restrict__ qblk,
                const uint8_t* __restrict__ qsqm, const __half* __restrict__ ddm,
                float* __restrict__ y, int OUT, int IN, int xbits, const GemvJob jb, int n0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= OUT) return;
    const int NB = IN / 32, NSB = NB / 8, BB = 16 + 4 * xbits;
    float acc[R];
#pragma unroll
    for (int n = 0; n < R; n++) acc[n] = 0.f;
    for (int p = lane; p < NB; p += 32) {
        uint8_t nib[32];
        sb6_block_codes(qblk + ((int64_t)row * NB + p) * BB, xbits, nib);
        float s, m;
        sb6_block_scales(qsqm, ddm, row, NB, NSB, p, s, m);
#pragma unroll
        for (int n = 0; n < R; n++) {
            const TX* xp = x + (int64_t)n * IN + p * 32;
            float dv = 0.f, xs = 0.f;
#pragma unroll
            for (int c = 0; c < 32; c++) {
                const float xv = to_f(xp[c]);
                dv = fmaf(xv, (float)nib[c], dv);
                xs += xv;
            }
            acc[n] = fmaf(s, dv, fmaf(m, xs, acc[n]));
        }
    }
#pragma unroll
    for (int n = 0; n < R; n++) {
        const float v = warp_sum(acc[n]);
        if (lane == 0) {
            if constexpr (EP) epilogue(jb, row, n0 + n, v);
            else y[(int64_t)n * OUT + row] = v;
        }
    }
}

// sb6 -> MLX affine container (group 32, bits 4+xbits).  The 32 codes of a
// block fill exactly `bits` u32 words, so every thread owns whole words.
__global__ void sb6_to_affine_kernel(const uint8_t* __restrict__ qblk, const uint8_t* __restrict__ qsqm,
                                     const __half* __restrict__ ddm, uint32_t* __restrict__ wq,
                                     float* __restrict__ scales, float* __restrict__ biases,
                                     int* __restrict__ fp16_bad, int OUT, int IN, int xbits) {
    const int NB = IN / 32, NSB = NB / 8, BB = 16 + 4 * xbits, bits = 4 + xbits;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)OUT * NB) return;
    const int64_t row = idx / NB;
    const int blk = (int)(idx % NB);
    uint8_t nib[32];
    sb6_block_codes(qblk + (row * NB + blk) * BB, xbits, nib);
    float s, m;
    sb6_block_scales(qsqm, ddm, row, NB, NSB, blk, s, m);
    const float s32 = fmaxf(s, 1e-8f);
    const float s16 = rnd_half(s32);
    if (s16 != s32) {
        for (int c = 0; c < 32; c++)
            if ((float)nib[c] * s16 + m != (float)nib[c] * s32 + m) atomicExch(fp16_bad, 1);
    }
    scales[row * NB + blk] = s32;
    biases[row * NB + blk] = m;
    uint32_t words[6] = {0, 0, 0, 0, 0, 0};
    for (int c = 0; c < 32; c++) {
        const int bit = c * bits, w0 = bit >> 5, off = bit & 31;
        words[w0] |= (uint32_t)nib[c] << off;
        if (off + bits > 32) words[w0 + 1] |= (uint32_t)nib[c] >> (32 - off);
    }
    uint32_t* wp = wq + row * ((int64_t)NB * bits) + (int64_t)blk * bits;
    for (int i = 0; i < bits; i++) wp[i] = words[i];
}

// ------------------------------------------------------------------------ sym

// Pairs are 24 bytes: read as u32 words (8-byte alignment at best).
__device__ __forceinline__ void sym6_pair_codes(const uint8_t* pb, int code[32]) {
    const uint32_t* bw = reinterpret_cast<const uint32_t*>(pb);
    const uint32_t wds[4] = {bw[0], bw[1], bw[2], bw[3]};
#pragma unroll
    for (int blk = 0; blk < 2; blk++)
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int bi = blk * 8 + j;
            const uint8_t byte = (uint8_t)(wds[bi >> 2] >> (8 * (bi & 3)));
            code[blk * 16 + j] = byte & 0xF;
            code[blk * 16 + j + 8] = byte >> 4;
        }
    const uint32_t hb = *reinterpret_cast<const uint32_t*>(pb + 16);
    const uint32_t hb2 = *reinterpret_cast<const uint32_t*>(pb + 20);
#pragma unroll
    for (int c = 0; c < 32; c++) code[c] |= (int)((((hb >> c) & 1u) << 4) | (((hb2 >> c) & 1u) << 5));
}

// One thread per (row, 16-block).  F16 multiplies in half, F32/BF16 in float.
template <typename TO>
__global__ void sym_dequant_kernel(const uint8_t* __restrict__ qblk, const int8_t* __restrict__ qs,
                                   const __half* __restrict__ d, TO* __restrict__ out, int OUT,
                                   int IN, int bits) {
    const int NB = IN / 16, NSB = (IN + 255) / 256;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)OUT * NB) return;
    const int64_t row = idx / NB;
    const int blk = (int)(idx % NB);
    const float s = rnd_half((float)qs[row * NB + blk] * __half2float(d[row * NSB + blk / 16]));
    int code[16];
    if (bits == 8) {
#pragma unroll
        for (int c = 0; c < 16; c++) code[c] = (int8_t)qblk[row * IN + blk * 16 + c];
    } else {
        int pc[32];
        sym6_pair_codes(qblk + (row * (IN / 32) + blk / 2) * 24, pc);
#pragma unroll
        for (int c = 0; c < 16; c++) code[c] = pc[(blk & 1) * 16 + c] - 32;
    }
    TO* o = out + row * IN + blk * 16;
#pragma unroll
    for (int c = 0; c < 16; c++) o[c] = from_f<TO>((float)code[c] * s);
}

template <typename TX, int R, bool EP = false>
__global__ void __launch_bounds__(256)
sym_gemv_kernel(const TX* __restrict__ x, const uint8_t* __restrict__ qblk,
                const int8_t* __restrict__ qs, const __half* __restrict__ d, float* __restrict__ y,
                int OUT, int IN, int bits, int out_per, const GemvJob jb, int n0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= OUT) return;
    const int NB = IN / 16, NSB = IN / 256, NK = OUT / out_per;
    const int xi = row / out_per;
    float acc[R];
#pragma unroll
    for (int n = 0; n < R; n++) acc[n] = 0.f;
    if (bits == 8) {
        for (int p = lane; p < NB; p += 32) {
            const float s = rnd_half((float)qs[(int64_t)row * NB + p] *
                                     __half2float(d[(int64_t)row * NSB + p / 16]));
            const uint4 q4 = *reinterpret_cast<const uint4*>(qblk + (int64_t)row * IN + p * 16);
            const int8_t* cq = reinterpret_cast<const int8_t*>(&q4);
#pragma unroll
            for (int n = 0; n < R; n++) {
                const TX* xp = x + ((int64_t)n * NK + xi) * IN + p * 16;
                float dv = 0.f;
#pragma unroll
                for (int c = 0; c < 16; c++) dv = fmaf(to_f(xp[c]), (float)cq[c], dv);
                acc[n] = fmaf(s, dv, acc[n]);
            }
        }
    } else {
        for (int p = lane; p < IN / 32; p += 32) {
            int cc[32];
            sym6_pair_codes(qblk + ((int64_t)row * (IN / 32) + p) * 24, cc);
            const float dsb = __half2float(d[(int64_t)row * NSB + p / 8]);
            const float s0 = rnd_half((float)qs[(int64_t)row * NB + 2 * p] * dsb);
            const float s1 = rnd_half((float)qs[(int64_t)row * NB + 2 * p + 1] * dsb);
#pragma unroll
            for (int n = 0; n < R; n++) {
                const TX* xp = x + ((int64_t)n * NK + xi) * IN + p * 32;
                float dv0 = 0.f, dv1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    const float x0 = to_f(xp[c]), x1 = to_f(xp[16 + c]);
                    dv0 = fmaf(x0, (float)cc[c], dv0);
                    dv1 = fmaf(x1, (float)cc[16 + c], dv1);
                    b0 += x0;
                    b1 += x1;
                }
                acc[n] = fmaf(s0, dv0 - 32.0f * b0, fmaf(s1, dv1 - 32.0f * b1, acc[n]));
            }
        }
    }
#pragma unroll
    for (int n = 0; n < R; n++) {
        const float v = warp_sum(acc[n]);
        if (lane == 0) {
            if constexpr (EP) epilogue(jb, row, n0 + n, v);
            else y[(int64_t)n * OUT + row] = v;
        }
    }
}

__global__ void sym_rows_kernel(const int32_t* __restrict__ ids, int n_ids,
                                const int8_t* __restrict__ codes, const int8_t* __restrict__ qs,
                                const __half* __restrict__ d, __half* __restrict__ out, int vocab,
                                int IN) {
    const int NB = IN / 16, NSB = (IN + 255) / 256;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)n_ids * NB) return;
    const int n = (int)(idx / NB), blk = (int)(idx % NB);
    int64_t row = ids[n];
    if (row < 0 || row >= vocab) row = 0;
    const float s = rnd_half((float)qs[row * NB + blk] * __half2float(d[row * NSB + blk / 16]));
    __half* o = out + (int64_t)n * IN + blk * 16;
#pragma unroll
    for (int c = 0; c < 16; c++) o[c] = __float2half_rn((float)codes[row * IN + blk * 16 + c] * s);
}

// ------------------------------------------------------------------ launchers

int launch_sb6_dequant(const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm, int odtype,
                       void* out, int OUT, int IN, int xbits, cudaStream_t st) {
    const int64_t n = (int64_t)OUT * (IN / 32);
    return dispatch_dtype(odtype, [&]<typename TO>() {
        sb6_dequant_kernel<TO><<<ceil_div(n, 256), 256, 0, st>>>(qblk, qsqm, (const __half*)ddm,
                                                                 (TO*)out, OUT, IN, xbits);
        return check_launch("sb6_dequant_kernel");
    });
}

int launch_sb6_gemv(int xdtype, const void* x, const uint8_t* qblk, const uint8_t* qsqm,
                    const uint16_t* ddm, float* y, int rows, int OUT, int IN, int xbits,
                    cudaStream_t st) {
    const size_t xe = xdtype == RWKV_F32 ? 4 : 2;
    return dispatch_dtype(xdtype, [&]<typename TX>() {
        for (int n0 = 0; n0 < rows; n0 += 4) {
            const int r = min(4, rows - n0);
            const TX* xp = (const TX*)((const char*)x + (size_t)n0 * IN * xe);
            float* yp = y + (size_t)n0 * OUT;
            const int blocks = ceil_div(OUT, 8);
            switch (r) {
#define SB6C(RR)                                                                         \
    case RR:                                                                             \
        sb6_gemv_kernel<TX, RR><<<blocks, 256, 0, st>>>(xp, qblk, qsqm, (const __half*)ddm, \
                                                        yp, OUT, IN, xbits, GemvJob{}, 0); \
        break;
                SB6C(1) SB6C(2) SB6C(3) SB6C(4)
#undef SB6C
            }
            int rc = check_launch("sb6_gemv_kernel");
            if (rc) return rc;
        }
        return ok();
    });
}

int launch_sb6_to_affine(const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm,
                         uint32_t* wq, float* scales, float* biases, int* fp16_bad_dev, int OUT,
                         int IN, int xbits, cudaStream_t st) {
    const int64_t n = (int64_t)OUT * (IN / 32);
    sb6_to_affine_kernel<<<ceil_div(n, 256), 256, 0, st>>>(qblk, qsqm, (const __half*)ddm, wq,
                                                           scales, biases, fp16_bad_dev, OUT, IN,
                                                           xbits);
    return check_launch("sb6_to_affine_kernel");
}

int launch_sym_dequant(const uint8_t* qblk, const uint8_t* qs, const uint16_t* d, int odtype,
                       void* out, int OUT, int IN, int bits, cudaStream_t st) {
    const int64_t n = (int64_t)OUT * (IN / 16);
    return dispatch_dtype(odtype, [&]<typename TO>() {
        sym_dequant_kernel<TO><<<ceil_div(n, 256), 256, 0, st>>>(qblk, (const int8_t*)qs,
                                                                 (const __half*)d, (TO*)out, OUT,
                                                                 IN, bits);
        return check_launch("sym_dequant_kernel");
    });
}

int launch_sym_gemv(int xdtype, const void* x, const uint8_t* qblk, const uint8_t* qs,
                    const uint16_t* d, float* y, int nn, int OUT, int IN, int bits, int out_per,
                    cudaStream_t st) {
    const size_t xe = xdtype == RWKV_F32 ? 4 : 2;
    const int NK = OUT / out_per;
    return dispatch_dtype(xdtype, [&]<typename TX>() {
        for (int n0 = 0; n0 < nn; n0 += 4) {
            const int r = min(4, nn - n0);
            const TX* xp = (const TX*)((const char*)x + (size_t)n0 * NK * IN * xe);
            float* yp = y + (size_t)n0 * OUT;
            const int blocks = ceil_div(OUT, 8);
            switch (r) {
#define SYMC(RR)                                                                             \
    case RR:                                                                                 \
        sym_gemv_kernel<TX, RR><<<blocks, 256, 0, st>>>(xp, qblk, (const int8_t*)qs,        \
                                                        (const __half*)d, yp, OUT, IN, bits, \
                                                        out_per, GemvJob{}, 0);              \
        break;
                SYMC(1) SYMC(2) SYMC(3) SYMC(4)
#undef SYMC
            }
            int rc = check_launch("sym_gemv_kernel");
            if (rc) return rc;
        }
        return ok();
    });
}

// A decode-runtime job on a .rwkvq matrix (GemvJob.wfmt WFMT_SB6 / WFMT_SYM):
// y = x W^T through the sb6 / sym GEMV, at most 4 activation rows per launch
// (the reference's sym kernel takes up to 4, its sb6 kernel 1), with the job's
// epilogue (activation, fp16 / fp32 / += output).  x rows are contiguous
// (x_stride == IN); xdtype is the activation type.
int launch_rwkvq_job(int xdtype, const GemvJob& j, int R, cudaStream_t st) {
    const size_t xe = xdtype == RWKV_F32 ? 4 : 2;
    return dispatch_dtype(xdtype, [&]<typename TX>() {
        const int blocks = ceil_div(j.OUT, 8);
        for (int n0 = 0; n0 < R; n0 += 4) {
            const int r = min(4, R - n0);
            const TX* xp = (const TX*)((const char*)j.x + (size_t)n0 * j.IN * xe);
            if (j.wfmt == WFMT_SB6) {
                const uint8_t* qb = (const uint8_t*)j.w;
                const uint8_t* qsqm = (const uint8_t*)j.scales;
                const __half* ddm = (const __half*)j.biases;
                switch (r) {
#define SB6J(RR) \
    case RR: sb6_gemv_kernel<TX, RR, true><<<blocks, 256, 0, st>>>(xp, qb, qsqm, ddm, nullptr, j.OUT, j.IN, j.wbits, j, n0); break;
                    SB6J(1) SB6J(2) SB6J(3) SB6J(4)
#undef SB6J
                }
            } else {
                const uint8_t* qb = (const uint8_t*)j.w;
                const int8_t* qs = (const int8_t*)j.scales;
                const __half* d = (const __half*)j.biases;
                switch (r) {
#define SYMJ(RR) \
    case RR: sym_gemv_kernel<TX, RR, true><<<blocks, 256, 0, st>>>(xp, qb, qs, d, nullptr, j.OUT, j.IN, j.wbits, j.OUT, j, n0); break;
                    SYMJ(1) SYMJ(2) SYMJ(3) SYMJ(4)
#undef SYMJ
                }
            }
            int rc = check_launch("rwkvq_gemv_kernel");
            if (rc) return rc;
        }
        return ok();
    });
}

int launch_sym_rows(const int32_t* ids, int n_ids, const uint8_t* codes, const uint8_t* qs,
                    const uint16_t* d, uint16_t* out, int vocab, int IN, cudaStream_t st) {
    const int64_t n = (int64_t)n_ids * (IN / 16);
    sym_rows_kernel<<<ceil_div(n, 256), 256, 0, st>>>(ids, n_ids, (const int8_t*)codes,
                                                      (const int8_t*)qs, (const __half*)d,
                                                      (__half*)out, vocab, IN);
    return check_launch("sym_rows_kernel");
}

}  // namespace rwkv
