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
#include "gemv_tile.cuh"

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

// One 128-code sb6 unit (4 blocks of 32, NV words each: 16 bytes of nibbles
// + xbits bit-planes of 4 bytes) of an output row against R staged rows:
// per block s = half(qs * d), m = half(qm * dm), acc += s * sum(q x) + m *
// sum(x), codes summed in column order.  xs: staged rows (xidx layout, RS
// floats per row); bs: block sums (BSR per row); cu: the unit's first column.
template <int R, int XB>
__device__ __forceinline__ void sb6_unit(const uint32_t (&wd)[24], uint2 sq, __half2 dd, const float* xs, int RS,
                                         const float* bs, int BSR, int cu, float (&acc)[R]) {
    constexpr int xbits = XB, NV = (16 + 4 * XB) / 4;
    const float d = __low2float(dd), dm = __high2float(dd);
#pragma unroll
    for (int b = 0; b < 4; b++) {
        const uint32_t pair = (b < 2 ? sq.x : sq.y) >> (16 * (b & 1));
        const float s = rnd_half((float)(pair & 0xFF) * d);
        const float m = rnd_half((float)(int8_t)(pair >> 8) * dm);
        const int wb = b * NV;  // the block's first word: NV words per block
        const uint32_t qh = xbits >= 1 ? wd[wb + 4] : 0u, qh2 = xbits >= 2 ? wd[wb + 5] : 0u;
        const int cb = cu + 32 * b;  // column of the block in the staged rows
        // the block's 32 codes as floats, column order (bytes j: low nibble col j, high col j + 16)
        float q[32];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t nw = wd[wb + i];
            uint32_t lo = nw & 0x0F0F0F0Fu, hi = (nw >> 4) & 0x0F0F0F0Fu;
            if (xbits >= 1) {
                lo |= spread4(qh >> (4 * i)) << 4;
                hi |= spread4(qh >> (16 + 4 * i)) << 4;
            }
            if (xbits >= 2) {
                lo |= spread4(qh2 >> (4 * i)) << 5;
                hi |= spread4(qh2 >> (16 + 4 * i)) << 5;
            }
#pragma unroll
            for (int k = 0; k < 4; k++) {
                q[4 * i + k] = code_f(lo, k);
                q[16 + 4 * i + k] = code_f(hi, k);
            }
        }
#pragma unroll
        for (int n = 0; n < R; n++) {
            const float* xb = xs + n * RS + xidx(cb);  // the block: 32 contiguous floats
            float dv = 0.f;
#pragma unroll
            for (int c4 = 0; c4 < 8; c4++) {
                const float4 xv = reinterpret_cast<const float4*>(xb)[c4];
                dv = fmaf(xv.x, q[4 * c4], dv);
                dv = fmaf(xv.y, q[4 * c4 + 1], dv);
                dv = fmaf(xv.z, q[4 * c4 + 2], dv);
                dv = fmaf(xv.w, q[4 * c4 + 3], dv);
            }
            acc[n] = fmaf(s, dv, fmaf(m, bs[n * BSR + cb / 32], acc[n]));
        }
    }
}

// TM: the most threads (128-code units) per output row and window: 16, or 32
// for the runtime's one-row launches (8192-column rows then take two windows
// and twice the CTAs).
template <typename TX, int R, bool EP, int XB, int TM = 16>
__global__ void __launch_bounds__(TG_T)
sb6_gemv_tile_kernel(const TX* __restrict__ x_, const uint8_t* __restrict__ qblk_, const uint8_t* __restrict__ qsqm_,
                     const __half* __restrict__ ddm_, float* __restrict__ y, int OUT_, int IN_, int rows,
                     const GemvJobs jobs, int n0) {
    constexpr int xbits = XB;
    __shared__ __align__(16) float xs[R * TM * TG_USTR];
    __shared__ float bs[R * TM * TG_UNIT / 32];
    // EP: the matrix, activations and epilogue of job blockIdx.y (a runtime
    // projection); else the arguments
    const GemvJob& jb = jobs.j[blockIdx.y];
    const int OUT = EP ? jb.OUT : OUT_, IN = EP ? jb.IN : IN_;
    const int64_t xstride = EP ? (int64_t)jb.x_stride : (int64_t)IN;
    const TX* __restrict__ x = EP ? (const TX*)jb.x + n0 * xstride : x_;
    const uint8_t* __restrict__ qblk = EP ? (const uint8_t*)jb.w : qblk_;
    const uint8_t* __restrict__ qsqm = EP ? (const uint8_t*)jb.scales : qsqm_;
    const __half* __restrict__ ddm = EP ? jb.biases : ddm_;
    const int TPR = tg_tpr(IN, TM), RPC = TG_T / TPR, W = TPR * TG_UNIT;
    if ((int)blockIdx.x * RPC >= OUT) return;  // a smaller job of the launch
    const int tid = threadIdx.x, lr = tid / TPR, u = tid - lr * TPR;
    const int row = blockIdx.x * RPC + lr;
    const int NB = IN / 32, NSB = NB / 8;
    constexpr int BB = 16 + 4 * xbits, NV = BB / 4;  // block bytes; 16-byte vectors per unit = words per block
    const int64_t rowc = min(row, OUT - 1);
    float acc[R];
#pragma unroll
    for (int n = 0; n < R; n++) acc[n] = 0.f;
    for (int k0 = 0; k0 < IN; k0 += W) {
        tg_stage<TX, R, 32>(x, xstride, k0, W, rows, xs, bs, TM * TG_USTR);
        const int blk0 = (k0 + u * TG_UNIT) / 32;  // first of the unit's 4 blocks
        const uint4* src = reinterpret_cast<const uint4*>(qblk + (rowc * NB + blk0) * BB);
        uint32_t wd[24];
#pragma unroll
        for (int v = 0; v < 6; v++) {
            if (v < NV) {
                const uint4 q = __ldg(src + v);
                wd[4 * v] = q.x; wd[4 * v + 1] = q.y; wd[4 * v + 2] = q.z; wd[4 * v + 3] = q.w;
            }
        }
        const uint2 sq = __ldg(reinterpret_cast<const uint2*>(qsqm + 2 * (rowc * NB + blk0)));
        const __half2 dd = __ldg(reinterpret_cast<const __half2*>(ddm) + rowc * NSB + blk0 / 8);
        sb6_unit<R, XB>(wd, sq, dd, xs, TM * TG_USTR, bs, W / 32, u * TG_UNIT, acc);
        __syncthreads();  // the window may be overwritten
    }
#pragma unroll
    for (int n = 0; n < R; n++) {
        float v = acc[n];
        for (int o = TPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (u == 0 && row < OUT && n < rows) {
            if constexpr (EP) epilogue(jb, row, n0 + n, v);
            else y[(int64_t)n * OUT + row] = v;
        }
    }
}

// sym: a unit is 8 16-blocks (8-bit: 8 vectors) or 4 32-code pairs (6-bit: 6
// vectors); x of matrix xi = row / out_per (every row of a CTA in one matrix).
template <typename TX, int R, bool EP, int TM = 16>
__global__ void __launch_bounds__(TG_T)
sym_gemv_tile_kernel(const TX* __restrict__ x_, const uint8_t* __restrict__ qblk_, const int8_t* __restrict__ qs_,
                     const __half* __restrict__ d_, float* __restrict__ y, int OUT_, int IN_, int bits_, int out_per_,
                     int rows, const GemvJobs jobs, int n0) {
    __shared__ __align__(16) float xs[R * TM * TG_USTR];
    __shared__ float bs[R * TM * TG_UNIT / 16];
    // EP: the matrix, activations and epilogue of job blockIdx.y (a runtime
    // projection, one matrix per job); else the arguments
    const GemvJob& jb = jobs.j[blockIdx.y];
    const int OUT = EP ? jb.OUT : OUT_, IN = EP ? jb.IN : IN_, bits = EP ? jb.wbits : bits_;
    const int out_per = EP ? jb.OUT : out_per_;
    const TX* __restrict__ x = EP ? (const TX*)jb.x + n0 * (int64_t)jb.x_stride : x_;
    const uint8_t* __restrict__ qblk = EP ? (const uint8_t*)jb.w : qblk_;
    const int8_t* __restrict__ qs = EP ? (const int8_t*)jb.scales : qs_;
    const __half* __restrict__ d = EP ? jb.biases : d_;
    const int TPR = tg_tpr(IN, TM), RPC = TG_T / TPR, W = TPR * TG_UNIT;
    if ((int)blockIdx.x * RPC >= OUT) return;  // a smaller job of the launch
    const int tid = threadIdx.x, lr = tid / TPR, u = tid - lr * TPR;
    const int row = blockIdx.x * RPC + lr;
    const int NB = IN / 16, NSB = IN / 256, NK = OUT / out_per, xi = (blockIdx.x * RPC) / out_per;
    const int64_t rowc = min(row, OUT - 1);
    const TX* xm = x + (int64_t)xi * IN;
    const int64_t xstride = EP ? (int64_t)jb.x_stride : (int64_t)NK * IN;
    float acc[R];
#pragma unroll
    for (int n = 0; n < R; n++) acc[n] = 0.f;
    for (int k0 = 0; k0 < IN; k0 += W) {
        tg_stage<TX, R, 16>(xm, xstride, k0, W, rows, xs, bs, TM * TG_USTR);
        const int blk0 = (k0 + u * TG_UNIT) / 16;  // first of the unit's 8 16-blocks
        const int cu = u * TG_UNIT;                 // the unit's column inside the window
        const uint2 q8 = __ldg(reinterpret_cast<const uint2*>(qs + rowc * NB + blk0));
        const float dsb = __half2float(__ldg(d + rowc * NSB + blk0 / 16));
        float sc[8];
#pragma unroll
        for (int b = 0; b < 8; b++)
            sc[b] = rnd_half((float)(int8_t)((b < 4 ? q8.x : q8.y) >> (8 * (b & 3))) * dsb);
        if (bits == 8) {
            const uint4* src = reinterpret_cast<const uint4*>(qblk + rowc * IN + (int64_t)blk0 * 16);
#pragma unroll
            for (int b = 0; b < 8; b++) {
                const uint4 qv = __ldg(src + b);
                const uint32_t wd[4] = {qv.x, qv.y, qv.z, qv.w};
                // int8 codes: bytes ^ 0x80 -> 0..255 under 2^23, less 2^23 + 128
                float q[16];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint32_t u8 = wd[i] ^ 0x80808080u;
#pragma unroll
                    for (int k = 0; k < 4; k++) q[4 * i + k] = code_f(u8, k) - 128.f;
                }
#pragma unroll
                for (int n = 0; n < R; n++) {
                    const float* xb = xs + n * (TM * TG_USTR) + xidx(cu + 16 * b);  // 16 contiguous floats
                    float dv = 0.f;
#pragma unroll
                    for (int c4 = 0; c4 < 4; c4++) {
                        const float4 xv = reinterpret_cast<const float4*>(xb)[c4];
                        dv = fmaf(xv.x, q[4 * c4], dv);
                        dv = fmaf(xv.y, q[4 * c4 + 1], dv);
                        dv = fmaf(xv.z, q[4 * c4 + 2], dv);
                        dv = fmaf(xv.w, q[4 * c4 + 3], dv);
                    }
                    acc[n] = fmaf(sc[b], dv, acc[n]);
                }
            }
        } else {
            const uint4* src = reinterpret_cast<const uint4*>(qblk + (rowc * (IN / 32) + blk0 / 2) * 24);
            uint32_t wd[24];
#pragma unroll
            for (int v = 0; v < 6; v++) {
                const uint4 q = __ldg(src + v);
                wd[4 * v] = q.x; wd[4 * v + 1] = q.y; wd[4 * v + 2] = q.z; wd[4 * v + 3] = q.w;
            }
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const uint32_t* pw = wd + 6 * p;
                const uint32_t hb = pw[4], hb2 = pw[5];
                // the pair's 32 codes (+32) as floats, column order: block q's bytes 0..7
                // (words 2q, 2q+1) give columns j (low nibble) and j + 8 (high) of the block
                float q[32];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int blk = i >> 1, half = i & 1;  // word i: block blk, bytes 4 half .. 4 half + 3
                    const uint32_t nw = pw[i];
                    const int cl = 16 * blk + 4 * half, ch = cl + 8;  // columns of the low / high nibbles
                    const uint32_t lo = (nw & 0x0F0F0F0Fu) | (spread4(hb >> cl) << 4) | (spread4(hb2 >> cl) << 5);
                    const uint32_t hi = ((nw >> 4) & 0x0F0F0F0Fu) | (spread4(hb >> ch) << 4) | (spread4(hb2 >> ch) << 5);
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        q[cl + k] = code_f(lo, k);
                        q[ch + k] = code_f(hi, k);
                    }
                }
#pragma unroll
                for (int n = 0; n < R; n++) {
                    const float* xp = xs + n * (TM * TG_USTR) + xidx(cu + 32 * p);  // the pair: 32 contiguous floats
                    float dv0 = 0.f, dv1 = 0.f;
#pragma unroll
                    for (int c = 0; c < 16; c++) {
                        dv0 = fmaf(xp[c], q[c], dv0);
                        dv1 = fmaf(xp[16 + c], q[16 + c], dv1);
                    }
                    const int bi = (cu + 32 * p) / 16;
                    acc[n] = fmaf(sc[2 * p], dv0 - 32.0f * bs[n * (W / 16) + bi],
                                  fmaf(sc[2 * p + 1], dv1 - 32.0f * bs[n * (W / 16) + bi + 1], acc[n]));
                }
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int n = 0; n < R; n++) {
        float v = acc[n];
        for (int o = TPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (u == 0 && row < OUT && n < rows) {
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

// sb6 tile kernel for xbits 0..2 and 1 or up to 4 activation rows
// (EP: grid.y jobs of one format)
template <typename TX, bool EP, int TM = 16>
static cudaError_t sb6_tile_launch(int xbits, int r, dim3 grid, cudaStream_t st, const TX* x, const uint8_t* qblk,
                                   const uint8_t* qsqm, const __half* ddm, float* y, int OUT, int IN,
                                   const GemvJobs& jobs, int n0) {
    auto go = [&](auto kern) {
        kern<<<grid, TG_T, 0, st>>>(x, qblk, qsqm, ddm, y, OUT, IN, r, jobs, n0);
        return cudaGetLastError();
    };
    if (r == 1) {
        if (xbits == 0) return go(sb6_gemv_tile_kernel<TX, 1, EP, 0, TM>);
        if (xbits == 1) return go(sb6_gemv_tile_kernel<TX, 1, EP, 1, TM>);
        return go(sb6_gemv_tile_kernel<TX, 1, EP, 2, TM>);
    }
    if (xbits == 0) return go(sb6_gemv_tile_kernel<TX, 4, EP, 0>);
    if (xbits == 1) return go(sb6_gemv_tile_kernel<TX, 4, EP, 1>);
    return go(sb6_gemv_tile_kernel<TX, 4, EP, 2>);
}

int launch_sb6_gemv(int xdtype, const void* x, const uint8_t* qblk, const uint8_t* qsqm,
                    const uint16_t* ddm, float* y, int rows, int OUT, int IN, int xbits,
                    cudaStream_t st) {
    const size_t xe = xdtype == RWKV_F32 ? 4 : 2;
    const int blocks = ceil_div(OUT, TG_T / tg_tpr(IN));
    return dispatch_dtype(xdtype, [&]<typename TX>() {
        for (int n0 = 0; n0 < rows; n0 += 4) {
            const int r = min(4, rows - n0);
            const TX* xp = (const TX*)((const char*)x + (size_t)n0 * IN * xe);
            float* yp = y + (size_t)n0 * OUT;
            sb6_tile_launch<TX, false>(xbits, r, dim3(blocks), st, xp, qblk, qsqm, (const __half*)ddm, yp, OUT, IN,
                                       GemvJobs{}, 0);
            int rc = check_launch("sb6_gemv_tile_kernel");
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
    const int NK = OUT / out_per, rpc = TG_T / tg_tpr(IN);
    const bool tiled = out_per % rpc == 0;  // every CTA's rows inside one fused matrix
    return dispatch_dtype(xdtype, [&]<typename TX>() {
        for (int n0 = 0; n0 < nn; n0 += 4) {
            const int r = min(4, nn - n0);
            const TX* xp = (const TX*)((const char*)x + (size_t)n0 * NK * IN * xe);
            float* yp = y + (size_t)n0 * OUT;
            if (tiled) {
                const int blocks = ceil_div(OUT, rpc);
                if (r == 1)
                    sym_gemv_tile_kernel<TX, 1, false><<<blocks, TG_T, 0, st>>>(
                        xp, qblk, (const int8_t*)qs, (const __half*)d, yp, OUT, IN, bits, out_per, r, GemvJobs{}, 0);
                else
                    sym_gemv_tile_kernel<TX, 4, false><<<blocks, TG_T, 0, st>>>(
                        xp, qblk, (const int8_t*)qs, (const __half*)d, yp, OUT, IN, bits, out_per, r, GemvJobs{}, 0);
            } else {
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
// Runtime projections on .rwkvq matrices: jobs of one format (WFMT_SB6 with
// one xbits, or WFMT_SYM with one bit width), fp16 / bf16 / fp32 activations
// with the jobs' row strides, up to 4 rows per launch, grid.y = the jobs.
// (Plain launches: as programmatic dependents the early CTAs, parked at the
// wait, took the previous kernel's SM slots -- sym 6-bit decode at 1 row
// 1.17 -> 1.47 ms.)
int launch_rwkvq_jobs(int xdtype, const GemvJobs& jobs, int nj, int R, cudaStream_t st) {
    // one row: up to 32 threads per output row (two windows and twice the CTAs
    // for 8192-column rows); more rows: up to 16 (the window staged per row)
    const int tm = R == 1 ? 32 : 16;
    int blocks = 0;
    for (int i = 0; i < nj; i++)
        blocks = std::max(blocks, ceil_div(jobs.j[i].OUT, TG_T / tg_tpr(jobs.j[i].IN, tm)));
    const dim3 grid(blocks, nj);
    const GemvJob& j0 = jobs.j[0];
    return dispatch_dtype(xdtype, [&]<typename TX>() {
        for (int n0 = 0; n0 < R; n0 += 4) {
            const int r = min(4, R - n0);
            cudaError_t e;
            if (j0.wfmt == WFMT_SB6) {
                e = R == 1 ? sb6_tile_launch<TX, true, 32>(j0.wbits, r, grid, st, nullptr, nullptr, nullptr, nullptr,
                                                           nullptr, 0, 0, jobs, n0)
                           : sb6_tile_launch<TX, true>(j0.wbits, r, grid, st, nullptr, nullptr, nullptr, nullptr,
                                                       nullptr, 0, 0, jobs, n0);
            } else {
                auto go = [&](auto kern) {
                    kern<<<grid, TG_T, 0, st>>>((const TX*)nullptr, (const uint8_t*)nullptr, (const int8_t*)nullptr,
                                                (const __half*)nullptr, (float*)nullptr, 0, 0, 0, 1, r, jobs, n0);
                    return cudaGetLastError();
                };
                e = R == 1 ? go(sym_gemv_tile_kernel<TX, 1, true, 32>) : r == 1 ? go(sym_gemv_tile_kernel<TX, 1, true>)
                                                                           : go(sym_gemv_tile_kernel<TX, 4, true>);
            }
            if (e != cudaSuccess) return fail(RWKV_E_CUDA, "rwkvq_gemv_tile_kernel: %s", cudaGetErrorString(e));
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
