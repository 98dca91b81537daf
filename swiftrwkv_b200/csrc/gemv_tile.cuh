// Tiled GEMV building blocks shared by the .rwkvq (sb6 / sym) and the MLX
// affine 4-bit GEMVs: a 256-thread CTA owns 16 output rows x 16 threads per
// row (fewer threads per row when IN / 128 is small), each thread one
// 128-code unit of every K window; the window of the activations and their
// per-block sums are staged in shared memory once for all rows of the CTA.
#pragma once

#include "common.cuh"

namespace rwkv {

// Four codes packed in the bytes of a word -> exact floats: byte k placed
// under the exponent of 2^23 (one PRMT), less 2^23 (one FADD).
__device__ __forceinline__ float code_f(uint32_t packed, int k) {
    return __int_as_float(__byte_perm(packed, 0x4B000000u, (uint32_t)k | 0x7540u)) - 8388608.f;
}
// Bits 0..3 of b, one per byte (bit i -> bit 0 of byte i).
__device__ __forceinline__ uint32_t spread4(uint32_t b) { return ((b & 0xFu) * 0x00204081u) & 0x01010101u; }

// ---- tiled GEMVs (the launchers' path): CTA = 256 threads; TPR = min(16,
// IN / 128) threads per output row (RPC = 256 / TPR rows per CTA); thread
// (row, u) owns unit u of every K window -- a unit is 128 codes (4 sb6 blocks
// or 8 sym 16-blocks), loaded as 16-byte vectors with its scales in one load.
// Each window (TPR units per row) of the activations, and the per-block sums
// of x, are staged in shared memory for all rows of the CTA.  Per block the
// arithmetic is the row-per-warp kernels' (codes summed sequentially, fp32
// s * sum(q x) + m * sum(x)); the TPR partials of a row are summed by a fixed
// shuffle tree.
constexpr int TG_T = 256;
constexpr int TG_UNIT = 128;

// threads per row: the largest power of two <= cap (<= 16) that divides IN / 128
__host__ __device__ __forceinline__ int tg_tpr(int IN, int cap = 16) {
    const int u = IN / TG_UNIT;
    int t = cap;
    while (t > 1 && u % t) t >>= 1;
    return t;
}

// Staged window layout: a 32-column sub-block takes 36 floats and a 128-column
// unit 148 (4 x 36 + 4), so the threads of a row -- one unit each -- read
// distinct banks (16-byte vectors stay aligned).  xidx: the offset of column c
// of a row inside the window; TG_RS: the floats of one row (16 units).
constexpr int TG_SUB = 36, TG_USTR = 148, TG_RS = 16 * TG_USTR;
__device__ __forceinline__ int xidx(int c) { return (c >> 7) * TG_USTR + ((c >> 5) & 3) * TG_SUB + (c & 31); }

// x rows of the window [k0, k0 + W) into xs (fp32, the layout above, RS
// floats per row), block sums (blocks of BS codes, summed in column order)
// into bs[n][W / BS].  Element loads, not vectors: the tiled kernels run many
// CTAs per SM, and a vector staging pass raised their register count (and
// cut their occupancy) by more than it saved.
template <typename TX, int R, int BS>
__device__ __forceinline__ void tg_stage(const TX* __restrict__ x, int64_t xstride, int k0, int W, int rows,
                                         float* xs, float* bs, int RS = TG_RS) {
    for (int e = threadIdx.x; e < R * W; e += TG_T) {
        const int n = e / W, c = e - n * W;
        xs[n * RS + xidx(c)] = n < rows ? to_f(x[(int64_t)n * xstride + k0 + c]) : 0.f;
    }
    __syncthreads();
    const int nb = W / BS;
    for (int e = threadIdx.x; e < R * nb; e += TG_T) {
        const int n = e / nb, b = e - n * nb;
        constexpr int SB = BS < 32 ? BS : 32;  // a block is contiguous within each 32-column sub-block
        float t = 0.f;
#pragma unroll
        for (int h = 0; h < BS / SB; h++) {
            const float* p = xs + n * RS + xidx(b * BS + h * SB);
#pragma unroll
            for (int c = 0; c < SB; c++) t += p[c];
        }
        bs[e] = t;
    }
    __syncthreads();
}

}  // namespace rwkv
