// Skinny GEMM  y[n, o] = sum_k x[n, k] * W[o, k]  for n < R (R small: decode
// rows), on the tensor cores with mma.sync.m16n8k16 (fp16 x fp16 -> fp32).
//
// Weight formats:
//  * Q4G64: MLX affine container, 4-bit codes LSB-first in u32 words, fp16
//    scale/bias per 64-column group (the QLoRA base).  The product is
//    computed as  scale * sum(q*x) + bias * sum(x)  per group: the tensor
//    core multiplies the exact integer codes (as fp16) by x and accumulates
//    in fp32; scale and bias are applied once per group in fp32.
//  * F16: dense fp16 rows (the x070 low-rank branches).
//
// K permutation (Q4G64).  Inside an MMA the k index only has to agree
// between A and B, so each lane's four k-slots {2t, 2t+1, 2t+8, 2t+9}
// (t = lane % 4) are mapped to nibbles of the two u32 words 2t, 2t+1 of the
// 64-column group: at k-step j (0..3) the slot pairs are the nibble pairs
// (j, j+4) of word 2t and of word 2t+1.  One LOP3 turns a word shifted by 4j
// into the half2 (1024 + q_j, 1024 + q_{j+4}); subtracting 1024 gives the
// exact codes.  B is permuted the same way from x[n][16t .. 16t+15].
//
// The pipelined kernels that use these pieces are in gemm_w4.cuh.
#pragma once

#include "common.cuh"

namespace rwkv {

constexpr int MMA_WARPS = 8;

__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// half2 (q_j, q_{j+4}) of a packed word, exact.
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int j) {
    uint32_t h = ((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
    __half2 v = __hsub2(*reinterpret_cast<__half2*>(&h), __half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400)));
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint4 ldg128(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint2 ldg64(const void* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }

// One job of a multi-job launch.  x is [R, x_stride] (fp16 for the tensor-core
// kernels, fp16 or fp32 for the CUDA-core ones); W rows [OUT, IN].
struct GemvJob {
    const void* w;        // Q4G64: u32 words; F16: __half
    const __half* scales; // Q4G64 only, [OUT, IN/64]
    const __half* biases;
    const void* x;
    int x_stride;         // elements between x rows
    int OUT, IN;
    int act;              // Act: function applied to the dot product
    int out;              // Out: how the result is written
    void* y;
    int y_stride;
    const float* bias;    // per-output-row bias for ACT_DECAY / ACT_SIGMOID_BIAS
    float alpha;          // ACT_SCALE factor
    // weight container: WFMT_AFFINE (w / scales / biases above), or a .rwkvq
    // matrix: WFMT_SB6 (w = qblk, scales = qsqm, biases = ddm; wbits = xbits)
    // or WFMT_SYM (w = qblk, scales = qs, biases = d; wbits = 6 or 8)
    int wfmt;
    int wbits;
};
enum WFmt : int { WFMT_AFFINE = 0, WFMT_SB6 = 1, WFMT_SYM = 2 };

enum Act : int {
    ACT_NONE = 0,
    ACT_RELU2 = 1,         // max(v, 0)^2                       (cmix key)
    ACT_TANH = 2,          // tanh(v)                            (w branch, down)
    ACT_SIGMOID = 3,       // sigmoid(v)                         (g branch, down)
    ACT_DECAY = 4,         // exp(-0.606531 * sigmoid(v + bias)) (w branch, up)
    ACT_SIGMOID_BIAS = 5,  // sigmoid(v + bias)                  (a / v branches, up)
    ACT_SCALE = 6,         // alpha * v                          (LoRA adapter, down)
};
enum Out : int { OUT_F32 = 0, OUT_F16 = 1, OUT_ADD_F32 = 2, OUT_BF16 = 3 };

__device__ __forceinline__ void epilogue(const GemvJob& jb, int o, int n, float v) {
    switch (jb.act) {
        case ACT_RELU2: v = fmaxf(v, 0.f); v = v * v; break;
        case ACT_TANH: v = tanhf(v); break;
        case ACT_SIGMOID: v = 1.0f / (1.0f + expf(-v)); break;
        case ACT_DECAY: v = expf(-0.606531f * (1.0f / (1.0f + expf(-(v + jb.bias[o]))))); break;
        case ACT_SIGMOID_BIAS: v = 1.0f / (1.0f + expf(-(v + jb.bias[o]))); break;
        case ACT_SCALE: v *= jb.alpha; break;
        default: break;
    }
    const int64_t idx = (int64_t)n * jb.y_stride + o;
    if (jb.out == OUT_F32)
        ((float*)jb.y)[idx] = v;
    else if (jb.out == OUT_F16)
        ((__half*)jb.y)[idx] = __float2half_rn(v);
    else if (jb.out == OUT_BF16)
        ((__nv_bfloat16*)jb.y)[idx] = __float2bfloat16_rn(v);
    else
        ((float*)jb.y)[idx] += v;
}

// B fragments for one 64-column group of x row `xr` (NULL = zero row):
// b[j][0] = (x[16t+j], x[16t+j+4]), b[j][1] = (x[16t+j+8], x[16t+j+12]);
// also returns the fp32 sum of the lane's 16 values.
__device__ __forceinline__ float q4_bfrag(const __half* xr, int t, uint32_t b[4][2]) {
    if (xr == nullptr) {
#pragma unroll
        for (int j = 0; j < 4; j++) b[j][0] = b[j][1] = 0u;
        return 0.f;
    }
    const uint4 lo = ldg128(xr + 16 * t);
    const uint4 hi = ldg128(xr + 16 * t + 8);
    const uint32_t h[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};  // h[i] = (x_{2i}, x_{2i+1})
    // x_j lives in h[j/2] half (j&1); pair (x_j, x_{j+4}) = halves of h[j/2] and h[j/2+2]
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;  // pick high or low halves
        b[j][0] = __byte_perm(h[j >> 1], h[(j >> 1) + 2], sel);
        b[j][1] = __byte_perm(h[(j >> 1) + 4], h[(j >> 1) + 6], sel);
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
        s += f.x + f.y;
    }
    return s;
}

constexpr int MAX_JOBS = 4;
struct GemvJobs {
    GemvJob j[MAX_JOBS];
};

}  // namespace rwkv
