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
// Tiling: a CTA owns 16 output rows; its 8 warps split the K groups; each
// warp keeps per-(row, n) fp32 totals for NT tiles of 8 input rows; partials
// are reduced across warps in shared memory and handed to the epilogue.
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
};

enum Act : int {
    ACT_NONE = 0,
    ACT_RELU2 = 1,         // max(v, 0)^2                       (cmix key)
    ACT_TANH = 2,          // tanh(v)                            (w branch, down)
    ACT_SIGMOID = 3,       // sigmoid(v)                         (g branch, down)
    ACT_DECAY = 4,         // exp(-0.606531 * sigmoid(v + bias)) (w branch, up)
    ACT_SIGMOID_BIAS = 5,  // sigmoid(v + bias)                  (a / v branches, up)
};
enum Out : int { OUT_F32 = 0, OUT_F16 = 1, OUT_ADD_F32 = 2 };

__device__ __forceinline__ void epilogue(const GemvJob& jb, int o, int n, float v) {
    switch (jb.act) {
        case ACT_RELU2: v = fmaxf(v, 0.f); v = v * v; break;
        case ACT_TANH: v = tanhf(v); break;
        case ACT_SIGMOID: v = 1.0f / (1.0f + expf(-v)); break;
        case ACT_DECAY: v = expf(-0.606531f * (1.0f / (1.0f + expf(-(v + jb.bias[o]))))); break;
        case ACT_SIGMOID_BIAS: v = 1.0f / (1.0f + expf(-(v + jb.bias[o]))); break;
        default: break;
    }
    const int64_t idx = (int64_t)n * jb.y_stride + o;
    if (jb.out == OUT_F32)
        ((float*)jb.y)[idx] = v;
    else if (jb.out == OUT_F16)
        ((__half*)jb.y)[idx] = __float2half_rn(v);
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

// Q4G64 job.  NT = number of 8-row tiles of x (R <= 8*NT).
template <int NT>
__device__ __forceinline__ void q4_job(const GemvJob& jb, int R, float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int m0 = blockIdx.x * 16;
    const int NG = jb.IN / 64;
    const int wpr = jb.IN / 8;
    const uint32_t* W = (const uint32_t*)jb.w;
    const int r0 = min(m0 + g, jb.OUT - 1), r1 = min(m0 + g + 8, jb.OUT - 1);
    const uint32_t* w0 = W + (int64_t)r0 * wpr + 2 * t;
    const uint32_t* w1 = W + (int64_t)r1 * wpr + 2 * t;

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    for (int G = warp; G < NG; G += MMA_WARPS) {
        const uint2 A0 = ldg64(w0 + 8 * G);
        const uint2 A1 = ldg64(w1 + 8 * G);
        const float s0 = __half2float(jb.scales[(int64_t)r0 * NG + G]);
        const float s1 = __half2float(jb.scales[(int64_t)r1 * NG + G]);
        const float c0 = __half2float(jb.biases[(int64_t)r0 * NG + G]);
        const float c1 = __half2float(jb.biases[(int64_t)r1 * NG + G]);
        uint32_t a[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            a[j][0] = nib_pair(A0.x, j);  // row g,   slots 2t,2t+1  <- word 2t
            a[j][1] = nib_pair(A1.x, j);  // row g+8
            a[j][2] = nib_pair(A0.y, j);  // row g,   slots 2t+8,2t+9 <- word 2t+1
            a[j][3] = nib_pair(A1.y, j);  // row g+8
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int n = nt * 8 + g;
            uint32_t b[4][2];
            const __half* xr = (n < R) ? (const __half*)jb.x + (int64_t)n * jb.x_stride + 64 * G : nullptr;
            float xs = q4_bfrag(xr, t, b);
            xs += __shfl_xor_sync(0xffffffffu, xs, 1);
            xs += __shfl_xor_sync(0xffffffffu, xs, 2);  // sum of x row n over the group
            const float X0 = __shfl_sync(0xffffffffu, xs, 8 * t);      // column 2t
            const float X1 = __shfl_sync(0xffffffffu, xs, 8 * t + 4);  // column 2t+1
            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 4; j++) mma16816(d, a[j], b[j]);
            acc[nt][0] = fmaf(s0, d[0], fmaf(c0, X0, acc[nt][0]));
            acc[nt][1] = fmaf(s0, d[1], fmaf(c0, X1, acc[nt][1]));
            acc[nt][2] = fmaf(s1, d[2], fmaf(c1, X0, acc[nt][2]));
            acc[nt][3] = fmaf(s1, d[3], fmaf(c1, X1, acc[nt][3]));
        }
    }
    // partials -> shared [warp][16 rows][8*NT cols]
    const int C = 8 * NT;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        float* p = red + (size_t)warp * 16 * C;
        p[g * C + nt * 8 + 2 * t] = acc[nt][0];
        p[g * C + nt * 8 + 2 * t + 1] = acc[nt][1];
        p[(g + 8) * C + nt * 8 + 2 * t] = acc[nt][2];
        p[(g + 8) * C + nt * 8 + 2 * t + 1] = acc[nt][3];
    }
}

// Dense fp16 job: natural k order (a0 = W[g][16j+2t..], a2 = W[g][16j+2t+8..]).
template <int NT>
__device__ __forceinline__ void f16_job(const GemvJob& jb, int R, float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int m0 = blockIdx.x * 16;
    const int KS = jb.IN / 16;  // k-steps
    const __half* W = (const __half*)jb.w;
    const int r0 = min(m0 + g, jb.OUT - 1), r1 = min(m0 + g + 8, jb.OUT - 1);
    const __half* w0 = W + (int64_t)r0 * jb.IN + 2 * t;
    const __half* w1 = W + (int64_t)r1 * jb.IN + 2 * t;
    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    for (int ks = warp; ks < KS; ks += MMA_WARPS) {
        uint32_t a[4];
        a[0] = *reinterpret_cast<const uint32_t*>(w0 + 16 * ks);
        a[1] = *reinterpret_cast<const uint32_t*>(w1 + 16 * ks);
        a[2] = *reinterpret_cast<const uint32_t*>(w0 + 16 * ks + 8);
        a[3] = *reinterpret_cast<const uint32_t*>(w1 + 16 * ks + 8);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int n = nt * 8 + g;
            uint32_t b[2] = {0u, 0u};
            if (n < R) {
                const __half* xr = (const __half*)jb.x + (int64_t)n * jb.x_stride + 16 * ks + 2 * t;
                b[0] = *reinterpret_cast<const uint32_t*>(xr);
                b[1] = *reinterpret_cast<const uint32_t*>(xr + 8);
            }
            mma16816(acc[nt], a, b);
        }
    }
    const int C = 8 * NT;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        float* p = red + (size_t)warp * 16 * C;
        p[g * C + nt * 8 + 2 * t] = acc[nt][0];
        p[g * C + nt * 8 + 2 * t + 1] = acc[nt][1];
        p[(g + 8) * C + nt * 8 + 2 * t] = acc[nt][2];
        p[(g + 8) * C + nt * 8 + 2 * t + 1] = acc[nt][3];
    }
}

constexpr int MAX_JOBS = 4;
struct GemvJobs {
    GemvJob j[MAX_JOBS];
};

// grid (max_j ceil(OUT_j/16), n_jobs, ceil(R / (8*NT))), block 256.
// FMT 0 = Q4G64, 1 = F16.
template <int FMT, int NT>
__global__ void __launch_bounds__(MMA_WARPS * 32)
gemv_mma_kernel(const GemvJobs jobs, int R) {
    extern __shared__ float red[];  // [MMA_WARPS][16][8*NT]
    GemvJob jb = jobs.j[blockIdx.y];
    if ((int)blockIdx.x * 16 >= jb.OUT) return;
    // this CTA's slice of input rows
    const int n0 = blockIdx.z * 8 * NT;
    jb.x = (const __half*)jb.x + (int64_t)n0 * jb.x_stride;
    const int Rz = min(R - n0, 8 * NT);
    if (FMT == 0)
        q4_job<NT>(jb, Rz, red);
    else
        f16_job<NT>(jb, Rz, red);
    __syncthreads();
    const int C = 8 * NT;
    for (int e = threadIdx.x; e < 16 * C; e += blockDim.x) {
        const int row = e / C, n = e % C;
        const int o = blockIdx.x * 16 + row;
        if (o >= jb.OUT || n >= Rz) continue;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < MMA_WARPS; w++) v += red[(size_t)w * 16 * C + e];
        epilogue(jb, o, n0 + n, v);
    }
}

// Host launcher.  Returns a cudaError_t.  R >= 1; NT picked from R.
template <int FMT>
inline cudaError_t launch_gemv_mma(const GemvJobs& jobs, int njobs, int R, cudaStream_t st) {
    int maxo = 0;
    for (int i = 0; i < njobs; i++) maxo = max(maxo, jobs.j[i].OUT);
    const int gx = (maxo + 15) / 16;
    auto go = [&](auto nt_tag) {
        constexpr int NT = decltype(nt_tag)::value;
        const size_t smem = (size_t)MMA_WARPS * 16 * 8 * NT * sizeof(float);
        dim3 grid(gx, njobs, (R + 8 * NT - 1) / (8 * NT));
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(gemv_mma_kernel<FMT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        gemv_mma_kernel<FMT, NT><<<grid, MMA_WARPS * 32, smem, st>>>(jobs, R);
        return cudaGetLastError();
    };
    if (R <= 8) return go(std::integral_constant<int, 1>{});
    if (R <= 16) return go(std::integral_constant<int, 2>{});
    if (R <= 32) return go(std::integral_constant<int, 4>{});
    return go(std::integral_constant<int, 8>{});
}

}  // namespace rwkv
