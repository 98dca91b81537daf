// Device side of a data-parallel state-tuning step over the WKV-7 path.
//
// The trainable parameter is each layer's initial WKV state [H, N, N] fp32
// (StateTrainableSet, Sources/RWKVGen/InitialState.swift:176-251), shared by
// every sequence of the batch.  Per layer:
//   rwkv_state_broadcast   the state into h_in [B, H, N, N] for the forward
//   rwkv_state_grad_sum    the backward's dh_in summed over the batch into the
//                          layer's gradient (fixed order: deterministic)
// and once per step, after the gradients of all ranks have been summed:
//   rwkv_adamw_clip_step   average, clip by global norm, AdamW
// which is the optimizer step of Trainer.run (Sources/RWKVGen/Training/
// Trainer.swift:141-161, clip at :182-189) in the same order, every
// operation rounded to fp32 as the reference's elementwise MLX ops do (no
// fused multiply-add).  The step reads the global norm from device memory, so
// no value travels to the host between the gradients and the update.
#include "common.cuh"

namespace rwkv {
namespace {

constexpr int ST_THREADS = 256;
constexpr int ADAM_MAX_BLOCKS = 1024;   // norm partials (one double each)
constexpr int64_t ADAM_PER_BLOCK = (int64_t)ST_THREADS * 16;

__global__ void __launch_bounds__(ST_THREADS)
state_broadcast_kernel(const float4* __restrict__ s, float4* __restrict__ h, int64_t per4, int B) {
    for (int64_t i = blockIdx.x * (int64_t)ST_THREADS + threadIdx.x; i < per4; i += (int64_t)gridDim.x * ST_THREADS) {
        const float4 x = s[i];
        for (int b = 0; b < B; b++) h[(int64_t)b * per4 + i] = x;
    }
}

__global__ void __launch_bounds__(ST_THREADS)
state_grad_sum_kernel(const float4* __restrict__ dh, float4* __restrict__ g, int64_t per4, int B, int accumulate) {
    for (int64_t i = blockIdx.x * (int64_t)ST_THREADS + threadIdx.x; i < per4; i += (int64_t)gridDim.x * ST_THREADS) {
        float4 acc = accumulate ? g[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        for (int b = 0; b < B; b++) {
            const float4 x = dh[(int64_t)b * per4 + i];
            acc.x = __fadd_rn(acc.x, x.x);
            acc.y = __fadd_rn(acc.y, x.y);
            acc.z = __fadd_rn(acc.z, x.z);
            acc.w = __fadd_rn(acc.w, x.w);
        }
        g[i] = acc;
    }
}

// Sum of squares of the scaled gradient over block `blockIdx.x`'s fixed
// range, in double; one partial per block.
__global__ void __launch_bounds__(ST_THREADS)
adam_sumsq_kernel(const float* __restrict__ grad, int64_t n, float grad_scale, int64_t per_block,
                  double* __restrict__ partial) {
    __shared__ double red[ST_THREADS / 32];
    const int64_t lo = blockIdx.x * per_block, hi = min(n, lo + per_block);
    double acc = 0.0;
    for (int64_t i = lo + threadIdx.x; i < hi; i += ST_THREADS) {
        const float g = __fmul_rn(grad[i], grad_scale);
        acc += (double)__fmul_rn(g, g);
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < ST_THREADS / 32; w++) s += red[w];
        partial[blockIdx.x] = s;
    }
}

struct AdamArgs {
    float* param;
    float* m;
    float* v;
    const float* grad;
    int64_t n, per_block;
    float grad_scale, clip, lr, beta1, beta2, eps, weight_decay, c1, c2;
    const double* partial;
    int nparts;
    float* norm_out;
};

__global__ void __launch_bounds__(ST_THREADS) adam_update_kernel(AdamArgs a) {
    __shared__ double red[ST_THREADS];
    __shared__ float s_scale;
    // every block reduces the same partials in the same order: one norm
    double x = 0.0;
    for (int i = threadIdx.x; i < a.nparts; i += ST_THREADS) x += a.partial[i];
    red[threadIdx.x] = x;
    __syncthreads();
    for (int o = ST_THREADS / 2; o; o >>= 1) {
        if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        // sqrt of the fp32 sum of squares, as (g * g).sum() then sqrt in fp32
        const float norm = sqrtf((float)red[0]);
        float s = 1.f;
        if (a.clip > 0.f) s = fminf(1.f, __fdiv_rn(a.clip, __fadd_rn(norm, 1e-6f)));
        s_scale = s;
        if (blockIdx.x == 0 && a.norm_out) *a.norm_out = norm;
    }
    __syncthreads();
    const float s = s_scale;
    const float ob1 = __fsub_rn(1.f, a.beta1), ob2 = __fsub_rn(1.f, a.beta2);
    const int64_t lo = blockIdx.x * a.per_block, hi = min(a.n, lo + a.per_block);
    for (int64_t i = lo + threadIdx.x; i < hi; i += ST_THREADS) {
        float g = __fmul_rn(a.grad[i], a.grad_scale);
        if (a.clip > 0.f) g = __fmul_rn(g, s);
        const float m = __fadd_rn(__fmul_rn(a.beta1, a.m[i]), __fmul_rn(ob1, g));
        const float v = __fadd_rn(__fmul_rn(a.beta2, a.v[i]), __fmul_rn(ob2, __fmul_rn(g, g)));
        const float mhat = __fdiv_rn(m, a.c1), vhat = __fdiv_rn(v, a.c2);
        float upd = __fdiv_rn(mhat, __fadd_rn(__fsqrt_rn(vhat), a.eps));
        const float p = a.param[i];
        if (a.weight_decay > 0.f) upd = __fadd_rn(upd, __fmul_rn(a.weight_decay, p));
        a.m[i] = m;
        a.v[i] = v;
        a.param[i] = __fsub_rn(p, __fmul_rn(a.lr, upd));
    }
}

int adam_blocks(int64_t n, int64_t* per_block) {
    int64_t blocks = (n + ADAM_PER_BLOCK - 1) / ADAM_PER_BLOCK;
    int64_t per = ADAM_PER_BLOCK;
    if (blocks > ADAM_MAX_BLOCKS) {
        per = (n + ADAM_MAX_BLOCKS - 1) / ADAM_MAX_BLOCKS;
        blocks = (n + per - 1) / per;
    }
    *per_block = per;
    return (int)blocks;
}

int grid_for(int64_t n4) {
    int64_t g = (n4 + ST_THREADS - 1) / ST_THREADS;
    return (int)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 8));
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace
}  // namespace rwkv

using namespace rwkv;

extern "C" int rwkv_state_broadcast(const float* state, float* h, int B, int H, int N,
                                    rwkv_stream_t stream) {
    const char* fn = "rwkv_state_broadcast";
    RWKV_REQUIRE(state && h, RWKV_E_NULL, "%s: NULL pointer", fn);
    RWKV_REQUIRE(B >= 1 && H >= 1 && N >= 1, RWKV_E_SHAPE, "%s: B=%d H=%d N=%d must be >= 1", fn, B, H, N);
    RWKV_REQUIRE(N == RWKV_WKV7_HEAD_SIZE, RWKV_E_UNSUPPORTED, "%s: N=%d, kernels take N=64", fn, N);
    RWKV_REQUIRE(aligned16(state) && aligned16(h), RWKV_E_UNSUPPORTED, "%s: pointers must be 16-byte aligned", fn);
    const int64_t per4 = (int64_t)H * N * N / 4;
    state_broadcast_kernel<<<grid_for(per4), ST_THREADS, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const float4*>(state), reinterpret_cast<float4*>(h), per4, B);
    return check_launch(fn);
}

extern "C" int rwkv_state_grad_sum(const float* dh_in, float* grad, int B, int H, int N, int accumulate,
                                   rwkv_stream_t stream) {
    const char* fn = "rwkv_state_grad_sum";
    RWKV_REQUIRE(dh_in && grad, RWKV_E_NULL, "%s: NULL pointer", fn);
    RWKV_REQUIRE(B >= 1 && H >= 1 && N >= 1, RWKV_E_SHAPE, "%s: B=%d H=%d N=%d must be >= 1", fn, B, H, N);
    RWKV_REQUIRE(N == RWKV_WKV7_HEAD_SIZE, RWKV_E_UNSUPPORTED, "%s: N=%d, kernels take N=64", fn, N);
    RWKV_REQUIRE(aligned16(dh_in) && aligned16(grad), RWKV_E_UNSUPPORTED, "%s: pointers must be 16-byte aligned", fn);
    const int64_t per4 = (int64_t)H * N * N / 4;
    state_grad_sum_kernel<<<grid_for(per4), ST_THREADS, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const float4*>(dh_in), reinterpret_cast<float4*>(grad), per4, B, accumulate != 0);
    return check_launch(fn);
}

extern "C" int64_t rwkv_adamw_workspace_size(int64_t n) {
    if (n < 1) return 0;
    int64_t per = 0;
    const int blocks = adam_blocks(n, &per);
    return ((int64_t)blocks * (int64_t)sizeof(double) + 255) / 256 * 256;
}

extern "C" int rwkv_adamw_clip_step(float* param, float* m, float* v, const float* grad, int64_t n,
                                    float grad_scale, float clip, float lr, float beta1, float beta2,
                                    float eps, float weight_decay, float bias_c1, float bias_c2,
                                    float* norm_out, void* workspace, int64_t workspace_bytes,
                                    rwkv_stream_t stream) {
    const char* fn = "rwkv_adamw_clip_step";
    RWKV_REQUIRE(param && m && v && grad, RWKV_E_NULL, "%s: NULL parameter, moment or gradient", fn);
    RWKV_REQUIRE(n >= 1, RWKV_E_SHAPE, "%s: n=%lld must be >= 1", fn, (long long)n);
    RWKV_REQUIRE(bias_c1 > 0.f && bias_c2 > 0.f, RWKV_E_SHAPE,
                 "%s: bias corrections c1=%g c2=%g must be > 0 (step t >= 1)", fn, bias_c1, bias_c2);
    const int64_t need = rwkv_adamw_workspace_size(n);
    RWKV_REQUIRE(workspace != nullptr && workspace_bytes >= need, RWKV_E_WORKSPACE,
                 "%s: workspace of %lld bytes, need %lld", fn, (long long)workspace_bytes, (long long)need);
    RWKV_REQUIRE(((uintptr_t)workspace & 7u) == 0, RWKV_E_UNSUPPORTED, "%s: workspace not 8-byte aligned", fn);
    int64_t per = 0;
    const int blocks = adam_blocks(n, &per);
    double* partial = static_cast<double*>(workspace);
    cudaStream_t st = (cudaStream_t)stream;
    adam_sumsq_kernel<<<blocks, ST_THREADS, 0, st>>>(grad, n, grad_scale, per, partial);
    if (int rc = check_launch("adam_sumsq_kernel")) return rc;
    AdamArgs a{param, m, v, grad, n, per, grad_scale, clip, lr, beta1, beta2, eps, weight_decay,
               bias_c1, bias_c2, partial, blocks, norm_out};
    adam_update_kernel<<<blocks, ST_THREADS, 0, st>>>(a);
    return check_launch("adam_update_kernel");
}
