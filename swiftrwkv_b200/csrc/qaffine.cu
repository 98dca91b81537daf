// MLX affine container kernels (the QLoRA base of X070Backbone, 4-bit group-64
// by default): y = x W^T with W = scale*q + bias per group, dequant to dense,
// embedding-row gather and the quantiser.
//
// Container (Sources/RWKVQuant/RwkvqNative.swift:28-31,161-175): each weight
// row is a stream of `bits`-bit codes packed LSB-first into u32 words; the
// field of column p starts at bit p*bits of the row.  For bits 2/4/8 a word
// holds whole codes; for 3/5/6 fields may straddle two words.
//
// The GEMV here is the CUDA-core path (x rows <= 8 per launch tile): weight
// words are streamed with 16-byte loads, each lane owning a 16-byte quad per
// step, codes unpacked in registers, products accumulated in fp32 as
//   acc += scale * sum(q*x) + bias * sum(x)     per quad (inside one group),
// then reduced across the warp with shuffles.  Two output rows per warp share
// the x loads and the x sums.
#include "common.cuh"
#include <mutex>
#include <unordered_map>

#include "gemm_dx.cuh"
#include "gemv_stream.cuh"
#include "gemm_tc.cuh"
#include "gemm_w4_wide.cuh"

namespace rwkv {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* o);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* o) {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float* o) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 f = __half22float2(h[i]);
        o[2 * i] = f.x;
        o[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* o) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 f = __bfloat1622float2(h[i]);
        o[2 * i] = f.x;
        o[2 * i + 1] = f.y;
    }
}

// Code p of a row (LSB-first bit stream).
__device__ __forceinline__ uint32_t get_code(const uint32_t* row, int64_t p, int bits) {
    const int64_t bit = p * bits;
    const int64_t w0 = bit >> 5;
    const int off = (int)(bit & 31);
    uint64_t word = row[w0];
    if (off + bits > 32) word |= (uint64_t)row[w0 + 1] << 32;
    return (uint32_t)(word >> off) & ((1u << bits) - 1u);
}

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_RW = 2;  // output rows per warp
constexpr int GEMV_MAXR = 8;

// bits in {4, 8}: whole codes per word, 16-byte quads.  R = x rows (<= 8).
template <typename TX, typename TS, typename TY, int BITS, int R>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
q_gemv_quad_kernel(const TX* __restrict__ x, const uint32_t* __restrict__ wq,
                   const TS* __restrict__ scales, const TS* __restrict__ biases,
                   TY* __restrict__ y, int rows, int OUT, int IN, int group, int x_stride,
                   int y_stride) {
    constexpr int CPW = 32 / BITS;     // codes per word
    constexpr int CPQ = 4 * CPW;       // codes per 16-byte quad
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o0 = (blockIdx.x * GEMV_WARPS + warp) * GEMV_RW;
    if (o0 >= OUT) return;
    const int wpr = IN * BITS / 32;
    const int nq = wpr / 4;
    const int NG = IN / group;
    float acc[GEMV_RW][R];
#pragma unroll
    for (int j = 0; j < GEMV_RW; j++)
#pragma unroll
        for (int n = 0; n < R; n++) acc[j][n] = 0.f;

    for (int qi = lane; qi < nq; qi += 32) {
        const int col0 = qi * CPQ;
        const int g = col0 / group;
        uint4 wv[GEMV_RW];
        float sc[GEMV_RW], bi[GEMV_RW];
#pragma unroll
        for (int j = 0; j < GEMV_RW; j++) {
            const int o = min(o0 + j, OUT - 1);
            wv[j] = __ldg(reinterpret_cast<const uint4*>(wq + (int64_t)o * wpr) + qi);
            sc[j] = to_f(scales[(int64_t)o * NG + g]);
            bi[j] = to_f(biases[(int64_t)o * NG + g]);
        }
#pragma unroll
        for (int n = 0; n < R; n++) {
            if (n >= rows) break;
            const TX* xp = x + (int64_t)n * x_stride + col0;
            float dq[GEMV_RW];
#pragma unroll
            for (int j = 0; j < GEMV_RW; j++) dq[j] = 0.f;
            float xs = 0.f;
#pragma unroll
            for (int c8 = 0; c8 < CPQ; c8 += 8) {
                float xv[8];
                load8<TX>(xp + c8, xv);
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int c = c8 + u;  // code index inside the quad
                    xs += xv[u];
#pragma unroll
                    for (int j = 0; j < GEMV_RW; j++) {
                        const uint32_t word = (&wv[j].x)[c / CPW];
                        const uint32_t qv = (word >> ((c % CPW) * BITS)) & ((1u << BITS) - 1u);
                        dq[j] = fmaf((float)qv, xv[u], dq[j]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < GEMV_RW; j++) acc[j][n] = fmaf(sc[j], dq[j], fmaf(bi[j], xs, acc[j][n]));
        }
    }
#pragma unroll
    for (int j = 0; j < GEMV_RW; j++)
#pragma unroll
        for (int n = 0; n < R; n++) {
            const float s = warp_sum(acc[j][n]);
            if (lane == 0 && o0 + j < OUT && n < rows) y[(int64_t)n * y_stride + o0 + j] = from_f<TY>(s);
        }
}

// Any bits in 2..8: per-code extraction, lanes strided over codes.
template <typename TX, typename TS, typename TY>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
q_gemv_generic_kernel(const TX* __restrict__ x, const uint32_t* __restrict__ wq,
                      const TS* __restrict__ scales, const TS* __restrict__ biases,
                      TY* __restrict__ y, int rows, int OUT, int IN, int group, int bits,
                      int x_stride, int y_stride) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o = blockIdx.x * GEMV_WARPS + warp;
    if (o >= OUT) return;
    const int64_t wpr = (int64_t)IN * bits / 32;
    const int NG = IN / group;
    const uint32_t* row = wq + (int64_t)o * wpr;
    float acc[GEMV_MAXR];
#pragma unroll
    for (int n = 0; n < GEMV_MAXR; n++) acc[n] = 0.f;
    for (int c = lane; c < IN; c += 32) {
        const float qv = (float)get_code(row, c, bits);
        const int g = c / group;
        const float wv = qv * to_f(scales[(int64_t)o * NG + g]) + to_f(biases[(int64_t)o * NG + g]);
#pragma unroll
        for (int n = 0; n < GEMV_MAXR; n++)
            if (n < rows) acc[n] = fmaf(wv, to_f(x[(int64_t)n * x_stride + c]), acc[n]);
    }
#pragma unroll
    for (int n = 0; n < GEMV_MAXR; n++) {
        const float s = warp_sum(acc[n]);
        if (lane == 0 && n < rows) y[(int64_t)n * y_stride + o] = from_f<TY>(s);
    }
}

// Dense dequant: one thread per (row, 32-column span).
template <typename TS, typename TO>
__global__ void q_dequant_kernel(const uint32_t* __restrict__ wq, const TS* __restrict__ scales,
                                 const TS* __restrict__ biases, TO* __restrict__ out,
                                 const int32_t* __restrict__ ids, int OUT, int IN, int group,
                                 int bits, int vocab) {
    const int spans = IN / 32;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)OUT * spans) return;
    const int orow = (int)(idx / spans), sp = (int)(idx % spans);
    int64_t row = orow;
    if (ids) {
        row = ids[orow];
        if (row < 0 || row >= vocab) row = 0;  // ids are checked on the host when possible
    }
    const int64_t wpr = (int64_t)IN * bits / 32;
    const int NG = IN / group;
    const uint32_t* rp = wq + row * wpr;
    const int c0 = sp * 32;
    const float s = to_f(scales[row * NG + c0 / group]);
    const float b = to_f(biases[row * NG + c0 / group]);
    TO* op = out + (int64_t)orow * IN + c0;
    if (bits == 4) {
        const uint4 wv = *reinterpret_cast<const uint4*>(rp + c0 / 8);
#pragma unroll
        for (int wi = 0; wi < 4; wi++) {
            const uint32_t word = (&wv.x)[wi];
#pragma unroll
            for (int u = 0; u < 8; u++) op[wi * 8 + u] = from_f<TO>((float)((word >> (4 * u)) & 15u) * s + b);
        }
    } else {
        for (int c = 0; c < 32; c++) op[c] = from_f<TO>((float)get_code(rp, c0 + c, bits) * s + b);
    }
}

// Quantiser: one thread per (row, group); the restated MLX affine_quantize
// (scale from the group's range, edge snapped to the integer grid).
template <typename TW, typename TS>
__global__ void q_quantize_kernel(const TW* __restrict__ W, uint32_t* __restrict__ wq,
                                  TS* __restrict__ scales, TS* __restrict__ biases, int OUT,
                                  int IN, int group, int bits) {
    const int NG = IN / group;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)OUT * NG) return;
    const int o = (int)(idx / NG), g = (int)(idx % NG);
    const TW* xp = W + (int64_t)o * IN + (int64_t)g * group;
    float wmax = to_f(xp[0]), wmin = wmax;
    for (int i = 1; i < group; i++) {
        const float v = to_f(xp[i]);
        wmax = fmaxf(wmax, v);
        wmin = fminf(wmin, v);
    }
    const float n_bins = (float)((1 << bits) - 1);
    const bool mask = fabsf(wmin) > fabsf(wmax);
    float scale = __fdiv_rn(__fsub_rn(wmax, wmin), n_bins);
    scale = fmaxf(scale, 1e-7f);
    if (!mask) scale = -scale;
    const float edge = mask ? wmin : wmax;
    const float q0 = rintf(__fdiv_rn(edge, scale));
    if (q0 != 0.0f) scale = __fdiv_rn(edge, q0);
    const float bias = (q0 == 0.0f) ? 0.0f : edge;
    scales[idx] = from_f<TS>(scale);
    biases[idx] = from_f<TS>(bias);
    // group * bits is a multiple of 32, so the group owns whole words.
    const int64_t wpr = (int64_t)IN * bits / 32;
    uint32_t* rp = wq + (int64_t)o * wpr + (int64_t)g * group * bits / 32;
    const int nw = group * bits / 32;
    for (int wi = 0; wi < nw; wi++) rp[wi] = 0u;
    for (int i = 0; i < group; i++) {
        float q = rintf(__fdiv_rn(__fsub_rn(to_f(xp[i]), bias), scale));
        q = fminf(fmaxf(q, 0.f), n_bins);
        const uint32_t qv = (uint32_t)q;
        const int bit = i * bits, w0 = bit >> 5, off = bit & 31;
        rp[w0] |= qv << off;
        if (off + bits > 32) rp[w0 + 1] |= qv >> (32 - off);
    }
}

// ------------------------------------------------------------------ launchers

template <typename F>
static int dispatch_sdtype(int dt, F&& f) {
    switch (dt) {
        case RWKV_F32: return f.template operator()<float>();
        case RWKV_BF16: return f.template operator()<__nv_bfloat16>();
        case RWKV_F16: return f.template operator()<__half>();
        default: return fail(RWKV_E_DTYPE, "unknown scale dtype %d", dt);
    }
}

// Library-owned split-K workspace of rwkv_q_gemm, one per device, allocated on
// first use and kept until exit.
struct GemmScratch {
    float* ws = nullptr;
    int* tickets = nullptr;
    int* err = nullptr;  // set by a tensor-core GEMM wait that gave up
    TcWaitFlag flag;     // err and its mapped host record
    size_t floats = 0, tickets_n = 0;
    int sm_count = 148;
    std::mutex mu;
};

static GemmScratch* gemm_scratch() {
    static std::mutex m;
    static std::unordered_map<int, GemmScratch*> per_dev;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(m);
    auto it = per_dev.find(dev);
    if (it != per_dev.end()) return it->second;
    GemmScratch* s = new GemmScratch();
    cudaDeviceGetAttribute(&s->sm_count, cudaDevAttrMultiProcessorCount, dev);
    s->floats = (size_t)(4 * s->sm_count + 64) * GW_BM * 64;
    s->tickets_n = 8192;
    if (cudaMalloc(&s->ws, s->floats * 4) != cudaSuccess ||
        cudaMalloc(&s->tickets, (s->tickets_n + 1) * 4) != cudaSuccess ||
        cudaMemset(s->tickets, 0, (s->tickets_n + 1) * 4) != cudaSuccess) {
        delete s;
        return nullptr;
    }
    s->err = s->tickets + s->tickets_n;
    if (!s->flag.init(s->err)) {
        delete s;
        return nullptr;
    }
    per_dev[dev] = s;
    return s;
}

template <typename TX, typename TS, typename TY, int BITS>
static void launch_quad(const void* x, const uint32_t* wq, const void* sc, const void* bi, void* y,
                        int r, int OUT, int IN, int group, int xs, int ys, cudaStream_t st) {
    const int blocks = ceil_div(OUT, GEMV_WARPS * GEMV_RW);
    const TX* xx = (const TX*)x;
    TY* yy = (TY*)y;
    const int rr = r <= 1 ? 1 : r <= 2 ? 2 : r <= 4 ? 4 : 8;
    switch (rr) {
#define QCASE(RR)                                                                           \
    case RR:                                                                                \
        q_gemv_quad_kernel<TX, TS, TY, BITS, RR><<<blocks, GEMV_WARPS * 32, 0, st>>>(      \
            xx, wq, (const TS*)sc, (const TS*)bi, yy, r, OUT, IN, group, xs, ys);           \
        break;
        QCASE(1) QCASE(2) QCASE(4) QCASE(8)
#undef QCASE
    }
}

int launch_q_gemm(int xdtype, const void* x, const uint32_t* wq, const void* scales,
                  const void* biases, int sdtype, int ydtype, void* y, int rows, int OUT, int IN,
                  int group, int bits, cudaStream_t st) {
    const size_t xe = xdtype == RWKV_F32 ? 4 : 2, ye = ydtype == RWKV_F32 ? 4 : 2;
    // fp16 activations on the 4-bit group-64 container: tensor-core path.
    if (xdtype == RWKV_F16 && sdtype == RWKV_F16 && bits == 4 && group == 64 &&
        (ydtype == RWKV_F32 || ydtype == RWKV_F16)) {
        GemvJobs jobs{};
        GemvJob& j = jobs.j[0];
        j.w = wq;
        j.scales = (const __half*)scales;
        j.biases = (const __half*)biases;
        j.x = x;
        j.x_stride = IN;
        j.OUT = OUT;
        j.IN = IN;
        j.act = ACT_NONE;
        j.out = ydtype == RWKV_F32 ? OUT_F32 : OUT_F16;
        j.y = y;
        j.y_stride = OUT;
        GemmScratch* sc = gemm_scratch();
        if (!sc) return fail(RWKV_E_CUDA, "rwkv_q_gemm: workspace allocation failed");
        // a wait of an earlier call on this device gave up: report it once
        // (sticky until this call), clear it, launch nothing
        if (sc->flag.take(st))
            return fail(RWKV_E_TIMEOUT, "rwkv_q_gemm: a tensor-core GEMM wait of an earlier call gave up; "
                                        "its outputs are not valid (flag cleared, nothing launched)");
        // 1..2 rows: the streaming CUDA-core GEMV (gemv_stream.cuh)
        if (q4_stream_eligible(jobs, 1, rows)) {
            cudaError_t e = launch_q4_gemv_stream(jobs, 1, rows, sc->sm_count, false, st);
            if (e != cudaSuccess) return fail(RWKV_E_CUDA, "q4_gemv_stream_kernel: %s", cudaGetErrorString(e));
            return ok();
        }
        // more than 8 rows: tcgen05 (TMA + TMEM) when the shapes allow it
        const TcPlan tp = plan_tc(TC_Q4, jobs, 1, rows, sc->sm_count);
        if (tp.ok) {
            cudaError_t e = launch_tc(TC_Q4, jobs, 1, rows, tp, sc->err, sc->flag.host_dev, st);
            if (e != cudaSuccess) return fail(RWKV_E_CUDA, "gemm_tc_kernel: %s", cudaGetErrorString(e));
            return ok();
        }
        GemmPlan p = plan_any(jobs, 1, rows, sc->sm_count);
        if (p.ws_floats > sc->floats || p.tickets > sc->tickets_n) {
            p.S = 1;
            p.ws_floats = p.tickets = 0;
        }
        GemmArgs ga{};
        ga.jobs = jobs;
        ga.njobs = 1;
        ga.R = rows;
        ga.ws = sc->ws;
        ga.tickets = sc->tickets;
        // the split-K workspace is shared by every call on the device: calls are
        // serialised on the stream they are issued to
        std::lock_guard<std::mutex> lk(sc->mu);
        cudaError_t e = launch_any<0>(ga, p, st);
        if (e != cudaSuccess) return fail(RWKV_E_CUDA, "gemm_w4_kernel: %s", cudaGetErrorString(e));
        return ok();
    }
    return dispatch_dtype(xdtype, [&]<typename TX>() {
        return dispatch_sdtype(sdtype, [&]<typename TS>() {
            return dispatch_dtype(ydtype, [&]<typename TY>() {
                for (int n0 = 0; n0 < rows; n0 += GEMV_MAXR) {
                    const int r = min(GEMV_MAXR, rows - n0);
                    const void* xp = (const char*)x + (size_t)n0 * IN * xe;
                    void* yp = (char*)y + (size_t)n0 * OUT * ye;
                    if (bits == 4) {
                        launch_quad<TX, TS, TY, 4>(xp, wq, scales, biases, yp, r, OUT, IN, group,
                                                   IN, OUT, st);
                    } else if (bits == 8) {
                        launch_quad<TX, TS, TY, 8>(xp, wq, scales, biases, yp, r, OUT, IN, group,
                                                   IN, OUT, st);
                    } else {
                        q_gemv_generic_kernel<TX, TS, TY>
                            <<<ceil_div(OUT, GEMV_WARPS), GEMV_WARPS * 32, 0, st>>>(
                                (const TX*)xp, wq, (const TS*)scales, (const TS*)biases, (TY*)yp,
                                r, OUT, IN, group, bits, IN, OUT);
                    }
                    int rc = check_launch("q_gemv_kernel");
                    if (rc) return rc;
                }
                return ok();
            });
        });
    });
}

// Projection backward dX = bf16(bf16(dY) W_bf16) (gemm_dx.cuh).  wfmt DX_BF16:
// `w` dense bf16 [OUT, IN]; DX_Q4: the 4-bit group-64 container (fp16 scales).
// Shares rwkv_q_gemm's wait-error record.  Arguments are checked by the caller.
int launch_gemm_dx_any(int wfmt, const void* dy, const void* w, const uint32_t* wq, const void* scales,
                       const void* biases, int dx_dtype, void* dx, int rows, int OUT, int IN, int accumulate,
                       cudaStream_t st) {
    GemmScratch* sc = gemm_scratch();
    if (!sc) return fail(RWKV_E_CUDA, "rwkv_gemm_dx: workspace allocation failed");
    if (sc->flag.take(st))
        return fail(RWKV_E_TIMEOUT, "rwkv_gemm_dx: a tensor-core GEMM wait of an earlier call gave up; "
                                    "its outputs are not valid (flag cleared, nothing launched)");
    DxArgs a{};
    a.scales = (const __half*)scales;
    a.biases = (const __half*)biases;
    a.dx = dx;
    a.dx_dtype = dx_dtype;
    a.accumulate = accumulate;
    a.rows = rows;
    a.OUT = OUT;
    a.IN = IN;
    a.err = sc->err;
    a.err_host = sc->flag.host_dev;
    cudaError_t e = launch_gemm_dx(wfmt, a, dy, w, wq, sc->sm_count, st);
    if (e != cudaSuccess) return fail(RWKV_E_CUDA, "gemm_dx_kernel: %s", cudaGetErrorString(e));
    return ok();
}

int q_gemm_status(cudaStream_t st) {
    GemmScratch* sc = gemm_scratch();
    if (!sc) return fail(RWKV_E_CUDA, "rwkv_q_gemm_status: workspace allocation failed");
    return sc->flag.status(st, "rwkv_q_gemm");
}

int q_gemm_inject_wait_error(int host_record, cudaStream_t st) {
    GemmScratch* sc = gemm_scratch();
    if (!sc) return fail(RWKV_E_CUDA, "rwkv_q_gemm_inject_wait_error: workspace allocation failed");
    return sc->flag.inject(host_record, st);
}

int launch_q_dequant(const uint32_t* wq, const void* scales, const void* biases, int sdtype,
                     int odtype, void* out, const int32_t* ids, int OUT, int IN, int group,
                     int bits, int vocab, cudaStream_t st) {
    const int64_t n = (int64_t)OUT * (IN / 32);
    return dispatch_sdtype(sdtype, [&]<typename TS>() {
        return dispatch_dtype(odtype, [&]<typename TO>() {
            q_dequant_kernel<TS, TO><<<ceil_div(n, 256), 256, 0, st>>>(
                wq, (const TS*)scales, (const TS*)biases, (TO*)out, ids, OUT, IN, group, bits, vocab);
            return check_launch("q_dequant_kernel");
        });
    });
}

int launch_q_quantize(int wdtype, const void* W, uint32_t* wq, void* scales, void* biases,
                      int OUT, int IN, int group, int bits, cudaStream_t st) {
    const int64_t n = (int64_t)OUT * (IN / group);
    return dispatch_dtype(wdtype, [&]<typename TW>() {
        q_quantize_kernel<TW, TW><<<ceil_div(n, 128), 128, 0, st>>>(
            (const TW*)W, wq, (TW*)scales, (TW*)biases, OUT, IN, group, bits);
        return check_launch("q_quantize_kernel");
    });
}

}  // namespace rwkv
