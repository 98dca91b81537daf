// Shared helpers for librwkvcuda: status reporting, element-type access and
// small warp primitives.  Everything here is header-only and sm_100a-only.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/rwkv_cuda.h"

namespace rwkv {

// ------------------------------------------------------------ error reporting

// Thread-local text of the calling thread's last failure (rwkv_last_error).
std::string& last_error();

inline int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    last_error() = buf;
    return code;
}

inline int ok() {
    last_error().clear();
    return RWKV_OK;
}

// Checks the launch that was just issued; converts a CUDA error to a status.
inline int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(RWKV_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return ok();
}

#define RWKV_REQUIRE(cond, code, ...)              \
    do {                                           \
        if (!(cond)) return ::rwkv::fail(code, __VA_ARGS__); \
    } while (0)

inline bool valid_dtype(int dt) { return dt == RWKV_F32 || dt == RWKV_BF16 || dt == RWKV_F16; }

// ------------------------------------------------------------- element access

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Runtime-dtype dispatch: calls f.template operator()<T>() with T the element
// type of `dt`.
template <typename F>
inline int dispatch_dtype(int dt, F&& f) {
    switch (dt) {
        case RWKV_F32: return f.template operator()<float>();
        case RWKV_BF16: return f.template operator()<__nv_bfloat16>();
        case RWKV_F16: return f.template operator()<__half>();
        default: return fail(RWKV_E_DTYPE, "unknown dtype %d", dt);
    }
}

// ------------------------------------------------------------ warp utilities

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over aligned groups of G consecutive lanes (G a power of two <= 32).
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while its predecessor in the stream is still running: it must call
// pdl_wait() before it reads or writes anything the predecessor touches
// (outside a PDL launch both are no-ops).  pdl_trigger() lets the successor
// launch once every CTA of this grid has issued it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Base-weight formats of the projection backward (gemm_dx.cuh): dense bf16,
// or the MLX affine 4-bit group-64 container dequantised on the fly.
enum : int { DX_BF16 = 0, DX_Q4 = 1 };

}  // namespace rwkv
