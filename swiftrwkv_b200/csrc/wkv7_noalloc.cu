// rwkv_wkv7_backward_noalloc: the WKV-7 backward for callers that cannot
// allocate device memory.
//
// Who needs it: a host that hands this library only the tensors of the op
// itself.  An autograd or custom-function bridge typically owns every device
// buffer through its own allocator and passes the kernel its declared inputs
// and outputs, with no way to request a temporary; a serving or training
// process that has reserved its whole memory budget up front cannot have a
// plugin call cudaMalloc behind its back (the call can fail, and it
// synchronises the device).  rwkv_wkv7_backward needs a caller-supplied
// workspace for the recomputed chunk states; this entry point takes that
// scratch from a fixed array compiled into the library instead.
//
// The array holds NOALLOC_MAX_HEADS (batch, head) pairs of 17 fp32 64x64
// states: 240 x 272 KiB = 63.75 MiB on every GPU that loads this library,
// held until the process exits.  Larger B*H is rejected with RWKV_E_SHAPE.
//
// No allocation: the array's device address is looked up once per device
// (cudaGetSymbolAddress, with that device current) on the first call there;
// that first call on a device should therefore come before any stream
// capture.  The address is kept with the id of the context it was looked up
// in; a call in another context on that device (after a cudaDeviceReset, say)
// looks it up again.  The kernel is the same one rwkv_wkv7_backward launches.
//
// Sharing: every call on a device uses the same array, and the array keeps
// the previous call's contents.  Nothing in it has to start at zero -- each
// chunk's 17 state slots are written before they are read -- so nothing is
// cleared.  Two calls in flight on the same device at the same time (on
// different streams, or from different threads without ordering) race on the
// array and give wrong gradients; order them on one stream.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace rwkv {

int64_t wkv7_bwd_seq_workspace(int, int);
int launch_wkv7_bwd_seq(int, const void*, const void*, const void*, const void*, const void*,
                        const void*, const float*, const float*, const void*, const float*, void*,
                        void*, void*, void*, void*, void*, float*, int, int, int, float*,
                        cudaStream_t);

namespace {

constexpr int NOALLOC_MAX_HEADS = RWKV_NOALLOC_MAX_HEADS;
constexpr int64_t NOALLOC_HEAD_BYTES = (int64_t)(RWKV_WKV7_CHUNK + 1) * 64 * 64 * 4;
constexpr int64_t NOALLOC_BYTES = NOALLOC_MAX_HEADS * NOALLOC_HEAD_BYTES;
static_assert(NOALLOC_BYTES % 16 == 0, "scratch rows stay 16-byte aligned");

// In host code this name only stands for the device array; its device
// address comes from cudaGetSymbolAddress.
static __device__ __align__(256) float g_bwd_scratch[NOALLOC_BYTES / 4];

constexpr int MAX_DEVICES = 64;

// Unique id of the calling thread's current context (0 when the driver entry
// points are unavailable: the cached address is then kept per device).
unsigned long long current_context_id() {
    static PFN_cuCtxGetCurrent_v4000 get_cur = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_cur = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_cur && get_id && get_cur(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS) return id;
    return 0;
}

// Device address of g_bwd_scratch on the current device, looked up on the
// first call there, and again when the device's current context has changed
// (nullptr and the error recorded on failure).
float* scratch_on_current_device() {
    static std::mutex mu;
    static float* addr[MAX_DEVICES] = {};
    static unsigned long long ctx_of[MAX_DEVICES] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        fail(RWKV_E_CUDA, "rwkv_wkv7_backward_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
        return nullptr;
    }
    if (dev < 0 || dev >= MAX_DEVICES) {
        fail(RWKV_E_UNSUPPORTED, "rwkv_wkv7_backward_noalloc: device %d beyond %d", dev, MAX_DEVICES);
        return nullptr;
    }
    // 0 until the runtime has made the device's context current (the lookup
    // below does), else the id that tells a reset device's new context apart
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev] || ctx_of[dev] != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_bwd_scratch);
        if (e != cudaSuccess || p == nullptr) {
            fail(RWKV_E_CUDA, "rwkv_wkv7_backward_noalloc: scratch address on device %d: %s", dev,
                 cudaGetErrorString(e));
            return nullptr;
        }
        addr[dev] = static_cast<float*>(p);
        ctx_of[dev] = current_context_id();
    }
    return addr[dev];
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace
}  // namespace rwkv

using namespace rwkv;

extern "C" int rwkv_wkv7_backward_noalloc(int dtype, const void* r, const void* w, const void* k,
                                          const void* v, const void* a, const void* b,
                                          const float* h_in, const float* h_ckpt, const void* dy,
                                          const float* dh_out, void* dr, void* dw, void* dk,
                                          void* dv, void* da, void* db, float* dh_in, int B, int T,
                                          int H, int N, rwkv_stream_t stream) {
    const char* fn = "rwkv_wkv7_backward_noalloc";
    RWKV_REQUIRE(dtype == RWKV_F32 || dtype == RWKV_BF16 || dtype == RWKV_F16, RWKV_E_DTYPE,
                 "%s: dtype %d", fn, dtype);
    const void* req[] = {r, w, k, v, a, b, h_ckpt, dy, dr, dw, dk, dv, da, db};
    for (int i = 0; i < 14; i++)
        RWKV_REQUIRE(req[i] != nullptr, RWKV_E_NULL, "%s: required pointer #%d is NULL", fn, i);
    RWKV_REQUIRE(B >= 1 && T >= 1 && H >= 1, RWKV_E_SHAPE, "%s: B=%d T=%d H=%d must be >= 1", fn, B, T, H);
    RWKV_REQUIRE(N == RWKV_WKV7_HEAD_SIZE, RWKV_E_UNSUPPORTED, "%s: N=%d, kernels take N=64", fn, N);
    RWKV_REQUIRE(T % RWKV_WKV7_CHUNK == 0, RWKV_E_SHAPE, "%s: T=%d must be a multiple of 16", fn, T);
    RWKV_REQUIRE((int64_t)B * T * H * N < (1ll << 40), RWKV_E_SHAPE, "%s: tensor too large", fn);
    RWKV_REQUIRE((int64_t)B * H <= NOALLOC_MAX_HEADS, RWKV_E_SHAPE,
                 "%s: B*H=%lld exceeds the built-in scratch of %d (batch, head) pairs "
                 "(%lld bytes); use rwkv_wkv7_backward with a workspace",
                 fn, (long long)B * H, NOALLOC_MAX_HEADS, (long long)NOALLOC_BYTES);
    for (int i = 0; i < 14; i++)
        RWKV_REQUIRE(aligned16(req[i]), RWKV_E_UNSUPPORTED, "%s: pointer #%d not 16-byte aligned", fn, i);
    RWKV_REQUIRE(wkv7_bwd_seq_workspace(B, H) <= NOALLOC_BYTES, RWKV_E_SHAPE, "%s: scratch too small", fn);
    float* scratch = scratch_on_current_device();
    if (!scratch) return RWKV_E_CUDA;
    return launch_wkv7_bwd_seq(dtype, r, w, k, v, a, b, h_in, h_ckpt, dy, dh_out, dr, dw, dk, dv,
                               da, db, dh_in, B, T, H, scratch, (cudaStream_t)stream);
}
