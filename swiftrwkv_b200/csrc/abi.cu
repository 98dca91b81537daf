// extern "C" entry points of librwkvcuda (declared in include/rwkv_cuda.h).
// Each wrapper validates its arguments on the host -- null pointers, shapes,
// element types, alignment -- and returns a status before anything launches.
#include <string>

#include "common.cuh"

namespace rwkv {

std::string& last_error() {
    static thread_local std::string s;
    return s;
}

// kernels (defined in the other translation units)
int launch_wkv7_seq(int, const void*, const void*, const void*, const void*, const void*,
                    const void*, const float*, void*, float*, float*, float*, int, int, int,
                    cudaStream_t);
int launch_wkv7_step(int, const void*, const void*, const void*, const void*, const void*,
                     const void*, float*, void*, int, int, cudaStream_t);
int launch_wkv7_step_tail(const float*, const float*, const float*, const float*, const float*,
                          const float*, float*, const float*, const float*, const float*,
                          const float*, float*, int, int, float, cudaStream_t);
int launch_wkv_tail(const float*, const float*, const float*, const float*, const float*,
                    const float*, const float*, const float*, float*, int, int, int, float,
                    cudaStream_t);
int launch_wkv7_chunk_fwd(int, const void*, const void*, const void*, const void*, const void*,
                          const void*, const float*, void*, float*, float*, float*, int, int, int,
                          void*, cudaStream_t);
int64_t wkv7_chunk_workspace(int, int, int);
int64_t wkv7_chunk_bwd_workspace(int, int, int);
int launch_wkv7_chunk_bwd(int, const void*, const void*, const void*, const void*, const void*,
                          const void*, const float*, const float*, const void*, const float*, void*,
                          void*, void*, void*, void*, void*, float*, int, int, int, void*,
                          cudaStream_t);
int64_t wkv7_bwd_seq_workspace(int, int);
int launch_wkv7_bwd_seq(int, const void*, const void*, const void*, const void*, const void*,
                        const void*, const float*, const float*, const void*, const float*, void*,
                        void*, void*, void*, void*, void*, float*, int, int, int, float*,
                        cudaStream_t);
int launch_q_gemm(int, const void*, const uint32_t*, const void*, const void*, int, int, void*,
                  int, int, int, int, int, cudaStream_t);
int q_gemm_status(cudaStream_t);
int launch_gemm_dx_any(int, const void*, const void*, const uint32_t*, const void*, const void*, int, void*, int,
                       int, int, int, cudaStream_t);
int q_gemm_inject_wait_error(int, cudaStream_t);
int launch_q_dequant(const uint32_t*, const void*, const void*, int, int, void*, const int32_t*,
                     int, int, int, int, int, cudaStream_t);
int launch_q_quantize(int, const void*, uint32_t*, void*, void*, int, int, int, int, cudaStream_t);
int launch_sb6_dequant(const uint8_t*, const uint8_t*, const uint16_t*, int, void*, int, int, int,
                       cudaStream_t);
int launch_sb6_gemv(int, const void*, const uint8_t*, const uint8_t*, const uint16_t*, float*, int,
                    int, int, int, cudaStream_t);
int launch_sb6_to_affine(const uint8_t*, const uint8_t*, const uint16_t*, uint32_t*, float*,
                         float*, int*, int, int, int, cudaStream_t);
int launch_sym_dequant(const uint8_t*, const uint8_t*, const uint16_t*, int, void*, int, int, int,
                       cudaStream_t);
int launch_sym_gemv(int, const void*, const uint8_t*, const uint8_t*, const uint16_t*, float*, int,
                    int, int, int, int, cudaStream_t);
int launch_sym_rows(const int32_t*, int, const uint8_t*, const uint8_t*, const uint16_t*,
                    uint16_t*, int, int, cudaStream_t);

static inline bool al16(const void* p) { return p == nullptr || ((uintptr_t)p & 15u) == 0; }

static int check_wkv_common(int dtype, const void* const* req, int nreq, int B, int T, int H,
                            int N, const char* fn) {
    RWKV_REQUIRE(valid_dtype(dtype), RWKV_E_DTYPE, "%s: dtype %d", fn, dtype);
    for (int i = 0; i < nreq; i++)
        RWKV_REQUIRE(req[i] != nullptr, RWKV_E_NULL, "%s: required pointer #%d is NULL", fn, i);
    RWKV_REQUIRE(B >= 1 && T >= 1 && H >= 1, RWKV_E_SHAPE, "%s: B=%d T=%d H=%d must be >= 1", fn, B,
                 T, H);
    RWKV_REQUIRE(N == RWKV_WKV7_HEAD_SIZE, RWKV_E_UNSUPPORTED, "%s: N=%d, kernels take N=64", fn, N);
    RWKV_REQUIRE((int64_t)B * T * H * N < (1ll << 40), RWKV_E_SHAPE, "%s: tensor too large", fn);
    for (int i = 0; i < nreq; i++)
        RWKV_REQUIRE(al16(req[i]), RWKV_E_UNSUPPORTED, "%s: pointer #%d not 16-byte aligned", fn, i);
    return RWKV_OK;
}

static bool valid_bits(int bits) {
    return bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8;
}

static int check_affine(int OUT, int IN, int group, int bits, const char* fn) {
    RWKV_REQUIRE(OUT >= 1 && IN >= 1, RWKV_E_SHAPE, "%s: OUT=%d IN=%d", fn, OUT, IN);
    RWKV_REQUIRE(valid_bits(bits), RWKV_E_UNSUPPORTED, "%s: bits=%d not in {2,3,4,5,6,8}", fn, bits);
    RWKV_REQUIRE(group == 32 || group == 64 || group == 128, RWKV_E_UNSUPPORTED,
                 "%s: group=%d not in {32,64,128}", fn, group);
    RWKV_REQUIRE(IN % group == 0, RWKV_E_SHAPE, "%s: IN=%d not a multiple of group %d", fn, IN, group);
    return RWKV_OK;
}

}  // namespace rwkv

using namespace rwkv;

extern "C" {

int rwkv_version(void) { return 100; }

const char* rwkv_status_string(int s) {
    switch (s) {
        case RWKV_OK: return "ok";
        case RWKV_E_NULL: return "null pointer";
        case RWKV_E_SHAPE: return "bad shape";
        case RWKV_E_DTYPE: return "bad dtype";
        case RWKV_E_UNSUPPORTED: return "unsupported";
        case RWKV_E_CUDA: return "cuda error";
        case RWKV_E_TIMEOUT: return "device wait timed out";
        case RWKV_E_WORKSPACE: return "workspace missing or too small";
        default: return "unknown status";
    }
}

const char* rwkv_last_error(void) { return last_error().c_str(); }

int rwkv_wkv7_forward(int dtype, const void* r, const void* w, const void* k, const void* v,
                      const void* a, const void* b, const float* h_in, void* y, float* h_out,
                      int B, int T, int H, int N, rwkv_stream_t stream) {
    const void* req[] = {r, w, k, v, a, b, y};
    if (int rc = check_wkv_common(dtype, req, 7, B, T, H, N, "rwkv_wkv7_forward")) return rc;
    RWKV_REQUIRE(al16(h_in) && al16(h_out), RWKV_E_UNSUPPORTED, "rwkv_wkv7_forward: state not 16-byte aligned");
    return launch_wkv7_seq(dtype, r, w, k, v, a, b, h_in, y, h_out, nullptr, nullptr, B, T, H,
                           (cudaStream_t)stream);
}

int64_t rwkv_wkv7_forward_chunked_workspace_size(int B, int T, int H, int N) {
    (void)N;
    if (B < 1 || T < 1 || H < 1) return 0;
    return wkv7_chunk_workspace(B, T, H);
}

int rwkv_wkv7_forward_chunked(int dtype, const void* r, const void* w, const void* k, const void* v,
                              const void* a, const void* b, const float* h_in, void* y, float* h_out,
                              float* sa, int B, int T, int H, int N, void* workspace,
                              int64_t workspace_bytes, rwkv_stream_t stream) {
    const void* req[] = {r, w, k, v, a, b, y};
    if (int rc = check_wkv_common(dtype, req, 7, B, T, H, N, "rwkv_wkv7_forward_chunked")) return rc;
    const int64_t need = wkv7_chunk_workspace(B, T, H);
    RWKV_REQUIRE(workspace != nullptr && workspace_bytes >= need, RWKV_E_WORKSPACE,
                 "rwkv_wkv7_forward_chunked: workspace %lld bytes, need %lld",
                 (long long)workspace_bytes, (long long)need);
    RWKV_REQUIRE(al16(workspace), RWKV_E_UNSUPPORTED, "rwkv_wkv7_forward_chunked: workspace not 16-byte aligned");
    return launch_wkv7_chunk_fwd(dtype, r, w, k, v, a, b, h_in, y, h_out, sa, nullptr, B, T, H,
                                 workspace, (cudaStream_t)stream);
}

int rwkv_wkv7_train_forward_chunked(int dtype, const void* r, const void* w, const void* k,
                                    const void* v, const void* a, const void* b, const float* h_in,
                                    void* y, float* h_out, float* sa, float* h_ckpt, int B, int T,
                                    int H, int N, void* workspace, int64_t workspace_bytes,
                                    rwkv_stream_t stream) {
    const char* fn = "rwkv_wkv7_train_forward_chunked";
    const void* req[] = {r, w, k, v, a, b, y, h_ckpt};
    if (int rc = check_wkv_common(dtype, req, 8, B, T, H, N, fn)) return rc;
    RWKV_REQUIRE(T % RWKV_WKV7_CHUNK == 0, RWKV_E_SHAPE, "%s: T=%d must be a multiple of 16", fn, T);
    RWKV_REQUIRE(al16(h_in) && al16(h_out), RWKV_E_UNSUPPORTED, "%s: state not 16-byte aligned", fn);
    const int64_t need = wkv7_chunk_workspace(B, T, H);
    RWKV_REQUIRE(workspace != nullptr && workspace_bytes >= need, RWKV_E_WORKSPACE,
                 "%s: workspace %lld bytes, need %lld", fn, (long long)workspace_bytes, (long long)need);
    RWKV_REQUIRE(al16(workspace), RWKV_E_UNSUPPORTED, "%s: workspace not 16-byte aligned", fn);
    return launch_wkv7_chunk_fwd(dtype, r, w, k, v, a, b, h_in, y, h_out, sa, h_ckpt, B, T, H,
                                 workspace, (cudaStream_t)stream);
}

int64_t rwkv_wkv7_backward_chunked_workspace_size(int B, int T, int H, int N) {
    (void)N;
    if (B < 1 || T < RWKV_WKV7_CHUNK || H < 1) return 0;
    return wkv7_chunk_bwd_workspace(B, T, H);
}

int rwkv_wkv7_backward_chunked(int dtype, const void* r, const void* w, const void* k, const void* v,
                               const void* a, const void* b, const float* h_in, const float* h_ckpt,
                               const void* dy, const float* dh_out, void* dr, void* dw, void* dk,
                               void* dv, void* da, void* db, float* dh_in, int B, int T, int H, int N,
                               void* workspace, int64_t workspace_bytes, rwkv_stream_t stream) {
    const char* fn = "rwkv_wkv7_backward_chunked";
    const void* req[] = {r, w, k, v, a, b, h_ckpt, dy, dr, dw, dk, dv, da, db};
    if (int rc = check_wkv_common(dtype, req, 14, B, T, H, N, fn)) return rc;
    RWKV_REQUIRE(T % RWKV_WKV7_CHUNK == 0, RWKV_E_SHAPE, "%s: T=%d must be a multiple of 16", fn, T);
    RWKV_REQUIRE(al16(h_in) && al16(h_ckpt) && al16(dh_out) && al16(dh_in), RWKV_E_UNSUPPORTED,
                 "%s: state not 16-byte aligned", fn);
    const int64_t need = wkv7_chunk_bwd_workspace(B, T, H);
    RWKV_REQUIRE(workspace != nullptr && workspace_bytes >= need, RWKV_E_WORKSPACE,
                 "%s: workspace %lld bytes, need %lld", fn, (long long)workspace_bytes, (long long)need);
    RWKV_REQUIRE(al16(workspace), RWKV_E_UNSUPPORTED, "%s: workspace not 16-byte aligned", fn);
    return launch_wkv7_chunk_bwd(dtype, r, w, k, v, a, b, h_in, h_ckpt, dy, dh_out, dr, dw, dk, dv,
                                 da, db, dh_in, B, T, H, workspace, (cudaStream_t)stream);
}

int rwkv_wkv7_train_forward(int dtype, const void* r, const void* w, const void* k,
                            const void* v, const void* a, const void* b, const float* h_in,
                            void* y, float* h_out, float* sa, float* h_ckpt, int B, int T,
                            int H, int N, rwkv_stream_t stream) {
    const void* req[] = {r, w, k, v, a, b, y, h_ckpt};
    if (int rc = check_wkv_common(dtype, req, 8, B, T, H, N, "rwkv_wkv7_train_forward")) return rc;
    RWKV_REQUIRE(T % RWKV_WKV7_CHUNK == 0, RWKV_E_SHAPE,
                 "rwkv_wkv7_train_forward: T=%d must be a multiple of 16", T);
    RWKV_REQUIRE(al16(h_in) && al16(h_out), RWKV_E_UNSUPPORTED, "rwkv_wkv7_train_forward: state not 16-byte aligned");
    return launch_wkv7_seq(dtype, r, w, k, v, a, b, h_in, y, h_out, sa, h_ckpt, B, T, H,
                           (cudaStream_t)stream);
}

int64_t rwkv_wkv7_backward_workspace_size(int B, int T, int H, int N) {
    (void)T;
    (void)N;
    if (B < 1 || H < 1) return 0;
    return wkv7_bwd_seq_workspace(B, H);
}

int rwkv_wkv7_backward(int dtype, const void* r, const void* w, const void* k, const void* v,
                       const void* a, const void* b, const float* h_in, const float* h_ckpt,
                       const void* dy, const float* dh_out, void* dr, void* dw, void* dk,
                       void* dv, void* da, void* db, float* dh_in, int B, int T, int H, int N,
                       void* workspace, int64_t workspace_bytes, rwkv_stream_t stream) {
    const void* req[] = {r, w, k, v, a, b, h_ckpt, dy, dr, dw, dk, dv, da, db};
    if (int rc = check_wkv_common(dtype, req, 14, B, T, H, N, "rwkv_wkv7_backward")) return rc;
    RWKV_REQUIRE(T % RWKV_WKV7_CHUNK == 0, RWKV_E_SHAPE,
                 "rwkv_wkv7_backward: T=%d must be a multiple of 16", T);
    const int64_t need = wkv7_bwd_seq_workspace(B, H);
    RWKV_REQUIRE(workspace != nullptr && workspace_bytes >= need, RWKV_E_WORKSPACE,
                 "rwkv_wkv7_backward: workspace %lld bytes, need %lld",
                 (long long)workspace_bytes, (long long)need);
    RWKV_REQUIRE(al16(workspace), RWKV_E_UNSUPPORTED, "rwkv_wkv7_backward: workspace not 16-byte aligned");
    return launch_wkv7_bwd_seq(dtype, r, w, k, v, a, b, h_in, h_ckpt, dy, dh_out, dr, dw, dk, dv,
                               da, db, dh_in, B, T, H, (float*)workspace, (cudaStream_t)stream);
}

int rwkv_wkv7_step(int dtype, const void* r, const void* w, const void* k, const void* v,
                   const void* a, const void* b, float* h, void* y, int rows, int H, int N,
                   rwkv_stream_t stream) {
    const void* req[] = {r, w, k, v, a, b, h, y};
    if (int rc = check_wkv_common(dtype, req, 8, rows, 1, H, N, "rwkv_wkv7_step")) return rc;
    return launch_wkv7_step(dtype, r, w, k, v, a, b, h, y, rows, H, (cudaStream_t)stream);
}

int rwkv_wkv_tail(const float* wkv, const float* r, const float* k, const float* v,
                  const float* rk, const float* ln_w, const float* ln_b, const float* g,
                  float* out, int rows, int H, int S, float eps, rwkv_stream_t stream) {
    const void* req[] = {wkv, r, k, v, rk, ln_w, ln_b, g, out};
    for (int i = 0; i < 9; i++)
        RWKV_REQUIRE(req[i] != nullptr, RWKV_E_NULL, "rwkv_wkv_tail: pointer #%d is NULL", i);
    RWKV_REQUIRE(rows >= 1 && H >= 1 && S >= 1, RWKV_E_SHAPE, "rwkv_wkv_tail: rows=%d H=%d S=%d", rows, H, S);
    RWKV_REQUIRE(S % 32 == 0 && S <= 256, RWKV_E_UNSUPPORTED,
                 "rwkv_wkv_tail: head size %d must be a multiple of 32 (wkvTailApplies)", S);
    return launch_wkv_tail(wkv, r, k, v, rk, ln_w, ln_b, g, out, rows, H, S, eps, (cudaStream_t)stream);
}

int rwkv_wkv7_step_tail(const float* r, const float* w, const float* k, const float* v,
                        const float* a, const float* b, float* h, const float* rk,
                        const float* ln_w, const float* ln_b, const float* g, float* out,
                        int rows, int H, int N, float eps, rwkv_stream_t stream) {
    const void* req[] = {r, w, k, v, a, b, h, rk, ln_w, ln_b, g, out};
    if (int rc = check_wkv_common(RWKV_F32, req, 12, rows, 1, H, N, "rwkv_wkv7_step_tail")) return rc;
    return launch_wkv7_step_tail(r, w, k, v, a, b, h, rk, ln_w, ln_b, g, out, rows, H, eps,
                                 (cudaStream_t)stream);
}

int rwkv_q_gemm(int xdtype, const void* x, const uint32_t* wq, const void* scales,
                const void* biases, int sdtype, int ydtype, void* y, int rows, int OUT, int IN,
                int group, int bits, rwkv_stream_t stream) {
    RWKV_REQUIRE(x && wq && scales && biases && y, RWKV_E_NULL, "rwkv_q_gemm: NULL argument");
    RWKV_REQUIRE(valid_dtype(xdtype) && valid_dtype(sdtype) && valid_dtype(ydtype), RWKV_E_DTYPE,
                 "rwkv_q_gemm: dtypes x=%d s=%d y=%d", xdtype, sdtype, ydtype);
    RWKV_REQUIRE(rows >= 1, RWKV_E_SHAPE, "rwkv_q_gemm: rows=%d", rows);
    if (int rc = check_affine(OUT, IN, group, bits, "rwkv_q_gemm")) return rc;
    RWKV_REQUIRE(al16(x) && al16(wq), RWKV_E_UNSUPPORTED, "rwkv_q_gemm: x / wq not 16-byte aligned");
    return launch_q_gemm(xdtype, x, wq, scales, biases, sdtype, ydtype, y, rows, OUT, IN, group,
                         bits, (cudaStream_t)stream);
}

static int check_dx(int dy_dtype, const void* dy, int dx_dtype, void* dx, int rows, int OUT, int IN,
                    int accumulate, const char* fn) {
    RWKV_REQUIRE(dy && dx, RWKV_E_NULL, "%s: NULL argument", fn);
    RWKV_REQUIRE(dy_dtype == RWKV_BF16, RWKV_E_DTYPE,
                 "%s: dY dtype %d; the backward takes the cotangent in bf16 (cast it first)", fn, dy_dtype);
    RWKV_REQUIRE(dx_dtype == RWKV_F32 || dx_dtype == RWKV_BF16 || dx_dtype == RWKV_F16, RWKV_E_DTYPE,
                 "%s: dX dtype %d", fn, dx_dtype);
    RWKV_REQUIRE(accumulate == 0 || dx_dtype == RWKV_F32, RWKV_E_DTYPE, "%s: accumulate needs an fp32 dX", fn);
    RWKV_REQUIRE(rows >= 1 && OUT >= 1 && IN >= 1, RWKV_E_SHAPE, "%s: rows=%d OUT=%d IN=%d", fn, rows, OUT, IN);
    RWKV_REQUIRE(IN % 128 == 0 && OUT % 64 == 0, RWKV_E_UNSUPPORTED,
                 "%s: IN=%d must be a multiple of 128 and OUT=%d of 64", fn, IN, OUT);
    RWKV_REQUIRE(al16(dy), RWKV_E_UNSUPPORTED, "%s: dY not 16-byte aligned", fn);
    return RWKV_OK;
}

int rwkv_gemm_dx(int dy_dtype, const void* dy, int w_dtype, const void* w, int dx_dtype, void* dx, int rows,
                 int OUT, int IN, int accumulate, rwkv_stream_t stream) {
    if (int rc = check_dx(dy_dtype, dy, dx_dtype, dx, rows, OUT, IN, accumulate, "rwkv_gemm_dx")) return rc;
    RWKV_REQUIRE(w, RWKV_E_NULL, "rwkv_gemm_dx: NULL weight");
    RWKV_REQUIRE(w_dtype == RWKV_BF16, RWKV_E_DTYPE, "rwkv_gemm_dx: weight dtype %d (bf16 only)", w_dtype);
    RWKV_REQUIRE(al16(w), RWKV_E_UNSUPPORTED, "rwkv_gemm_dx: weight not 16-byte aligned");
    return launch_gemm_dx_any(DX_BF16, dy, w, nullptr, nullptr, nullptr, dx_dtype, dx, rows, OUT, IN, accumulate,
                              (cudaStream_t)stream);
}

int rwkv_q_gemm_dx(int dy_dtype, const void* dy, const uint32_t* wq, const void* scales, const void* biases,
                   int sdtype, int dx_dtype, void* dx, int rows, int OUT, int IN, int group, int bits,
                   int accumulate, rwkv_stream_t stream) {
    if (int rc = check_dx(dy_dtype, dy, dx_dtype, dx, rows, OUT, IN, accumulate, "rwkv_q_gemm_dx")) return rc;
    RWKV_REQUIRE(wq && scales && biases, RWKV_E_NULL, "rwkv_q_gemm_dx: NULL weight buffer");
    RWKV_REQUIRE(group == 64 && bits == 4 && sdtype == RWKV_F16, RWKV_E_UNSUPPORTED,
                 "rwkv_q_gemm_dx: group=%d bits=%d scale dtype %d (4-bit group 64, fp16 scales)", group, bits,
                 sdtype);
    RWKV_REQUIRE(al16(wq), RWKV_E_UNSUPPORTED, "rwkv_q_gemm_dx: wq not 16-byte aligned");
    return launch_gemm_dx_any(DX_Q4, dy, nullptr, wq, scales, biases, dx_dtype, dx, rows, OUT, IN, accumulate,
                              (cudaStream_t)stream);
}

int rwkv_q_gemm_status(rwkv_stream_t stream) { return q_gemm_status((cudaStream_t)stream); }

int rwkv_q_gemm_inject_wait_error(int host_record, rwkv_stream_t stream) {
    return q_gemm_inject_wait_error(host_record, (cudaStream_t)stream);
}

int rwkv_q_dequant(const uint32_t* wq, const void* scales, const void* biases, int sdtype,
                   int odtype, void* w_out, int OUT, int IN, int group, int bits,
                   rwkv_stream_t stream) {
    RWKV_REQUIRE(wq && scales && biases && w_out, RWKV_E_NULL, "rwkv_q_dequant: NULL argument");
    RWKV_REQUIRE(valid_dtype(sdtype) && valid_dtype(odtype), RWKV_E_DTYPE, "rwkv_q_dequant: dtypes");
    if (int rc = check_affine(OUT, IN, group, bits, "rwkv_q_dequant")) return rc;
    RWKV_REQUIRE(al16(wq), RWKV_E_UNSUPPORTED, "rwkv_q_dequant: wq not 16-byte aligned");
    return launch_q_dequant(wq, scales, biases, sdtype, odtype, w_out, nullptr, OUT, IN, group, bits,
                            OUT, (cudaStream_t)stream);
}

int rwkv_q_rows(const int32_t* ids, int n_ids, const uint32_t* wq, const void* scales,
                const void* biases, int sdtype, int odtype, void* out, int vocab, int IN,
                int group, int bits, rwkv_stream_t stream) {
    RWKV_REQUIRE(ids && wq && scales && biases && out, RWKV_E_NULL, "rwkv_q_rows: NULL argument");
    RWKV_REQUIRE(valid_dtype(sdtype) && valid_dtype(odtype), RWKV_E_DTYPE, "rwkv_q_rows: dtypes");
    RWKV_REQUIRE(n_ids >= 1, RWKV_E_SHAPE, "rwkv_q_rows: n_ids=%d", n_ids);
    if (int rc = check_affine(vocab, IN, group, bits, "rwkv_q_rows")) return rc;
    RWKV_REQUIRE(al16(wq), RWKV_E_UNSUPPORTED, "rwkv_q_rows: wq not 16-byte aligned");
    return launch_q_dequant(wq, scales, biases, sdtype, odtype, out, ids, n_ids, IN, group, bits,
                            vocab, (cudaStream_t)stream);
}

int rwkv_q_quantize(int wdtype, const void* W, uint32_t* wq, void* scales, void* biases,
                    int OUT, int IN, int group, int bits, rwkv_stream_t stream) {
    RWKV_REQUIRE(W && wq && scales && biases, RWKV_E_NULL, "rwkv_q_quantize: NULL argument");
    RWKV_REQUIRE(valid_dtype(wdtype), RWKV_E_DTYPE, "rwkv_q_quantize: dtype %d", wdtype);
    if (int rc = check_affine(OUT, IN, group, bits, "rwkv_q_quantize")) return rc;
    return launch_q_quantize(wdtype, W, wq, scales, biases, OUT, IN, group, bits,
                             (cudaStream_t)stream);
}

static int check_sb6(const void* qblk, const void* qsqm, const void* ddm, int OUT, int IN,
                     int xbits, const char* fn) {
    RWKV_REQUIRE(qblk && qsqm && ddm, RWKV_E_NULL, "%s: NULL buffer", fn);
    RWKV_REQUIRE(OUT >= 1 && IN >= 1, RWKV_E_SHAPE, "%s: OUT=%d IN=%d", fn, OUT, IN);
    RWKV_REQUIRE(xbits >= 0 && xbits <= 2, RWKV_E_SHAPE, "%s: xbits=%d not in 0..2", fn, xbits);
    RWKV_REQUIRE(IN % 256 == 0, RWKV_E_UNSUPPORTED, "%s: IN=%d not a multiple of 256", fn, IN);
    RWKV_REQUIRE(al16(qblk), RWKV_E_UNSUPPORTED, "%s: qblk not 16-byte aligned", fn);
    return RWKV_OK;
}

int rwkv_sb6_dequant(const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm, int odtype,
                     void* out, int OUT, int IN, int xbits, rwkv_stream_t stream) {
    if (int rc = check_sb6(qblk, qsqm, ddm, OUT, IN, xbits, "rwkv_sb6_dequant")) return rc;
    RWKV_REQUIRE(out != nullptr, RWKV_E_NULL, "rwkv_sb6_dequant: out is NULL");
    RWKV_REQUIRE(valid_dtype(odtype), RWKV_E_DTYPE, "rwkv_sb6_dequant: dtype %d", odtype);
    return launch_sb6_dequant(qblk, qsqm, ddm, odtype, out, OUT, IN, xbits, (cudaStream_t)stream);
}

int rwkv_sb6_gemv(int xdtype, const void* x, const uint8_t* qblk, const uint8_t* qsqm,
                  const uint16_t* ddm, float* y, int rows, int OUT, int IN, int xbits,
                  rwkv_stream_t stream) {
    if (int rc = check_sb6(qblk, qsqm, ddm, OUT, IN, xbits, "rwkv_sb6_gemv")) return rc;
    RWKV_REQUIRE(x && y, RWKV_E_NULL, "rwkv_sb6_gemv: NULL x / y");
    RWKV_REQUIRE(valid_dtype(xdtype), RWKV_E_DTYPE, "rwkv_sb6_gemv: dtype %d", xdtype);
    RWKV_REQUIRE(rows >= 1, RWKV_E_SHAPE, "rwkv_sb6_gemv: rows=%d", rows);
    return launch_sb6_gemv(xdtype, x, qblk, qsqm, ddm, y, rows, OUT, IN, xbits, (cudaStream_t)stream);
}

int rwkv_sb6_to_affine(const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm,
                       uint32_t* wq, float* scales, float* biases, int* fp16_ok_host, int OUT,
                       int IN, int xbits, rwkv_stream_t stream) {
    if (int rc = check_sb6(qblk, qsqm, ddm, OUT, IN, xbits, "rwkv_sb6_to_affine")) return rc;
    RWKV_REQUIRE(wq && scales && biases && fp16_ok_host, RWKV_E_NULL, "rwkv_sb6_to_affine: NULL output");
    cudaStream_t st = (cudaStream_t)stream;
    int* flag = nullptr;
    if (cudaMallocAsync((void**)&flag, sizeof(int), st) != cudaSuccess)
        return fail(RWKV_E_CUDA, "rwkv_sb6_to_affine: flag allocation failed");
    cudaMemsetAsync(flag, 0, sizeof(int), st);
    int rc = launch_sb6_to_affine(qblk, qsqm, ddm, wq, scales, biases, flag, OUT, IN, xbits, st);
    int bad = 0;
    if (rc == RWKV_OK) {
        cudaMemcpyAsync(&bad, flag, sizeof(int), cudaMemcpyDeviceToHost, st);
        cudaFreeAsync(flag, st);
        if (cudaStreamSynchronize(st) != cudaSuccess)
            return fail(RWKV_E_CUDA, "rwkv_sb6_to_affine: %s", cudaGetErrorString(cudaGetLastError()));
        *fp16_ok_host = bad ? 0 : 1;
        return ok();
    }
    cudaFreeAsync(flag, st);
    return rc;
}

static int check_sym(const void* qblk, const void* qs, const void* d, int OUT, int IN, int bits,
                     const char* fn) {
    RWKV_REQUIRE(qblk && qs && d, RWKV_E_NULL, "%s: NULL buffer", fn);
    RWKV_REQUIRE(OUT >= 1 && IN >= 1, RWKV_E_SHAPE, "%s: OUT=%d IN=%d", fn, OUT, IN);
    RWKV_REQUIRE(bits == 6 || bits == 8, RWKV_E_SHAPE, "%s: bits=%d not in {6,8}", fn, bits);
    RWKV_REQUIRE(IN % (bits == 8 ? 16 : 32) == 0, RWKV_E_SHAPE, "%s: IN=%d", fn, IN);
    return RWKV_OK;
}

int rwkv_sym_dequant(const uint8_t* qblk, const uint8_t* qs, const uint16_t* d, int odtype,
                     void* out, int OUT, int IN, int bits, rwkv_stream_t stream) {
    if (int rc = check_sym(qblk, qs, d, OUT, IN, bits, "rwkv_sym_dequant")) return rc;
    RWKV_REQUIRE(out != nullptr, RWKV_E_NULL, "rwkv_sym_dequant: out is NULL");
    RWKV_REQUIRE(valid_dtype(odtype), RWKV_E_DTYPE, "rwkv_sym_dequant: dtype %d", odtype);
    RWKV_REQUIRE(al16(qblk), RWKV_E_UNSUPPORTED, "rwkv_sym_dequant: qblk not 16-byte aligned");
    return launch_sym_dequant(qblk, qs, d, odtype, out, OUT, IN, bits, (cudaStream_t)stream);
}

int rwkv_sym_gemv(int xdtype, const void* x, const uint8_t* qblk, const uint8_t* qs,
                  const uint16_t* d, float* y, int nn, int OUT, int IN, int bits, int out_per,
                  rwkv_stream_t stream) {
    if (int rc = check_sym(qblk, qs, d, OUT, IN, bits, "rwkv_sym_gemv")) return rc;
    RWKV_REQUIRE(x && y, RWKV_E_NULL, "rwkv_sym_gemv: NULL x / y");
    RWKV_REQUIRE(valid_dtype(xdtype), RWKV_E_DTYPE, "rwkv_sym_gemv: dtype %d", xdtype);
    RWKV_REQUIRE(nn >= 1, RWKV_E_SHAPE, "rwkv_sym_gemv: nn=%d", nn);
    RWKV_REQUIRE(IN % 256 == 0, RWKV_E_UNSUPPORTED, "rwkv_sym_gemv: IN=%d not a multiple of 256", IN);
    RWKV_REQUIRE(out_per >= 4 && out_per % 4 == 0 && OUT % out_per == 0, RWKV_E_UNSUPPORTED,
                 "rwkv_sym_gemv: out_per=%d must divide OUT=%d and be a multiple of 4", out_per, OUT);
    RWKV_REQUIRE(al16(qblk), RWKV_E_UNSUPPORTED, "rwkv_sym_gemv: qblk not 16-byte aligned");
    return launch_sym_gemv(xdtype, x, qblk, qs, d, y, nn, OUT, IN, bits, out_per, (cudaStream_t)stream);
}

int rwkv_sym_rows(const int32_t* ids, int n_ids, const uint8_t* codes, const uint8_t* qs,
                  const uint16_t* d, uint16_t* out, int vocab, int IN, rwkv_stream_t stream) {
    RWKV_REQUIRE(ids && codes && qs && d && out, RWKV_E_NULL, "rwkv_sym_rows: NULL argument");
    RWKV_REQUIRE(n_ids >= 1 && vocab >= 1 && IN >= 16 && IN % 16 == 0, RWKV_E_SHAPE,
                 "rwkv_sym_rows: n_ids=%d vocab=%d IN=%d", n_ids, vocab, IN);
    return launch_sym_rows(ids, n_ids, codes, qs, d, out, vocab, IN, (cudaStream_t)stream);
}

}  // extern "C"
