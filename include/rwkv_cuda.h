/*
 * rwkv_cuda.h -- C ABI of the B200 (sm_100a) WKV-7 and quantised-GEMV library
 * (librwkvcuda.so).
 *
 * Conventions (shared by every entry point):
 *  - Every function returns an int status: RWKV_OK (0) or a negative
 *    RWKV_E_* code.  Nothing traps; rwkv_last_error() gives a one-line reason
 *    for the calling thread's last failure.
 *  - Every buffer is a caller-owned DEVICE pointer unless stated otherwise.
 *    Calls are asynchronous on the given stream (NULL = the legacy default
 *    stream); argument checks happen on the host before anything launches.
 *  - Element types are explicit (RWKV_F32 / RWKV_BF16 / RWKV_F16).  WKV state
 *    is always fp32, laid out [.., H, N, N] with rows = value index dv and
 *    columns = key index dk; sequence tensors are [B, T, H, N] row-major.
 *  - Optional tensors may be NULL, mirroring the reference's Swift optionals
 *    (h_in = NULL means a zero state; an output that is NULL is not written).
 *  - Shapes a kernel does not take return RWKV_E_UNSUPPORTED (the reference's
 *    `nil` fall-back); there is no CPU fallback behind any entry point.
 *
 * Each declaration cites the reference interface (RafaelUI/SwiftRWKV, file:line)
 * it replaces.
 */
#ifndef RWKV_CUDA_H
#define RWKV_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* rwkv_stream_t; /* == cudaStream_t */

enum {
    RWKV_OK = 0,
    RWKV_E_NULL = -1,        /* a required pointer is NULL */
    RWKV_E_SHAPE = -2,       /* inconsistent or out-of-range sizes */
    RWKV_E_DTYPE = -3,       /* element type not accepted by this entry point */
    RWKV_E_UNSUPPORTED = -4, /* valid shape the kernel does not take */
    RWKV_E_CUDA = -5,        /* a CUDA runtime call failed */
    RWKV_E_TIMEOUT = -6,     /* a bounded device-side wait gave up */
    RWKV_E_WORKSPACE = -7    /* workspace missing or too small */
};

enum { RWKV_F32 = 0, RWKV_BF16 = 1, RWKV_F16 = 2 };

#define RWKV_WKV7_HEAD_SIZE 64 /* WKV7_HEAD_SIZE, Sources/RWKVKernel/WKV7.swift:7 */
#define RWKV_WKV7_CHUNK 16     /* WKV7_CHUNK, Sources/RWKVKernel/WKV7.swift:8 */

/* ---------------------------------------------------------------- library */

int rwkv_version(void);                  /* 100*major + minor */
const char* rwkv_status_string(int status);
const char* rwkv_last_error(void);       /* thread-local, "" when none */

/* ------------------------------------------------------------------ WKV-7
 * r, w, k, v, a, b, y: [B, T, H, N] in `dtype`; h_in/h_out: [B, H, N, N] fp32.
 * N must be 64.  The recurrence per head, row dv (Sources/RWKVKernel/
 * WKV7Reference.swift:47-74): sa = S a;  S <- S diag(w) + v k^T + sa b^T;
 * y = S r (on the updated S).
 */

/* Frozen forward over the whole sequence, any T >= 1.
 * Replaces wkv7SequenceForward (Sources/RWKVKernel/WKV7.swift:242-264), and
 * with it wkv7ForwardWithState / wkv7ForwardChunked / wkv7Forward
 * (WKV7.swift:96-148), which give the same result. */
int rwkv_wkv7_forward(int dtype, const void* r, const void* w, const void* k, const void* v,
                      const void* a, const void* b, const float* h_in, void* y, float* h_out,
                      int B, int T, int H, int N, rwkv_stream_t stream);

/* Prefill form of rwkv_wkv7_forward, chunked (same arguments and results to
 * fp32 rounding, ~1e-6 relative).  16-token chunks in the normalised DPLR
 * form: each chunk's transition S -> S A_c + B_c is built in parallel over
 * chunks (tensor cores), a scan applies them (one 64x64x64 fp32 product per
 * chunk and head, split over 8 CTAs of 8 state rows), and each chunk's
 * outputs come from its start state -- so the T-sequential depth drops
 * sixteen-fold.  Unlike rwkv_wkv7_forward it does not
 * promise the bitwise identities of the sequential form (step = forward at
 * T=1, split = contiguous).  h_in / h_out as in rwkv_wkv7_forward; sa
 * [B,T,H,N] fp32 (may be NULL) receives S_{t-1} a_t as the training forward
 * does.  `workspace`: rwkv_wkv7_forward_chunked_workspace_size bytes of device
 * memory (3 states per chunk and head).  Replaces wkv7SequenceForward /
 * wkv7ForwardWithState on the prefill path (Sources/RWKVKernel/WKV7.swift:
 * 96-148, :242-264). */
int64_t rwkv_wkv7_forward_chunked_workspace_size(int B, int T, int H, int N);
int rwkv_wkv7_forward_chunked(int dtype, const void* r, const void* w, const void* k,
                              const void* v, const void* a, const void* b, const float* h_in,
                              void* y, float* h_out, float* sa, int B, int T, int H, int N,
                              void* workspace, int64_t workspace_bytes, rwkv_stream_t stream);

/* Differentiable forward of the training path: as rwkv_wkv7_forward, plus
 * sa [B,T,H,N] fp32 (may be NULL) and h_ckpt [B, H, T/16, N, N] fp32, the state
 * after every 16 steps (the last one equals h_out).  T % 16 == 0.
 * Replaces wkv7TrainWithState's forward kernel (Sources/RWKVKernel/
 * WKV7Train.swift:26-97, :375-468) and wkv7Train (:472-475). */
int rwkv_wkv7_train_forward(int dtype, const void* r, const void* w, const void* k,
                            const void* v, const void* a, const void* b, const float* h_in,
                            void* y, float* h_out, float* sa, float* h_ckpt, int B, int T,
                            int H, int N, rwkv_stream_t stream);

/* Chunked form of rwkv_wkv7_train_forward (same arguments and results to fp32
 * rounding, plus a workspace of rwkv_wkv7_forward_chunked_workspace_size
 * bytes): the chunked prefill kernels with each chunk's end state written to
 * h_ckpt [B, H, T/16, N, N].  T % 16 == 0.  Replaces wkv7TrainWithState's
 * forward kernel (Sources/RWKVKernel/WKV7Train.swift:26-97, :375-468) on the
 * prefill-sized path. */
int rwkv_wkv7_train_forward_chunked(int dtype, const void* r, const void* w, const void* k,
                                    const void* v, const void* a, const void* b, const float* h_in,
                                    void* y, float* h_out, float* sa, float* h_ckpt, int B, int T,
                                    int H, int N, void* workspace, int64_t workspace_bytes,
                                    rwkv_stream_t stream);

/* Workspace bytes rwkv_wkv7_backward needs for these sizes. */
int64_t rwkv_wkv7_backward_workspace_size(int B, int T, int H, int N);

/* Gradients of (y, h_out) w.r.t. (r, w, k, v, a, b, h_in).  h_in (NULL = zero)
 * and h_ckpt come from the forward; dh_out may be NULL (zero); dh_in may be
 * NULL (not written).  States inside a chunk are recomputed from the chunk's
 * starting checkpoint (no division by w).  Deterministic.  T % 16 == 0.
 * `workspace` is device memory of rwkv_wkv7_backward_workspace_size bytes.
 * Replaces the VJP of wkv7TrainWithState: ckptBwdKernelV2 / ckptBwdKernel
 * (Sources/RWKVKernel/WKV7Train.swift:99-339, :410-420). */
int rwkv_wkv7_backward(int dtype, const void* r, const void* w, const void* k, const void* v,
                       const void* a, const void* b, const float* h_in, const float* h_ckpt,
                       const void* dy, const float* dh_out, void* dr, void* dw, void* dk,
                       void* dv, void* da, void* db, float* dh_in, int B, int T, int H, int N,
                       void* workspace, int64_t workspace_bytes, rwkv_stream_t stream);

/* Chunked (DPLR) form of rwkv_wkv7_backward: same arguments and results to
 * fp32 rounding, deterministic, T % 16 == 0.  The gradient at every chunk
 * boundary comes from a reverse scan (Q' = Q A_c^T + DY B', built per chunk in
 * parallel), then each chunk's gradients come from its start state (the
 * h_ckpt / h_in checkpoint) and its boundary gradient as tensor-core products,
 * so the T-sequential depth is one 64x64x64 product per 16 tokens.  Chunks
 * whose decays underflow (smallest c_16 < 1e-30) are done token by token.
 * `workspace`: rwkv_wkv7_backward_chunked_workspace_size bytes (3 states per
 * chunk and head).  Replaces the VJP of wkv7TrainWithState (Sources/
 * RWKVKernel/WKV7Train.swift:99-339, :410-420) on the training path. */
int64_t rwkv_wkv7_backward_chunked_workspace_size(int B, int T, int H, int N);
int rwkv_wkv7_backward_chunked(int dtype, const void* r, const void* w, const void* k, const void* v,
                               const void* a, const void* b, const float* h_in, const float* h_ckpt,
                               const void* dy, const float* dh_out, void* dr, void* dw, void* dk,
                               void* dv, void* da, void* db, float* dh_in, int B, int T, int H, int N,
                               void* workspace, int64_t workspace_bytes, rwkv_stream_t stream);

/* rwkv_wkv7_backward without a workspace argument and without allocating.
 * No counterpart in the reference: it exists for hosts that cannot allocate
 * device memory for this library -- a framework bridge that passes the op only
 * its own input and output tensors, or a process whose memory budget is
 * reserved up front, where a cudaMalloc could fail and would synchronise the
 * device.  The recompute scratch is a fixed array built into the library:
 * RWKV_NOALLOC_MAX_HEADS (batch, head) pairs x 272 KiB = 63.75 MiB, held by
 * every GPU that loads the library until the process exits; B*H above the
 * limit returns RWKV_E_SHAPE.  The first call on a device, and the first
 * after the device's context changed (a cudaDeviceReset), looks the array's
 * address up (make that call before any stream capture).  All calls on a device share the array:
 * calls that overlap on the GPU race, so order them on one stream.  Same
 * arguments and results as rwkv_wkv7_backward otherwise. */
#define RWKV_NOALLOC_MAX_HEADS 240
int rwkv_wkv7_backward_noalloc(int dtype, const void* r, const void* w, const void* k,
                               const void* v, const void* a, const void* b, const float* h_in,
                               const float* h_ckpt, const void* dy, const float* dh_out, void* dr,
                               void* dw, void* dk, void* dv, void* da, void* db, float* dh_in,
                               int B, int T, int H, int N, rwkv_stream_t stream);

/* One-token decode step for `rows` independent rows: r..b, y [rows, H, N];
 * h [rows, H, N, N] fp32 updated in place.
 * Replaces wkv7StepForward (Sources/RWKVKernel/WKV7DecodeKernels.swift:73-89). */
int rwkv_wkv7_step(int dtype, const void* r, const void* w, const void* k, const void* v,
                   const void* a, const void* b, float* h, void* y, int rows, int H, int N,
                   rwkv_stream_t stream);

/* Fused tmix tail: per (row, head) GroupNorm (two-pass, eps) of wkv, plus the
 * bonus (sum r*k*r_k)*v, times the gate:
 *   out = ((norm(wkv)*ln_w + ln_b) + (sum r*k*r_k) * v) * g.
 * wkv, r, k, v, g, out: [rows, H*S] fp32; rk, ln_w, ln_b: [H*S] fp32.
 * Replaces wkvTail (Sources/RWKVKernel/WKV7DecodeKernels.swift:106-178). */
int rwkv_wkv_tail(const float* wkv, const float* r, const float* k, const float* v,
                  const float* rk, const float* ln_w, const float* ln_b, const float* g,
                  float* out, int rows, int H, int S, float eps, rwkv_stream_t stream);

/* The decode step and the tail in one launch (the pair of calls at
 * Sources/RWKVGen/X070Generation.swift:280-291): updates h, writes the tail
 * output [rows, H*N] fp32.  Inputs fp32. */
int rwkv_wkv7_step_tail(const float* r, const float* w, const float* k, const float* v,
                        const float* a, const float* b, float* h, const float* rk,
                        const float* ln_w, const float* ln_b, const float* g, float* out,
                        int rows, int H, int N, float eps, rwkv_stream_t stream);

/* ------------------------------------------- MLX affine container (QLoRA base)
 * wq: uint32 [OUT, IN*bits/32], each row an LSB-first bit stream of `bits`-bit
 * codes (Sources/RWKVQuant/RwkvqNative.swift:28-31,161-175); scales, biases:
 * [OUT, IN/group] in `sdtype` (F16, BF16 or F32); w = scale*q + bias.
 * bits in {2,3,4,5,6,8}; group in {32, 64, 128}; IN % group == 0.
 */

/* y[n, o] = sum_i x[n, i] * W[o, i]   (quantizedMM with transpose: true).
 * x: [rows, IN] in xdtype; y: [rows, OUT] in ydtype; accumulation in fp32.
 * fp16 x on the 4-bit group-64 container: 1-2 rows on the streaming CUDA-core
 * GEMV (IN % 128 == 0), 3-8 rows on the mma.sync GEMV -- both MLX's
 * matrix-vector numerics, scale * sum(q x) + bias * sum(x) per group --, more
 * rows on the tcgen05 GEMM over the weight dequantised into fp16 (MLX's
 * quantized-matmul numerics).
 * Replaces the quantizedMM call of X070Backbone.baseProj
 * (Sources/RWKVGen/X070Backbone.swift:678-681) and RwkvqNativeWeight
 * (Sources/RWKVQuant/RwkvqNative.swift:48-51). */
int rwkv_q_gemm(int xdtype, const void* x, const uint32_t* wq, const void* scales,
                const void* biases, int sdtype, int ydtype, void* y, int rows, int OUT, int IN,
                int group, int bits, rwkv_stream_t stream);

/* Wait errors of rwkv_q_gemm's tensor-core path (fp16 x, 4-bit group 64,
 * rows > 8).  Its pipeline waits are bounded in time; a wait that gives up
 * leaves that call's output invalid and records it per device.  The next
 * rwkv_q_gemm on that device returns RWKV_E_TIMEOUT, clears the record and
 * launches nothing (a launch still in flight may record it later).
 * rwkv_q_gemm_status synchronises `stream`, then returns RWKV_E_TIMEOUT (and
 * clears the record) if one is set, else RWKV_OK: a host that must know
 * whether the outputs it is about to use are valid calls it.  No counterpart
 * in the reference, whose Metal kernels have no bounded waits. */
int rwkv_q_gemm_status(rwkv_stream_t stream);
/* Sets the record as a wait that gives up would: the device flag, which makes
 * the next tensor-core launch skip its work, and with host_record != 0 also
 * the host record.  For testing a host's handling of RWKV_E_TIMEOUT without a
 * device fault.  No counterpart in the reference. */
int rwkv_q_gemm_inject_wait_error(int host_record, rwkv_stream_t stream);

/* Projection backward through a frozen base: the VJP X070Backbone gives a
 * base projection y = x W^T (baseMatmul, Sources/RWKVGen/X070Backbone.swift:
 * 337-356: matmul(cotangent.asType(bf16), weight(bf16)), a bf16 result cast
 * to the primal's type):
 *     dX[n, i] = bf16( sum_o dY[n, o] * Wb[o, i] )     (fp32 accumulation)
 * dY [rows, OUT] bf16 (the host casts the cotangent, as the reference does);
 * dX [rows, IN] in dx_dtype F32 / BF16 / F16 (the bf16-rounded sum, widened
 * or narrowed: F16 rounds twice, like the reference's asType); accumulate != 0
 * adds into an F32 dX (gradients of one input summed over its projections).
 * rwkv_gemm_dx: Wb a dense bf16 [OUT, IN] (a dense target, or a base
 * dequantised to bf16 by rwkv_q_dequant / rwkv_sb6_dequant / rwkv_sym_dequant
 * as the reference's rwkvqWeight does, X070Backbone.swift:669-672).
 * rwkv_q_gemm_dx: Wb = bf16(float(q) * scale + bias) of the MLX affine 4-bit
 * group-64 container (fp16 scales), dequantised inside the kernel; bitwise
 * the same as rwkv_q_dequant to bf16 followed by rwkv_gemm_dx.
 * IN % 128 == 0, OUT % 64 == 0, dY / W / wq 16-byte aligned.  tcgen05 tensor
 * cores; shares rwkv_q_gemm's wait-error record (rwkv_q_gemm_status).  The
 * reference's optional fp32 backward (rwkvqBackwardDType = .float32) is not
 * provided. */
int rwkv_gemm_dx(int dy_dtype, const void* dy, int w_dtype, const void* w, int dx_dtype, void* dx, int rows,
                 int OUT, int IN, int accumulate, rwkv_stream_t stream);
int rwkv_q_gemm_dx(int dy_dtype, const void* dy, const uint32_t* wq, const void* scales, const void* biases,
                   int sdtype, int dx_dtype, void* dx, int rows, int OUT, int IN, int group, int bits,
                   int accumulate, rwkv_stream_t stream);

/* Dense W [OUT, IN] in odtype: float(q)*float(scale) + float(bias), one
 * rounding.  Replaces MLX `dequantized` as used at
 * Sources/RWKVGen/X070Backbone.swift:759-766 and RwkvqModelTests. */
int rwkv_q_dequant(const uint32_t* wq, const void* scales, const void* biases, int sdtype,
                   int odtype, void* w_out, int OUT, int IN, int group, int bits,
                   rwkv_stream_t stream);

/* Embedding rows: out[n, :] = dequantised row ids[n] (int32, device), odtype.
 * Replaces X070Backbone.embed's quantised branch (X070Backbone.swift:758-767). */
int rwkv_q_rows(const int32_t* ids, int n_ids, const uint32_t* wq, const void* scales,
                const void* biases, int sdtype, int odtype, void* out, int vocab, int IN,
                int group, int bits, rwkv_stream_t stream);

/* Affine quantiser writing the MLX container from W [OUT, IN] (wdtype);
 * scales/biases written in wdtype (F16/BF16) or F32.  Replaces MLX `quantized`
 * at Sources/RWKVGen/LoRA.swift:68 (quantizeWeight / quantizeBaseModel). */
int rwkv_q_quantize(int wdtype, const void* W, uint32_t* wq, void* scales, void* biases,
                    int OUT, int IN, int group, int bits, rwkv_stream_t stream);

/* ------------------------------------------------------ .rwkvq sb6 (K3 layout)
 * qblk: uint8 [OUT, (IN/32)*(16+4*xbits)]; qsqm: uint8 [OUT, (IN/32)*2];
 * ddm: fp16 [OUT, (IN/256)*2]; superblock 8; xbits in {0,1,2}; IN % 256 == 0.
 */

/* Dense [OUT, IN] in odtype; combine in fp32, one rounding at store.
 * Replaces rwkvqDequantDense (Sources/RWKVQuant/RwkvqDequant.swift:160-183). */
int rwkv_sb6_dequant(const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm, int odtype,
                     void* out, int OUT, int IN, int xbits, rwkv_stream_t stream);

/* y [rows, OUT] fp32 = x [rows, IN] (xdtype) times W^T.  The reference takes
 * one row; any rows >= 1 here.
 * Replaces rwkvqSb6GEMV / RwkvqSidecar.sb6GEMV
 * (Sources/RWKVQuant/RwkvqSb6GEMV.swift:170-208). */
int rwkv_sb6_gemv(int xdtype, const void* x, const uint8_t* qblk, const uint8_t* qsqm,
                  const uint16_t* ddm, float* y, int rows, int OUT, int IN, int xbits,
                  rwkv_stream_t stream);

/* Lossless relayout into the MLX affine container (group 32, bits 4+xbits):
 * wq [OUT, (IN/32)*bits] u32, scales/biases [OUT, IN/32] fp32 (scale clamped
 * at 1e-8).  *fp16_ok_host (host int, written after a stream sync) is 1 when
 * fp16 scales/biases would change no weight.
 * Replaces RwkvqSidecar.nativeAffine (Sources/RWKVQuant/RwkvqNative.swift:78-196). */
int rwkv_sb6_to_affine(const uint8_t* qblk, const uint8_t* qsqm, const uint16_t* ddm,
                       uint32_t* wq, float* scales, float* biases, int* fp16_ok_host, int OUT,
                       int IN, int xbits, rwkv_stream_t stream);

/* --------------------------------------------------- .rwkvq sym (6 / 8 bit)
 * qblk: 8-bit: int8 codes [OUT, IN]; 6-bit: [OUT, (IN/32)*24] (pairs of
 * 16-blocks: 16 nibble bytes + 2 bit-planes, codes stored +32);
 * qs: int8 [OUT, IN/16]; d: fp16 [OUT, ceil(IN/256)].
 */

/* Dense [OUT, IN]: F32 and BF16 multiply in float, F16 multiplies in half.
 * Replaces rwkvqDequantSym (Sources/RWKVQuant/RwkvqDequant.swift:409-431). */
int rwkv_sym_dequant(const uint8_t* qblk, const uint8_t* qs, const uint16_t* d, int odtype,
                     void* out, int OUT, int IN, int bits, rwkv_stream_t stream);

/* y [nn, OUT] fp32.  K = OUT/out_per matrices share one launch; matrix j
 * (rows j*out_per ..) reads input row n*K + j of x [nn*K, IN].  out_per = OUT
 * is a plain GEMV over nn input rows.  IN % 256 == 0, out_per % 4 == 0.
 * Replaces rwkvqSymGEMV and symGEMVFused
 * (Sources/RWKVQuant/RwkvqSymGEMV.swift:223-247, :343-358). */
int rwkv_sym_gemv(int xdtype, const void* x, const uint8_t* qblk, const uint8_t* qs,
                  const uint16_t* d, float* y, int nn, int OUT, int IN, int bits, int out_per,
                  rwkv_stream_t stream);

/* Embedding rows of an 8-bit sym table, fp16 out [n_ids, IN]:
 * out = half(code * half(qs*d)).  Replaces RwkvqSymRowTable.rows
 * (Sources/RWKVQuant/RwkvqSymRows.swift:26-78). */
int rwkv_sym_rows(const int32_t* ids, int n_ids, const uint8_t* codes, const uint8_t* qs,
                  const uint16_t* d, uint16_t* out, int vocab, int IN, rwkv_stream_t stream);


/* --------------------------------------------- x070 recurrent decode runtime
 * The host side of X070Backbone's decode over the kernels above, for a 4-bit
 * group-64 QLoRA base or a dense bf16 base: embedding -> per layer (ln1, token shift, r/k/v
 * GEMVs, low-rank w/a/v/g branches, WKV step + tail, o GEMV, ln2, cmix
 * key/value GEMVs) -> ln_out -> head GEMV -> greedy argmax.  Each row of a
 * batch carries its own state; one step is captured into a CUDA graph per
 * row count and replayed.  Replaces X070Backbone.step / stepEager
 * (Sources/RWKVGen/X070Generation.swift:449-498), generate
 * (Sources/RWKVGen/Generate.swift:112-202) and generateBatch's step loop
 * (Sources/RWKVGen/BatchGenerate.swift:54-116), greedy sampling
 * (Sources/RWKVGen/GPUSampler.swift:90).
 */
typedef struct rwkv_x070* rwkv_x070_t;

typedef struct {
    int n_layer, n_embd, head_size, vocab, ffn; /* X070Config (X070Backbone.swift:24-37) */
    int rank_w, rank_a, rank_v, rank_g;         /* low-rank sizes (X070Init.swift:46-52) */
    int quant_bits, quant_group;                /* 4, 64 (LoRA.swift:28-91); or 0: dense bf16 base */
    /* 4-bit base: RWKV_F16 (fp16 activations, tensor-core GEMMs) or RWKV_F32;
     * dense bf16 base: RWKV_BF16 (bf16 activations, tensor-core GEMMs) or
     * RWKV_F32.  Other pairings return RWKV_E_DTYPE: a tensor-core product
     * takes both operands in one type. */
    int act_dtype;
    int max_rows;   /* rows (batch) the state and workspace are sized for */
} rwkv_x070_config;

int rwkv_x070_create(const rwkv_x070_config* cfg, rwkv_x070_t* out);
int rwkv_x070_destroy(rwkv_x070_t model);
/* Parameter by its reference name ("emb.weight", "blocks.3.tmix.r_proj.weight",
 * ...), from a HOST fp32 array of n elements; the big matrices are quantised
 * on the device (rwkv_q_quantize), the low-rank matrices stored fp16.
 * LoRA adapters (Sources/RWKVGen/LoRA.swift:118-127, applied as in
 * X070Backbone.proj, X070Backbone.swift:746-752: base + scale (x A^T) B^T) use
 * the reference's keys "<target>.lora_a" [rank, IN] and "<target>.lora_b"
 * [OUT, rank], plus "<target>.lora_scale" [1] (alpha / rank), for target
 * "blocks.L.tmix.{r,k,v,o}_proj", "blocks.L.cmix.{key,value}" or "head";
 * rank a multiple of 16, at most 256; stored fp16.  Changing an adapter drops
 * the captured step graphs. */
int rwkv_x070_set_param(rwkv_x070_t model, const char* name, const float* host, int64_t n);
/* A projection or head matrix (set_param's names "blocks.L.tmix.{r,k,v,o}_proj.weight",
 * "blocks.L.cmix.{key,value}.weight", "head.weight") from .rwkvq buffers
 * in the loader's layout, HOST memory, used as stored (no requantisation):
 * kind 1 = sb6 (bits = xbits 0..2; b1 = qblk [OUT, IN/32 * (16 + 4 xbits)],
 * b2 = qsqm [OUT, IN/32 * 2], b3 = ddm [OUT, IN/256] fp16 pairs); kind 2 =
 * sym (bits 6 or 8; b1 = qblk, b2 = qs [OUT, IN/16] int8, b3 = d [OUT,
 * IN/256] fp16); n1..n3 their byte counts; IN % 256 == 0.  The step then
 * runs that matrix through rwkv_sb6_gemv / rwkv_sym_gemv's kernels (at most 4
 * activation rows per launch) with the projection's epilogue, as the
 * reference's decode takes rwkvqSb6GEMV / rwkvqSymGEMV for sidecar matrices
 * (X070Backbone.swift:708-732).  set_param with fp32 values returns the
 * matrix to the model's own base container.  Steps with such matrices take
 * the per-kernel path. */
int rwkv_x070_set_param_rwkvq(rwkv_x070_t model, const char* name, int kind, int bits, const void* b1, int64_t n1,
                              const void* b2, int64_t n2, const void* b3, int64_t n3);
/* Random init with the x070 recipe (Sources/RWKVGen/Training/X070Init.swift:79-206),
 * drawn on the device from `seed`. */
int rwkv_x070_init_random(rwkv_x070_t model, uint64_t seed);
/* Zero the state of rows 0..rows-1 (RWKVState(cfg:), X070Generation.swift:34-41). */
int rwkv_x070_reset_state(rwkv_x070_t model, int rows, rwkv_stream_t stream);
/* One token per row.  ids: device int32 [rows] (NULL = the previous step's
 * argmax, kept on the device); logits: device fp32 [rows, vocab] or NULL;
 * next_ids: device int32 [rows] or NULL.  use_graph != 0 replays the
 * captured step (the stream must not be the legacy default stream during
 * the first, capturing call). */
int rwkv_x070_step(rwkv_x070_t model, const int32_t* ids, int rows, float* logits,
                   int32_t* next_ids, int use_graph, rwkv_stream_t stream);
/* Parallel prefill of right-padded prompts: ids device int32 [rows, T];
 * lengths_host HOST int32 [rows], each in 1..T (NULL = all T; positions past
 * a row's length are padding).  Runs whole blocks of positions per launch
 * (sequence-mode glue, the projections as tensor-core GEMMs over every token
 * of the block, the chunked WKV-7 forward), masking padding so that w = 1,
 * k = 0, b = 0 there -- the state of a row stops at its last real token --
 * and takes each row's token-shift state at that token.  Continues from the
 * rows' current state (reset first for a fresh start).  logits: device fp32
 * [rows, vocab] of each row's last real token, or NULL; next_ids: device
 * int32 [rows] (their argmax) or NULL; the argmax is also kept as the next
 * step's input (rwkv_x070_step with ids = NULL).  Block buffers are
 * allocated on first use and kept by the model.
 * Replaces prefill / prefillBatch over bodyWithState (Sources/RWKVGen/
 * X070Generation.swift:344-355, BatchGenerate.swift:36-51,
 * X070Backbone.swift:1011-1048; padding mask RWKVBlock.swift:221-237,
 * lastRealIndex RWKVBatchState.swift:159-175). */
int rwkv_x070_prefill(rwkv_x070_t model, const int32_t* ids, const int32_t* lengths_host, int rows, int T,
                      float* logits, int32_t* next_ids, rwkv_stream_t stream);
/* Greedy generation with HOST buffers: prompts [rows, prompt_len] prefilled
 * in parallel (rwkv_x070_prefill), then n_new tokens per row into out
 * [rows, n_new].  Continues from the rows' current state. */
int rwkv_x070_generate(rwkv_x070_t model, const int32_t* prompt_host, int rows, int prompt_len,
                       int n_new, int32_t* out_host, rwkv_stream_t stream);
/* generateBatch with ragged prompts and stop tokens, HOST buffers: prompts
 * [rows, max_len] right-padded, lengths_host [rows] (NULL = all max_len);
 * rows start from a zero state; greedy; a row stops after emitting one of
 * the n_stop ids in stop_host (the stop id is kept) or after n_new tokens,
 * and a stopped row leaves the batch (its state rows are compacted away, so
 * later steps run on the live rows only).  out_host [rows, n_new] receives
 * each row's tokens, out_len_host [rows] their counts.
 * Replaces X070Backbone.generateBatch (Sources/RWKVGen/BatchGenerate.swift:
 * 69-116) with the argmax sampler. */
int rwkv_x070_generate_batch(rwkv_x070_t model, const int32_t* prompts_host, const int32_t* lengths_host,
                             int rows, int max_len, int n_new, const int32_t* stop_host, int n_stop,
                             int32_t* out_host, int32_t* out_len_host, rwkv_stream_t stream);
/* Wait errors of the model's tensor-core GEMMs (bounded pipeline waits; see
 * rwkv_q_gemm_status): a step after one gave up returns RWKV_E_TIMEOUT,
 * clears the record and launches nothing; rwkv_x070_generate checks it at
 * the end too.  rwkv_x070_status synchronises `stream` and reports (and
 * clears) the record: RWKV_E_TIMEOUT means the state and outputs since the
 * last report are not valid.  rwkv_x070_inject_wait_error sets it as a wait
 * that gives up would (the device flag; with host_record also the host
 * record), for testing a host's error handling without a device fault.  No
 * counterpart in the reference. */
int rwkv_x070_status(rwkv_x070_t model, rwkv_stream_t stream);
int rwkv_x070_inject_wait_error(rwkv_x070_t model, int host_record, rwkv_stream_t stream);
/* Step profiler (tracing): one eager step with a CUDA event after every
 * launch; writes per-launch device milliseconds to ms_host[0..*count) and the
 * launch names, '\n'-separated, to names_host.  Advances the state like a step.
 * Stands in for DecodeBench's --step-profile (Sources/DecodeBench/main.swift:146-196). */
int rwkv_x070_profile_step(rwkv_x070_t model, int rows, float* ms_host, int cap, char* names_host,
                           int names_cap, int* count, rwkv_stream_t stream);
/* How a decode step runs.  path 0 (the default): the per-kernel sequence
 * captured in a CUDA graph.  path 1: for 1..64 rows with fp16 activations on
 * the 4-bit base and no LoRA adapters, the whole step is ONE cooperative
 * launch of a persistent kernel (one CTA per SM, phases separated by grid
 * barriers, weights streamed ahead of their phase): 1..8 rows on exact-code
 * mma.sync GEMVs, 9..64 rows on the tcgen05 GEMM; other steps keep the graph.
 * The arithmetic is the per-kernel path's for the row count (the exact
 * dequantised weight up to 8 rows, the fp16-dequantised weight above); sums
 * are grouped differently.  On the 1.5B step the persistent kernels are the
 * slower (1 row 1.48 vs 0.89 ms, 8 rows 1.87 vs 1.52 ms, 64 rows 2.70 vs
 * 2.11 ms), hence the default.  rwkv_x070_decode_path returns 1 when a step
 * on `rows` rows takes the persistent kernel.  No counterpart in the reference (MLX schedules the
 * reference's kernels). */
int rwkv_x070_set_decode_path(rwkv_x070_t model, int path);
/* The raw %globaltimer trace of the last rwkv_x070_profile_step that ran the
 * persistent kernel (CTA 0: phase boundaries at [0, 1024); per pipeline stage
 * j < 2048: weight copy issued [1024 + j], activation copy issued
 * [3072 + j], MMA inputs ready [5120 + j], dequantised [7168 + j]; 0 where
 * nothing was recorded), up to cap entries into out_host. */
int rwkv_x070_trace(rwkv_x070_t model, uint64_t* out_host, int cap, int* count);
int rwkv_x070_decode_path(rwkv_x070_t model, int rows);
int64_t rwkv_x070_weight_bytes(rwkv_x070_t model);
int rwkv_x070_launches_per_step(rwkv_x070_t model);

/* ------------------------------------------------ state tuning (WKV path)
 * The trainable initial WKV state of a layer, [H, N, N] fp32, shared by every
 * sequence of the batch (StateTrainableSet, Sources/RWKVGen/InitialState.swift:
 * 176-251).  N must be 64; pointers 16-byte aligned. */

/* h[b] = state for b < B: the forward's h_in [B, H, N, N] (the state broadcast
 * of InitialLayerState.broadcast, InitialState.swift:59-73). */
int rwkv_state_broadcast(const float* state, float* h, int B, int H, int N, rwkv_stream_t stream);
/* grad (+)= sum over b of dh_in[b], b = 0..B-1 in order (deterministic); the
 * gradient of the shared state from the backward's dh_in.  accumulate = 0
 * overwrites grad. */
int rwkv_state_grad_sum(const float* dh_in, float* grad, int B, int H, int N, int accumulate,
                        rwkv_stream_t stream);
/* Workspace bytes rwkv_adamw_clip_step needs for n parameters. */
int64_t rwkv_adamw_workspace_size(int64_t n);
/* One optimizer step of Trainer.run (Sources/RWKVGen/Training/Trainer.swift:
 * 141-161) over n fp32 parameters, in its order: g = grad * grad_scale (the
 * average: 1/gradAccum, or 1/world after a data-parallel sum); global-norm
 * clip g *= min(1, clip / (||g|| + 1e-6)) when clip > 0 (clipByGlobalNorm,
 * :182-189); m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2; upd = (m/c1) /
 * (sqrt(v/c2) + eps) [+ weight_decay * p]; p -= lr * upd.  c1 = 1 - b1^t and
 * c2 = 1 - b2^t come from the host's step count t.  Every operation rounds to
 * fp32 (no fused multiply-add); the norm's sum of squares is taken in double
 * in a fixed order.  ||g|| (before clipping) goes to *norm_out (device, may be
 * NULL).  Nothing returns to the host. */
int rwkv_adamw_clip_step(float* param, float* m, float* v, const float* grad, int64_t n,
                         float grad_scale, float clip, float lr, float beta1, float beta2, float eps,
                         float weight_decay, float bias_c1, float bias_c2, float* norm_out,
                         void* workspace, int64_t workspace_bytes, rwkv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RWKV_CUDA_H */
