// x070 (RWKV-7 "Goose") recurrent decode runtime over the hot-path kernels:
// the host side of X070Backbone.step / generate / generateBatch for a 4-bit
// QLoRA base (Sources/RWKVGen/X070Generation.swift:449-498,
// BatchGenerate.swift:54-116), in C++.
//
// Weights live on the device: the big matrices (r/k/v/o projections, cmix
// key/value, head, embedding) in the MLX affine container (4-bit, group 64,
// fp16 scale/bias), the low-rank branches in fp16, vectors in fp32.  Every
// row has its own state: WKV [L, rows, H, 64, 64] fp32 and the two token-shift
// rows per layer.  One decode step is a fixed sequence of launches on one
// stream; it is captured once per row count into a CUDA graph and replayed.
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemm_w4_wide.cuh"
#include "gemv_stream.cuh"
#include "x070_kernels.cuh"
#include "x070_persist.cuh"
#include "x070_small.cuh"

namespace rwkv {
int launch_rwkvq_jobs(int xdtype, const GemvJobs& jobs, int nj, int R, cudaStream_t st);
}

namespace rwkv {

int launch_q_quantize(int, const void*, uint32_t*, void*, void*, int, int, int, int, cudaStream_t);
int64_t wkv7_chunk_workspace(int, int, int);
int launch_wkv7_chunk_fwd(int, const void*, const void*, const void*, const void*, const void*, const void*,
                          const float*, void*, float*, float*, float*, int, int, int, void*, cudaStream_t);

// Prefill processes the prompts in blocks of Ts positions of every row, with
// rows * Ts <= PF_TOKENS token rows per block (Ts a multiple of 16), so its
// buffers stay bounded whatever the prompt length.
constexpr int PF_TOKENS = 8192;

// weight formats of the runtime's matrices
enum : int { WF_Q4 = 0, WF_F16 = 1, WF_BF16 = 2 };

// -------------------------------------------------------- device init helpers

__device__ __forceinline__ uint64_t splitmix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// mode 0: uniform(lo, hi); mode 1: normal(0, lo); counter-based, seeded.
template <typename T>
__global__ void fill_kernel(T* out, int64_t n, int mode, float lo, float hi, uint64_t seed) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t z = splitmix(seed ^ splitmix((uint64_t)i));
        const float u1 = ((z >> 40) + 0.5f) * (1.0f / 16777216.0f);
        float v;
        if (mode == 0) {
            v = lo + (hi - lo) * u1;
        } else {
            const float u2 = (((z >> 16) & 0xFFFFFF) + 0.5f) * (1.0f / 16777216.0f);
            v = lo * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        }
        out[i] = from_f<T>(v);
    }
}

template <typename T>
__global__ void f32_to_kernel(const float* in, T* out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = from_f<T>(in[i]);
}

// ------------------------------------------------------------------- model

// A base matrix: the MLX 4-bit group-64 container, or dense bf16 (`dense`).
struct QMat {
    uint32_t* wq = nullptr;
    __half* sc = nullptr;
    __half* bi = nullptr;
    __nv_bfloat16* dense = nullptr;
    __half2* sbr = nullptr;  // (scale, bias) repacked per 128-row block and 256-code stage (persistent step)
    __half* sbs = nullptr;   // (scale, bias) blocks per 16-row tile and 2048-code piece (1..8-row persistent step)
    // set: the matrix is a .rwkvq sb6 / sym matrix (WFMT_SB6 / WFMT_SYM, qbits
    // = xbits / bits) used as stored: qblk, q2 = qsqm / qs, qd = ddm / d
    int fmt = WFMT_AFFINE, qbits = 0;
    uint8_t* qblk = nullptr;
    uint8_t* q2 = nullptr;
    __half* qd = nullptr;
    int OUT = 0, IN = 0;
};

// (scale, bias) pairs of an MLX 4-bit group-64 matrix, repacked for the
// persistent step's 1-D bulk copies: out[((mb * S + st) * 128 + r) * 4 + j] =
// (scale, bias) of row mb * 128 + r, group 4 st + j  (S = IN / 256).
__global__ void x070_repack_sb_kernel(const __half* __restrict__ sc, const __half* __restrict__ bi,
                                      __half2* __restrict__ out, int OUT, int IN) {
    const int NG = IN / 64, S = IN / 256;
    const int64_t n = (int64_t)OUT * NG;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int o = (int)(i / NG), gi = (int)(i % NG);
        const int mb = o / 128, r = o % 128, st = gi / 4, j = gi % 4;
        out[(((int64_t)mb * S + st) * 128 + r) * 4 + j] = __halves2half2(sc[i], bi[i]);
    }
}

// A LoRA adapter on a projection (LoRA.swift:118-127, X070Backbone.swift:
// 746-752): y = base(x) + scale * (x A^T) B^T with A [rank, IN], B [OUT, rank]
// stored in fp16; active once A and B are both set with the same rank.
struct Adapter {
    __half* A = nullptr;
    __half* B = nullptr;
    int rank_a = 0, rank_b = 0;
    float scale = 1.f;
    bool on() const { return A && B && rank_a == rank_b; }
};
constexpr int LORA_MAX_RANK = 256;
enum { AD_R, AD_K, AD_V, AD_O, AD_KEY, AD_VALUE, AD_N };

struct LayerW {
    float *ln1w = nullptr, *ln1b = nullptr, *ln2w = nullptr, *ln2b = nullptr;
    float* coef6 = nullptr;  // [6, C]: r, w, k, v, a, g
    float *kkw = nullptr, *kaw = nullptr, *rkw = nullptr, *lnxw = nullptr, *lnxb = nullptr;
    float* cxk = nullptr;
    float *wbias = nullptr, *abias = nullptr, *vbias = nullptr;
    __half *wA = nullptr, *wB = nullptr, *aA = nullptr, *aB = nullptr;
    __half *gA = nullptr, *gB = nullptr, *vA = nullptr, *vB = nullptr;
    QMat r, k, v, o, key, value;
    Adapter ad[AD_N];   // LoRA on r, k, v, o (tmix) and key, value (cmix)
};

struct X070 {
    rwkv_x070_config cfg{};
    int L, C, H, V, F, Rmax;
    int rw, ra, rv, rg, hid;  // low-rank sizes and hidden width
    bool f16act;   // 16-bit activations (fp16 or bf16): the tensor-core GEMM path
    bool bf16act;  // bf16 activations (with the dense bf16 base)
    bool dense;    // dense bf16 base instead of the 4-bit container
    int base_wf, lr_wf;  // weight formats (WF_*) of the base and the low-rank / adapter matrices
    std::vector<void*> allocs;
    std::vector<LayerW> lw;
    QMat emb, head;
    Adapter head_ad;             // LoRA on the head
    void* lora_z = nullptr;      // [3][Rmax][LORA_MAX_RANK] adapter down outputs (activation type)
    float* key_tmp = nullptr;    // [Rmax, F] cmix key pre-activation when it has an adapter
    float *ln0w, *ln0b, *lnow, *lnob;
    // state
    float *wkv, *tshift, *cshift;
    // workspace
    float *x, *r, *k, *v, *wdec, *a, *vv, *g, *vfirst, *logits;
    void *mix, *hidden, *tail, *xk, *ffn, *lnout;
    int32_t* ids;
    unsigned long long* amax_keys;
    size_t act_bytes;
    std::map<int, cudaGraphExec_t> graphs;
    int64_t weight_bytes = 0;
    int64_t wver = 0;  // bumped by every weight change (the persistent step's repacked scales follow it)
    // A capture cannot run on the legacy default stream: graph work requested
    // there is forwarded to this stream, ordered by events on both sides.
    cudaStream_t own = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    // The low-rank branches (down + up) of a layer run on `side`, beside the
    // r/k/v GEMM, when both take the tensor-core path (which keeps no shared
    // workspace): fork after tmix_in, join before the WKV step.
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    // split-K partials and tickets of the tensor-core GEMMs
    float* gws = nullptr;
    int* gtickets = nullptr;
    float* gws_side = nullptr;   // the same for launches on `side` (the low-rank branch)
    int* gtickets_side = nullptr;
    int* gerr = nullptr;  // set by a tensor-core GEMM wait that gave up
    TcWaitFlag gflag;     // gerr and its mapped host record
    size_t gws_floats = 0, gtickets_n = 0;
    int sm_count = 148;
    // step profiler: an event node after every launch of a captured step
    bool profiling = false;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<std::string> prof_names;
    cudaStream_t prof_stream = nullptr;
    void mark(const char* name) {
        if (!profiling) return;
        if (prof_names.size() >= prof_ev.size()) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            prof_ev.push_back(e);
        }
        cudaEventRecordWithFlags(prof_ev[prof_names.size()], prof_stream, cudaEventRecordExternal);
        prof_names.push_back(name);
    }

    bool alloc_failed = false;

    // Device allocation owned by the model (freed by the destructor); a
    // failure is recorded and reported by rwkv_x070_create.
    template <typename T>
    T* alloc(size_t n, bool zero = true) {
        void* p = nullptr;
        if (n == 0) n = 1;
        if (alloc_failed || cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
            alloc_failed = true;
            return nullptr;
        }
        if (zero) cudaMemset(p, 0, n * sizeof(T));
        allocs.push_back(p);
        return (T*)p;
    }
    QMat qmat(int OUT, int IN) {
        QMat q;
        q.OUT = OUT;
        q.IN = IN;
        if (dense) {
            q.dense = alloc<__nv_bfloat16>((size_t)OUT * IN);
            weight_bytes += (int64_t)OUT * IN * 2;
            return q;
        }
        q.wq = alloc<uint32_t>((size_t)OUT * IN / 8);
        q.sc = alloc<__half>((size_t)OUT * IN / 64);
        q.bi = alloc<__half>((size_t)OUT * IN / 64);
        weight_bytes += (int64_t)OUT * IN / 2 + (int64_t)OUT * IN / 64 * 4;
        return q;
    }
    __half* hmat(size_t n) {
        weight_bytes += (int64_t)n * 2;
        return alloc<__half>(n);
    }

    explicit X070(const rwkv_x070_config& c) : cfg(c) {
        L = c.n_layer; C = c.n_embd; H = C / c.head_size; V = c.vocab; F = c.ffn; Rmax = c.max_rows;
        rw = c.rank_w; ra = c.rank_a; rv = c.rank_v; rg = c.rank_g;
        hid = rw + ra + rv + rg;
        f16act = c.act_dtype == RWKV_F16 || c.act_dtype == RWKV_BF16;
        bf16act = c.act_dtype == RWKV_BF16;
        dense = c.quant_bits == 0;
        base_wf = dense ? WF_BF16 : WF_Q4;
        lr_wf = bf16act || (dense && !f16act) ? WF_BF16 : WF_F16;
        act_bytes = f16act ? 2 : 4;
        emb = qmat(V, C);
        head = qmat(V, C);
        ln0w = alloc<float>(C); ln0b = alloc<float>(C); lnow = alloc<float>(C); lnob = alloc<float>(C);
        lw.resize(L);
        for (int l = 0; l < L; l++) {
            LayerW& w = lw[l];
            w.ln1w = alloc<float>(C); w.ln1b = alloc<float>(C); w.ln2w = alloc<float>(C); w.ln2b = alloc<float>(C);
            w.coef6 = alloc<float>(6 * (size_t)C);
            w.kkw = alloc<float>(C); w.kaw = alloc<float>(C); w.rkw = alloc<float>(C);
            w.lnxw = alloc<float>(C); w.lnxb = alloc<float>(C); w.cxk = alloc<float>(C);
            w.wbias = alloc<float>(C); w.abias = alloc<float>(C); w.vbias = alloc<float>(C);
            w.wA = hmat((size_t)rw * C); w.wB = hmat((size_t)C * rw);
            w.aA = hmat((size_t)ra * C); w.aB = hmat((size_t)C * ra);
            w.gA = hmat((size_t)rg * C); w.gB = hmat((size_t)C * rg);
            if (l > 0) { w.vA = hmat((size_t)rv * C); w.vB = hmat((size_t)C * rv); }
            w.r = qmat(C, C); w.k = qmat(C, C); w.v = qmat(C, C); w.o = qmat(C, C);
            w.key = qmat(F, C); w.value = qmat(C, F);
            weight_bytes += (int64_t)C * 4 * 20;
        }
        const size_t RC = (size_t)Rmax * C;
        wkv = alloc<float>((size_t)L * Rmax * H * 64 * 64);
        tshift = alloc<float>((size_t)L * RC);
        cshift = alloc<float>((size_t)L * RC);
        x = alloc<float>(RC); r = alloc<float>(RC); k = alloc<float>(RC); v = alloc<float>(RC);
        wdec = alloc<float>(RC); a = alloc<float>(RC); vv = alloc<float>(RC); g = alloc<float>(RC);
        vfirst = alloc<float>(RC);
        logits = alloc<float>((size_t)Rmax * V);
        mix = alloc<char>(6 * RC * act_bytes);
        hidden = alloc<char>((size_t)Rmax * hid * act_bytes);
        tail = alloc<char>(RC * act_bytes);
        xk = alloc<char>(RC * act_bytes);
        ffn = alloc<char>((size_t)Rmax * F * act_bytes);
        lnout = alloc<char>(RC * act_bytes);
        ids = alloc<int32_t>(Rmax);
        amax_keys = alloc<unsigned long long>(Rmax);
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
        // split-K never exceeds ~2 waves of 64 x 64 tiles: (2*SMs + tiles) * 4096 floats
        gws_floats = (size_t)(4 * sm_count + 64) * GW_BM * 64;
        gtickets_n = 8192;
        gws = alloc<float>(gws_floats);
        gtickets = alloc<int>(gtickets_n + 1);
        gerr = gtickets + gtickets_n;
        gws_side = alloc<float>(gws_floats);
        gtickets_side = alloc<int>(gtickets_n);
        if (!alloc_failed && !gflag.init(gerr)) alloc_failed = true;
        cudaStreamCreateWithFlags(&own, cudaStreamNonBlocking);
        cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming);
        cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming);
        cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking);
        cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming);
        cudaEventCreateWithFlags(&ev_join, cudaEventDisableTiming);
    }

    ~X070() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        for (cudaEvent_t e : prof_ev) cudaEventDestroy(e);
        for (void* p : allocs) cudaFree(p);
        for (void* p : pk_allocs) cudaFree(p);
        auto free_q = [](QMat& q) {
            if (q.qblk) cudaFree(q.qblk);
            if (q.q2) cudaFree(q.q2);
            if (q.qd) cudaFree(q.qd);
        };
        free_q(head);
        for (LayerW& w : lw) {
            free_q(w.r); free_q(w.k); free_q(w.v); free_q(w.o); free_q(w.key); free_q(w.value);
        }
        pf_free();
        if (pf_prompt) cudaFree(pf_prompt);
        gflag.release();
        if (own) cudaStreamDestroy(own);
        if (ev_in) cudaEventDestroy(ev_in);
        if (ev_out) cudaEventDestroy(ev_out);
        if (side) cudaStreamDestroy(side);
        if (ev_fork) cudaEventDestroy(ev_fork);
        if (ev_join) cudaEventDestroy(ev_join);
    }

    // ----- parameters

    int upload_q(QMat& q, const float* host, int64_t n) {
        RWKV_REQUIRE(n == (int64_t)q.OUT * q.IN, RWKV_E_SHAPE, "matrix size %lld, expected %d x %d",
                     (long long)n, q.OUT, q.IN);
        if (q.fmt != WFMT_AFFINE) {  // back to the model's own container: the launch sequence changes
            q.fmt = WFMT_AFFINE;
            drop_graphs();
        }
        if (dense) {
            float* t32 = nullptr;
            if (cudaMalloc(&t32, n * 4) != cudaSuccess) return fail(RWKV_E_CUDA, "set_param: staging allocation failed");
            cudaMemcpy(t32, host, n * 4, cudaMemcpyHostToDevice);
            f32_to_kernel<__nv_bfloat16><<<1024, 256>>>(t32, q.dense, n);
            cudaDeviceSynchronize();
            cudaFree(t32);
            return check_launch("f32_to_kernel");
        }
        float* tmp = nullptr;
        __half* h16 = nullptr;
        if (cudaMalloc(&tmp, n * 4) != cudaSuccess || cudaMalloc(&h16, n * 2) != cudaSuccess)
            return fail(RWKV_E_CUDA, "set_param: staging allocation failed");
        cudaMemcpy(tmp, host, n * 4, cudaMemcpyHostToDevice);
        f32_to_kernel<__half><<<1024, 256>>>(tmp, h16, n);
        int rc = launch_q_quantize(RWKV_F16, h16, q.wq, q.sc, q.bi, q.OUT, q.IN, 64, 4, 0);
        cudaDeviceSynchronize();
        cudaFree(tmp);
        cudaFree(h16);
        return rc;
    }
    int upload_h(__half* dst, int64_t expect, const float* host, int64_t n) {
        RWKV_REQUIRE(dst != nullptr, RWKV_E_SHAPE, "set_param: this layer has no such matrix");
        RWKV_REQUIRE(n == expect, RWKV_E_SHAPE, "matrix size %lld, expected %lld", (long long)n, (long long)expect);
        float* tmp = nullptr;
        if (cudaMalloc(&tmp, n * 4) != cudaSuccess) return fail(RWKV_E_CUDA, "set_param: staging allocation failed");
        cudaMemcpy(tmp, host, n * 4, cudaMemcpyHostToDevice);
        // 16-bit storage in the low-rank format: fp16, or bf16 beside bf16 activations
        if (lr_wf == WF_BF16) f32_to_kernel<__nv_bfloat16><<<1024, 256>>>(tmp, (__nv_bfloat16*)dst, n);
        else f32_to_kernel<__half><<<1024, 256>>>(tmp, dst, n);
        cudaDeviceSynchronize();
        cudaFree(tmp);
        return check_launch("f32_to_kernel");
    }
    int upload_f(float* dst, int64_t expect, const float* host, int64_t n) {
        RWKV_REQUIRE(n == expect, RWKV_E_SHAPE, "vector size %lld, expected %lld", (long long)n, (long long)expect);
        return cudaMemcpy(dst, host, n * 4, cudaMemcpyHostToDevice) == cudaSuccess
                   ? ok() : fail(RWKV_E_CUDA, "set_param: copy failed");
    }

    void drop_graphs() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
    }
    // "<target>.lora_a" [rank, IN], ".lora_b" [OUT, rank], ".lora_scale" [1]
    // (the reference's adapter keys, LoRA.swift:170-200; scale = alpha / rank).
    // A change invalidates the captured step graphs (the launch sequence changes).
    int set_adapter(Adapter& a, const std::string& part, int IN, int OUT, bool key, const float* host, int64_t n) {
        if (part == "scale") {
            RWKV_REQUIRE(n == 1, RWKV_E_SHAPE, "set_param: lora_scale takes one value, got %lld", (long long)n);
            a.scale = host[0];
            drop_graphs();
            return ok();
        }
        const bool isA = part == "a";
        RWKV_REQUIRE(isA || part == "b", RWKV_E_SHAPE, "set_param: unknown adapter tensor 'lora_%s'", part.c_str());
        const int64_t dim = isA ? IN : OUT;
        RWKV_REQUIRE(n > 0 && n % dim == 0, RWKV_E_SHAPE, "set_param: lora_%s size %lld is not rank x %lld",
                     part.c_str(), (long long)n, (long long)dim);
        const int rank = (int)(n / dim);
        RWKV_REQUIRE(rank % 16 == 0 && rank <= LORA_MAX_RANK, RWKV_E_UNSUPPORTED,
                     "set_param: adapter rank %d must be a multiple of 16, at most %d", rank, LORA_MAX_RANK);
        __half*& dst = isA ? a.A : a.B;
        int& rk = isA ? a.rank_a : a.rank_b;
        if (!dst || rk != rank) {
            dst = alloc<__half>((size_t)rank * dim);
            weight_bytes += (int64_t)rank * dim * 2;
        }
        rk = rank;
        if (!lora_z) lora_z = alloc<char>((size_t)3 * Rmax * LORA_MAX_RANK * act_bytes);
        if (key && !key_tmp) key_tmp = alloc<float>((size_t)Rmax * F);
        RWKV_REQUIRE(!alloc_failed && dst && lora_z && (!key || key_tmp), RWKV_E_CUDA, "set_param: adapter allocation failed");
        drop_graphs();
        return upload_h(dst, n, host, n);
    }

    // The base matrix `name` (set_param's names of the projection / head
    // matrices) from .rwkvq buffers used as stored: kind WFMT_SB6 (bits =
    // xbits 0..2; b1 = qblk, b2 = qsqm, b3 = ddm) or WFMT_SYM (bits 6 or 8;
    // b1 = qblk, b2 = qs, b3 = d).
    int set_param_rwkvq(const std::string& name, int kind, int bits, const void* b1, int64_t n1, const void* b2,
                        int64_t n2, const void* b3, int64_t n3) {
        QMat* q = nullptr;
        if (name == "head.weight") q = &head;
        else if (name.compare(0, 7, "blocks.") == 0) {
            const size_t dot = name.find('.', 7);
            const int l = dot == std::string::npos ? -1 : atoi(name.c_str() + 7);
            if (l >= 0 && l < L) {
                const std::string sfx = name.substr(dot + 1);
                LayerW& w = lw[l];
                if (sfx == "tmix.r_proj.weight") q = &w.r;
                else if (sfx == "tmix.k_proj.weight") q = &w.k;
                else if (sfx == "tmix.v_proj.weight") q = &w.v;
                else if (sfx == "tmix.o_proj.weight") q = &w.o;
                else if (sfx == "cmix.key.weight") q = &w.key;
                else if (sfx == "cmix.value.weight") q = &w.value;
            }
        }
        RWKV_REQUIRE(q, RWKV_E_SHAPE, "set_param_rwkvq: '%s' is not a projection or head matrix", name.c_str());
        const int64_t OUT = q->OUT, IN = q->IN;
        RWKV_REQUIRE(IN % 256 == 0, RWKV_E_UNSUPPORTED, "set_param_rwkvq: IN=%lld not a multiple of 256", (long long)IN);
        int64_t e1, e2, e3;
        if (kind == WFMT_SB6) {
            RWKV_REQUIRE(bits >= 0 && bits <= 2, RWKV_E_UNSUPPORTED, "set_param_rwkvq: sb6 xbits %d", bits);
            e1 = OUT * (IN / 32) * (16 + 4 * bits);
            e2 = OUT * (IN / 32) * 2;
            e3 = OUT * (IN / 256) * 4;
        } else if (kind == WFMT_SYM) {
            RWKV_REQUIRE(bits == 6 || bits == 8, RWKV_E_UNSUPPORTED, "set_param_rwkvq: sym bits %d", bits);
            e1 = bits == 8 ? OUT * IN : OUT * (IN / 32) * 24;
            e2 = OUT * (IN / 16);
            e3 = OUT * (IN / 256) * 2;
        } else {
            return fail(RWKV_E_UNSUPPORTED, "set_param_rwkvq: kind %d (1 sb6, 2 sym)", kind);
        }
        RWKV_REQUIRE(b1 && b2 && b3, RWKV_E_NULL, "set_param_rwkvq: NULL buffer");
        RWKV_REQUIRE(n1 == e1 && n2 == e2 && n3 == e3, RWKV_E_SHAPE,
                     "set_param_rwkvq: '%s' buffers %lld / %lld / %lld bytes, expected %lld / %lld / %lld",
                     name.c_str(), (long long)n1, (long long)n2, (long long)n3, (long long)e1, (long long)e2,
                     (long long)e3);
        if (q->qblk) cudaFree(q->qblk);
        if (q->q2) cudaFree(q->q2);
        if (q->qd) cudaFree(q->qd);
        q->qblk = q->q2 = nullptr;
        q->qd = nullptr;
        if (cudaMalloc(&q->qblk, n1) != cudaSuccess || cudaMalloc(&q->q2, n2) != cudaSuccess ||
            cudaMalloc(&q->qd, n3) != cudaSuccess)
            return fail(RWKV_E_CUDA, "set_param_rwkvq: allocation failed");
        cudaMemcpy(q->qblk, b1, n1, cudaMemcpyHostToDevice);
        cudaMemcpy(q->q2, b2, n2, cudaMemcpyHostToDevice);
        cudaMemcpy(q->qd, b3, n3, cudaMemcpyHostToDevice);
        q->fmt = kind;
        q->qbits = bits;
        wver++;
        drop_graphs();
        return check_launch("set_param_rwkvq");
    }

    int set_param(const std::string& name, const float* host, int64_t n) {
        wver++;
        if (name.compare(0, 10, "head.lora_") == 0) return set_adapter(head_ad, name.substr(10), C, V, false, host, n);
        if (name == "emb.weight") return upload_q(emb, host, n);
        if (name == "head.weight") return upload_q(head, host, n);
        if (name == "ln0.weight") return upload_f(ln0w, C, host, n);
        if (name == "ln0.bias") return upload_f(ln0b, C, host, n);
        if (name == "ln_out.weight") return upload_f(lnow, C, host, n);
        if (name == "ln_out.bias") return upload_f(lnob, C, host, n);
        int l = -1, used = 0;
        if (sscanf(name.c_str(), "blocks.%d.%n", &l, &used) != 1 || l < 0 || l >= L)
            return fail(RWKV_E_SHAPE, "set_param: unknown parameter '%s'", name.c_str());
        const std::string s = name.substr(used);
        LayerW& w = lw[l];
        static const char* mixn[6] = {"tmix.x_r", "tmix.x_w", "tmix.x_k", "tmix.x_v", "tmix.x_a", "tmix.x_g"};
        for (int m = 0; m < 6; m++)
            if (s == mixn[m]) return upload_f(w.coef6 + (size_t)m * C, C, host, n);
        if (s == "ln1.weight") return upload_f(w.ln1w, C, host, n);
        if (s == "ln1.bias") return upload_f(w.ln1b, C, host, n);
        if (s == "ln2.weight") return upload_f(w.ln2w, C, host, n);
        if (s == "ln2.bias") return upload_f(w.ln2b, C, host, n);
        if (s == "tmix.k_k") return upload_f(w.kkw, C, host, n);
        if (s == "tmix.k_a") return upload_f(w.kaw, C, host, n);
        if (s == "tmix.r_k") return upload_f(w.rkw, C, host, n);
        if (s == "tmix.ln_x.weight") return upload_f(w.lnxw, C, host, n);
        if (s == "tmix.ln_x.bias") return upload_f(w.lnxb, C, host, n);
        if (s == "cmix.x_k") return upload_f(w.cxk, C, host, n);
        if (s == "tmix.w_lora_B.bias") return upload_f(w.wbias, C, host, n);
        if (s == "tmix.a_lora_B.bias") return upload_f(w.abias, C, host, n);
        if (s == "tmix.v_lora_B.bias") return upload_f(w.vbias, C, host, n);
        if (s == "tmix.w_lora_A.weight") return upload_h(w.wA, (int64_t)rw * C, host, n);
        if (s == "tmix.w_lora_B.weight") return upload_h(w.wB, (int64_t)C * rw, host, n);
        if (s == "tmix.a_lora_A.weight") return upload_h(w.aA, (int64_t)ra * C, host, n);
        if (s == "tmix.a_lora_B.weight") return upload_h(w.aB, (int64_t)C * ra, host, n);
        if (s == "tmix.g_lora_A.weight") return upload_h(w.gA, (int64_t)rg * C, host, n);
        if (s == "tmix.g_lora_B.weight") return upload_h(w.gB, (int64_t)C * rg, host, n);
        if (s == "tmix.v_lora_A.weight") return upload_h(w.vA, (int64_t)rv * C, host, n);
        if (s == "tmix.v_lora_B.weight") return upload_h(w.vB, (int64_t)C * rv, host, n);
        if (s == "tmix.r_proj.weight") return upload_q(w.r, host, n);
        if (s == "tmix.k_proj.weight") return upload_q(w.k, host, n);
        if (s == "tmix.v_proj.weight") return upload_q(w.v, host, n);
        if (s == "tmix.o_proj.weight") return upload_q(w.o, host, n);
        if (s == "cmix.key.weight") return upload_q(w.key, host, n);
        if (s == "cmix.value.weight") return upload_q(w.value, host, n);
        static const char* adn[AD_N] = {"tmix.r_proj", "tmix.k_proj", "tmix.v_proj", "tmix.o_proj", "cmix.key",
                                        "cmix.value"};
        for (int t = 0; t < AD_N; t++) {
            const std::string pre = std::string(adn[t]) + ".lora_";
            if (s.compare(0, pre.size(), pre) == 0)
                return set_adapter(w.ad[t], s.substr(pre.size()), t == AD_VALUE ? F : C, t == AD_KEY ? F : C,
                                   t == AD_KEY, host, n);
        }
        return fail(RWKV_E_SHAPE, "set_param: unknown parameter '%s'", name.c_str());
    }

    // Random init on the device with the x070 recipe (X070Init.swift:79-206):
    // orthogonal matrices are drawn as Gaussians of the same element scale.
    int init_random(uint64_t seed) {
        wver++;
        const size_t maxn = std::max((size_t)V * C, (size_t)F * C);
        __half* h16 = nullptr;
        if (cudaMalloc(&h16, maxn * 2) != cudaSuccess) return fail(RWKV_E_CUDA, "init: staging allocation failed");
        uint64_t salt = 0;
        // low-rank matrices in their storage format (fp16, or bf16 beside bf16 activations)
        auto fill = [&](__half* dst, int64_t n, int mode, float a, float b) {
            const uint64_t sd = seed * 0x9E3779B97F4A7C15ull + (++salt);
            if (lr_wf == WF_BF16) fill_kernel<__nv_bfloat16><<<2048, 256>>>((__nv_bfloat16*)dst, n, mode, a, b, sd);
            else fill_kernel<__half><<<2048, 256>>>(dst, n, mode, a, b, sd);
        };
        auto qfill = [&](QMat& q, int mode, float a, float b) {
            const uint64_t sd = seed * 0x9E3779B97F4A7C15ull + (++salt);
            if (dense) {
                fill_kernel<__nv_bfloat16><<<2048, 256>>>(q.dense, (int64_t)q.OUT * q.IN, mode, a, b, sd);
                return check_launch("fill_kernel");
            }
            fill_kernel<__half><<<2048, 256>>>(h16, (int64_t)q.OUT * q.IN, mode, a, b, sd);
            return launch_q_quantize(RWKV_F16, h16, q.wq, q.sc, q.bi, q.OUT, q.IN, 64, 4, 0);
        };
        const float s = 0.5f / sqrtf((float)C);
        int rc = qfill(emb, 0, -1e-4f, 1e-4f);
        if (!rc) rc = qfill(head, 1, (V > C ? 0.5f * sqrtf((float)V / C) : 0.5f) / sqrtf((float)std::max(V, C)), 0);
        std::vector<float> ones(C, 1.f), zeros(C, 0.f), tmp(C);
        cudaMemcpy(ln0w, ones.data(), C * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(lnow, ones.data(), C * 4, cudaMemcpyHostToDevice);
        const int N = cfg.head_size;
        std::vector<float> lin(C), zz(C);
        for (int i = 0; i < C; i++) {
            lin[i] = (float)i / (C - 1) - 0.5f;
            const float z = ((float)(i % N) - (N - 1) / 2.0f) / ((N - 1) / 2.0f);
            zz[i] = z * fabsf(z);
        }
        auto curve = [&](double kk) {
            for (int i = 0; i < C; i++) tmp[i] = (float)(1.0 - pow((double)i / C, kk));
            return tmp.data();
        };
        for (int l = 0; l < L && !rc; l++) {
            LayerW& w = lw[l];
            const double r01 = L > 1 ? (double)l / (L - 1) : 0.0, r1a = 1.0 - (double)l / L;
            cudaMemcpy(w.ln1w, ones.data(), C * 4, cudaMemcpyHostToDevice);
            cudaMemcpy(w.ln2w, ones.data(), C * 4, cudaMemcpyHostToDevice);
            const double ks[6] = {0.2, 0.9, 0.7, 0.7, 0.9, 0.2};
            for (int m = 0; m < 6; m++)
                cudaMemcpy(w.coef6 + (size_t)m * C, curve(ks[m] * r1a), C * 4, cudaMemcpyHostToDevice);
            const double ex = 1.0 + pow(r01, 0.3);
            for (int i = 0; i < C; i++)
                tmp[i] = (float)(-6.0 + 6.0 * pow((double)i / (C - 1), ex)) + 0.5f + zz[i] * 2.5f;
            cudaMemcpy(w.wbias, tmp.data(), C * 4, cudaMemcpyHostToDevice);
            for (int i = 0; i < C; i++) tmp[i] = -0.19f + zz[i] * 0.3f + lin[i] * 0.4f;
            cudaMemcpy(w.abias, tmp.data(), C * 4, cudaMemcpyHostToDevice);
            for (int i = 0; i < C; i++) tmp[i] = 0.73f - lin[i] * 0.4f;
            cudaMemcpy(w.vbias, tmp.data(), C * 4, cudaMemcpyHostToDevice);
            for (int i = 0; i < C; i++) tmp[i] = 0.71f - lin[i] * 0.1f;
            cudaMemcpy(w.kkw, tmp.data(), C * 4, cudaMemcpyHostToDevice);
            std::fill(tmp.begin(), tmp.end(), 1.02f);
            cudaMemcpy(w.kaw, tmp.data(), C * 4, cudaMemcpyHostToDevice);
            std::fill(tmp.begin(), tmp.end(), -0.04f);
            cudaMemcpy(w.rkw, tmp.data(), C * 4, cudaMemcpyHostToDevice);
            std::fill(tmp.begin(), tmp.end(), (float)pow((double)(l + 1) / L, 0.7));
            cudaMemcpy(w.lnxw, tmp.data(), C * 4, cudaMemcpyHostToDevice);
            cudaMemcpy(w.cxk, curve(pow(r1a, 4)), C * 4, cudaMemcpyHostToDevice);
            // low-rank: A = 0 (already zero), B ~ orthogonal * 0.1
            fill(w.wB, (int64_t)C * rw, 1, 0.1f / sqrtf((float)C), 0);
            fill(w.aB, (int64_t)C * ra, 1, 0.1f / sqrtf((float)C), 0);
            fill(w.gB, (int64_t)C * rg, 1, 0.1f / sqrtf((float)C), 0);
            if (l > 0) fill(w.vB, (int64_t)C * rv, 1, 0.1f / sqrtf((float)C), 0);
            rc = qfill(w.r, 0, -s, s);
            if (!rc) rc = qfill(w.k, 0, -0.1f * s, 0.1f * s);
            if (!rc) rc = qfill(w.v, 0, -s, s);
            if (!rc) rc = qfill(w.o, 0, 0.f, 0.f);
            if (!rc) rc = qfill(w.key, 0, -s, s);
            if (!rc) rc = qfill(w.value, 0, 0.f, 0.f);
        }
        cudaDeviceSynchronize();
        cudaFree(h16);
        if (rc) return rc;
        return check_launch("init_random");
    }

    // ----- one decode step on `R` rows: ids -> logits, ids <- argmax

    static int pdl_check(cudaError_t e, const char* name) {
        return e == cudaSuccess ? RWKV_OK : fail(RWKV_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    }

    // row kernels: GV = 16-byte column groups per thread, C <= 1024 GV
    template <typename F>
    int row_launch(F&& f, const char* name) const {
        const int gv = (C + 4 * GLUE_T - 1) / (4 * GLUE_T);
        cudaError_t e = gv <= 1 ? f.template operator()<1>() : gv == 2 ? f.template operator()<2>()
                      : gv == 3 ? f.template operator()<3>() : f.template operator()<4>();
        return pdl_check(e, name);
    }

    // fmt 0: the base matrices (4-bit, or dense bf16); 1: the low-rank / adapter matrices
    int gemv(int fmt, GemvJobs& jobs, int nj, int R, cudaStream_t st) {
        const int wf = fmt == 0 ? base_wf : lr_wf;
        if (fmt == 0) {
            // .rwkvq matrices go to their own GEMV kernels, the rest below
            GemvJobs rest{};
            int nr = 0;
            bool done[MAX_JOBS] = {};
            for (int i = 0; i < nj; i++) {
                if (jobs.j[i].wfmt == WFMT_AFFINE) {
                    rest.j[nr++] = jobs.j[i];
                } else if (!done[i]) {
                    // at 1 row one launch per (format, bit width) for the jobs that
                    // share it (1.5B sb6 / sym 6-bit decode 1.24 / 1.42 -> 1.12 / 1.17 ms);
                    // above 1 row one launch per job (grouped: 8-row sb6 4.92 -> 5.18 ms)
                    GemvJobs g{};
                    int ng = 0;
                    for (int k = i; k < nj && (R == 1 || k == i); k++)
                        if (!done[k] && jobs.j[k].wfmt == jobs.j[i].wfmt && jobs.j[k].wbits == jobs.j[i].wbits) {
                            g.j[ng++] = jobs.j[k];
                            done[k] = true;
                        }
                    const int xdt = bf16act ? RWKV_BF16 : f16act ? RWKV_F16 : RWKV_F32;
                    if (int rc = launch_rwkvq_jobs(xdt, g, ng, R, st)) return rc;
                }
            }
            if (nr == 0) return RWKV_OK;
            if (nr < nj) {
                jobs = rest;
                nj = nr;
            }
        }
        if (f16act) {
            // 1..2 rows of fp16 activations on the 4-bit base: the streaming CUDA-core GEMV
            if (fmt == 0 && wf == WF_Q4 && !bf16act && q4_stream_eligible(jobs, nj, R)) {
                cudaError_t e = launch_q4_gemv_stream(jobs, nj, R, sm_count, /*pdl=*/true, st);
                return e == cudaSuccess ? RWKV_OK : fail(RWKV_E_CUDA, "q4_gemv_stream: %s", cudaGetErrorString(e));
            }
            // and the dense fp16 low-rank branches: the small fp16 GEMV
            if (fmt == 1 && wf == WF_F16 && !bf16act && f16_small_eligible(jobs, nj, R)) {
                cudaError_t e = launch_f16_gemv_small(jobs, nj, R, /*pdl=*/true, st);
                return e == cudaSuccess ? RWKV_OK : fail(RWKV_E_CUDA, "f16_gemv_small: %s", cudaGetErrorString(e));
            }
            const int tfmt = wf == WF_Q4 ? TC_Q4 : wf == WF_F16 ? TC_F16 : TC_BF16;
            const TcPlan tp = plan_tc(tfmt, jobs, nj, R, sm_count);
            if (tp.ok) {
                cudaError_t e = launch_tc(tfmt, jobs, nj, R, tp, gerr, gflag.host_dev, st, /*pdl=*/true);
                return e == cudaSuccess ? RWKV_OK : fail(RWKV_E_CUDA, "gemm_tc: %s", cudaGetErrorString(e));
            }
            if (wf == WF_BF16)
                return fail(RWKV_E_UNSUPPORTED, "gemm: bf16 matrices take the tensor-core path only (16-byte rows)");
            GemmPlan p = plan_any(jobs, nj, R, sm_count);
            if (p.ws_floats > gws_floats || p.tickets > gtickets_n)
                return fail(RWKV_E_WORKSPACE, "gemm: split-K plan exceeds the workspace");
            GemmArgs ga{};
            // the side stream runs beside the main one: its own split-K workspace
            const bool on_side = st == side;
            ga.jobs = jobs; ga.njobs = nj; ga.R = R;
            ga.ws = on_side ? gws_side : gws;
            ga.tickets = on_side ? gtickets_side : gtickets;
            cudaError_t e = fmt == 0 ? launch_any<0>(ga, p, st, true) : launch_any<1>(ga, p, st, true);
            return e == cudaSuccess ? RWKV_OK : fail(RWKV_E_CUDA, "gemm: %s", cudaGetErrorString(e));
        }
        int maxo = 0;
        for (int i = 0; i < nj; i++) maxo = std::max(maxo, jobs.j[i].OUT);
        dim3 grid((maxo + 7) / 8, nj, (R + 7) / 8);
        if (wf == WF_Q4) gemv_cc_kernel<0><<<grid, 256, 0, st>>>(jobs, R);
        else if (wf == WF_F16) gemv_cc_kernel<1><<<grid, 256, 0, st>>>(jobs, R);
        else gemv_cc_kernel<2><<<grid, 256, 0, st>>>(jobs, R);
        return check_launch("gemv_cc_kernel");
    }

    // whether gemv() takes the tensor-core path for these jobs
    bool tc_path(int fmt, const GemvJobs& jobs, int nj, int R) const {
        const int wf = fmt == 0 ? base_wf : lr_wf;
        for (int i = 0; i < nj; i++)
            if (jobs.j[i].wfmt != WFMT_AFFINE) return false;
        return f16act && plan_tc(wf == WF_Q4 ? TC_Q4 : wf == WF_F16 ? TC_F16 : TC_BF16, jobs, nj, R, sm_count).ok;
    }
    // output type of an activation-typed GEMM result
    int aout() const { return !f16act ? OUT_F32 : bf16act ? OUT_BF16 : OUT_F16; }

    static GemvJob qjob(const QMat& q, const void* x, int xs, int act, int out, void* y, int ys,
                        const float* bias = nullptr) {
        GemvJob j{};
        if (q.dense) j.w = q.dense;
        else j.w = q.wq;
        j.scales = q.sc; j.biases = q.bi; j.x = x; j.x_stride = xs;
        if (q.fmt != WFMT_AFFINE) {
            j.w = q.qblk;
            j.scales = (const __half*)q.q2;
            j.biases = q.qd;
            j.wfmt = q.fmt;
            j.wbits = q.qbits;
        }
        j.OUT = q.OUT; j.IN = q.IN; j.act = act; j.out = out; j.y = y; j.y_stride = ys; j.bias = bias;
        return j;
    }
    static GemvJob hjob(const __half* W, int OUT, int IN, const void* x, int xs, int act, int out,
                        void* y, int ys, const float* bias = nullptr) {
        GemvJob j{};
        j.w = W; j.x = x; j.x_stride = xs; j.OUT = OUT; j.IN = IN; j.act = act; j.out = out;
        j.y = y; j.y_stride = ys; j.bias = bias;
        return j;
    }

    // LoRA adapters of up to three projections sharing one down and one up
    // launch: z = scale * (x A^T) (activation type), y += z B^T.
    struct LoraJob {
        const Adapter* ad;
        const void* x;
        int xs, IN, OUT;
        float* y;
        int ys;
    };
    // zbuf: [3][zrows][LORA_MAX_RANK] of the activation type, zrows >= R.
    template <typename A>
    int lora_apply(const LoraJob* lj, int n, int R, cudaStream_t st, void* zbuf = nullptr, int zrows = 0) {
        if (!zbuf) {
            zbuf = lora_z;
            zrows = Rmax;
        }
        GemvJobs D{}, U{};
        int nd = 0;
        for (int i = 0; i < n; i++) {
            const Adapter& ad = *lj[i].ad;
            if (!ad.on()) continue;
            A* z = (A*)zbuf + (size_t)nd * zrows * LORA_MAX_RANK;
            GemvJob d = hjob(ad.A, ad.rank_a, lj[i].IN, lj[i].x, lj[i].xs, ACT_SCALE, aout(), z,
                             ad.rank_a);
            d.alpha = ad.scale;
            D.j[nd] = d;
            U.j[nd] = hjob(ad.B, lj[i].OUT, ad.rank_a, z, ad.rank_a, ACT_NONE, OUT_ADD_F32, lj[i].y, lj[i].ys);
            nd++;
        }
        if (nd == 0) return RWKV_OK;
        int rc = gemv(1, D, nd, R, st);
        if (rc) return rc;
        mark("lora_adapter_down");
        rc = gemv(1, U, nd, R, st);
        if (rc) return rc;
        mark("lora_adapter_up");
        return RWKV_OK;
    }

    template <typename A>
    int step_body(int R, cudaStream_t st) {
        const size_t RC = (size_t)R * C;
        const int aout = this->aout();
        A* mixp = (A*)mix;
        A* hidp = (A*)hidden;
        int rc;
        if ((rc = pdl_check(launch_pdl(x070_embed_kernel, R, GLUE_T, 0, st, (const int32_t*)ids, (const uint32_t*)emb.wq,
                                       (const __half*)emb.sc, (const __half*)emb.bi, (const __nv_bfloat16*)emb.dense,
                                       (const float*)ln0w, (const float*)ln0b, x, C, V), "x070_embed_kernel")))
            return rc;
        mark("embed");
        for (int l = 0; l < L; l++) {
            LayerW& w = lw[l];
            float* ts = tshift + (size_t)l * Rmax * C;
            float* cs = cshift + (size_t)l * Rmax * C;
            float* st8 = wkv + (size_t)l * Rmax * H * 64 * 64;
            if ((rc = row_launch([&]<int GV>() {
                     return launch_pdl(x070_tmix_in_kernel<A, GV>, R, GLUE_T, 0, st, (const float*)x,
                                       (const float*)w.ln1w, (const float*)w.ln1b, ts,
                                       (const float*)w.coef6, mixp, R, C);
                 }, "x070_tmix_in_kernel")))
                return rc;
            mark("tmix_in");
            auto M = [&](int m) { return (const void*)(mixp + (size_t)m * RC); };
            GemvJobs J{};
            J.j[0] = qjob(w.r, M(0), C, ACT_NONE, OUT_F32, r, C);
            J.j[1] = qjob(w.k, M(2), C, ACT_NONE, OUT_F32, k, C);
            J.j[2] = qjob(w.v, M(3), C, ACT_NONE, OUT_F32, v, C);
            // low-rank down: w (tanh), a, g (sigmoid), v
            GemvJobs D{};
            int nd = 0;
            D.j[nd++] = hjob(w.wA, rw, C, M(1), C, ACT_TANH, aout, hidp, hid);
            D.j[nd++] = hjob(w.aA, ra, C, M(4), C, ACT_NONE, aout, hidp + rw, hid);
            D.j[nd++] = hjob(w.gA, rg, C, M(5), C, ACT_SIGMOID, aout, hidp + rw + ra, hid);
            if (l > 0) D.j[nd++] = hjob(w.vA, rv, C, M(3), C, ACT_NONE, aout, hidp + rw + ra + rg, hid);
            GemvJobs U{};
            int nu = 0;
            U.j[nu++] = hjob(w.wB, C, rw, hidp, hid, ACT_DECAY, OUT_F32, wdec, C, w.wbias);
            U.j[nu++] = hjob(w.aB, C, ra, hidp + rw, hid, ACT_SIGMOID_BIAS, OUT_F32, a, C, w.abias);
            U.j[nu++] = hjob(w.gB, C, rg, hidp + rw + ra, hid, ACT_NONE, OUT_F32, g, C);
            if (l > 0) U.j[nu++] = hjob(w.vB, C, rv, hidp + rw + ra + rg, hid, ACT_SIGMOID_BIAS, OUT_F32, vv, C, w.vbias);
            // the low-rank branch reads only tmix_in's mixes and writes only
            // w/a/g/v': beside the r/k/v GEMM (launches on `side` have their
            // own split-K workspace; the step profiler keeps one stream)
            const bool fork = side && !profiling;
            cudaStream_t sb = fork ? side : st;
            if (fork) {
                cudaEventRecord(ev_fork, st);
                cudaStreamWaitEvent(side, ev_fork, 0);
            }
            if ((rc = gemv(1, D, nd, R, sb))) return rc;
            mark("lora_down");
            if ((rc = gemv(1, U, nu, R, sb))) return rc;
            mark("lora_up");
            if (fork) cudaEventRecord(ev_join, side);
            if ((rc = gemv(0, J, 3, R, st))) return rc;
            mark("gemm_rkv");
            {
                const LoraJob lj[3] = {{&w.ad[AD_R], M(0), C, C, C, r, C}, {&w.ad[AD_K], M(2), C, C, C, k, C},
                                       {&w.ad[AD_V], M(3), C, C, C, v, C}};
                if ((rc = lora_apply<A>(lj, 3, R, st))) return rc;
            }
            if (fork) cudaStreamWaitEvent(st, ev_join, 0);
            if ((rc = pdl_check(launch_pdl(x070_wkv_kernel<A>, R * H, 128, 0, st, (const float*)r,
                                           (const float*)wdec, (const float*)k, (const float*)v,
                                           (const float*)a, (const float*)vv, vfirst, (const float*)w.kkw,
                                           (const float*)w.kaw, (const float*)w.rkw, (const float*)w.lnxw,
                                           (const float*)w.lnxb, (const float*)g, st8, (A*)tail, H,
                                           (int)(l == 0)), "x070_wkv_kernel")))
                return rc;
            mark("wkv_step_tail");
            GemvJobs O{};
            O.j[0] = qjob(w.o, tail, C, ACT_NONE, OUT_ADD_F32, x, C);
            if ((rc = gemv(0, O, 1, R, st))) return rc;
            mark("gemm_o");
            {
                const LoraJob lj[1] = {{&w.ad[AD_O], tail, C, C, C, x, C}};
                if ((rc = lora_apply<A>(lj, 1, R, st))) return rc;
            }
            if ((rc = row_launch([&]<int GV>() {
                     return launch_pdl(x070_cmix_in_kernel<A, GV>, R, GLUE_T, 0, st, (const float*)x,
                                       (const float*)w.ln2w, (const float*)w.ln2b, cs,
                                       (const float*)w.cxk, (A*)xk, C);
                 }, "x070_cmix_in_kernel")))
                return rc;
            mark("cmix_in");
            GemvJobs K{};
            if (!w.ad[AD_KEY].on()) {
                K.j[0] = qjob(w.key, xk, C, ACT_RELU2, aout, ffn, F);
                if ((rc = gemv(0, K, 1, R, st))) return rc;
                mark("gemm_key");
            } else {
                // the adapter is added before relu^2: pre-activation in fp32, then the activation
                K.j[0] = qjob(w.key, xk, C, ACT_NONE, OUT_F32, key_tmp, F);
                if ((rc = gemv(0, K, 1, R, st))) return rc;
                mark("gemm_key");
                const LoraJob lj[1] = {{&w.ad[AD_KEY], xk, C, C, F, key_tmp, F}};
                if ((rc = lora_apply<A>(lj, 1, R, st))) return rc;
                const int n = R * F;
                if ((rc = pdl_check(launch_pdl(x070_relu2_cast_kernel<A>, std::min((n + 255) / 256, 4 * sm_count), 256, 0,
                                               st, (const float*)key_tmp, (A*)ffn, n), "x070_relu2_cast_kernel")))
                    return rc;
                mark("relu2");
            }
            GemvJobs Vv{};
            Vv.j[0] = qjob(w.value, ffn, F, ACT_NONE, OUT_ADD_F32, x, C);
            if ((rc = gemv(0, Vv, 1, R, st))) return rc;
            mark("gemm_value");
            {
                const LoraJob lj[1] = {{&w.ad[AD_VALUE], ffn, F, F, C, x, C}};
                if ((rc = lora_apply<A>(lj, 1, R, st))) return rc;
            }
        }
        if ((rc = row_launch([&]<int GV>() {
                 return launch_pdl(x070_ln_out_kernel<A, GV>, R, GLUE_T, 0, st, (const float*)x,
                                   (const float*)lnow, (const float*)lnob, (A*)lnout, C);
             }, "x070_ln_out_kernel")))
            return rc;
        mark("ln_out");
        GemvJobs Hd{};
        Hd.j[0] = qjob(head, lnout, C, ACT_NONE, OUT_F32, logits, V);
        if ((rc = gemv(0, Hd, 1, R, st))) return rc;
        mark("gemm_head");
        {
            const LoraJob lj[1] = {{&head_ad, lnout, C, C, V, logits, V}};
            if ((rc = lora_apply<A>(lj, 1, R, st))) return rc;
        }
        if ((rc = pdl_check(launch_pdl(x070_argmax_kernel, dim3((V + ARGMAX_SLICE - 1) / ARGMAX_SLICE, R), GLUE_T, 0,
                                       st, (const float*)logits, V, amax_keys), "x070_argmax_kernel")))
            return rc;
        mark("argmax");
        rc = pdl_check(launch_pdl(x070_argmax_finish_kernel, (R + 127) / 128, 128, 0, st, amax_keys, ids, R),
                       "x070_argmax_finish_kernel");
        mark("argmax_finish");
        return rc;
    }

    // ----- persistent decode step (x070_persist.cuh): one launch per step

    // 0 (default): the per-kernel graph; 1: the persistent step where it
    // applies (measured slower on the 1.5B step: 2.70 vs 2.11 ms at 64 rows)
    int decode_path = 0;
    struct PkProgram {
        int BN = 0, nphases = 0, nitems_max = 0, ntiles_max = 0;
        std::vector<std::string> names;  // per phase, for the step profiler
        pk::Job* jobs = nullptr;
        pk::Item* items = nullptr;
        pk::Phase* phases = nullptr;
        pk::Layer* layers = nullptr;
        float* ws = nullptr;
        int* tickets = nullptr;
    };
    std::map<int, PkProgram> pk_progs;
    std::vector<void*> pk_allocs;
    unsigned int* pk_bar = nullptr;    // grid barrier counter
    unsigned long long* pk_trace = nullptr;  // per-phase timestamps when profiling
    std::vector<unsigned long long> pk_last_trace;  // the last profiled step's trace (rwkv_x070_trace)
    int64_t pk_wver = -1;
    int pk_occ = -1;  // CTAs of the persistent kernel per SM (cached)

    bool any_rwkvq() const {
        if (head.fmt != WFMT_AFFINE) return true;
        for (const LayerW& w : lw)
            if (w.r.fmt || w.k.fmt || w.v.fmt || w.o.fmt || w.key.fmt || w.value.fmt) return true;
        return false;
    }
    bool any_adapter() const {
        if (head_ad.on()) return true;
        for (const LayerW& w : lw)
            for (int t = 0; t < AD_N; t++)
                if (w.ad[t].on()) return true;
        return false;
    }
    // Whether a step on R rows takes the persistent kernel.
    bool pk_eligible(int R) const {
        return decode_path == 1 && f16act && !bf16act && !dense && R > 8 && R <= 64 && C % 256 == 0 && C <= 4 * pk::WT * 2 &&
               F % 256 == 0 && V % 128 == 0 && !any_adapter() && !any_rwkvq();
    }
    template <typename T>
    T* pk_alloc(size_t n) {
        void* p = nullptr;
        if (cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)) != cudaSuccess) return nullptr;
        pk_allocs.push_back(p);
        return (T*)p;
    }
    // Repacked (scale, bias) of every 4-bit matrix, refreshed after weight changes.
    int pk_repack(cudaStream_t st) {
        if (pk_wver == wver) return RWKV_OK;
        std::vector<QMat*> qs = {&head};
        for (LayerW& w : lw) {
            QMat* m[6] = {&w.r, &w.k, &w.v, &w.o, &w.key, &w.value};
            for (QMat* q : m) qs.push_back(q);
        }
        for (QMat* q : qs) {
            if (!q->sbr && !(q->sbr = pk_alloc<__half2>((size_t)q->OUT * q->IN / 64)))
                return fail(RWKV_E_CUDA, "persistent step: scale repack allocation failed");
            x070_repack_sb_kernel<<<std::min(ceil_div((int64_t)q->OUT * q->IN / 64, 256), 8 * sm_count), 256, 0, st>>>(
                q->sc, q->bi, q->sbr, q->OUT, q->IN);
        }
        pk_wver = wver;
        return check_launch("x070_repack_sb_kernel");
    }

    // The step as a program of phases for R rows (tensor maps, work items).
    int pk_build(int R, PkProgram& P) {
        auto enc = tensor_map_encoder();
        if (!enc) return fail(RWKV_E_CUDA, "persistent step: no tensor-map encoder");
        const int BN = R <= 16 ? 16 : R <= 32 ? 32 : 64;
        const int G = sm_count;
        std::vector<pk::Job> jobs;
        std::vector<pk::Item> items;
        std::vector<pk::Phase> phases;
        bool bad = false;
        auto xmap = [&](CUtensorMap& m, const void* x, int IN, int xs) {
            cuuint64_t dims[2] = {(cuuint64_t)IN, (cuuint64_t)R};
            cuuint64_t strides[1] = {(cuuint64_t)xs * 2};
            cuuint32_t box[2] = {64, (cuuint32_t)BN};
            cuuint32_t es[2] = {1, 1};
            if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)x, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                bad = true;
        };
        auto qj = [&](const QMat& q, const void* x, int xs, int act, int out, void* y, int ys,
                      const float* bias = nullptr) {
            pk::Job j{};
            cuuint64_t dims[2] = {(cuuint64_t)(q.IN / 8), (cuuint64_t)q.OUT};
            cuuint64_t strides[1] = {(cuuint64_t)q.IN / 2};
            cuuint32_t box[2] = {32, 128};
            cuuint32_t es[2] = {1, 1};
            if (enc(&j.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, (void*)q.wq, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                bad = true;
            xmap(j.xmap, x, q.IN, xs);
            j.sb = (const unsigned char*)q.sbr;
            j.g = qjob(q, x, xs, act, out, y, ys, bias);
            j.fmt = pk::FMT_Q4;
            j.sb_stages = q.IN / 256;
            jobs.push_back(j);
            return (int)jobs.size() - 1;
        };
        auto hj = [&](const __half* W, int OUT, int IN, const void* x, int xs, int act, int out, void* y, int ys,
                      const float* bias = nullptr) {
            pk::Job j{};
            cuuint64_t dims[2] = {(cuuint64_t)IN, (cuuint64_t)OUT};
            cuuint64_t strides[1] = {(cuuint64_t)IN * 2};
            cuuint32_t box[2] = {64, 128};
            cuuint32_t es[2] = {1, 1};
            if (enc(&j.wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)W, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                bad = true;
            xmap(j.xmap, x, IN, xs);
            j.g = hjob(W, OUT, IN, x, xs, act, out, y, ys, bias);
            j.fmt = pk::FMT_F16;
            jobs.push_back(j);
            return (int)jobs.size() - 1;
        };
        // A GEMM phase over jobs js: every 128-row tile split along K so that
        // the phase has about one work item per CTA (items of a tile adjacent).
        int max_items = 1, tiles = 0;  // tiles numbered across the program
        auto gemm = [&](std::initializer_list<int> js, int layer) {
            auto stages = [&](const pk::Job& j) { return j.fmt == pk::FMT_Q4 ? j.g.IN / 256 : (j.g.IN + 63) / 64; };
            int64_t T = 0;
            for (int ji : js) T += (int64_t)((jobs[ji].g.OUT + 127) / 128) * stages(jobs[ji]);
            const int target = (int)std::max<int64_t>(1, (T + G - 1) / G);
            pk::Phase ph{pk::PH_GEMM, (int)items.size(), 0, layer};
            int& tile = tiles;
            for (int ji : js) {
                const int S = stages(jobs[ji]);
                const int nz = std::min(16, (S + target - 1) / target);  // the kernel sums at most 16 partials
                for (int m0 = 0; m0 < jobs[ji].g.OUT; m0 += 128, tile++)
                    for (int z = 0; z < nz; z++) {
                        const int a = (int)((int64_t)S * z / nz), b = (int)((int64_t)S * (z + 1) / nz);
                        pk::Item itm{ji, m0, a, b - a, tile, z, nz, (int)items.size() - ph.i0, jobs[ji].fmt, 0, nullptr};
                        if (jobs[ji].fmt == pk::FMT_Q4)
                            itm.sb = jobs[ji].sb + (size_t)(m0 / 128) * jobs[ji].sb_stages * pk::WSB;
                        items.push_back(itm);
                    }
            }
            ph.i1 = (int)items.size();
            max_items = std::max(max_items, ph.i1 - ph.i0);
            phases.push_back(ph);
        };
        std::vector<std::string> names;
        auto named = [&](const char* n) { names.resize(phases.size() - 1); names.push_back(n); };
        __half* mixp = (__half*)mix;
        __half* hidp = (__half*)hidden;
        const size_t RC = (size_t)R * C;
        auto M = [&](int m) { return (const void*)(mixp + (size_t)m * RC); };
        phases.push_back({pk::PH_EMBED, 0, 0, -1});
        named("embed");
        for (int l = 0; l < L; l++) {
            LayerW& w = lw[l];
            phases.push_back({pk::PH_TMIX, 0, 0, l});
            named("tmix_in");
            const int jr = qj(w.r, M(0), C, ACT_NONE, OUT_F32, r, C);
            const int jk = qj(w.k, M(2), C, ACT_NONE, OUT_F32, k, C);
            const int jv = qj(w.v, M(3), C, ACT_NONE, OUT_F32, v, C);
            const int dw = hj(w.wA, rw, C, M(1), C, ACT_TANH, OUT_F16, hidp, hid);
            const int da = hj(w.aA, ra, C, M(4), C, ACT_NONE, OUT_F16, hidp + rw, hid);
            const int dg = hj(w.gA, rg, C, M(5), C, ACT_SIGMOID, OUT_F16, hidp + rw + ra, hid);
            const int uw = hj(w.wB, C, rw, hidp, hid, ACT_DECAY, OUT_F32, wdec, C, w.wbias);
            const int ua = hj(w.aB, C, ra, hidp + rw, hid, ACT_SIGMOID_BIAS, OUT_F32, a, C, w.abias);
            const int ug = hj(w.gB, C, rg, hidp + rw + ra, hid, ACT_NONE, OUT_F32, g, C);
            if (l > 0) {
                const int dv = hj(w.vA, rv, C, M(3), C, ACT_NONE, OUT_F16, hidp + rw + ra + rg, hid);
                const int uv = hj(w.vB, C, rv, hidp + rw + ra + rg, hid, ACT_SIGMOID_BIAS, OUT_F32, vv, C, w.vbias);
                gemm({jr, jk, jv, dw, da, dg, dv}, l);
                named("gemm_rkv_lowrank_down");
                gemm({uw, ua, ug, uv}, l);
                named("gemm_lowrank_up");
            } else {
                gemm({jr, jk, jv, dw, da, dg}, l);
                named("gemm_rkv_lowrank_down");
                gemm({uw, ua, ug}, l);
                named("gemm_lowrank_up");
            }
            phases.push_back({pk::PH_WKV, 0, 0, l});
            named("wkv_step_tail");
            gemm({qj(w.o, tail, C, ACT_NONE, OUT_ADD_F32, x, C)}, l);
            named("gemm_o");
            phases.push_back({pk::PH_CMIX, 0, 0, l});
            named("cmix_in");
            gemm({qj(w.key, xk, C, ACT_RELU2, OUT_F16, ffn, F)}, l);
            named("gemm_key");
            gemm({qj(w.value, ffn, F, ACT_NONE, OUT_ADD_F32, x, C)}, l);
            named("gemm_value");
        }
        phases.push_back({pk::PH_LNOUT, 0, 0, -1});
        named("ln_out");
        gemm({qj(head, lnout, C, ACT_NONE, OUT_F32, logits, V)}, -1);
        named("gemm_head");
        phases.push_back({pk::PH_ARGMAX, 0, 0, -1});
        named("argmax");
        phases.push_back({pk::PH_ARGFIN, 0, 0, -1});
        named("argmax_finish");
        if (bad) return fail(RWKV_E_CUDA, "persistent step: tensor map encoding failed");
        if ((int)phases.size() > pk::MAX_PHASES)
            return fail(RWKV_E_UNSUPPORTED, "persistent step: %d phases, at most %d", (int)phases.size(), pk::MAX_PHASES);
        std::vector<pk::Layer> layers(L);
        for (int l = 0; l < L; l++) {
            const LayerW& w = lw[l];
            layers[l] = {w.ln1w, w.ln1b, w.ln2w, w.ln2b, w.coef6, w.kkw, w.kaw, w.rkw, w.lnxw, w.lnxb, w.cxk,
                         wkv + (size_t)l * Rmax * H * 64 * 64, tshift + (size_t)l * Rmax * C, cshift + (size_t)l * Rmax * C};
        }
        P.BN = BN;
        P.names = names;
        P.nphases = (int)phases.size();
        P.nitems_max = max_items;
        P.ntiles_max = std::max(1, tiles);
        P.jobs = pk_alloc<pk::Job>(jobs.size());
        P.items = pk_alloc<pk::Item>(items.size());
        P.phases = pk_alloc<pk::Phase>(phases.size());
        P.layers = pk_alloc<pk::Layer>(layers.size());
        P.ws = pk_alloc<float>((size_t)max_items * BN * 128);
        P.tickets = pk_alloc<int>(P.ntiles_max);
        if (!P.jobs || !P.items || !P.phases || !P.layers || !P.ws || !P.tickets)
            return fail(RWKV_E_CUDA, "persistent step: program allocation failed");
        cudaMemcpy(P.jobs, jobs.data(), jobs.size() * sizeof(pk::Job), cudaMemcpyHostToDevice);
        cudaMemcpy(P.items, items.data(), items.size() * sizeof(pk::Item), cudaMemcpyHostToDevice);
        cudaMemcpy(P.phases, phases.data(), phases.size() * sizeof(pk::Phase), cudaMemcpyHostToDevice);
        cudaMemcpy(P.layers, layers.data(), layers.size() * sizeof(pk::Layer), cudaMemcpyHostToDevice);
        cudaMemset(P.tickets, 0, (size_t)P.ntiles_max * sizeof(int));
        return check_launch("persistent step: program upload");
    }

    template <int BN>
    cudaError_t pk_launch(const pk::Args& a, cudaStream_t st) {
        auto kern = pk::x070_persist_kernel<BN>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pk::SMEM);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(sm_count);
        cfg.blockDim = dim3(pk::THREADS);
        cfg.dynamicSmemBytes = pk::SMEM;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (grid barriers)
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kern, a);
    }

    int pk_step(int R, cudaStream_t st) {
        if (int rc = pk_repack(st)) return rc;
        const size_t bar_words = 32;
        if (!pk_bar && !(pk_bar = pk_alloc<unsigned int>(bar_words)))
            return fail(RWKV_E_CUDA, "persistent step: allocation failed");
        auto it = pk_progs.find(R);
        if (it == pk_progs.end()) {
            PkProgram P;
            if (int rc = pk_build(R, P)) return rc;
            it = pk_progs.emplace(R, P).first;
        }
        const PkProgram& P = it->second;
        if (pk_occ < 0) {
            int n = 0;
            cudaFuncSetAttribute(pk::x070_persist_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, pk::SMEM);
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, pk::x070_persist_kernel<64>, pk::THREADS, pk::SMEM) !=
                cudaSuccess)
                n = 0;
            cudaGetLastError();
            pk_occ = n;
        }
        if (pk_occ < 1) return fail(RWKV_E_UNSUPPORTED, "persistent step: the kernel does not fit on an SM");
        pk::Args a{};
        a.jobs = P.jobs; a.items = P.items; a.phases = P.phases; a.layers = P.layers;
        a.nphases = P.nphases; a.R = R; a.C = C; a.H = H; a.V = V;
        a.x = x; a.r = r; a.k = k; a.v = v; a.wdec = wdec; a.a = this->a; a.g = g; a.vv = vv; a.vfirst = vfirst;
        a.logits = logits; a.ws = P.ws;
        a.mix = (__half*)mix; a.tail = (__half*)tail; a.xk = (__half*)xk; a.lnout = (__half*)lnout;
        a.ids = ids; a.amax_keys = amax_keys;
        a.emb_wq = emb.wq; a.emb_sc = emb.sc; a.emb_bi = emb.bi;
        a.ln0w = ln0w; a.ln0b = ln0b; a.lnow = lnow; a.lnob = lnob;
        a.tickets = P.tickets; a.bar = pk_bar; a.err = gerr; a.err_host = gflag.host_dev;
        if (profiling) {
            if (!pk_trace && !(pk_trace = pk_alloc<unsigned long long>(pk::T_END)))
                return fail(RWKV_E_CUDA, "persistent step: trace allocation failed");
            if (P.nphases + 1 > 1024) return fail(RWKV_E_UNSUPPORTED, "persistent step: too many phases to trace");
            a.trace = pk_trace;
        }
        cudaMemsetAsync(pk_bar, 0, bar_words * sizeof(unsigned int), st);
        cudaMemsetAsync(P.tickets, 0, (size_t)P.ntiles_max * sizeof(int), st);
        const cudaError_t e = P.BN == 16 ? pk_launch<16>(a, st) : P.BN == 32 ? pk_launch<32>(a, st) : pk_launch<64>(a, st);
        if (e != cudaSuccess) return fail(RWKV_E_CUDA, "x070_persist_kernel: %s", cudaGetErrorString(e));
        return RWKV_OK;
    }

    // ----- persistent decode step for 1..8 rows (x070_small.cuh)

    bool sp_eligible(int R) const {
        return decode_path == 1 && f16act && !bf16act && !dense && R >= 1 && R <= 8 && C % 128 == 0 &&
               C <= 4 * pk::WT * 2 && F % 128 == 0 && !any_adapter() && !any_rwkvq();
    }
    struct SpProgram {
        int nphases = 0;
        std::vector<std::string> names;
        sp::Job* jobs = nullptr;
        sp::Item* items = nullptr;
        int* ofs = nullptr;
        sp::Phase* phases = nullptr;
        pk::Layer* layers = nullptr;
    };
    std::map<int, SpProgram> sp_progs;
    int sp_occ[4] = {-1, -1, -1, -1};
    int64_t sp_wver = -1;

    // The (scale, bias) blocks of every 4-bit matrix, refreshed after weight changes.
    int sp_repack(cudaStream_t st) {
        if (sp_wver == wver) return RWKV_OK;
        std::vector<QMat*> qs = {&head};
        for (LayerW& w : lw) {
            QMat* m[6] = {&w.r, &w.k, &w.v, &w.o, &w.key, &w.value};
            for (QMat* q : m) qs.push_back(q);
        }
        for (QMat* q : qs) {
            const size_t n = (size_t)ceil_div(q->OUT, sp::TR) * ceil_div(q->IN, sp::KPQ) * (sp::SBB / 2);
            if (!q->sbs && !(q->sbs = pk_alloc<__half>(n)))
                return fail(RWKV_E_CUDA, "small-row persistent step: scale repack allocation failed");
            x070_repack_sb_small_kernel_launch(q, st);
        }
        sp_wver = wver;
        return check_launch("x070_repack_sb_small_kernel");
    }
    void x070_repack_sb_small_kernel_launch(QMat* q, cudaStream_t st) {
        const int64_t n = (int64_t)ceil_div(q->OUT, sp::TR) * ceil_div(q->IN, sp::KPQ) * (sp::SBB / 2);
        sp::x070_repack_sb_small_kernel<<<(int)std::min<int64_t>(ceil_div(n, 256), 8 * sm_count), 256, 0, st>>>(
            q->sc, q->bi, q->sbs, q->OUT, q->IN);
    }

    int sp_build(int R, SpProgram& P) {
        const int G = sm_count;
        std::vector<sp::Job> jobs;
        std::vector<sp::Item> items;
        std::vector<int> ofs;
        std::vector<sp::Phase> phases;
        std::vector<std::string> names;
        auto named = [&](const char* n) { names.resize(phases.size() - 1); names.push_back(n); };
        auto qj = [&](const QMat& q, const void* xx, int xs, int act, int out, void* y, int ys, const float* bias = nullptr) {
            jobs.push_back({qjob(q, xx, xs, act, out, y, ys, bias), q.sbs, sp::FMT_Q4, ceil_div(q.IN, sp::KPQ)});
            return (int)jobs.size() - 1;
        };
        auto hj = [&](const __half* W, int OUT, int IN, const void* xx, int xs, int act, int out, void* y, int ys,
                      const float* bias = nullptr) {
            jobs.push_back({hjob(W, OUT, IN, xx, xs, act, out, y, ys, bias), nullptr, sp::FMT_F16, ceil_div(IN, sp::KPH)});
            return (int)jobs.size() - 1;
        };
        // A GEMV phase over jobs js: 16-row tiles, each cut along K into pieces
        // (4-bit: 2048 codes, fp16: 512 columns); whole tiles go to CTAs in
        // order so that every CTA gets about the same number of pieces.
        auto gemv = [&](std::initializer_list<int> js, int layer, const char* name) {
            struct Tile { int job, o0, np; };
            std::vector<Tile> tiles;
            int64_t T = 0;
            for (int ji : js) {
                const int KP = jobs[ji].fmt == sp::FMT_Q4 ? sp::KPQ : sp::KPH;
                const int np = (jobs[ji].g.IN + KP - 1) / KP;
                for (int o0 = 0; o0 < jobs[ji].g.OUT; o0 += sp::TR) {
                    tiles.push_back({ji, o0, np});
                    T += np;
                }
            }
            phases.push_back({pk::PH_GEMM, (int)ofs.size(), layer, 0});
            named(name);
            size_t ti = 0;
            int64_t done = 0;
            for (int c = 0; c < G; c++) {
                ofs.push_back((int)items.size());
                const int64_t until = T * (c + 1) / G;
                while (ti < tiles.size() && done < until) {
                    const Tile& t = tiles[ti++];
                    const int KP = jobs[t.job].fmt == sp::FMT_Q4 ? sp::KPQ : sp::KPH, IN = jobs[t.job].g.IN;
                    for (int q = 0; q < t.np; q++) {
                        const int k0 = q * KP;
                        items.push_back({t.job, t.o0, k0, std::min(KP, IN - k0), q == t.np - 1, 0, 0, 0});
                    }
                    done += t.np;
                }
            }
            ofs.push_back((int)items.size());
        };
        __half* mixp = (__half*)mix;
        __half* hidp = (__half*)hidden;
        const size_t RC = (size_t)R * C;
        auto M = [&](int m) { return (const void*)(mixp + (size_t)m * RC); };
        phases.push_back({pk::PH_EMBED, 0, -1, 0});
        named("embed");
        for (int l = 0; l < L; l++) {
            LayerW& w = lw[l];
            phases.push_back({pk::PH_TMIX, 0, l, 0});
            named("tmix_in");
            const int jr = qj(w.r, M(0), C, ACT_NONE, OUT_F32, r, C);
            const int jk = qj(w.k, M(2), C, ACT_NONE, OUT_F32, k, C);
            const int jv = qj(w.v, M(3), C, ACT_NONE, OUT_F32, v, C);
            const int dw = hj(w.wA, rw, C, M(1), C, ACT_TANH, OUT_F16, hidp, hid);
            const int da = hj(w.aA, ra, C, M(4), C, ACT_NONE, OUT_F16, hidp + rw, hid);
            const int dg = hj(w.gA, rg, C, M(5), C, ACT_SIGMOID, OUT_F16, hidp + rw + ra, hid);
            const int uw = hj(w.wB, C, rw, hidp, hid, ACT_DECAY, OUT_F32, wdec, C, w.wbias);
            const int ua = hj(w.aB, C, ra, hidp + rw, hid, ACT_SIGMOID_BIAS, OUT_F32, a, C, w.abias);
            const int ug = hj(w.gB, C, rg, hidp + rw + ra, hid, ACT_NONE, OUT_F32, g, C);
            if (l > 0) {
                const int dv = hj(w.vA, rv, C, M(3), C, ACT_NONE, OUT_F16, hidp + rw + ra + rg, hid);
                const int uv = hj(w.vB, C, rv, hidp + rw + ra + rg, hid, ACT_SIGMOID_BIAS, OUT_F32, vv, C, w.vbias);
                gemv({jr, jk, jv, dw, da, dg, dv}, l, "gemm_rkv_lowrank_down");
                gemv({uw, ua, ug, uv}, l, "gemm_lowrank_up");
            } else {
                gemv({jr, jk, jv, dw, da, dg}, l, "gemm_rkv_lowrank_down");
                gemv({uw, ua, ug}, l, "gemm_lowrank_up");
            }
            phases.push_back({pk::PH_WKV, 0, l, 0});
            named("wkv_step_tail");
            gemv({qj(w.o, tail, C, ACT_NONE, OUT_ADD_F32, x, C)}, l, "gemm_o");
            phases.push_back({pk::PH_CMIX, 0, l, 0});
            named("cmix_in");
            gemv({qj(w.key, xk, C, ACT_RELU2, OUT_F16, ffn, F)}, l, "gemm_key");
            gemv({qj(w.value, ffn, F, ACT_NONE, OUT_ADD_F32, x, C)}, l, "gemm_value");
        }
        phases.push_back({pk::PH_LNOUT, 0, -1, 0});
        named("ln_out");
        gemv({qj(head, lnout, C, ACT_NONE, OUT_F32, logits, V)}, -1, "gemm_head");
        phases.push_back({pk::PH_ARGMAX, 0, -1, 0});
        named("argmax");
        phases.push_back({pk::PH_ARGFIN, 0, -1, 0});
        named("argmax_finish");
        if ((int)phases.size() > pk::MAX_PHASES)
            return fail(RWKV_E_UNSUPPORTED, "small-row persistent step: %d phases, at most %d", (int)phases.size(),
                        pk::MAX_PHASES);
        std::vector<pk::Layer> layers(L);
        for (int l = 0; l < L; l++) {
            const LayerW& w = lw[l];
            layers[l] = {w.ln1w, w.ln1b, w.ln2w, w.ln2b, w.coef6, w.kkw, w.kaw, w.rkw, w.lnxw, w.lnxb, w.cxk,
                         wkv + (size_t)l * Rmax * H * 64 * 64, tshift + (size_t)l * Rmax * C, cshift + (size_t)l * Rmax * C};
        }
        P.names = names;
        P.nphases = (int)phases.size();
        P.jobs = pk_alloc<sp::Job>(jobs.size());
        P.items = pk_alloc<sp::Item>(items.size());
        P.ofs = pk_alloc<int>(ofs.size());
        P.phases = pk_alloc<sp::Phase>(phases.size());
        P.layers = pk_alloc<pk::Layer>(layers.size());
        if (!P.jobs || !P.items || !P.ofs || !P.phases || !P.layers)
            return fail(RWKV_E_CUDA, "small-row persistent step: program allocation failed");
        cudaMemcpy(P.jobs, jobs.data(), jobs.size() * sizeof(sp::Job), cudaMemcpyHostToDevice);
        cudaMemcpy(P.items, items.data(), items.size() * sizeof(sp::Item), cudaMemcpyHostToDevice);
        cudaMemcpy(P.ofs, ofs.data(), ofs.size() * sizeof(int), cudaMemcpyHostToDevice);
        cudaMemcpy(P.phases, phases.data(), phases.size() * sizeof(sp::Phase), cudaMemcpyHostToDevice);
        cudaMemcpy(P.layers, layers.data(), layers.size() * sizeof(pk::Layer), cudaMemcpyHostToDevice);
        return check_launch("small-row persistent step: program upload");
    }

    template <int RB>
    int sp_launch(const sp::Args& sa, cudaStream_t st) {
        auto kern = sp::x070_small_kernel<2, RB>;
        constexpr int SM = sp::Cfg<RB>::SMEM;
        const int ri = RB == 1 ? 0 : RB == 2 ? 1 : RB == 4 ? 2 : 3;
        if (sp_occ[ri] < 0) {
            int n = 0;
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM);
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, sp::THREADS, SM) != cudaSuccess) n = 0;
            cudaGetLastError();
            sp_occ[ri] = n;
        }
        if (sp_occ[ri] < 1) return fail(RWKV_E_UNSUPPORTED, "small-row persistent step: the kernel does not fit on an SM");
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(sm_count);
        cfg.blockDim = dim3(sp::THREADS);
        cfg.dynamicSmemBytes = SM;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (grid barriers)
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, sa);
        if (e != cudaSuccess) return fail(RWKV_E_CUDA, "x070_small_kernel: %s", cudaGetErrorString(e));
        return RWKV_OK;
    }

    int sp_step(int R, cudaStream_t st) {
        if (int rc = sp_repack(st)) return rc;
        const size_t bar_words = 32;
        if (!pk_bar && !(pk_bar = pk_alloc<unsigned int>(bar_words)))
            return fail(RWKV_E_CUDA, "small-row persistent step: allocation failed");
        auto it = sp_progs.find(R);
        if (it == sp_progs.end()) {
            SpProgram P;
            if (int rc = sp_build(R, P)) return rc;
            it = sp_progs.emplace(R, P).first;
        }
        const SpProgram& P = it->second;
        sp::Args sa{};
        pk::Args& a = sa.g;
        a.layers = P.layers;
        a.nphases = P.nphases; a.R = R; a.C = C; a.H = H; a.V = V;
        a.x = x; a.r = r; a.k = k; a.v = v; a.wdec = wdec; a.a = this->a; a.g = g; a.vv = vv; a.vfirst = vfirst;
        a.logits = logits;
        a.mix = (__half*)mix; a.tail = (__half*)tail; a.xk = (__half*)xk; a.lnout = (__half*)lnout;
        a.ids = ids; a.amax_keys = amax_keys;
        a.emb_wq = emb.wq; a.emb_sc = emb.sc; a.emb_bi = emb.bi;
        a.ln0w = ln0w; a.ln0b = ln0b; a.lnow = lnow; a.lnob = lnob;
        a.bar = pk_bar; a.err = gerr; a.err_host = gflag.host_dev;
        if (profiling) {
            if (!pk_trace && !(pk_trace = pk_alloc<unsigned long long>(pk::T_END)))
                return fail(RWKV_E_CUDA, "small-row persistent step: trace allocation failed");
            if (P.nphases + 1 > 1024) return fail(RWKV_E_UNSUPPORTED, "small-row persistent step: too many phases to trace");
            a.trace = pk_trace;
        }
        sa.jobs = P.jobs; sa.items = P.items; sa.ofs = P.ofs; sa.phases = P.phases; sa.nphases = P.nphases;
        cudaMemsetAsync(pk_bar, 0, bar_words * sizeof(unsigned int), st);
        return R <= 1 ? sp_launch<1>(sa, st) : R <= 2 ? sp_launch<2>(sa, st) : R <= 4 ? sp_launch<4>(sa, st)
                                                                            : sp_launch<8>(sa, st);
    }

    // Whether a step on R rows is one persistent launch, and that launch.
    bool persist_eligible(int R) const { return pk_eligible(R) || sp_eligible(R); }
    int persist_step(int R, cudaStream_t st) { return sp_eligible(R) ? sp_step(R, st) : pk_step(R, st); }

    int run_step(int R, cudaStream_t st) {
        if (persist_eligible(R)) return persist_step(R, st);
        return bf16act ? step_body<__nv_bfloat16>(R, st) : f16act ? step_body<__half>(R, st) : step_body<float>(R, st);
    }

    int graph_step(int R, cudaStream_t st) {
        if (persist_eligible(R)) return run_step(R, st);  // one launch per step: nothing to capture
        auto it = graphs.find(R);
        if (it == graphs.end()) {
            cudaGraph_t gph;
            if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
                return fail(RWKV_E_CUDA, "graph capture could not start (the stream must not be the legacy default stream)");
            int rc = run_step(R, st);
            cudaError_t e = cudaStreamEndCapture(st, &gph);
            if (rc) return rc;
            if (e != cudaSuccess) return fail(RWKV_E_CUDA, "graph capture: %s", cudaGetErrorString(e));
            cudaGraphExec_t ex;
            e = cudaGraphInstantiate(&ex, gph, 0);
            cudaGraphDestroy(gph);
            if (e != cudaSuccess) return fail(RWKV_E_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
            it = graphs.emplace(R, ex).first;
        }
        cudaError_t e = cudaGraphLaunch(it->second, st);
        return e == cudaSuccess ? ok() : fail(RWKV_E_CUDA, "graph launch: %s", cudaGetErrorString(e));
    }

    // One eager step with an event after every launch; per-launch device
    // milliseconds into ms[] (up to cap) and their names, '\n'-separated.
    // The step captured into a graph with an event node after every launch,
    // replayed once: device-side per-launch milliseconds into ms[] (up to
    // cap) and their names, '\n'-separated.
    int profile_step(int R, cudaStream_t st, float* ms, int cap, char* names, int names_cap, int* count) {
        if (persist_eligible(R)) return profile_persistent(R, st, ms, cap, names, names_cap, count);
        cudaStream_t cs = st ? st : own;
        if (!st) {
            cudaEventRecord(ev_in, st);
            cudaStreamWaitEvent(own, ev_in, 0);
        }
        cudaEvent_t e0;
        cudaEventCreate(&e0);
        prof_stream = cs;
        prof_names.clear();
        cudaGraph_t gph;
        if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
            return fail(RWKV_E_CUDA, "profile: capture could not start");
        cudaEventRecordWithFlags(e0, cs, cudaEventRecordExternal);
        profiling = true;
        int rc = run_step(R, cs);
        profiling = false;
        cudaError_t e = cudaStreamEndCapture(cs, &gph);
        if (rc == RWKV_OK && e != cudaSuccess) rc = fail(RWKV_E_CUDA, "profile capture: %s", cudaGetErrorString(e));
        if (rc == RWKV_OK) {
            cudaGraphExec_t ex;
            e = cudaGraphInstantiate(&ex, gph, 0);
            if (e == cudaSuccess) {
                cudaGraphLaunch(ex, cs);
                if (cudaStreamSynchronize(cs) != cudaSuccess) rc = fail(RWKV_E_CUDA, "profile: replay failed");
                cudaGraphExecDestroy(ex);
            } else {
                rc = fail(RWKV_E_CUDA, "profile instantiate: %s", cudaGetErrorString(e));
            }
        }
        if (e == cudaSuccess || rc != RWKV_OK) cudaGraphDestroy(gph);
        std::string all;
        int n = 0;
        cudaEvent_t prev = e0;
        for (size_t i = 0; i < prof_names.size() && rc == RWKV_OK; i++) {
            float t = 0.f;
            cudaEventElapsedTime(&t, prev, prof_ev[i]);
            if (n < cap) ms[n++] = t;
            all += prof_names[i];
            all += "\n";
            prev = prof_ev[i];
        }
        cudaEventDestroy(e0);
        prof_names.clear();
        *count = n;
        if (names && names_cap > 0) {
            strncpy(names, all.c_str(), names_cap - 1);
            names[names_cap - 1] = 0;
        }
        if (!st) {
            cudaEventRecord(ev_out, own);
            cudaStreamWaitEvent(st, ev_out, 0);
        }
        return rc;
    }

    // The persistent step's phases: device milliseconds between CTA 0's
    // passes through consecutive grid barriers (%globaltimer), one entry per
    // phase named after what it runs.
    int profile_persistent(int R, cudaStream_t st, float* ms, int cap, char* names, int names_cap, int* count) {
        profiling = true;
        prof_names.clear();
        int rc = persist_step(R, st);
        profiling = false;
        prof_names.clear();
        if (rc) return rc;
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail(RWKV_E_CUDA, "profile: persistent step failed");
        const bool small = sp_eligible(R);
        const int nph = small ? sp_progs.at(R).nphases : pk_progs.at(R).nphases;
        const std::vector<std::string>& pnames = small ? sp_progs.at(R).names : pk_progs.at(R).names;
        pk_last_trace.resize(pk::T_END);
        cudaMemcpy(pk_last_trace.data(), pk_trace, pk::T_END * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        std::vector<unsigned long long> t(nph + 1);
        cudaMemcpy(t.data(), pk_trace, t.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        std::string all;
        int n = 0;
        for (int p = 0; p < nph; p++) {
            if (n < cap) ms[n++] = (float)((t[p + 1] - t[p]) * 1e-6);
            all += pnames[p];
            all += "\n";
        }
        *count = n;
        if (names && names_cap > 0) {
            strncpy(names, all.c_str(), names_cap - 1);
            names[names_cap - 1] = 0;
        }
        return check_launch("rwkv_x070_profile_step");
    }

    // graph_step on any stream, the legacy default stream included.
    int graph_step_any(int R, cudaStream_t st) {
        if (st != nullptr) return graph_step(R, st);
        cudaEventRecord(ev_in, st);
        cudaStreamWaitEvent(own, ev_in, 0);
        int rc = graph_step(R, own);
        cudaEventRecord(ev_out, own);
        cudaStreamWaitEvent(st, ev_out, 0);
        return rc;
    }

    // ----- parallel prefill (bodyWithState over right-padded prompts)

    std::vector<void*> pf_allocs;
    int pf_cap = 0;      // token rows the block buffers hold
    int pf_prompt_cap = 0;
    float *pf_x = nullptr, *pf_ln1 = nullptr, *pf_ln2 = nullptr, *pf_r = nullptr, *pf_k = nullptr, *pf_v = nullptr;
    float *pf_w = nullptr, *pf_a = nullptr, *pf_g = nullptr, *pf_vv = nullptr, *pf_vfirst = nullptr;
    float *pf_aw = nullptr, *pf_bw = nullptr, *pf_y = nullptr, *pf_keytmp = nullptr;
    void *pf_mix = nullptr, *pf_hidden = nullptr, *pf_tail = nullptr, *pf_xk = nullptr, *pf_ffn = nullptr;
    void *pf_z = nullptr, *pf_ws = nullptr;
    int32_t *pf_ids = nullptr, *pf_len = nullptr, *pf_prompt = nullptr, *pf_keep = nullptr;
    float* pf_gather = nullptr;  // one layer of WKV state rows, for the row drop

    void pf_free() {
        for (void* p : pf_allocs) cudaFree(p);
        pf_allocs.clear();
        pf_cap = 0;
    }
    template <typename T>
    T* pf_alloc(size_t n, bool& bad) {
        void* p = nullptr;
        if (bad || cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)) != cudaSuccess) {
            bad = true;
            return nullptr;
        }
        pf_allocs.push_back(p);
        return (T*)p;
    }
    // Block buffers for `ntok` token rows (allocated on first use, grown when
    // a larger block comes; the model keeps them until it is destroyed).
    int ensure_prefill(int ntok, int Ts, int rows) {
        const int64_t ws_need = wkv7_chunk_workspace(rows, Ts, H);
        if (ntok <= pf_cap && ws_need <= pf_ws_bytes) return RWKV_OK;
        cudaDeviceSynchronize();  // a previous block may still use the old buffers
        pf_free();
        bool bad = false;
        const size_t NC = (size_t)ntok * C;
        float** f32s[] = {&pf_x, &pf_ln1, &pf_ln2, &pf_r, &pf_k, &pf_v, &pf_w, &pf_a, &pf_g, &pf_vv, &pf_vfirst,
                          &pf_aw, &pf_bw, &pf_y};
        for (float** q : f32s) *q = pf_alloc<float>(NC, bad);
        pf_mix = pf_alloc<char>(6 * NC * act_bytes, bad);
        pf_hidden = pf_alloc<char>((size_t)ntok * hid * act_bytes, bad);
        pf_tail = pf_alloc<char>(NC * act_bytes, bad);
        pf_xk = pf_alloc<char>(NC * act_bytes, bad);
        pf_ffn = pf_alloc<char>((size_t)ntok * F * act_bytes, bad);
        pf_z = pf_alloc<char>((size_t)3 * ntok * LORA_MAX_RANK * act_bytes, bad);
        pf_keytmp = pf_alloc<float>((size_t)ntok * F, bad);
        pf_ws_bytes = std::max<int64_t>(ws_need, wkv7_chunk_workspace(std::max(1, ntok / 16), 16, H));
        pf_ws = pf_alloc<char>((size_t)pf_ws_bytes, bad);
        pf_ids = pf_alloc<int32_t>(ntok, bad);
        pf_len = pf_alloc<int32_t>(Rmax, bad);
        pf_keep = pf_alloc<int32_t>(Rmax, bad);
        pf_gather = pf_alloc<float>(std::max((size_t)Rmax * H * 4096, (size_t)Rmax * C), bad);
        if (bad) {
            pf_free();
            return fail(RWKV_E_CUDA, "prefill: block buffer allocation failed (%d token rows)", ntok);
        }
        pf_cap = ntok;
        return RWKV_OK;
    }
    int64_t pf_ws_bytes = 0;

    // Block size: Ts positions per row, a multiple of 16, rows * Ts <= PF_TOKENS.
    int prefill_block(int rows, int T) const {
        const int T16 = (T + 15) / 16 * 16;
        const int fit = std::max(16, PF_TOKENS / rows / 16 * 16);
        return std::min(T16, fit);
    }

    // One block of Ts positions through every layer (rows' state advances);
    // rows whose last real token lies in the block get ln_out of it in lnout.
    template <typename A>
    int prefill_block_body(const int32_t* prompt, int T, int rows, int p0, int Ts, cudaStream_t st) {
        const int N = rows * Ts;
        const size_t NC = (size_t)N * C;
        const int aout = this->aout();
        A* mixp = (A*)pf_mix;
        A* hidp = (A*)pf_hidden;
        x070_pf_ids_kernel<<<(N + 255) / 256, 256, 0, st>>>(prompt, T, p0, Ts, rows, pf_ids);
        x070_embed_kernel<<<N, GLUE_T, 0, st>>>(pf_ids, emb.wq, emb.sc, emb.bi, emb.dense, ln0w, ln0b, pf_x, C, V);
        int rc = check_launch("x070 prefill embed");
        if (rc) return rc;
        auto rows_launch = [&](auto&& f, const char* name) { return row_launch(f, name); };
        for (int l = 0; l < L; l++) {
            LayerW& w = lw[l];
            float* ts = tshift + (size_t)l * Rmax * C;
            float* cs = cshift + (size_t)l * Rmax * C;
            float* st8 = wkv + (size_t)l * Rmax * H * 64 * 64;
            if ((rc = rows_launch([&]<int GV>() {
                     x070_ln_out_kernel<float, GV><<<N, GLUE_T, 0, st>>>(pf_x, w.ln1w, w.ln1b, pf_ln1, C);
                     x070_pf_tmix_mix_kernel<A, GV><<<N, GLUE_T, 0, st>>>(pf_ln1, ts, w.coef6, mixp, N, Ts, C);
                     return cudaGetLastError();
                 }, "x070 prefill tmix input")))
                return rc;
            auto M = [&](int m) { return (const void*)(mixp + (size_t)m * NC); };
            GemvJobs J{};
            J.j[0] = qjob(w.r, M(0), C, ACT_NONE, OUT_F32, pf_r, C);
            J.j[1] = qjob(w.k, M(2), C, ACT_NONE, OUT_F32, pf_k, C);
            J.j[2] = qjob(w.v, M(3), C, ACT_NONE, OUT_F32, pf_v, C);
            if ((rc = gemv(0, J, 3, N, st))) return rc;
            {
                const LoraJob lj[3] = {{&w.ad[AD_R], M(0), C, C, C, pf_r, C}, {&w.ad[AD_K], M(2), C, C, C, pf_k, C},
                                       {&w.ad[AD_V], M(3), C, C, C, pf_v, C}};
                if ((rc = lora_apply<A>(lj, 3, N, st, pf_z, pf_cap))) return rc;
            }
            GemvJobs D{};
            int nd = 0;
            D.j[nd++] = hjob(w.wA, rw, C, M(1), C, ACT_TANH, aout, hidp, hid);
            D.j[nd++] = hjob(w.aA, ra, C, M(4), C, ACT_NONE, aout, hidp + rw, hid);
            D.j[nd++] = hjob(w.gA, rg, C, M(5), C, ACT_SIGMOID, aout, hidp + rw + ra, hid);
            if (l > 0) D.j[nd++] = hjob(w.vA, rv, C, M(3), C, ACT_NONE, aout, hidp + rw + ra + rg, hid);
            if ((rc = gemv(1, D, nd, N, st))) return rc;
            GemvJobs U{};
            int nu = 0;
            U.j[nu++] = hjob(w.wB, C, rw, hidp, hid, ACT_DECAY, OUT_F32, pf_w, C, w.wbias);
            U.j[nu++] = hjob(w.aB, C, ra, hidp + rw, hid, ACT_SIGMOID_BIAS, OUT_F32, pf_a, C, w.abias);
            U.j[nu++] = hjob(w.gB, C, rg, hidp + rw + ra, hid, ACT_NONE, OUT_F32, pf_g, C);
            if (l > 0) U.j[nu++] = hjob(w.vB, C, rv, hidp + rw + ra + rg, hid, ACT_SIGMOID_BIAS, OUT_F32, pf_vv, C, w.vbias);
            if ((rc = gemv(1, U, nu, N, st))) return rc;
            x070_pf_prep_kernel<<<dim3(N, (H + 7) / 8), 256, 0, st>>>(pf_w, pf_k, pf_v, pf_a, pf_vv, pf_vfirst, pf_aw,
                                                                     pf_bw, w.kkw, w.kaw, pf_len, p0, Ts, H, (int)(l == 0));
            if ((rc = check_launch("x070_pf_prep_kernel"))) return rc;
            // the state advances in place: each scan CTA reads and writes only its own state rows
            if ((rc = launch_wkv7_chunk_fwd(RWKV_F32, pf_r, pf_w, pf_k, pf_v, pf_aw, pf_bw, st8, pf_y, st8, nullptr,
                                            nullptr, rows, Ts, H, pf_ws, st)))
                return rc;
            x070_pf_tail_kernel<A><<<dim3(N, (H + 7) / 8), 256, 0, st>>>(pf_y, pf_r, pf_k, pf_v, w.rkw, w.lnxw, w.lnxb,
                                                                        pf_g, (A*)pf_tail, H);
            if ((rc = check_launch("x070_pf_tail_kernel"))) return rc;
            GemvJobs O{};
            O.j[0] = qjob(w.o, pf_tail, C, ACT_NONE, OUT_ADD_F32, pf_x, C);
            if ((rc = gemv(0, O, 1, N, st))) return rc;
            {
                const LoraJob lj[1] = {{&w.ad[AD_O], pf_tail, C, C, C, pf_x, C}};
                if ((rc = lora_apply<A>(lj, 1, N, st, pf_z, pf_cap))) return rc;
            }
            if ((rc = rows_launch([&]<int GV>() {
                     x070_ln_out_kernel<float, GV><<<N, GLUE_T, 0, st>>>(pf_x, w.ln2w, w.ln2b, pf_ln2, C);
                     x070_pf_cmix_mix_kernel<A, GV><<<N, GLUE_T, 0, st>>>(pf_ln2, cs, w.cxk, (A*)pf_xk, Ts, C);
                     return cudaGetLastError();
                 }, "x070 prefill cmix input")))
                return rc;
            GemvJobs K{};
            if (!w.ad[AD_KEY].on()) {
                K.j[0] = qjob(w.key, pf_xk, C, ACT_RELU2, aout, pf_ffn, F);
                if ((rc = gemv(0, K, 1, N, st))) return rc;
            } else {
                K.j[0] = qjob(w.key, pf_xk, C, ACT_NONE, OUT_F32, pf_keytmp, F);
                if ((rc = gemv(0, K, 1, N, st))) return rc;
                const LoraJob lj[1] = {{&w.ad[AD_KEY], pf_xk, C, C, F, pf_keytmp, F}};
                if ((rc = lora_apply<A>(lj, 1, N, st, pf_z, pf_cap))) return rc;
                const int n = N * F;
                x070_relu2_cast_kernel<A><<<std::min((n + 255) / 256, 4 * sm_count), 256, 0, st>>>(pf_keytmp, (A*)pf_ffn, n);
                if ((rc = check_launch("x070_relu2_cast_kernel"))) return rc;
            }
            GemvJobs Vv{};
            Vv.j[0] = qjob(w.value, pf_ffn, F, ACT_NONE, OUT_ADD_F32, pf_x, C);
            if ((rc = gemv(0, Vv, 1, N, st))) return rc;
            {
                const LoraJob lj[1] = {{&w.ad[AD_VALUE], pf_ffn, F, F, C, pf_x, C}};
                if ((rc = lora_apply<A>(lj, 1, N, st, pf_z, pf_cap))) return rc;
            }
            x070_pf_commit_kernel<<<rows, 256, 0, st>>>(pf_ln1, pf_ln2, ts, cs, pf_len, p0, Ts, C);
            if ((rc = check_launch("x070_pf_commit_kernel"))) return rc;
        }
        return rows_launch([&]<int GV>() {
            x070_pf_lnout_kernel<A, GV><<<rows, GLUE_T, 0, st>>>(pf_x, lnow, lnob, (A*)lnout, pf_len, p0, Ts, C);
            return cudaGetLastError();
        }, "x070_pf_lnout_kernel");
    }

    // Prompts [rows, T] (device, right-padded) with host lengths (nullptr: all
    // T): every block, then the head over each row's last real token and the
    // greedy argmax into ids.  Continues from the rows' current state.
    int prefill(const int32_t* prompt, const int32_t* len_host, int rows, int T, cudaStream_t st) {
        std::vector<int32_t> lens(rows, T);
        int maxlen = 0;
        for (int i = 0; i < rows; i++) {
            if (len_host) lens[i] = len_host[i];
            RWKV_REQUIRE(lens[i] >= 1 && lens[i] <= T, RWKV_E_SHAPE,
                         "prefill: row %d length %d not in 1..%d (no empty prompt)", i, lens[i], T);
            maxlen = std::max(maxlen, lens[i]);
        }
        const int Ts = prefill_block(rows, maxlen);
        if (int rc = ensure_prefill(rows * Ts, Ts, rows)) return rc;
        cudaMemcpyAsync(pf_len, lens.data(), rows * sizeof(int32_t), cudaMemcpyHostToDevice, st);
        for (int p0 = 0; p0 < maxlen; p0 += Ts) {
            const int rc = bf16act ? prefill_block_body<__nv_bfloat16>(prompt, T, rows, p0, Ts, st)
                           : f16act ? prefill_block_body<__half>(prompt, T, rows, p0, Ts, st)
                                    : prefill_block_body<float>(prompt, T, rows, p0, Ts, st);
            if (rc) return rc;
        }
        // the head over the rows' hidden states, then greedy ids: the decode step's tail
        GemvJobs Hd{};
        Hd.j[0] = qjob(head, lnout, C, ACT_NONE, OUT_F32, logits, V);
        int rc = gemv(0, Hd, 1, rows, st);
        if (rc) return rc;
        {
            const LoraJob lj[1] = {{&head_ad, lnout, C, C, V, logits, V}};
            if ((rc = bf16act ? lora_apply<__nv_bfloat16>(lj, 1, rows, st)
                      : f16act ? lora_apply<__half>(lj, 1, rows, st) : lora_apply<float>(lj, 1, rows, st)))
                return rc;
        }
        x070_argmax_kernel<<<dim3((V + ARGMAX_SLICE - 1) / ARGMAX_SLICE, rows), GLUE_T, 0, st>>>(logits, V, amax_keys);
        x070_argmax_finish_kernel<<<(rows + 127) / 128, 128, 0, st>>>(amax_keys, ids, rows);
        return check_launch("x070 prefill head");
    }

    // Rows keep[0..nkeep) of the state move to rows 0..nkeep-1 (in order).
    int gather_rows(const int32_t* keep_host, int nkeep, cudaStream_t st) {
        if (!pf_gather) return fail(RWKV_E_CUDA, "gather_rows: no buffers");
        cudaMemcpyAsync(pf_keep, keep_host, nkeep * sizeof(int32_t), cudaMemcpyHostToDevice, st);
        const int64_t ES = (int64_t)H * 4096;
        const int grid = 4 * sm_count;
        for (int l = 0; l < L; l++) {
            float* blocks[3] = {wkv + (size_t)l * Rmax * ES, tshift + (size_t)l * Rmax * C, cshift + (size_t)l * Rmax * C};
            const int64_t E[3] = {ES, C, C};
            for (int q = 0; q < 3; q++) {
                x070_gather_rows_kernel<<<grid, 256, 0, st>>>(blocks[q], pf_gather, pf_keep, nkeep, E[q]);
                cudaMemcpyAsync(blocks[q], pf_gather, (size_t)nkeep * E[q] * 4, cudaMemcpyDeviceToDevice, st);
            }
        }
        return check_launch("x070_gather_rows_kernel");
    }

    // Device copy of host prompts [rows, T] for generate (its own buffer,
    // grown when needed, freed with the model).
    int stage_prompt(const int32_t* host, int rows, int T, cudaStream_t st) {
        const int n = rows * T;
        if (n > pf_prompt_cap) {
            cudaStreamSynchronize(st);  // an earlier prefill may still read the old buffer
            if (pf_prompt) cudaFree(pf_prompt);
            pf_prompt = nullptr;
            pf_prompt_cap = 0;
            if (cudaMalloc(&pf_prompt, (size_t)n * 4) != cudaSuccess) {
                pf_prompt = nullptr;
                return fail(RWKV_E_CUDA, "generate: prompt buffer allocation failed");
            }
            pf_prompt_cap = n;
        }
        cudaMemcpyAsync(pf_prompt, host, (size_t)n * 4, cudaMemcpyHostToDevice, st);
        return RWKV_OK;
    }

    int launches_per_step() const {
        int n = 1 + L * 10 + 4 + (head_ad.on() ? 2 : 0);
        for (const LayerW& w : lw) {
            if (w.ad[AD_R].on() || w.ad[AD_K].on() || w.ad[AD_V].on()) n += 2;
            n += (w.ad[AD_O].on() ? 2 : 0) + (w.ad[AD_KEY].on() ? 3 : 0) + (w.ad[AD_VALUE].on() ? 2 : 0);
        }
        return n;
    }
};

}  // namespace rwkv

using namespace rwkv;

extern "C" {

int rwkv_x070_create(const rwkv_x070_config* cfg, rwkv_x070_t* out) {
    RWKV_REQUIRE(cfg && out, RWKV_E_NULL, "rwkv_x070_create: NULL argument");
    const rwkv_x070_config& c = *cfg;
    RWKV_REQUIRE(c.n_layer >= 1 && c.vocab >= 1 && c.max_rows >= 1, RWKV_E_SHAPE, "rwkv_x070_create: sizes");
    RWKV_REQUIRE(c.head_size == 64 && c.n_embd % 64 == 0 && c.n_embd <= GLUE_T * GLUE_PER, RWKV_E_UNSUPPORTED,
                 "rwkv_x070_create: n_embd %d must be a multiple of 64 up to 4096, head 64", c.n_embd);
    RWKV_REQUIRE(c.ffn % 64 == 0, RWKV_E_UNSUPPORTED, "rwkv_x070_create: ffn %d must be a multiple of 64", c.ffn);
    RWKV_REQUIRE(c.rank_w % 16 == 0 && c.rank_a % 16 == 0 && c.rank_v % 16 == 0 && c.rank_g % 16 == 0,
                 RWKV_E_UNSUPPORTED, "rwkv_x070_create: low-rank sizes must be multiples of 16");
    RWKV_REQUIRE((c.quant_bits == 4 && c.quant_group == 64) || c.quant_bits == 0, RWKV_E_UNSUPPORTED,
                 "rwkv_x070_create: the base must be 4-bit group-64 (quant_bits 4) or dense bf16 (quant_bits 0)");
    RWKV_REQUIRE(c.act_dtype == RWKV_F16 || c.act_dtype == RWKV_F32 || c.act_dtype == RWKV_BF16, RWKV_E_DTYPE,
                 "rwkv_x070_create: act dtype");
    // a tensor-core product takes both operands in one type: the 4-bit base is
    // dequantised into fp16, the dense base is bf16
    RWKV_REQUIRE(c.act_dtype == RWKV_F32 || (c.quant_bits == 4) == (c.act_dtype == RWKV_F16), RWKV_E_DTYPE,
                 "rwkv_x070_create: fp16 activations go with the 4-bit base, bf16 with the dense bf16 base");
    X070* m = new X070(c);
    if (m->alloc_failed) {
        delete m;
        return fail(RWKV_E_CUDA, "rwkv_x070_create: device allocation failed");
    }
    *out = reinterpret_cast<rwkv_x070_t>(m);
    return ok();
}

int rwkv_x070_destroy(rwkv_x070_t h) {
    delete reinterpret_cast<X070*>(h);
    return ok();
}

int rwkv_x070_set_param(rwkv_x070_t h, const char* name, const float* host, int64_t n) {
    RWKV_REQUIRE(h && name && host, RWKV_E_NULL, "rwkv_x070_set_param: NULL argument");
    return reinterpret_cast<X070*>(h)->set_param(name, host, n);
}

int rwkv_x070_init_random(rwkv_x070_t h, uint64_t seed) {
    RWKV_REQUIRE(h, RWKV_E_NULL, "rwkv_x070_init_random: NULL handle");
    return reinterpret_cast<X070*>(h)->init_random(seed);
}

int rwkv_x070_reset_state(rwkv_x070_t h, int rows, rwkv_stream_t stream) {
    RWKV_REQUIRE(h, RWKV_E_NULL, "rwkv_x070_reset_state: NULL handle");
    X070& m = *reinterpret_cast<X070*>(h);
    RWKV_REQUIRE(rows >= 1 && rows <= m.Rmax, RWKV_E_SHAPE, "rows %d not in 1..%d", rows, m.Rmax);
    cudaStream_t st = (cudaStream_t)stream;
    for (int l = 0; l < m.L; l++) {
        cudaMemsetAsync(m.wkv + (size_t)l * m.Rmax * m.H * 4096, 0, (size_t)rows * m.H * 4096 * 4, st);
        cudaMemsetAsync(m.tshift + (size_t)l * m.Rmax * m.C, 0, (size_t)rows * m.C * 4, st);
        cudaMemsetAsync(m.cshift + (size_t)l * m.Rmax * m.C, 0, (size_t)rows * m.C * 4, st);
    }
    return check_launch("rwkv_x070_reset_state");
}

int rwkv_x070_step(rwkv_x070_t h, const int32_t* ids, int rows, float* logits, int32_t* next_ids,
                   int use_graph, rwkv_stream_t stream) {
    RWKV_REQUIRE(h, RWKV_E_NULL, "rwkv_x070_step: NULL handle");
    X070& m = *reinterpret_cast<X070*>(h);
    RWKV_REQUIRE(rows >= 1 && rows <= m.Rmax, RWKV_E_SHAPE, "rows %d not in 1..%d", rows, m.Rmax);
    cudaStream_t st = (cudaStream_t)stream;
    // a GEMM wait of an earlier step gave up: report it once, clear it, run nothing
    if (m.gflag.take(st))
        return fail(RWKV_E_TIMEOUT, "rwkv_x070_step: a tensor-core GEMM wait of an earlier step gave up; "
                                    "the state is not valid (flag cleared, nothing launched)");
    if (ids) cudaMemcpyAsync(m.ids, ids, rows * 4, cudaMemcpyDeviceToDevice, st);
    int rc = use_graph ? m.graph_step_any(rows, st) : m.run_step(rows, st);
    if (rc) return rc;
    if (logits) cudaMemcpyAsync(logits, m.logits, (size_t)rows * m.V * 4, cudaMemcpyDeviceToDevice, st);
    if (next_ids) cudaMemcpyAsync(next_ids, m.ids, rows * 4, cudaMemcpyDeviceToDevice, st);
    return check_launch("rwkv_x070_step");
}

int rwkv_x070_generate(rwkv_x070_t h, const int32_t* prompt_host, int rows, int prompt_len,
                       int n_new, int32_t* out_host, rwkv_stream_t stream) {
    RWKV_REQUIRE(h && prompt_host && out_host, RWKV_E_NULL, "rwkv_x070_generate: NULL argument");
    X070& m = *reinterpret_cast<X070*>(h);
    RWKV_REQUIRE(rows >= 1 && rows <= m.Rmax && prompt_len >= 1 && n_new >= 0, RWKV_E_SHAPE,
                 "rwkv_x070_generate: rows %d prompt %d new %d", rows, prompt_len, n_new);
    cudaStream_t st = (cudaStream_t)stream;
    if (m.gflag.take(st))
        return fail(RWKV_E_TIMEOUT, "rwkv_x070_generate: a tensor-core GEMM wait of an earlier step gave up "
                                    "(flag cleared, nothing launched)");
    std::vector<int32_t> col(rows);
    // the prompt in parallel (prefill), then one token per step
    if (int rc = m.stage_prompt(prompt_host, rows, prompt_len, st)) return rc;
    if (int rc = m.prefill(m.pf_prompt, nullptr, rows, prompt_len, st)) return rc;
    for (int s = 0; s < n_new; s++) {
        cudaMemcpyAsync(col.data(), m.ids, rows * 4, cudaMemcpyDeviceToHost, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail(RWKV_E_CUDA, "generate: sync failed");
        for (int n = 0; n < rows; n++) out_host[(size_t)n * n_new + s] = col[n];
        if (s + 1 < n_new)
            if (int rc = m.graph_step_any(rows, st)) return rc;
    }
    if (int rc = m.gflag.status(st, "rwkv_x070_generate")) return rc;
    return check_launch("rwkv_x070_generate");
}

int rwkv_x070_prefill(rwkv_x070_t h, const int32_t* ids, const int32_t* lengths_host, int rows, int T,
                      float* logits, int32_t* next_ids, rwkv_stream_t stream) {
    RWKV_REQUIRE(h && ids, RWKV_E_NULL, "rwkv_x070_prefill: NULL argument");
    X070& m = *reinterpret_cast<X070*>(h);
    RWKV_REQUIRE(rows >= 1 && rows <= m.Rmax && T >= 1, RWKV_E_SHAPE, "rwkv_x070_prefill: rows %d (1..%d), T %d",
                 rows, m.Rmax, T);
    cudaStream_t st = (cudaStream_t)stream;
    if (m.gflag.take(st))
        return fail(RWKV_E_TIMEOUT, "rwkv_x070_prefill: a tensor-core GEMM wait of an earlier call gave up "
                                    "(flag cleared, nothing launched)");
    if (int rc = m.prefill(ids, lengths_host, rows, T, st)) return rc;
    if (logits) cudaMemcpyAsync(logits, m.logits, (size_t)rows * m.V * 4, cudaMemcpyDeviceToDevice, st);
    if (next_ids) cudaMemcpyAsync(next_ids, m.ids, rows * 4, cudaMemcpyDeviceToDevice, st);
    return check_launch("rwkv_x070_prefill");
}

int rwkv_x070_generate_batch(rwkv_x070_t h, const int32_t* prompts_host, const int32_t* lengths_host, int rows,
                             int max_len, int n_new, const int32_t* stop_host, int n_stop, int32_t* out_host,
                             int32_t* out_len_host, rwkv_stream_t stream) {
    RWKV_REQUIRE(h && prompts_host && out_host && out_len_host, RWKV_E_NULL, "rwkv_x070_generate_batch: NULL argument");
    RWKV_REQUIRE(n_stop == 0 || stop_host, RWKV_E_NULL, "rwkv_x070_generate_batch: NULL stop list");
    X070& m = *reinterpret_cast<X070*>(h);
    RWKV_REQUIRE(rows >= 1 && rows <= m.Rmax && max_len >= 1 && n_new >= 0 && n_stop >= 0, RWKV_E_SHAPE,
                 "rwkv_x070_generate_batch: rows %d prompt %d new %d stops %d", rows, max_len, n_new, n_stop);
    cudaStream_t st = (cudaStream_t)stream;
    if (m.gflag.take(st))
        return fail(RWKV_E_TIMEOUT, "rwkv_x070_generate_batch: a tensor-core GEMM wait of an earlier call gave up "
                                    "(flag cleared, nothing launched)");
    for (int i = 0; i < rows; i++) out_len_host[i] = 0;
    if (int rc = rwkv_x070_reset_state(h, rows, stream)) return rc;
    if (int rc = m.stage_prompt(prompts_host, rows, max_len, st)) return rc;
    if (int rc = m.prefill(m.pf_prompt, lengths_host, rows, max_len, st)) return rc;
    std::vector<int> alive(rows);
    for (int i = 0; i < rows; i++) alive[i] = i;
    std::vector<int32_t> col(rows), next, keep;
    for (int s = 0; s < n_new; s++) {
        const int na = (int)alive.size();
        cudaMemcpyAsync(col.data(), m.ids, na * 4, cudaMemcpyDeviceToHost, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail(RWKV_E_CUDA, "generate_batch: sync failed");
        next.clear();
        keep.clear();
        for (int r = 0; r < na; r++) {
            const int i = alive[r];
            const int32_t id = col[r];
            out_host[(size_t)i * n_new + out_len_host[i]++] = id;
            bool stop = false;
            for (int q = 0; q < n_stop && !stop; q++) stop = stop_host[q] == id;
            if (stop) continue;
            next.push_back(id);
            keep.push_back(r);
        }
        if (keep.empty() || s + 1 >= n_new) break;
        if ((int)keep.size() < na) {
            // finished rows leave the batch (RWKVBatchState.gather)
            if (int rc = m.gather_rows(keep.data(), (int)keep.size(), st)) return rc;
            std::vector<int> a2(keep.size());
            for (size_t q = 0; q < keep.size(); q++) a2[q] = alive[keep[q]];
            alive.swap(a2);
        }
        cudaMemcpyAsync(m.ids, next.data(), next.size() * 4, cudaMemcpyHostToDevice, st);
        if (int rc = m.graph_step_any((int)next.size(), st)) return rc;
    }
    if (int rc = m.gflag.status(st, "rwkv_x070_generate_batch")) return rc;
    return check_launch("rwkv_x070_generate_batch");
}

int rwkv_x070_status(rwkv_x070_t h, rwkv_stream_t stream) {
    RWKV_REQUIRE(h, RWKV_E_NULL, "rwkv_x070_status: NULL handle");
    return reinterpret_cast<X070*>(h)->gflag.status((cudaStream_t)stream, "rwkv_x070");
}

int rwkv_x070_inject_wait_error(rwkv_x070_t h, int host_record, rwkv_stream_t stream) {
    RWKV_REQUIRE(h, RWKV_E_NULL, "rwkv_x070_inject_wait_error: NULL handle");
    return reinterpret_cast<X070*>(h)->gflag.inject(host_record, (cudaStream_t)stream);
}

int rwkv_x070_profile_step(rwkv_x070_t h, int rows, float* ms_host, int cap, char* names_host,
                           int names_cap, int* count, rwkv_stream_t stream) {
    RWKV_REQUIRE(h && ms_host && count, RWKV_E_NULL, "rwkv_x070_profile_step: NULL argument");
    X070& m = *reinterpret_cast<X070*>(h);
    RWKV_REQUIRE(rows >= 1 && rows <= m.Rmax, RWKV_E_SHAPE, "rows %d not in 1..%d", rows, m.Rmax);
    return m.profile_step(rows, (cudaStream_t)stream, ms_host, cap, names_host, names_cap, count);
}

int rwkv_x070_set_param_rwkvq(rwkv_x070_t h, const char* name, int kind, int bits, const void* b1, int64_t n1,
                              const void* b2, int64_t n2, const void* b3, int64_t n3) {
    RWKV_REQUIRE(h && name, RWKV_E_NULL, "rwkv_x070_set_param_rwkvq: NULL argument");
    return reinterpret_cast<X070*>(h)->set_param_rwkvq(name, kind, bits, b1, n1, b2, n2, b3, n3);
}

int rwkv_x070_set_decode_path(rwkv_x070_t h, int path) {
    RWKV_REQUIRE(h, RWKV_E_NULL, "rwkv_x070_set_decode_path: NULL handle");
    RWKV_REQUIRE(path == 0 || path == 1, RWKV_E_SHAPE, "rwkv_x070_set_decode_path: path %d (0 or 1)", path);
    reinterpret_cast<X070*>(h)->decode_path = path;
    return ok();
}

int rwkv_x070_trace(rwkv_x070_t h, uint64_t* out_host, int cap, int* count) {
    RWKV_REQUIRE(h && out_host && count, RWKV_E_NULL, "rwkv_x070_trace: NULL argument");
    const auto& t = reinterpret_cast<X070*>(h)->pk_last_trace;
    const int n = std::min<int>(cap, (int)t.size());
    for (int i = 0; i < n; i++) out_host[i] = t[i];
    *count = n;
    return ok();
}

int rwkv_x070_decode_path(rwkv_x070_t h, int rows) {
    return h && reinterpret_cast<X070*>(h)->persist_eligible(rows) ? 1 : 0;
}

int64_t rwkv_x070_weight_bytes(rwkv_x070_t h) { return h ? reinterpret_cast<X070*>(h)->weight_bytes : 0; }

int rwkv_x070_launches_per_step(rwkv_x070_t h) {
    return h ? reinterpret_cast<X070*>(h)->launches_per_step() : 0;
}

}  // extern "C"
