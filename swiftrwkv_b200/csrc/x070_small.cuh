// Persistent x070 decode step for 1..8 rows: the whole step (embedding, 24
// layers of tmix / projections / WKV / cmix, ln_out, head, greedy argmax) in
// ONE cooperative launch of one CTA per SM, fp16 activations on the 4-bit
// group-64 base (X070Generation.swift:449-498 over BatchGenerate.swift:54-116's
// batch).
//
// Why: at 1..8 rows every projection is a GEMV that streams 2-10 MB of weights.
// Launched one kernel at a time each pays a launch, a pipeline that fills from
// HBM and a split-K tail (9-15 us for what HBM moves in 0.4-1.5 us), and the
// step is ~245 such launches.  Here the CTAs stay resident; the step is a
// program of phases separated by grid barriers, and weights -- which do not
// depend on the activations -- stream into a shared-memory ring ahead of the
// phase they belong to, across barriers, glue phases and layers.
//
// CTA = 320 threads: warp 0 streams weight pieces (cp.async, 16-byte chunks,
// completion counted on the slot's mbarrier), warp 1 idles, warps 2-9 are the
// workers: glue phases (the decode glue kernels' arithmetic, shared with the
// 9..64-row persistent kernel), and the GEMV phases.
//
// A GEMV phase is a list of tiles (job = matrix, 16 weight rows); a tile is 1..4
// pieces along K (4-bit: <= 2048 codes, fp16: <= 512 columns per piece) and
// belongs wholly to one CTA, so nothing is reduced across CTAs.  All eight
// worker warps share a piece, each taking a run of its 64-column groups:
// mma.sync m16n8k16 on the exact codes (fp16 1024 + q, less 1024) against the
// fp16 activations staged in shared memory, fp32 per-group scaling
// (scale * sum(q x) + bias * sum(x)) -- the <= 8-row GEMV numerics of
// gemm_w4_kernel.  At the tile's last piece the warps' partials are summed in
// warp order (deterministic) and the job's epilogue runs.
//
// Every wait is bounded in time and watches the device error flag; once it is
// set every role skips the rest of the program.
#pragma once

#include "x070_persist.cuh"

namespace rwkv {
namespace sp {

constexpr int THREADS = pk::THREADS;          // 320: producer warp, idle warp, 8 worker warps
constexpr int WT = pk::WT;                    // 256 worker threads
constexpr int TR = 16;                        // weight rows per tile
constexpr int KPQ = 2048, KPH = 512;          // K per piece: 4-bit codes / fp16 columns
constexpr int WROWB = 1056;                   // slot row pitch: 2048 codes or 512 fp16 + 32 B
constexpr int SBB = 2 * TR * 32 * 2;          // a piece's (scale, bias) block: [2][16][32] fp16
constexpr int SB_OFF = TR * WROWB;
constexpr int SLOT = SB_OFF + SBB;            // 18944 B
constexpr int KW = 4096;                      // activation window (columns) staged at a time
constexpr int XROW = KW + 8;                  // staged activation row pitch (fp16)

// Shared-memory layout for RB staged activation rows (RB >= the step's rows):
// the weight ring takes what the activation window leaves.
template <int RB>
struct Cfg {
    static constexpr int X_OFF = 0;
    static constexpr int G_OFF = X_OFF + RB * XROW * 2;
    static constexpr int RED_OFF = G_OFF + pk::GLUE_SMEM;       // warp partials [8][16][8] fp32
    static constexpr int P_OFF = RED_OFF + 8 * TR * 8 * 4;
    static constexpr int T_OFF = P_OFF + pk::MAX_PHASES * 16;
    static constexpr int W_OFF = (T_OFF + 32 + 127) & ~127;
    static constexpr int NS = (227 * 1024 - W_OFF - 16 * 8 - 128) / SLOT;  // ring slots
    static constexpr int B_OFF = W_OFF + NS * SLOT;
    static constexpr int SMEM = B_OFF + 2 * NS * 8;
    static_assert(NS >= 4 && SMEM <= 227 * 1024, "shared memory per CTA");
    static_assert(G_OFF % 16 == 0 && W_OFF % 128 == 0 && SLOT % 128 == 0, "alignment");
};

enum : int { FMT_Q4 = 0, FMT_F16 = 1 };

// One matrix of a GEMV phase: the runtime's job (weights, activations,
// epilogue); 4-bit: sbp = its (scale, bias) blocks, one SBB-byte block per
// (16-row tile, piece), in that order (x070_repack_sb_small_kernel).
struct Job {
    GemvJob g;
    const __half* sbp;
    int fmt;
    int np;  // pieces per tile
};

// A piece: rows [o0, o0 + 16) of job `job`, K columns [k0, k0 + kn); `last`:
// the tile's final piece (its epilogue runs after it).
struct Item {
    int job, o0, k0, kn, last, pad0, pad1, pad2;
};

// A phase: type (pk::PH_*), layer, and for GEMV phases the CTA's pieces
// items[ofs[cta] .. ofs[cta + 1]) with ofs = A.ofs + i0 (G + 1 entries).
struct Phase {
    int type, i0, layer, pad;
};

struct Args {
    pk::Args g;            // glue buffers, layers, barrier, error flag, trace
    const Job* jobs;
    const Item* items;
    const int* ofs;        // per GEMV phase: G + 1 offsets into items
    const Phase* phases;
    int nphases;
};

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 16-byte-multiple global -> shared copy counted on mbarrier `bar` (tx bytes).
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(saddr(bar))
                 : "memory");
}

// ---- producer (one thread of warp 0): this CTA's pieces of every GEMV phase,
// in program order, each into ring slot seq % NS once the workers have
// released it: one bulk copy per weight row (the row's K range of the piece)
// and, for 4-bit pieces, one for the piece's (scale, bias) block.
template <int NS>
__device__ void produce(const Args& A, const Phase* phs, unsigned char* ring, uint64_t* full, uint64_t* empty,
                        int* err, bool& ok) {
    const int G = gridDim.x, cta = blockIdx.x;
    int seq = 0;
    for (int p = 0; p < A.nphases && ok; p++) {
        const Phase ph = phs[p];
        if (ph.type != pk::PH_GEMM) continue;
        const int* ofs = A.ofs + ph.i0;
        const int i1 = ofs[cta + 1];
        for (int i = ofs[cta]; i < i1; i++, seq++) {
            const Item it = A.items[i];
            const Job& jb = A.jobs[it.job];
            const int s = seq % NS;
            if (seq >= NS && !tc::mbar_wait(empty + s, ((seq / NS) - 1) & 1, err)) {
                ok = false;
                break;
            }
            const uint32_t dst = saddr(ring + s * SLOT);
            const int nr = min(TR, jb.g.OUT - it.o0);
            const bool q4 = jb.fmt == FMT_Q4;
            const uint32_t rowb = q4 ? it.kn / 2 : it.kn * 2;
            tc::mbar_expect_tx(full + s, nr * rowb + (q4 ? SBB : 0));
            const char* w = q4 ? (const char*)jb.g.w + ((int64_t)it.o0 * jb.g.IN + it.k0) / 2
                               : (const char*)jb.g.w + ((int64_t)it.o0 * jb.g.IN + it.k0) * 2;
            const int64_t pitch = q4 ? jb.g.IN / 2 : (int64_t)jb.g.IN * 2;
            for (int r = 0; r < nr; r++) bulk_copy(dst + r * WROWB, w + r * pitch, rowb, full + s);
            if (q4) bulk_copy(dst + SB_OFF, jb.sbp + ((size_t)(it.o0 / TR) * jb.np + it.k0 / KPQ) * (SBB / 2), SBB, full + s);
        }
    }
    // every copy issued here lands before the CTA may exit
    for (int q = max(0, seq - NS); q < seq; q++)
        if (!tc::mbar_wait_own(full + (q % NS), (q / NS) & 1, err)) ok = false;
}

// (scale, bias) of a 4-bit group-64 matrix [OUT, IN/64] into one SBB-byte
// block per (16-row tile, 2048-column piece), tile-major: [2][16][32] fp16
// (scales, then biases; rows past OUT and groups past IN are zero).
__global__ void x070_repack_sb_small_kernel(const __half* __restrict__ sc, const __half* __restrict__ bi,
                                            __half* __restrict__ out, int OUT, int IN) {
    constexpr int BH = SBB / 2;  // halves per block
    const int np = (IN + KPQ - 1) / KPQ, nt = (OUT + TR - 1) / TR, NG = IN / 64;
    const int64_t n = (int64_t)nt * np * BH;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = e / BH;
        const int within = (int)(e - blk * BH);
        const int tile = (int)(blk / np), piece = (int)(blk - (int64_t)tile * np);
        const int hb = within / (TR * 32), rr = (within / 32) % TR, gi = within % 32;
        const int o = tile * TR + rr, gg = piece * (KPQ / 64) + gi;
        __half v = __ushort_as_half(0);
        if (o < OUT && gg < NG) v = (hb ? bi : sc)[(int64_t)o * NG + gg];
        out[e] = v;
    }
}

// ---- activations: rows 0..R-1 of the job's x, columns [k0, k0 + KW) (clipped
// to IN, zero past IN up to whole 64-column groups), into the staged window
// xs[R][XROW] (fp16).  All 256 workers; the caller brackets it with worker
// barriers.
__device__ void stage_x(const GemvJob& g, int R, int k0, __half* xs, int wt) {
    const int kn = min(KW, g.IN - k0);
    const int kpad = (kn + 63) & ~63;  // whole 64-column groups are read
    const int cpr = kpad / 8;          // 16-byte chunks per row
    for (int e = wt; e < R * cpr; e += WT) {
        const int n = e / cpr, c = e - n * cpr;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (8 * c < kn) v = *reinterpret_cast<const uint4*>((const __half*)g.x + (int64_t)n * g.x_stride + k0 + 8 * c);
        *reinterpret_cast<uint4*>(xs + n * XROW + 8 * c) = v;
    }
}

// ---- one piece on the worker warps: warp w (0..7) accumulates its share of
// the piece's K into acc (rows g, g+8 of the 16-row tile x activation rows 2t,
// 2t+1: the m16n8k16 accumulator fragment).  slot: the piece's weights;
// xs: the staged activations (R rows; the MMA's columns R..7 read row R-1
// and are discarded), whose column 0 is K column xk0.
__device__ __forceinline__ void piece_q4(const unsigned char* slot, const __half* xs, int kx, int kn, int R, int w,
                                         int lane, float (&acc)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const int ngr = kn / 64, ga = ngr * w / 8, gb = ngr * (w + 1) / 8;
    const __half* sc = reinterpret_cast<const __half*>(slot + SB_OFF);
    const __half* bi = sc + TR * 32;
#pragma unroll 4
    for (int gi = ga; gi < gb; gi++) {
        // B fragments (nibble-pair order) and the group sums of activation rows 2t, 2t+1
        const __half* xr = xs + min(g, R - 1) * XROW + kx + 64 * gi;
        const uint4 lo = *reinterpret_cast<const uint4*>(xr + 16 * t);
        const uint4 hi = *reinterpret_cast<const uint4*>(xr + 16 * t + 8);
        const uint32_t h[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        uint32_t b[4][2];
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const uint32_t sel = (kk & 1) ? 0x7632u : 0x5410u;
            b[kk][0] = __byte_perm(h[kk >> 1], h[(kk >> 1) + 2], sel);
            b[kk][1] = __byte_perm(h[(kk >> 1) + 4], h[(kk >> 1) + 6], sel);
        }
        float sx = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
            sx += f.x + f.y;
        }
        sx += __shfl_xor_sync(0xffffffffu, sx, 1);
        sx += __shfl_xor_sync(0xffffffffu, sx, 2);
        const float X0 = __shfl_sync(0xffffffffu, sx, 8 * t), X1 = __shfl_sync(0xffffffffu, sx, 8 * t + 4);
        // A fragments: words 2t, 2t+1 of the group in rows g and g + 8, exact codes
        const uint2 A0 = *reinterpret_cast<const uint2*>(slot + g * WROWB + (8 * gi + 2 * t) * 4);
        const uint2 A1 = *reinterpret_cast<const uint2*>(slot + (g + 8) * WROWB + (8 * gi + 2 * t) * 4);
        uint32_t a[4][4];
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            a[kk][0] = nib_pair(A0.x, kk);
            a[kk][1] = nib_pair(A1.x, kk);
            a[kk][2] = nib_pair(A0.y, kk);
            a[kk][3] = nib_pair(A1.y, kk);
        }
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < 4; kk++) mma16816(d, a[kk], b[kk]);
        const float s0 = __half2float(sc[g * 32 + gi]), s1 = __half2float(sc[(g + 8) * 32 + gi]);
        const float c0 = __half2float(bi[g * 32 + gi]), c1 = __half2float(bi[(g + 8) * 32 + gi]);
        acc[0] = fmaf(s0, d[0], fmaf(c0, X0, acc[0]));
        acc[1] = fmaf(s0, d[1], fmaf(c0, X1, acc[1]));
        acc[2] = fmaf(s1, d[2], fmaf(c1, X0, acc[2]));
        acc[3] = fmaf(s1, d[3], fmaf(c1, X1, acc[3]));
    }
}

__device__ __forceinline__ void piece_f16(const unsigned char* slot, const __half* xs, int kx, int kn, int R, int w,
                                          int lane, float (&acc)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const int nks = kn / 16, ka = nks * w / 8, kb = nks * (w + 1) / 8;
    const __half* w0 = reinterpret_cast<const __half*>(slot + g * WROWB) + 2 * t;
    const __half* w1 = reinterpret_cast<const __half*>(slot + (g + 8) * WROWB) + 2 * t;
    const __half* xr = xs + min(g, R - 1) * XROW + kx + 2 * t;
#pragma unroll 4
    for (int ks = ka; ks < kb; ks++) {
        const int c = 16 * ks;
        const uint32_t a[4] = {*reinterpret_cast<const uint32_t*>(w0 + c), *reinterpret_cast<const uint32_t*>(w1 + c),
                               *reinterpret_cast<const uint32_t*>(w0 + c + 8),
                               *reinterpret_cast<const uint32_t*>(w1 + c + 8)};
        const uint32_t b[2] = {*reinterpret_cast<const uint32_t*>(xr + c), *reinterpret_cast<const uint32_t*>(xr + c + 8)};
        mma16816(acc, a, b);
    }
}


// Grid barrier among the workers of every CTA (pk::grid_barrier), with the
// status made uniform over the CTA: false when the wait failed or the error
// flag is set, as read by one thread after the barrier.
__device__ __forceinline__ bool grid_sync(unsigned int* bar, unsigned int gen, int* err, int wt, int* flag) {
    const bool okb = pk::grid_barrier(bar, gen, err, wt, flag);
    if (wt == 0) *flag = okb && *(volatile int*)err == 0;
    pk::wbar(1, WT);
    const bool r = *flag != 0;
    pk::wbar(1, WT);
    return r;
}

// Sum of the eight warps' partials of a 16-row tile (warp order) and the job's
// epilogue for its R activation rows; red: [8][16][8] fp32.
__device__ __forceinline__ void tile_out(const GemvJob& g, int o0, int R, float* red, const float (&acc)[4], int w,
                                         int lane, int wt, bool ok) {
    const int gq = lane >> 2, t = lane & 3;
    float* mine = red + w * TR * 8;
    mine[gq * 8 + 2 * t] = acc[0];
    mine[gq * 8 + 2 * t + 1] = acc[1];
    mine[(gq + 8) * 8 + 2 * t] = acc[2];
    mine[(gq + 8) * 8 + 2 * t + 1] = acc[3];
    pk::wbar(1, WT);
    if (ok && wt < TR * 8) {
        const int r = wt / 8, n = wt - r * 8;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < 8; q++) v += red[q * TR * 8 + wt];
        if (n < R && o0 + r < g.OUT) epilogue(g, o0 + r, n, v);
    }
    pk::wbar(1, WT);
}

template <int GV, int RB>
__global__ void __launch_bounds__(THREADS, 1) x070_small_kernel(const __grid_constant__ Args S) {
    using C = Cfg<RB>;
    constexpr int NS = C::NS;
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::B_OFF);
    uint64_t* empty = full + NS;
    Phase* phs = reinterpret_cast<Phase*>(smem + C::P_OFF);
    int* flag = reinterpret_cast<int*>(smem + C::T_OFF);
    float* glue = reinterpret_cast<float*>(smem + C::G_OFF);
    float* red = reinterpret_cast<float*>(smem + C::RED_OFF);
    __half* xs = reinterpret_cast<__half*>(smem + C::X_OFF);
    unsigned char* ring = smem + C::W_OFF;
    const pk::Args& A = S.g;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    int* err = A.err;

    for (int p = tid; p < S.nphases; p += THREADS) phs[p] = S.phases[p];
    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            tc::mbar_init(full + s, 1);    // the producer's expect_tx arrival (+ the copies' bytes)
            tc::mbar_init(empty + s, 8);   // one arrival per worker warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        flag[1] = *(volatile int*)err == 0;
    }
    __syncthreads();
    bool ok = flag[1] != 0;  // a wait of an earlier launch gave up: skip the program

    if (warp == 0) {
        if (ok && lane == 0) produce<NS>(S, phs, ring, full, empty, err, ok);
    } else if (warp >= 2) {
        const int wt = tid - 64, w = warp - 2;
        float* sh = glue + 2 * 12 * 64;  // reduction scratch of the glue phases
        const int R = A.R;
        int seq = 0, xjob = -1, xk0 = 0;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (A.trace && cta == 0 && wt == 0) A.trace[0] = tc::gtime();
        for (int p = 0; p < S.nphases; p++) {
            const Phase ph = phs[p];
            const pk::Layer* L = ph.layer >= 0 ? A.layers + ph.layer : nullptr;
            if (ok) {
                switch (ph.type) {
                    case pk::PH_EMBED:
                        for (int n = cta; n < R; n += G) pk::do_embed<GV>(A, n, sh, wt);
                        break;
                    case pk::PH_TMIX:
                        for (int n = cta; n < R; n += G) pk::do_tmix<GV>(A, *L, n, sh, wt);
                        break;
                    case pk::PH_CMIX:
                        for (int n = cta; n < R; n += G) pk::do_cmix<GV>(A, *L, n, sh, wt);
                        break;
                    case pk::PH_LNOUT:
                        for (int n = cta; n < R; n += G) pk::do_lnout<GV>(A, n, sh, wt);
                        break;
                    case pk::PH_WKV: {
                        const int half = wt >> 7, t = wt & 127, RH = R * A.H, l0 = ph.layer == 0;
                        for (int rh0 = 2 * cta; rh0 < RH; rh0 += 2 * G) {
                            const int rh = rh0 + half;
                            float4 st[8];
                            float f[9];
                            if (rh < RH) {
                                pk::wkv_load(*L, rh, t, st);
                                pk::wkv_vec_load(A, *L, rh, l0, t, f);
                                pk::do_wkv(A, *L, rh, l0, glue + half * 12 * 64, t, half, st, f);
                            }
                        }
                        break;
                    }
                    case pk::PH_ARGMAX: {
                        const int V = A.V, ns = (V + ARGMAX_SLICE - 1) / ARGMAX_SLICE;
                        for (int it = cta; it < R * ns; it += G) {
                            const int n = it / ns, c0 = (it % ns) * ARGMAX_SLICE, cend = min(V, c0 + ARGMAX_SLICE);
                            const float* lp = A.logits + (int64_t)n * V;
                            unsigned long long best = 0ull;
                            for (int c = c0 + wt; c < cend; c += WT) best = max(best, argmax_key(lp[c], c));
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
                            if (lane == 0) atomicMax(A.amax_keys + n, best);
                        }
                        break;
                    }
                    case pk::PH_ARGFIN:
                        for (int n = cta * WT + wt; n < R; n += G * WT) {
                            A.ids[n] = (int32_t)(0xFFFFFFFFu - (unsigned)(A.amax_keys[n] & 0xFFFFFFFFull));
                            A.amax_keys[n] = 0ull;
                        }
                        break;
                    default:
                        break;
                }
            }
            if (ph.type == pk::PH_GEMM) {
                // the loop's shape (and every worker barrier in it) does not
                // depend on `ok`, which may differ between threads after a wait
                // gave up; only the arithmetic is skipped
                xjob = -1;  // the activations are new in every phase
                const int* ofs = S.ofs + ph.i0;
                const int i1 = ofs[cta + 1];
                for (int i = ofs[cta]; i < i1; i++, seq++) {
                    const Item it = S.items[i];
                    const Job& jb = S.jobs[it.job];
                    if (it.job != xjob || it.k0 < xk0 || it.k0 + it.kn > xk0 + KW) {
                        pk::wbar(1, WT);
                        if (ok) stage_x(jb.g, R, it.k0, xs, wt);
                        pk::wbar(1, WT);
                        xjob = it.job;
                        xk0 = it.k0;
                    }
                    const int s = seq % NS;
                    if (ok && !tc::mbar_wait(full + s, (seq / NS) & 1, err)) ok = false;
                    if (ok) {
                        const unsigned char* slot = ring + s * SLOT;
                        if (jb.fmt == FMT_Q4) piece_q4(slot, xs, it.k0 - xk0, it.kn, R, w, lane, acc);
                        else piece_f16(slot, xs, it.k0 - xk0, it.kn, R, w, lane, acc);
                    }
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(empty + s);
                    if (it.last) {
                        tile_out(jb.g, it.o0, R, red, acc, w, lane, wt, ok);
                        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
                    }
                }
            }
            if (A.trace && wt == 0 && cta < 160 && p < 256) A.trace[pk::T_C + 160 * p + cta] = tc::gtime();
            ok = grid_sync(A.bar, (unsigned int)(p + 1), err, wt, flag);
            if (A.trace && cta == 0 && wt == 0) A.trace[p + 1] = tc::gtime();
        }
    }
    const int bad = __syncthreads_or(!ok && (warp >= 2 || lane == 0));
    if (tid == 0 && bad) {
        *(volatile int*)A.err_host = 1;
        __threadfence_system();
    }
}

}  // namespace sp
}  // namespace rwkv
