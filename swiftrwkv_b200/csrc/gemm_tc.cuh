// Batched-decode GEMM on the 5th-generation tensor cores (tcgen05 + TMA +
// TMEM):  y[n, o] = act( sum_k x[n, k] * W[o, k] )  with W in the MLX affine
// 4-bit group-64 container (fp16 scale / bias), x fp16, for activation rows
// R > 8 (BN = 16 .. 128 rows per n-block).
//
// CTA (576 threads) = one 128-row block of W x one BN-row block of x, K in
// stages of GPS 64-column groups:
//   warp 0      TMA producer: the stage's packed codes (128 rows x 32*GPS
//               bytes, swizzled) and GPS activation boxes (BN rows x 64 fp16,
//               128-byte swizzle, the K-major layout tcgen05.mma reads)
//   warp 1      TMEM owner and MMA issuer: 4*GPS tcgen05.mma (M=128, N=BN,
//               K=16) per stage, A read from TMEM, B from shared memory, D in
//               TMEM; tcgen05.commit frees the stage
//   warps 2-17  thread <-> weight row (its TMEM lane); the four warps of a
//               lane quadrant split each stage's code chunks.  They dequantise
//               with one HFMA2 per two weights, w = half(scale*q + bias),
//               exactly as the mma.sync wide path does, and store the fp16
//               weights into the A stage in TMEM (tcgen05.st); after the last
//               stage they drain the accumulator (tcgen05.ld) and run the
//               epilogue
// Keeping A in TMEM means the dequantised weights never touch shared memory:
// per group the CTA moves 4 KB of codes and BN*128 bytes of x through it.
//
// mbarriers: wfull[s] / xfull[s] (the stage's weight / activation bytes
// landed), sempty[s] (MMAs of smem stage s done), afull[a] (512 dequant arrivals), aempty[a] (MMAs reading TMEM stage
// a done), done (every MMA done).  Every mbarrier wait is bounded in time: on
// expiry the waiter sets *err, all roles wind down, the producer waits
// (bounded) for its copies in flight, and TMEM is freed after the final MMA
// commit.
//
// Split-K (S > 1): the S CTAs of one output tile form a (1, 1, S) cluster.
// After a cluster barrier each CTA stores rows [128z/S, 128(z+1)/S) of its
// fp32 partial into CTA z's shared memory (distributed shared memory, posted
// stores); after a second barrier CTA z sums its rows over the S partials in
// split order (deterministic) and applies the epilogue.  No global
// workspace, no atomics.
#pragma once

#include <cudaTypedefs.h>

#include "gemm_w4.cuh"

namespace rwkv {
namespace tc {

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}

constexpr uint64_t WAIT_LIMIT_NS = 200ull * 1000 * 1000;  // far beyond any healthy wait

// Wait for the phase with parity `parity` to complete.  Returns false (with
// *err set) when the wait expires or another role has already given up.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int* err) {
    if (mbar_try(b, parity)) return true;
    const uint64_t t0 = gtime();
    for (uint32_t it = 1;; it++) {
        if (mbar_try(b, parity)) return true;
        if ((it & 63) == 0) {
            if (*(volatile int*)err) return false;
            if (gtime() - t0 > WAIT_LIMIT_NS) {
                atomicExch(err, 1);
                return false;
            }
        }
    }
}

// The same wait, blind to *err: for asynchronous work this CTA started and
// must see finish before it moves on (TMA copies into its shared memory, the
// MMAs before the final commit).  Gives up only on its own time limit, and
// then sets *err.
__device__ __forceinline__ bool mbar_wait_own(uint64_t* b, uint32_t parity, int* err) {
    if (mbar_try(b, parity)) return true;
    const uint64_t t0 = gtime();
    for (uint32_t it = 1;; it++) {
        if (mbar_try(b, parity)) return true;
        if ((it & 63) == 0 && gtime() - t0 > WAIT_LIMIT_NS) {
            atomicExch(err, 1);
            return false;
        }
    }
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(saddr(dst)), "l"(map), "r"(saddr(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory operand descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;            // leading offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;  // stride offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;            // version
    d |= (uint64_t)2 << 61;            // SWIZZLE_128B
    return d;
}

// kind::f16 instruction descriptor: D f32, A and B f16 (bf16 = true: both
// bf16, format 1 in bits 7-9 and 10-12), both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16 = false) {
    return (1u << 4) | (bf16 ? (1u << 7) | (1u << 10) : 0u) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem]^T
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
// D[tmem] (+)= A[smem] * B[smem]^T
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar)) : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
          "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
          "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

template <int BYTES>
__device__ __forceinline__ void cp_async(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(saddr(dst)), "l"(src), "n"(BYTES) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// The 8 codes of packed word w (k = 8w .. 8w+7), dequantised to fp16 in
// natural k order: out[q] = (w_{2q}, w_{2q+1}).  Byte q holds codes 2q (low
// nibble) and 2q+1 (high nibble); placed in the two halves under the
// exponent of 1024 they read 1024 + c_lo and 1024 + 16 c_hi, and one exact
// HFMA2 by (1, 1/16) and (-1024, -64) turns them into (c_lo, c_hi).  The
// second HFMA2 is the rounding point, w = half(scale * q + bias).
__device__ __forceinline__ void dq_word(uint32_t w, __half2 s2, __half2 b2, uint32_t* out) {
    const __half2 mul = __halves2half2(__ushort_as_half(0x3C00), __ushort_as_half(0x2C00));  // (1, 1/16)
    const __half2 add = __halves2half2(__ushort_as_half(0xE400), __ushort_as_half(0xD400));  // (-1024, -64)
#pragma unroll
    for (int q = 0; q < 4; q++) {
        uint32_t h = (__byte_perm(w, 0, 0x4040u | (uint32_t)q | ((uint32_t)q << 8)) & 0x00F0000Fu) | 0x64006400u;
        const __half2 c = __hfma2(*reinterpret_cast<__half2*>(&h), mul, add);
        const __half2 v = __hfma2(c, s2, b2);
        out[q] = *reinterpret_cast<const uint32_t*>(&v);
    }
}

// 4 / 8 columns into raw registers; complete them with tmem_ld_wait()
__device__ __forceinline__ void tmem_ld4_async(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8_async(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

// whole-cluster barrier (every thread of every CTA), release / acquire
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// shared::cluster address of the same offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_rank(uint32_t smem_addr, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
// posted 16-byte store into a peer CTA's shared memory (ordered by the next cluster barrier)
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, const uint32_t* v) {
    asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]), "r"(v[1]), "r"(v[2]),
                 "r"(v[3]) : "memory");
}

}  // namespace tc

constexpr int TC_JOBS = 4;
constexpr int TC_BM = 128;
constexpr int TC_SRING = 4;    // scale / bias prefetch ring (stages)
constexpr int TC_MAX_SPLIT = 8;  // split-K CTAs of one tile form one cluster

// Weight formats: TC_Q4 = MLX affine 4-bit group-64 codes (dequantised into
// TMEM), TC_F16 / TC_BF16 = dense fp16 / bf16 [OUT, IN] (read by the MMA
// straight from shared memory; activations of the same type).
enum : int { TC_Q4 = 0, TC_F16 = 1, TC_BF16 = 2 };

struct alignas(64) TcJob {
    CUtensorMap wmap;  // TC_Q4: codes {IN/8, OUT} u32, box {8*GPS, 128}, swizzled;
                       // TC_F16: weights {IN, OUT} fp16, box {64, 128}, 128-byte swizzle
    CUtensorMap xmap;  // activations: dims {IN, R} fp16, box {64, BN}, 128-byte swizzle
    GemvJob g;         // scales, biases, OUT, IN, epilogue
};

// err: device flag that a wait which gives up sets (the other roles of every
// CTA of the launch watch it and wind down); a CTA that gave up, or that found
// the flag already set at entry and skipped its work, also writes 1 to
// err_host (mapped pinned host memory), so the host learns of it without a
// copy.  Neither is cleared by the kernel.
struct TcArgs {
    TcJob j[TC_JOBS];
    int njobs, R, S;
    int* err;
    int* err_host;
};

// QW dequant warps per TMEM lane quadrant; TMC TMEM columns: 512 (accumulator
// in [0, 256), A stages in [256, 512), one CTA per SM) or 256 (accumulator in
// [0, 64), A stages in [64, 256): BN <= 64, small enough -- with QW = 2 and a
// ~100 KB stage ring -- that two CTAs fit on an SM, so a launch's CTAs can
// become resident, and stream their weights, beside its predecessor's).
template <int FMT, int BN, int GPS, int ST, int QW_ = 4, int TMC_ = 512>
struct TcCfg {
    static constexpr int QW = QW_;
    static constexpr int DQW = 4 * QW;                    // dequant / epilogue warps
    static constexpr int THREADS = 64 + 32 * DQW;         // + producer warp + MMA warp
    static constexpr int TMC = TMC_;
    static constexpr int A_COL = TMC == 512 ? 256 : 64;
    static_assert(TMC == 512 || (TMC == 256 && BN <= 64), "TMEM layout");
    static constexpr int CROW = FMT == TC_Q4 ? 32 * GPS : 128 * GPS;  // weight bytes per row per stage
    static constexpr int C_BYTES = TC_BM * CROW;
    static constexpr int XBOX = BN * 128;                 // one x box (64 columns)
    static constexpr int X_BYTES = GPS * XBOX;
    static constexpr int STAGE = C_BYTES + X_BYTES;       // multiple of 1024
    static constexpr int ST_A = (TMC - A_COL) / (32 * GPS);
    static constexpr int CPR = 2 * GPS;                   // 16-byte code chunks per row per stage
    static constexpr int CPW = CPR / QW;                  // chunks per dequant warp per stage
    static constexpr int SLOT = 8;                        // ring slot: a 4-byte-aligned pair of scales + of biases
    static constexpr int SR_OFF = ST * STAGE;             // ring: [TC_SRING][32*DQW] slots
    static constexpr int B_OFF = SR_OFF + (FMT == TC_Q4 ? TC_SRING * 32 * DQW * SLOT : 0);
    static constexpr int NBAR = 3 * ST + 2 * ST_A + 1;
    static constexpr int T_OFF = B_OFF + NBAR * 8;
    static constexpr int TOTAL = T_OFF + 16 + 1024;       // + slack for 1024-byte alignment
    static_assert(STAGE % 1024 == 0, "stage bases stay 1024-byte aligned");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "M=128 needs N % 16 == 0, 16..256");
    static_assert(BN <= A_COL, "accumulator columns");
    static constexpr int RP = BN + 4;                     // split-K receive row pitch (floats): 16-byte rows, conflict-free
    static_assert(ST * STAGE >= (TC_BM + TC_MAX_SPLIT) * RP * 4, "split-K receive buffers reuse the stage buffers");
    static_assert(TOTAL <= 227 * 1024, "shared memory per CTA");
    static_assert(FMT != TC_Q4 || ST_A >= 1, "at least one A stage");
    static_assert(FMT != TC_Q4 || (CPR % QW == 0 && CPW >= 1 && CPW <= 2),
                  "a dequant warp's chunks lie in one group");
    static_assert(BN % (4 * QW) == 0, "accumulator columns per warp in units of 4");
};

// Byte offset of 16-byte chunk c of row r in a TMA tile with `rb`-byte rows
// written with the matching swizzle (128 B: Swizzle<3,4,3>; 64 B: Swizzle<2,4,3>).
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c, uint32_t rb) {
    const uint32_t off = r * rb + 16 * c;
    return off ^ (((off >> 7) & (rb / 16 - 1)) << 4);
}

template <int FMT, int BN, int GPS, int ST, int QW = 4, int TMC = 512>
__global__ void __launch_bounds__(TcCfg<FMT, BN, GPS, ST, QW, TMC>::THREADS, TMC == 512 ? 1 : 2)
gemm_tc_kernel(const __grid_constant__ TcArgs args) {
    using C = TcCfg<FMT, BN, GPS, ST, QW, TMC>;
    constexpr int TC_DQW = C::DQW, TC_QW = C::QW, TC_TMEM_COLS = C::TMC, TC_A_COL = C::A_COL;
    constexpr int ST_A = C::ST_A;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + C::B_OFF);
    uint64_t* xfull = wfull + ST;
    uint64_t* sempty = xfull + ST;
    uint64_t* afull = sempty + ST;
    uint64_t* aempty = afull + ST_A;
    uint64_t* done = aempty + ST_A;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::T_OFF);
    int* skip_slot = reinterpret_cast<int*>(smem + C::T_OFF + 8);

    const TcJob& jb = args.j[blockIdx.y];
    const int OUT = jb.g.OUT, IN = jb.g.IN;
    const int m0 = blockIdx.x * TC_BM;
    const int S = args.S;
    const int nblk = blockIdx.z / S, kz = blockIdx.z % S;  // kz = rank in the (1, 1, S) cluster
    const int n0 = nblk * BN;
    // uniform over the cluster (same x, y, n-block), before any barrier or TMEM use
    if (m0 >= OUT || n0 >= args.R) return;
    const int NG = (IN + 63) / 64, NS = NG / GPS;  // TC_Q4: IN % (64 GPS) == 0; TC_F16: GPS == 1
    const int s0 = (int)((int64_t)NS * kz / S), s1 = (int)((int64_t)NS * (kz + 1) / S);
    const int nst = s1 - s0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int* err = args.err;

    if (tid == 0) {
        pdl_trigger();
        for (int s = 0; s < ST; s++) {
            tc::mbar_init(wfull + s, 1);
            tc::mbar_init(xfull + s, 1);
            tc::mbar_init(sempty + s, 1);
        }
        for (int a = 0; a < ST_A; a++) {
            tc::mbar_init(afull + a, 32 * TC_DQW);
            tc::mbar_init(aempty + a, 1);
        }
        tc::mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // a wait of an earlier launch gave up and nobody has cleared the flag:
        // every role skips its work (no copies, no MMAs, no output), so the
        // launch ends at once and the host is told again
        *skip_slot = *(volatile int*)err;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(tc::saddr(tmem_slot)), "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc::tc_before();
    __syncthreads();
    tc::tc_after();
    const uint32_t tmem = *tmem_slot;
    const bool skip = *skip_slot != 0;
    bool ok = !skip;
    constexpr int CW = BN / TC_QW;  // accumulator columns per dequant warp
    uint32_t acc[CW];

    if (warp == 0) {
        if (lane == 0 && !skip) {  // ---- TMA producer
            // weights do not depend on the previous kernel: the first stages'
            // weights stream (and are dequantised) before its activations are ready
            auto load_w = [&](int i) {
                const int s = i % ST, g = (s0 + i) * GPS;
                unsigned char* st = smem + s * C::STAGE;
                tc::mbar_expect_tx(wfull + s, C::C_BYTES);
                if constexpr (FMT == TC_Q4) {
                    tc::tma_2d(st, &jb.wmap, wfull + s, 8 * g, m0);
                } else {
#pragma unroll
                    for (int q = 0; q < GPS; q++) tc::tma_2d(st + q * TC_BM * 128, &jb.wmap, wfull + s, 64 * (g + q), m0);
                }
            };
            auto load_x = [&](int i) {
                const int s = i % ST, g = (s0 + i) * GPS;
                unsigned char* st = smem + s * C::STAGE;
                tc::mbar_expect_tx(xfull + s, C::X_BYTES);
#pragma unroll
                for (int q = 0; q < GPS; q++)
                    tc::tma_2d(st + C::C_BYTES + q * C::XBOX, &jb.xmap, xfull + s, 64 * (g + q), n0);
            };
            const int pre = min(ST, nst);
            for (int i = 0; i < pre; i++) load_w(i);
            pdl_wait();
            for (int i = 0; i < pre; i++) load_x(i);
            int issued = pre;
            for (int i = pre; i < nst; i++) {
                const int s = i % ST;
                if (!tc::mbar_wait(sempty + s, ((i / ST) - 1) & 1, err)) {
                    ok = false;
                    break;
                }
                load_w(i);
                load_x(i);
                issued = i + 1;
            }
            // the copies this thread issued have landed before the CTA may
            // exit or reuse the stage buffers (whatever the other roles did)
            for (int i = max(0, issued - ST); i < issued; i++) {
                if (!tc::mbar_wait_own(wfull + (i % ST), (i / ST) & 1, err)) ok = false;
                if (!tc::mbar_wait_own(xfull + (i % ST), (i / ST) & 1, err)) ok = false;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            constexpr uint32_t IDESC = tc::idesc_f16(TC_BM, BN, FMT == TC_BF16);
            for (int i = 0; i < (skip ? 0 : nst); i++) {
                const int s = i % ST, a = i % ST_A;
                if (!tc::mbar_wait(wfull + s, (i / ST) & 1, err) || !tc::mbar_wait(xfull + s, (i / ST) & 1, err) ||
                    (FMT == TC_Q4 && !tc::mbar_wait(afull + a, (i / ST_A) & 1, err))) {
                    ok = false;
                    break;
                }
                tc::tc_after();
                const uint32_t xs = tc::saddr(smem + s * C::STAGE + C::C_BYTES);
                const uint32_t ta = tmem + TC_A_COL + a * (32 * GPS);
                const uint32_t ws = tc::saddr(smem + s * C::STAGE);
#pragma unroll
                for (int q = 0; q < GPS; q++) {
                    const uint64_t bd = tc::sw128_desc(xs + q * C::XBOX);
                    if constexpr (FMT == TC_Q4) {
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            tc::umma_ts(tmem, ta + q * 32 + kk * 8, bd + 2 * kk, IDESC, (i | q | kk) ? 1u : 0u);
                    } else {
                        const uint64_t ad = tc::sw128_desc(ws + q * TC_BM * 128);
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            tc::umma_ss(tmem, ad + 2 * kk, bd + 2 * kk, IDESC, (i | q | kk) ? 1u : 0u);
                    }
                }
                if constexpr (FMT == TC_Q4) tc::umma_commit(aempty + a);
                tc::umma_commit(sempty + s);
            }
            tc::umma_commit(done);  // after an early exit too: TMEM is freed only after the MMAs finish
        }
    } else {
        // ---- dequant: row rl = the warp's TMEM lane quadrant; the TC_QW warps of
        // a quadrant split each stage's code chunks (warp h: chunks [h*CPW, (h+1)*CPW),
        // all inside group q0 = h*CPW/2)
        constexpr int CPW = C::CPW;
        const int dt = tid - 64;
        const int q4 = warp & 3, h = (warp - 2) >> 2;
        const int rl = 32 * q4 + lane;
        const int orow = min(m0 + rl, OUT - 1);
        const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
        const int q0 = (h * CPW) >> 1, qpair = q0 & ~1;
        const __half* sc = (const __half*)jb.g.scales + (int64_t)orow * NG + qpair;
        const __half* bi = (const __half*)jb.g.biases + (int64_t)orow * NG + qpair;
        // ring slot of stage i for this thread: scales of groups (qpair, qpair+1), then biases
        __half* ring = reinterpret_cast<__half*>(smem + C::SR_OFF);
        auto slot = [&](int i) { return ring + ((i % TC_SRING) * (32 * TC_DQW) + dt) * 4; };
        auto fetch = [&](int i) {
            if (i < nst) {
                const int g = (s0 + i) * GPS;
                tc::cp_async<4>(slot(i), sc + g);
                tc::cp_async<4>(slot(i) + 2, bi + g);
            }
            tc::cp_commit();
        };
        if constexpr (FMT == TC_Q4) {
        if (!skip) {
#pragma unroll
        for (int i = 0; i < TC_SRING - 1; i++) fetch(i);
        for (int i = 0; i < nst; i++) {
            const int s = i % ST, a = i % ST_A;
            fetch(i + TC_SRING - 1);
            if (!tc::mbar_wait(wfull + s, (i / ST) & 1, err)) { ok = false; break; }
            if (i >= ST_A && !tc::mbar_wait(aempty + a, ((i / ST_A) - 1) & 1, err)) { ok = false; break; }
            tc::tc_after();
            tc::cp_wait<TC_SRING - 1>();
            const __half* sh = slot(i);
            const __half2 s2 = __half2half2(sh[q0 & 1]), b2 = __half2half2(sh[2 + (q0 & 1)]);
            const unsigned char* cs = smem + s * C::STAGE;
#pragma unroll
            for (int cc = 0; cc < CPW; cc++) {
                const int ch = h * CPW + cc;
                const uint4 cw = *reinterpret_cast<const uint4*>(cs + swz(rl, ch, C::CROW));
                uint32_t v[16];
                tc::dq_word(cw.x, s2, b2, v);
                tc::dq_word(cw.y, s2, b2, v + 4);
                tc::dq_word(cw.z, s2, b2, v + 8);
                tc::dq_word(cw.w, s2, b2, v + 12);
                tc::tmem_st16(tmem + lane_base + TC_A_COL + a * (32 * GPS) + ch * 16, v);
            }
            tc::tmem_st_wait();
            tc::tc_before();
            tc::mbar_arrive(afull + a);
        }
        tc::cp_wait<0>();
        }
        }
        // every MMA has finished before the accumulator is read, the stage
        // buffers are reused for the split-K exchange and TMEM is freed
        ok = tc::mbar_wait_own(done, 0, err) && ok;
        tc::tc_after();
        // returns at once when the producer's wait preceded the MMAs; in the
        // skip path it keeps the grid from completing before its predecessor,
        // whose completion the grid's dependents rely on
        pdl_wait();
        // ---- accumulator: row rl, this warp's half of the BN columns
        const GemvJob g = jb.g;  // a register copy: stores below cannot alias it
        const uint32_t tacc = tmem + lane_base;
        const int o = m0 + rl;
        // this thread's CW accumulator columns (row rl), all loads in flight at once
#pragma unroll
        for (int c = 0; c < CW; c += 4) tc::tmem_ld4_async(tacc + h * CW + c, acc + c);
        tc::tmem_ld_wait();
        if (S == 1 && ok && o < OUT) {
            const int c0 = n0 + h * CW;
            if (g.act == ACT_NONE && g.out == OUT_F32) {
                float* yo = (float*)g.y + (int64_t)c0 * g.y_stride + o;
#pragma unroll
                for (int c = 0; c < CW; c++)
                    if (c0 + c < args.R) yo[(int64_t)c * g.y_stride] = __uint_as_float(acc[c]);
            } else {
#pragma unroll
                for (int c = 0; c < CW; c++)
                    if (c0 + c < args.R) epilogue(g, o, c0 + c, __uint_as_float(acc[c]));
            }
        }
    }
    if (S > 1) {
        // Split-K over the (1, 1, S) cluster.  CTA z owns rows [128z/S, 128(z+1)/S)
        // of the tile and receives, from every split zs, those rows of its
        // partial into rbuf[zs][row][RP] (its own stage buffers, idle once
        // every CTA of the cluster has passed the first barrier), 16 bytes per
        // store.  Every thread of every CTA takes both barriers, on every path.
        constexpr int RP = C::RP;
        const int NRM = (TC_BM + S - 1) / S;
        const uint32_t rbuf = tc::saddr(smem);
        tc::cluster_sync();
        // a wait that gave up anywhere in the cluster set *err before the
        // barrier: read it now, its latency hidden behind the partial stores
        const int gave_up = warp >= 2 ? *(volatile int*)err : 0;
        if (warp >= 2) {
            const int rl = 32 * (warp & 3) + lane, h = (warp - 2) >> 2;
            const int zo = ((rl + 1) * S + TC_BM - 1) / TC_BM - 1;  // owner of row rl
            const int lr = rl - TC_BM * zo / S;
            const uint32_t dst = tc::map_rank(rbuf + (uint32_t)((kz * NRM + lr) * RP + h * CW) * 4, zo);
#pragma unroll
            for (int c = 0; c < CW; c += 4) tc::st_cluster_v4(dst + (uint32_t)c * 4, acc + c);
        }
        tc::cluster_sync();
        if (warp >= 2 && !gave_up) {
            // task = (row, 4 columns): the S partials summed in split order
            // (deterministic), then 4 outputs; lanes take consecutive rows, so
            // the reads are conflict-free and the stores coalesce along o
            const GemvJob g = jb.g;
            const int r0 = TC_BM * kz / S, nr = TC_BM * (kz + 1) / S - r0;
            const float* rb = reinterpret_cast<const float*>(smem);
            const bool plain = g.act == ACT_NONE && g.out == OUT_F32;
            for (int e = tid - 64; e < nr * (BN / 4); e += 32 * TC_DQW) {
                const int cq = e / nr, lr = e - cq * nr;
                const float* src = rb + lr * RP + 4 * cq;
                float4 v = *reinterpret_cast<const float4*>(src);
                for (int z = 1; z < S; z++) {
                    const float4 p = *reinterpret_cast<const float4*>(src + z * NRM * RP);
                    v.x += p.x;
                    v.y += p.y;
                    v.z += p.z;
                    v.w += p.w;
                }
                const int o = m0 + r0 + lr;
                if (o >= OUT) continue;
                const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int n = n0 + 4 * cq + j;
                    if (n < args.R) {
                        if (plain) ((float*)g.y)[(int64_t)n * g.y_stride + o] = vv[j];
                        else epilogue(g, o, n, vv[j]);
                    }
                }
            }
        }
    }
    tc::tc_before();
    const int bad = __syncthreads_or(!ok && (warp >= 2 || lane == 0));
    if (warp == 1) {
        tc::tc_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
    }
    if (tid == 0 && bad) {
        *(volatile int*)args.err_host = 1;
        __threadfence_system();
    }
}

// ------------------------------------------------------------------ host side

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

static __global__ void tc_set_flag_kernel(int* p, int v) { *p = v; }

// The wait-error record of the tensor-core GEMMs that share it: the device
// flag the kernel's waits watch (TcArgs::err) and a mapped pinned host int
// (TcArgs::err_host) that a CTA which gave up sets, so that the host can test
// it with a plain load.  The kernel never clears either: take() and status()
// report and clear them.
struct TcWaitFlag {
    int* dev = nullptr;       // device memory, owned by the caller
    int* host = nullptr;      // host view of the mapped int
    int* host_dev = nullptr;  // the same int, as the device addresses it

    bool init(int* dev_int) {
        dev = dev_int;
        if (cudaHostAlloc((void**)&host, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
            host = nullptr;
            return false;
        }
        *(volatile int*)host = 0;
        if (cudaHostGetDevicePointer((void**)&host_dev, host, 0) != cudaSuccess) return false;
        return true;
    }
    void release() {
        if (host) cudaFreeHost(host);
        host = host_dev = nullptr;
    }
    // Without synchronising: true when a CTA has recorded a wait that gave up
    // (a launch still running may record one later).  Clears both flags, the
    // device one in stream order on `st`.
    bool take(cudaStream_t st) {
        if (!host || *(volatile int*)host == 0) return false;
        *(volatile int*)host = 0;
        cudaMemsetAsync(dev, 0, sizeof(int), st);
        return true;
    }
    // Synchronises `st`, then reports and clears either flag.
    int status(cudaStream_t st, const char* who) {
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail(RWKV_E_CUDA, "%s: stream synchronisation failed", who);
        int d = 0;
        if (cudaMemcpy(&d, dev, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
            return fail(RWKV_E_CUDA, "%s: flag read failed", who);
        const bool h = host && *(volatile int*)host != 0;
        if (!d && !h) return ok();
        if (host) *(volatile int*)host = 0;
        cudaMemset(dev, 0, sizeof(int));
        return fail(RWKV_E_TIMEOUT, "%s: a tensor-core GEMM pipeline wait gave up; its outputs are not valid", who);
    }
    // Marks the record as a wait that gives up would: the device flag, and
    // with host_record also the host int.
    int inject(int host_record, cudaStream_t st) {
        tc_set_flag_kernel<<<1, 1, 0, st>>>(dev, 1);
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail(RWKV_E_CUDA, "inject: synchronisation failed");
        if (host_record && host) *(volatile int*)host = 1;
        return check_launch("tc_set_flag_kernel");
    }
};

struct TcPlan {
    int BN = 0, GPS = 0, S = 1, nnb = 0, mblocks = 0;
    bool ok = false;
};

// Whether a job can take the tcgen05 path: fp16 activations with rows
// 16-byte aligned, 16-byte aligned weights; TC_Q4: IN a multiple of 256
// (whole stages) and 8-byte aligned scales and biases; TC_F16: 16-byte rows.
inline bool tc_job_ok(int FMT, const GemvJob& j) {
    const bool common = j.OUT >= 1 && j.x_stride % 8 == 0 && ((uintptr_t)j.x & 15) == 0 &&
                        ((uintptr_t)j.w & 15) == 0;
    if (FMT != TC_Q4) return common && j.IN >= 8 && j.IN % 8 == 0;
    return common && j.IN % 256 == 0 && j.IN >= 256 && j.scales && j.biases &&
           ((uintptr_t)j.scales & 7) == 0 && ((uintptr_t)j.biases & 7) == 0;
}

// Kernel configurations (tile width BN, groups per stage GPS, stages ST,
// dequant warps per quadrant QW, TMEM columns TMC) per weight format;
// X(FMT, BN, GPS, ST, QW, TMC).  One CTA per SM.  (Two-per-SM variants --
// 128-deep stages, 8 dequant warps, 256 TMEM columns, so that a launch's CTAs
// could stream their weights beside its predecessor's -- measured slower on
// the 1.5B decode step: 64 rows 2.11 -> 2.36 ms.)
#define RWKV_TC_CONFIGS(FMT, X)                                                                 \
    switch (BN) {                                                                              \
        case 16: return FMT == TC_Q4 ? X(TC_Q4, 16, 4, 6, 4, 512) : FMT == TC_F16 ? X(TC_F16, 16, 1, 8, 4, 512)     \
                                                                   : X(TC_BF16, 16, 1, 8, 4, 512);                   \
        case 32: return FMT == TC_Q4 ? X(TC_Q4, 32, 4, 5, 4, 512) : FMT == TC_F16 ? X(TC_F16, 32, 1, 8, 4, 512)     \
                                                                   : X(TC_BF16, 32, 1, 8, 4, 512);                   \
        case 64: return FMT == TC_Q4 ? X(TC_Q4, 64, 4, 4, 4, 512) : FMT == TC_F16 ? X(TC_F16, 64, 1, 8, 4, 512)     \
                                                                   : X(TC_BF16, 64, 1, 8, 4, 512);                   \
        default: return FMT == TC_Q4 ? X(TC_Q4, 128, 2, 4, 4, 512) : FMT == TC_F16 ? X(TC_F16, 128, 1, 6, 4, 512)  \
                                                                    : X(TC_BF16, 128, 1, 6, 4, 512);                 \
    }

// How many (1, 1, S) clusters of this configuration the GPU holds at once
// (cached per configuration and S; 0 when the query fails).
template <int FMT, int BN, int GPS, int ST, int QW, int TMC>
inline int tc_max_clusters_t(int S) {
    static int cache[TC_MAX_SPLIT + 1] = {};
    if (S < 1 || S > TC_MAX_SPLIT) return 0;
    if (cache[S]) return cache[S] > 0 ? cache[S] : 0;
    using C = TcCfg<FMT, BN, GPS, ST, QW, TMC>;
    auto kern = gemm_tc_kernel<FMT, BN, GPS, ST, QW, TMC>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::TOTAL) == cudaSuccess) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(1, 1, S);
        cfg.blockDim = dim3(C::THREADS);
        cfg.dynamicSmemBytes = C::TOTAL;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = S;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    cache[S] = n > 0 ? n : -1;
    return n;
}

inline int tc_max_clusters(int FMT, int BN, int S) {
#define X_(F, B, G, T, Q, M) tc_max_clusters_t<F, B, G, T, Q, M>(S)
    RWKV_TC_CONFIGS(FMT, X_)
#undef X_
}

inline int tc_gps(int FMT, int BN) { return FMT != TC_Q4 ? 1 : BN <= 64 ? 4 : 2; }

inline TcPlan plan_tc(int FMT, const GemvJobs& jobs, int njobs, int R, int sm_count) {
    TcPlan p{};
    // decode batches (R <= 256) and prefill token blocks (R up to 64 Ki rows,
    // 128-row n-blocks, no split-K once the n-blocks fill the GPU)
    // (bf16 dense weights take it at any row count: no exact-GEMV numerics to keep)
    if ((R <= 8 && FMT != TC_BF16) || R < 1 || R > 65536 || njobs < 1 || njobs > TC_JOBS) return p;
    for (int i = 0; i < njobs; i++)
        if (!tc_job_ok(FMT, jobs.j[i])) return p;
    p.BN = R <= 16 ? 16 : R <= 32 ? 32 : R <= 64 ? 64 : 128;
    p.GPS = tc_gps(FMT, p.BN);
    p.nnb = (R + p.BN - 1) / p.BN;
    int maxo = 0, minst = 1 << 30;
    for (int i = 0; i < njobs; i++) {
        maxo = std::max(maxo, jobs.j[i].OUT);
        minst = std::min(minst, (jobs.j[i].IN + 63) / 64 / p.GPS);
    }
    p.mblocks = (maxo + TC_BM - 1) / TC_BM;
    int ctas = 0;
    for (int i = 0; i < njobs; i++) ctas += (jobs.j[i].OUT + TC_BM - 1) / TC_BM * p.nnb;
    // split K until about one CTA per SM, with at least two stages per split,
    // and only as far as every cluster of the launch is resident at once
    int S = (sm_count + ctas - 1) / ctas;
    S = std::max(1, std::min(std::min(S, minst / 2), TC_MAX_SPLIT));
    const int clusters = p.mblocks * njobs * p.nnb;
    while (S > 1 && tc_max_clusters(FMT, p.BN, S) < clusters) S--;
    p.S = S;
    p.ok = true;
    return p;
}

inline bool encode_tc_maps(int FMT, TcJob& t, const GemvJob& j, int R, int BN, int GPS) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    t.g = j;
    if (FMT == TC_Q4) {
        cuuint64_t dims[2] = {(cuuint64_t)(j.IN / 8), (cuuint64_t)j.OUT};
        cuuint64_t strides[1] = {(cuuint64_t)j.IN / 2};
        cuuint32_t box[2] = {(cuuint32_t)(8 * GPS), (cuuint32_t)TC_BM};
        cuuint32_t es[2] = {1, 1};
        if (enc(&t.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, (void*)j.w, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE,
                GPS == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    } else {
        cuuint64_t dims[2] = {(cuuint64_t)j.IN, (cuuint64_t)j.OUT};
        cuuint64_t strides[1] = {(cuuint64_t)j.IN * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)TC_BM};
        cuuint32_t es[2] = {1, 1};
        if (enc(&t.wmap, FMT == TC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                (void*)j.w, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)j.IN, (cuuint64_t)R};
        cuuint64_t strides[1] = {(cuuint64_t)j.x_stride * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)BN};
        cuuint32_t es[2] = {1, 1};
        if (enc(&t.xmap, FMT == TC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                (void*)j.x, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

template <int FMT, int BN, int GPS, int ST, int QW, int TMC>
inline cudaError_t launch_tc_t(const TcArgs& a, const TcPlan& p, bool pdl, cudaStream_t st) {
    using C = TcCfg<FMT, BN, GPS, ST, QW, TMC>;
    auto kern = gemm_tc_kernel<FMT, BN, GPS, ST, QW, TMC>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::TOTAL);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.mblocks, a.njobs, p.nnb * a.S);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (a.S > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = a.S;
        na++;
    }
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    if (a.S > 1 && tc_max_clusters_t<FMT, BN, GPS, ST, QW, TMC>(a.S) < 1) return cudaErrorLaunchOutOfResources;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// jobs -> tensor maps -> launch.  err: device int that a wait which gives up
// sets to 1; err_host: device-visible pointer to a mapped pinned host int
// that a CTA which gave up (or skipped its work) sets to 1.
// pdl: launch as a programmatic dependent of the previous kernel in the stream.
inline cudaError_t launch_tc(int FMT, const GemvJobs& jobs, int njobs, int R, const TcPlan& p,
                             int* err, int* err_host, cudaStream_t st, bool pdl = false) {
    TcArgs a{};
    for (int i = 0; i < njobs; i++)
        if (!encode_tc_maps(FMT, a.j[i], jobs.j[i], R, p.BN, p.GPS)) return cudaErrorInvalidValue;
    a.njobs = njobs;
    a.R = R;
    a.S = p.S;
    a.err = err;
    a.err_host = err_host;
    const int BN = p.BN;
#define X_(F, B, G, T, Q, M) launch_tc_t<F, B, G, T, Q, M>(a, p, pdl, st)
    RWKV_TC_CONFIGS(FMT, X_)
#undef X_
}

#undef RWKV_TC_CONFIGS

}  // namespace rwkv
