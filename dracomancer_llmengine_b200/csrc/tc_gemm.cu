// Grouped expert GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulators, TMA).
//
// One work item = (expert e, 128-row tile of weight rows, up to 128 of its tokens in
// expert-sorted order).  Per item the CTA computes D[row][tok] = sum_k W[row][k] * B[tok][k]
// with K = the matrix row length:
//   gate/up mode: the 128 rows are 64 gate rows and the same 64 rows of up, interleaved so
//                 that TMEM lanes i and i^8 of every warp quarter hold gate and up of one
//                 intermediate row; B = the tokens' activations; the epilogue writes
//                 act = silu(gate) * up as fp16, the B operand of the down GEMM;
//   down mode:    128 rows of the down matrix, B = act; the epilogue writes y (fp32).
//
// Data path per 256-value superblock column of the tile:
//   TMA copies (each CTA its own) the 128 rows' raw superblocks (Q4_K 144 B, Q6_K 224 B padded)
//   into a shared-memory ring -> 16 dequant warps (4 warpgroups, thread = TMEM lane) decode
//   64 values at a time to fp16 in registers and store them into TMEM (tcgen05.st), where
//   they are the MMA's A operand -> one elected thread issues tcgen05.mma.kind::f16 with the
//   activations' fp16 tile (TMA, 128-byte swizzle) as the B operand into one of two fp32
//   accumulators in TMEM -> an epilogue warpgroup reads the other accumulator back
//   (tcgen05.ld) while the next item's MMAs run.
// A K step is half a superblock column (8 MMAs of K = 16); four A slots are in flight and four
// or eight activation stages (token tiles of <= 128 or <= 64 tokens).  The
// issuing thread tests the readiness of step q + 1 before it issues step q (an mbarrier wait
// costs that thread a few hundred cycles during which it cannot issue), and one
// tcgen05.commit per step releases both the step's A slot and its activation stage.
// Every wait on an mbarrier is bounded; on a timeout the CTA records an error code, stops
// issuing work, drains what it issued and frees its TMEM.
//
// Weights are decoded as the reference decodes them (src/m5_kern_scalar.c:69-142) in fp32 and
// rounded once to fp16; activations are rounded to fp16; accumulation is fp32.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "kernels.cuh"
#include "tc_gemm.cuh"

#include <cstdio>
#include <mutex>

#ifndef DRACO_TC_RAW_STAGES_Q4K
#define DRACO_TC_RAW_STAGES_Q4K 5
#endif
#ifndef DRACO_TC_RAW_STAGES_Q6K
#define DRACO_TC_RAW_STAGES_Q6K 3
#endif
// 64-token tiles (decode and lightly loaded experts): 8 activation stages and 5 (Q4_K) / 3 (Q6_K)
// weight stages.  The MMAs of a K step need both its A slot and its activation stage, and an
// activation stage is reused only after the MMAs of the step it held finished, so with 4 stages
// the activation TMA latency (rows from L2) held the MMA warps (per-site wait counters, cfg2)
#ifndef DRACO_TC_B_STAGES_64
#define DRACO_TC_B_STAGES_64 8
#endif
#ifndef DRACO_TC_RAW_STAGES_Q4K_64
#define DRACO_TC_RAW_STAGES_Q4K_64 5
#endif
#ifndef DRACO_TC_RAW_STAGES_Q6K_64
#define DRACO_TC_RAW_STAGES_Q6K_64 3
#endif
// 64-token tiles: MMA issuer warps (2: even and odd K steps into separate accumulators) and
// A slots in TMEM (2 * issuers * 64 accumulator columns + 64 per slot <= 512)
#ifndef DRACO_TC_ISSUERS_64
#define DRACO_TC_ISSUERS_64 2
#endif
#ifndef DRACO_TC_SLOTS_64
#define DRACO_TC_SLOTS_64 4
#endif
#ifndef DRACO_TC_SUSPEND_NS
#define DRACO_TC_SUSPEND_NS 1000
#endif

namespace draco {
namespace tc {

constexpr int kDeqWarps = 16;                 // 4 warpgroups
constexpr int kProdWarp = 16;                 // TMA producer of the weight superblocks
constexpr int kMmaWarp = 17;                  // MMA issuer, TMEM owner
constexpr int kBProdWarp = 18;                // TMA producer of the activation tiles
constexpr int kEpiWarp0 = 19;                 // epilogue warpgroup: warps 19..22
constexpr int kMmaWarp2 = 23;                 // second MMA issuer (odd K steps; 64-token tiles)
constexpr int kMaxRawStages = 8;              // raw superblock-column stages
constexpr int kMaxSlots = 8;                  // A slots in TMEM (K steps decoded ahead of the MMAs), most
constexpr int kDone = 8;                      // ring of per-step completion barriers (>= every stage count)
constexpr int kMaxBStages = 8;                // activation stages
constexpr int kTmemCols = 512;
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // bounded waits give up after 2 s
// try_wait may suspend the polling thread up to this long (0: poll with test_wait)
constexpr uint32_t kSuspendNs = DRACO_TC_SUSPEND_NS;

// error codes written to *err
constexpr int kErrTimeout = 0x100;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    if (kSuspendNs == 0)
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
            : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: returns false (and raises the CTA's abort flag) after kWaitLimitNs, or when
// another role already aborted (checked every 64 polls).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int where) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; i++) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*abort_flag) return false;
            if (global_ns() - t0 > kWaitLimitNs) break;
        }
    }
    *abort_flag = 1;
    atomicOr(err, kErrTimeout | where);
    return false;
}

// The same for all 32 lanes of a warp, with a warp-uniform result (the caller goes on to
// warp-collective tcgen05 instructions).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int where) {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; i++) {
        const bool done = mbar_try(bar, parity);
        if (__all_sync(0xffffffffu, done)) return true;
        if ((i & 63) == 63) {
            int stop = 0;
            if ((threadIdx.x & 31) == 0) {
                if (*abort_flag) stop = 1;
                else if (t0 == 0) t0 = global_ns();
                else if (global_ns() - t0 > kWaitLimitNs) stop = 2;
            }
            stop = __shfl_sync(0xffffffffu, stop, 0);
            if (stop == 1) return false;
            if (stop == 2) break;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        *abort_flag = 1;
        atomicOr(err, kErrTimeout | where);
    }
    __syncwarp();
    return false;
}
// one lane of the (converged) warp
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(pred));
    return pred != 0;
}
// Non-blocking test of two barriers' phases in one instruction group (one pass through the
// shared-memory pipe instead of two)
__device__ __forceinline__ bool mbar_test2(uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %3;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 q, [%2], %4;\n\tand.pred p, p, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(a)), "r"(smem_u32(b)), "r"(pa), "r"(pb)
        : "memory");
    return ok != 0;
}
// Drain wait: bounded, does not give up early on the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1; !mbar_try(bar, parity); i++)
        if ((i & 63) == 0 && global_ns() - t0 > kWaitLimitNs) return;
}

// Optional wait statistics (kernels instantiated with STATS): cycles a role spends in each
// wait site, summed over warps (one lane per warp) into stats[site].
enum StatSite {
    kStProdRawEmpty = 0, kStProdBEmpty, kStMmaAccEmpty, kStMmaBFull, kStMmaAFull, kStDeqRawFull, kStDeqAEmpty,
    kStEpiAccFull, kStDeqTotal, kStMmaTotal, kStDeqDecode, kStDeqStore, kStEpiWork, kStMmaTest, kStMmaIssue,
    kStSites
};
template <bool EN>
struct StatTimer {
    unsigned long long acc[EN ? kStSites : 1];
    long long t;
    __device__ __forceinline__ void reset() {
        if (EN)
            for (int i = 0; i < kStSites; i++) acc[i] = 0;
    }
    __device__ __forceinline__ void start() {
        if (EN) t = clock64();
    }
    __device__ __forceinline__ void stop(int site) {
        if (EN) acc[site] += (unsigned long long)(clock64() - t);
    }
    __device__ __forceinline__ void total(int site, long long t0) {
        if (EN) acc[site] = (unsigned long long)(clock64() - t0);
    }
    __device__ void flush(unsigned long long* stats) {
        if (EN && stats)
            for (int i = 0; i < kStSites; i++)
                if (acc[i]) atomicAdd(stats + i, acc[i]);
    }
};

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
// the same with an L2 eviction-priority policy (createpolicy)
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16, fp32 accumulate
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]),
        "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]),
        "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// instruction descriptor: D fp32, A/B fp16, both K-major, M = 128, N = n
__device__ __forceinline__ uint32_t idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// shared-memory descriptor of a K-major, 128-byte-swizzled operand tile (rows of 128 B,
// 8-row atoms of 1024 B stacked densely): start >> 4, LBO 16 B, SBO 1024 B, version 1, SW128
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// ---------------------------------------------------------------- dequantisation (-> fp16)
// Operand K order.  A dequant thread turns one 32-bit word of packed codes into fp16 pairs with
// one LOP3 per pair: the two values of a pair are bytes 0 and 2 (or 1 and 3) of the word, i.e.
// K positions 4w + {0, 2} and 4w + {1, 3}.  Both operands of the MMAs therefore hold K in the
// order "positions 1 and 2 of every group of 4 swapped": the weights by construction here, the
// activations by the gather (gather_*_kernel) and by the gate/up epilogue, which writes the
// down GEMM's activation rows.  A dot product does not depend on the order of its terms'
// pairing, so the result is that of the natural order (up to fp32 accumulation order).
__host__ __device__ __forceinline__ int kperm(int i) { return (i & ~3) | ((i & 1) << 1) | ((i >> 1) & 1); }

__device__ __forceinline__ uint32_t lop_or_mask(uint32_t a, uint32_t mask, uint32_t bits) {
    // (a & mask) | bits in one LOP3
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bits));
    return r;
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ __half2 u2h2(uint32_t u) { return *reinterpret_cast<const __half2*>(&u); }
__device__ __forceinline__ uint32_t h22u(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }

// Q4_K 6-bit scale/min of sub-block j (0..7) from the 12 scale bytes held in three words
// (s0 = bytes 0-3, s1 = 4-7, s2 = 8-11; src/m5_kern_scalar.c:39-46), without indexing memory
__device__ __forceinline__ void q4k_sm_words(uint32_t s0, uint32_t s1, uint32_t s2, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63;
        mn = (s1 >> (8 * j)) & 63;
    } else {
        const int b = 8 * (j - 4);
        const uint32_t e2 = (s2 >> b) & 0xff;
        sc = (int)((e2 & 15) | (((s0 >> b) >> 6 & 3) << 4));
        mn = (int)((e2 >> 4) | (((s1 >> b) >> 6 & 3) << 4));
    }
}

// Per-sub-block constants of the Q4_K decode in fp16x2 arithmetic.  The reference's value is
// w = d*sc*q - dmin*m (src/m5_kern_scalar.c:73-83).  With H = 1024 + 16q (the nibble placed in
// mantissa bits 4-7 under exponent 10):
//   I = fma(H, sc/16, -72 sc) = sc*(q - 8)          exact (integer |I| <= 504)
//   w = fma(I, d, C),  C = fp16(8 d sc - dmin m)       one rounding of d*sc*(q-8) + C
// Centring q on 8 leaves C small wherever the sub-block's values are centred (the min term is
// about 8 scale steps), so w is the fp16 rounding of the exact value up to C's own rounding.
struct Q4Sub {
    __half2 sc16, off, d, c;
};
// small non-negative integer (< 2^23) to float without the conversion unit: 2^23 + v in the
// mantissa, minus 2^23 (exact)
__device__ __forceinline__ float small_int_f(int v) { return __int_as_float(0x4B000000 + v) - 8388608.f; }
// d_bits: the superblock's fp16 d; d, dmin: as floats
__device__ __forceinline__ Q4Sub q4_sub(uint32_t d_bits, float d, float dmin, int sc, int mn) {
    Q4Sub r;
    // sc / 16 exactly: fp16 1024 + sc (bits 0x6400 + sc) times 1/16 minus 64; both halves
    const __half2 h = u2h2((0x6400u + (uint32_t)sc) * 0x00010001u);
    r.sc16 = __hfma2(h, __float2half2_rn(0.0625f), __float2half2_rn(-64.f));
    r.off = __hmul2(r.sc16, __float2half2_rn(-1152.f));   // -72 sc, exact
    r.d = u2h2(d_bits * 0x00010001u);
    const float scf = small_int_f(sc), mnf = small_int_f(mn);
    const float cf = __fsub_rn(8.f * d * scf, dmin * mnf);
    r.c = __floats2half2_rn(cf, cf);
    return r;
}
__device__ __forceinline__ uint32_t q4_pair(uint32_t hbits, const Q4Sub& k) {
    const __half2 i = __hfma2(u2h2(hbits), k.sc16, k.off);
    return h22u(__hfma2(i, k.d, k.c));
}

// Q4_K: 64 values [64*kc, 64*kc+64) of one superblock row -> 32 fp16 pairs (kperm order)
__device__ __forceinline__ void deq_q4k(const uint8_t* blk, int kc, uint32_t (&out)[32]) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const float d = h2f((uint16_t)(hd.x & 0xffff)), dmin = h2f((uint16_t)(hd.x >> 16));
    int sc0, m0, sc1, m1;
    q4k_sm_words(hd.y, hd.z, hd.w, 2 * kc, sc0, m0);
    q4k_sm_words(hd.y, hd.z, hd.w, 2 * kc + 1, sc1, m1);
    const Q4Sub k0 = q4_sub(hd.x & 0xffffu, d, dmin, sc0, m0), k1 = q4_sub(hd.x & 0xffffu, d, dmin, sc1, m1);
    const uint4* qv = reinterpret_cast<const uint4*>(blk + 16 + 32 * kc);
    constexpr uint32_t kMask = 0x00F000F0u, kMagic = 0x64006400u;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint4 q = qv[h];
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint32_t word = c == 0 ? q.x : c == 1 ? q.y : c == 2 ? q.z : q.w;
            const int w = 4 * h + c;
            // low nibbles (sub-block 2kc) of bytes 0,2 and 1,3; high nibbles (2kc+1) likewise,
            // each moved to bits 4-7 of its half
            out[2 * w] = q4_pair(lop_or_mask(word << 4, kMask, kMagic), k0);
            out[2 * w + 1] = q4_pair(lop_or_mask(word >> 4, kMask, kMagic), k0);
            out[16 + 2 * w] = q4_pair(lop_or_mask(word, kMask, kMagic), k1);
            out[16 + 2 * w + 1] = q4_pair(lop_or_mask(word >> 8, kMask, kMagic), k1);
        }
    }
}

// Q6_K (224-byte padded superblock): values p in [64*kc, 64*kc+64)
//   ql byte (p>>7)*64 + (p&63), high nibble if (p>>6)&1; qh byte (p>>7)*32 + (p&31), shift
//   ((p>>5)&3)*2; scale sc[p>>4]; w = d * sc * (q - 32)   (src/m5_kern_scalar.c:115-142)
// fp16x2 arithmetic: H = 1024 + q (PRMT under the exponent byte 0x64), Q = H - 1056 = q - 32
// exact; S = d*sc exact in fp32 is split S = S_hi + S_lo (both fp16) and w = fma(Q, S_hi,
// Q*S_lo): the fp16 rounding of Q*S up to the tiny rounding of Q*S_lo.
__device__ __forceinline__ void deq_q6k(const uint8_t* blk, int kc, uint32_t (&out)[32]) {
    const int h = kc >> 1, nhi = kc & 1;
    const uint4* qlv = reinterpret_cast<const uint4*>(blk + h * 64);
    const uint4* qhv = reinterpret_cast<const uint4*>(blk + 128 + h * 32);
    const uint32_t scw = *reinterpret_cast<const uint32_t*>(blk + 192 + 4 * kc);
    const float d = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
    const int nsh = 4 * nhi;
    const __half2 m1056 = __float2half2_rn(-1056.f);
    // 4 groups of 16 values: group g covers p = 64kc + 16g .. +16 with scale sc[4kc + g];
    // ql byte 16g + i of this half, qh byte 16(g & 1) + i, 2-bit field at (2 nhi + g/2) * 2
#pragma unroll
    for (int g = 0; g < 4; g++) {
        // int8 scale to float without the conversion unit: (sc + 128) via the mantissa, minus 128
        const float S = d * (small_int_f((int)((scw >> (8 * g)) & 0xffu) ^ 0x80) - 128.f);
        const __half shi = __float2half_rn(S);
        const __half2 s_hi = __half2half2(shi);
        const __half2 s_lo = __float2half2_rn(__fsub_rn(S, __half2float(shi)));
        const uint4 l = qlv[g];
        const uint4 q2 = qhv[g & 1];
        const int shift = (2 * nhi + (g >> 1)) * 2;   // field -> bits 4-5 of each byte
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const uint32_t lw = w == 0 ? l.x : w == 1 ? l.y : w == 2 ? l.z : l.w;
            const uint32_t hw = w == 0 ? q2.x : w == 1 ? q2.y : w == 2 ? q2.z : q2.w;
            const uint32_t hs = shift >= 4 ? hw >> (shift - 4) : hw << (4 - shift);
            const uint32_t q6 = lop_or_mask(lw >> nsh, 0x0F0F0F0Fu, hs & 0x30303030u);
            const __half2 q02 = __hadd2(u2h2(__byte_perm(q6, 0x64646464u, 0x4240)), m1056);
            const __half2 q13 = __hadd2(u2h2(__byte_perm(q6, 0x64646464u, 0x4341)), m1056);
            out[8 * g + 2 * w] = h22u(__hfma2(q02, s_hi, __hmul2(q02, s_lo)));
            out[8 * g + 2 * w + 1] = h22u(__hfma2(q13, s_hi, __hmul2(q13, s_lo)));
        }
    }
}

// ---------------------------------------------------------------- the kernel
// NT = most tokens per item (64 or 128).  With 64-token tiles two warps issue the MMAs (even
// and odd K steps) into separate accumulators that the epilogue adds: both issuers' per-step
// overheads (readiness test, commit) then overlap.
template <int MODE, int CODE, int NT>
struct Cfg {
    static constexpr int kIssuers = NT == 64 ? DRACO_TC_ISSUERS_64 : 1;
    // TMEM: 2 accumulator buffers (kIssuers x NT columns each), then the A slots of 64 columns
    static constexpr int kABase = 2 * kIssuers * NT;
    static constexpr int kSlots = NT == 64 ? DRACO_TC_SLOTS_64 : 4;
    static constexpr int kThreads = 32 * (NT == 64 ? 24 : 23);
    // TMEM columns of accumulator (buffer b, issuer i): b * kAccStride + i * NT
    static constexpr int kAccStride = kIssuers * NT;
    static constexpr int kBB = CODE == DRACO_CODE_Q4_K ? 144 : kQ6Padded;   // raw bytes per row superblock
    static constexpr int kRawStage = 128 * kBB;
    // activation stages: one K step = two 64-wide chunks x NT tokens x 128 B
    static constexpr int kBStage = NT * 256;
    static constexpr int kBStages = NT == 64 ? DRACO_TC_B_STAGES_64 : 4;
    // weight stages next to them (227 KB per block)
    static constexpr int kRawStages = NT == 64 ? (CODE == DRACO_CODE_Q4_K ? DRACO_TC_RAW_STAGES_Q4K_64 : DRACO_TC_RAW_STAGES_Q6K_64)
                                               : (CODE == DRACO_CODE_Q4_K ? DRACO_TC_RAW_STAGES_Q4K : DRACO_TC_RAW_STAGES_Q6K);
    static constexpr int kBOff = kRawStages * kRawStage;                 // 1024-aligned below
    static constexpr int kBOffAligned = (kBOff + 1023) / 1024 * 1024;
    static constexpr int kBarOff = kBOffAligned + kBStages * kBStage;
    static constexpr int kSmem = kBarOff + 1024 + 1024;                    // barriers + alignment slack
    static_assert(kRawStages <= kMaxRawStages && kBStages <= kMaxBStages && kBStages <= kDone &&
                      kSlots <= kDone && kSlots <= kMaxSlots && kABase + 64 * kSlots <= kTmemCols &&
                      kSmem <= 232448,
                  "rings and shared memory");
};

// one copy of a map brings a K step's two 64-wide chunks for R tokens as two SW128 tiles of R
// rows (tile c at byte c * R * 128)
using ActMaps = TcActMaps;

struct Bars {
    uint64_t raw_full[kMaxRawStages], raw_empty[kMaxRawStages];
    uint64_t a_full[kMaxSlots], b_full[kMaxBStages];
    uint64_t done[kDone];                      // done[q % 8]: MMAs of K step q finished
    uint64_t acc_full[2], acc_empty[2], drain[2];
    uint32_t tmem_base;
    int abort_flag;
};

// TMEM lane m (= 32 * quarter + i) of a gate/up tile holds raw row
//   gate: 16*quarter + ((i & 16) >> 1) + (i & 7)         for (i & 8) == 0
//   up:   64 + the same                                  for (i & 8) != 0
// so lanes i and i^8 hold gate and up of one intermediate row; down tiles are unpermuted.
__device__ __forceinline__ int gu_row(int quarter, int i) { return 16 * quarter + ((i & 16) >> 1) + (i & 7); }

template <int MODE, int CODE, int NT, bool STATS>
__global__ void __launch_bounds__(Cfg<MODE, CODE, NT>::kThreads, 1)
    moe_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                  const __grid_constant__ ActMaps tmB, const int4* __restrict__ items,
                  const int* __restrict__ n_items_p, int rows_per_expert, int K, int out_ld,
                  __half* __restrict__ act_out, float* __restrict__ y_out, int* __restrict__ err,
                  unsigned long long* __restrict__ stats) {
    using C = Cfg<MODE, CODE, NT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-align the dynamic shared memory base (swizzled tiles need it) by pointer arithmetic
    // on the shared array, so every access below stays a shared-memory access
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* raw = smem;
    uint8_t* bt = smem + C::kBOffAligned;
    Bars* bars = reinterpret_cast<Bars*>(smem + C::kBarOff);
    volatile int* abort_flag = &bars->abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = *n_items_p;
    const int nb = K / 256;   // superblock columns per item; K steps per item = 2 * nb

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::kRawStages; i++) {
            mbar_init(&bars->raw_full[i], 1);
            mbar_init(&bars->raw_empty[i], kDeqWarps);
        }
        for (int i = 0; i < C::kSlots; i++) mbar_init(&bars->a_full[i], kDeqWarps / 2);
        for (int i = 0; i < C::kBStages; i++) mbar_init(&bars->b_full[i], 1);
        for (int i = 0; i < kDone; i++) mbar_init(&bars->done[i], 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&bars->acc_full[i], C::kIssuers);
            mbar_init(&bars->acc_empty[i], 4);
            mbar_init(&bars->drain[i], 1);
        }
        bars->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&bars->tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    StatTimer<STATS> st;
    st.reset();
    const long long t_begin = STATS ? clock64() : 0;

    // The three issuing roles run warp-converged loops (every lane waits and computes the same
    // values, so they stay in uniform registers) and one elected lane issues each TMA copy,
    // MMA and commit.
    if (warp == kProdWarp) {
        // ------------------------------------------------------------ weight producer
        const uint64_t pol = policy_evict_first();   // weights stream through L2 once
        uint32_t sq = 0;   // superblock columns issued so far
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const int4 item = items[it];
            const int row0 = item.x * rows_per_expert + item.y * (MODE == 0 ? 64 : 128);
            for (int sb = 0; sb < nb; sb++, sq++) {
                const int s = sq % C::kRawStages;
                st.start();
                ok = warp_wait(&bars->raw_empty[s], ((sq / C::kRawStages) & 1) ^ 1, abort_flag, err, 1);
                st.stop(kStProdRawEmpty);
                if (!ok) break;
                if (elect_one()) {
                    uint8_t* dst = raw + s * C::kRawStage;
                    mbar_expect_tx(&bars->raw_full[s], C::kRawStage);
                    tma_load_2d_hint(dst, &tmA0, sb * (C::kBB / 4), row0, &bars->raw_full[s], pol);
                    tma_load_2d_hint(dst + 64 * C::kBB, MODE == 0 ? &tmA1 : &tmA0, sb * (C::kBB / 4),
                                     MODE == 0 ? row0 : row0 + 64, &bars->raw_full[s], pol);
                }
                __syncwarp();
            }
        }
        if (!ok)   // drain: the most recent fills land before the CTA exits
            for (uint32_t k = 0; k < (uint32_t)C::kRawStages && k < sq; k++) {
                const uint32_t q = sq - 1 - k;
                mbar_drain(&bars->raw_full[q % C::kRawStages], (q / C::kRawStages) & 1);
            }
    } else if (warp == kBProdWarp) {
        // ------------------------------------------------------------ activation producer
        uint32_t q = 0;   // K steps issued so far
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const int4 item = items[it];
            const int p0 = item.z, nbox = (item.w + 15) >> 4;
            const CUtensorMap* map = &tmB.m[nbox - 1];
            for (int s2 = 0; s2 < 2 * nb; s2++, q++) {
                const int bs = q % C::kBStages;
                if (q >= (uint32_t)C::kBStages) {   // stage reused: step q - kBStages finished
                    const uint32_t r = q - C::kBStages;
                    st.start();
                    ok = warp_wait(&bars->done[r % kDone], (r / kDone) & 1, abort_flag, err, 2);
                    st.stop(kStProdBEmpty);
                    if (!ok) break;
                }
                if (elect_one()) {
                    mbar_expect_tx(&bars->b_full[bs], 2 * nbox * 16 * 128);
                    tma_load_3d(bt + bs * C::kBStage, map, 0, p0, 2 * s2, &bars->b_full[bs]);
                }
                __syncwarp();
            }
        }
        if (!ok)
            for (uint32_t k = 0; k < (uint32_t)C::kBStages && k < q; k++) {
                const uint32_t r = q - 1 - k;
                mbar_drain(&bars->b_full[r % C::kBStages], (r / C::kBStages) & 1);
            }
    } else if (warp == kMmaWarp || (C::kIssuers == 2 && warp == kMmaWarp2)) {
        // ------------------------------------------------------------ MMA issuer(s)
        const int iss = warp == kMmaWarp ? 0 : 1;   // issues the K steps with (step & 1) == iss
        const uint64_t desc0 = sdesc_sw128(smem_u32(bt));
        uint32_t q = 0, n_done = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, n_done++) {
            const int4 item = items[it];
            const int nbox = (item.w + 15) >> 4;
            const uint32_t idesc = idesc_f16(nbox * 16);
            const uint32_t sub = (uint32_t)nbox * (16 * 128 >> 4);   // second chunk's tile, 16-byte units
            const int buf = n_done & 1;
            if (n_done >= 2) {   // the epilogue of item n_done - 2 has read this buffer
                st.start();
                ok = warp_wait(&bars->acc_empty[buf], ((n_done >> 1) & 1) ^ 1, abort_flag, err, 3);
                st.stop(kStMmaAccEmpty);
                if (!ok) break;
                tc_fence_after();
            }
            const uint32_t d_tm = tmem + buf * C::kAccStride + iss * NT;
            const int nsteps = 2 * nb;   // even, so a step's parity is the same in every item
            uint32_t qi = q + (C::kIssuers == 2 ? iss : 0);   // this issuer's first step
            bool rdy = __all_sync(0xffffffffu, mbar_test2(&bars->a_full[qi % C::kSlots], (qi / C::kSlots) & 1,
                                                          &bars->b_full[qi % C::kBStages], (qi / C::kBStages) & 1));
            for (int s2 = qi - q; s2 < nsteps; s2 += C::kIssuers, qi += C::kIssuers) {
                const int sl = qi % C::kSlots, bs = qi % C::kBStages;
                if (!rdy) {
                    st.start();
                    ok = warp_wait(&bars->a_full[sl], (qi / C::kSlots) & 1, abort_flag, err, 5);
                    st.stop(kStMmaAFull);
                    if (!ok) break;
                    st.start();
                    ok = warp_wait(&bars->b_full[bs], (qi / C::kBStages) & 1, abort_flag, err, 4);
                    st.stop(kStMmaBFull);
                    if (!ok) break;
                }
                tc_fence_after();
                // readiness of this issuer's next step, tested before this step's MMAs are issued
                st.start();
                const uint32_t qn = qi + C::kIssuers;
                if (s2 + C::kIssuers < nsteps)
                    rdy = __all_sync(0xffffffffu,
                                     mbar_test2(&bars->a_full[qn % C::kSlots], (qn / C::kSlots) & 1,
                                                &bars->b_full[qn % C::kBStages], (qn / C::kBStages) & 1));
                st.stop(kStMmaTest);
                st.start();
                const uint32_t a_tm = tmem + C::kABase + 64 * sl;
                const uint64_t bd = desc0 + (uint64_t)(bs * (C::kBStage >> 4));
                const bool first = s2 < C::kIssuers;   // this accumulator's first step of the item
                if (elect_one()) {
#pragma unroll
                    for (int c = 0; c < 2; c++) {
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            tc_mma_ts(d_tm, a_tm + 32 * c + 8 * j, bd + (uint64_t)(c * sub + 2 * j), idesc,
                                      (!first || c || j) ? 1u : 0u);
                    }
                    tc_commit(&bars->done[qi % kDone]);
                }
                __syncwarp();
                st.stop(kStMmaIssue);
            }
            q += nsteps;
            if (ok && elect_one()) tc_commit(&bars->acc_full[buf]);
            __syncwarp();
        }
        // every issued MMA must finish before TMEM is released
        if (elect_one()) {
            tc_commit(&bars->drain[iss]);
            mbar_drain(&bars->drain[iss], 0);
        }
        __syncwarp();
    } else if (warp < kDeqWarps) {
        // ------------------------------------------------------------ dequant
        // warpgroup wg decodes the 64-value chunk wg of every superblock column, i.e. half
        // (wg & 1) of K step 2 * column + (wg >> 1)
        const int wg = warp >> 2, quarter = warp & 3;
        const int row = MODE == 0 ? ((lane >> 3) & 1) * 64 + gu_row(quarter, lane) : quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        uint32_t sq = 0;   // superblock columns consumed
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            for (int sb = 0; sb < nb; sb++, sq++) {
                const uint32_t q = 2 * sq + (wg >> 1);   // this warpgroup's K step
                const int rs = sq % C::kRawStages, sl = q % C::kSlots;
                st.start();
                ok = warp_wait(&bars->raw_full[rs], (sq / C::kRawStages) & 1, abort_flag, err, 7);
                st.stop(kStDeqRawFull);
                if (!ok) break;
                if (q >= (uint32_t)C::kSlots) {   // slot reused: step q - 4 finished
                    const uint32_t r = q - C::kSlots;
                    st.start();
                    ok = warp_wait(&bars->done[r % kDone], (r / kDone) & 1, abort_flag, err, 8);
                    st.stop(kStDeqAEmpty);
                    if (!ok) break;
                }
                tc_fence_after();
                uint32_t v[32];
                const uint8_t* blk = raw + rs * C::kRawStage + row * C::kBB;
                st.start();
                if (CODE == DRACO_CODE_Q4_K) deq_q4k(blk, wg, v);
                else deq_q6k(blk, wg, v);
                st.stop(kStDeqDecode);
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->raw_empty[rs]);
                st.start();
                tc_st32(tmem + lane_base + C::kABase + 64 * sl + 32 * (wg & 1), v);
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->a_full[sl]);
                st.stop(kStDeqStore);
            }
        }
        st.total(kStDeqTotal, t_begin);
    } else if (warp >= kEpiWarp0) {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        // 16 accumulator columns, the two issuers' partial sums added (even steps first)
        auto ld_acc = [&](uint32_t addr, uint32_t (&v)[16]) {
            tc_ld16(addr, v);
            if (C::kIssuers == 2) {
                uint32_t w[16];
                tc_ld16(addr + NT, w);
                tc_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] = __float_as_uint(__fadd_rn(__uint_as_float(v[i]), __uint_as_float(w[i])));
            } else {
                tc_wait_ld();
            }
        };
        uint32_t n_done = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, n_done++) {
            const int4 item = items[it];
            const int mt = item.y, p0 = item.z, ntok = item.w;
            const int buf = n_done & 1;
            st.start();
            const bool ok = warp_wait(&bars->acc_full[buf], (n_done >> 1) & 1, abort_flag, err, 9);
            st.stop(kStEpiAccFull);
            if (!ok) break;
            st.start();
            tc_fence_after();
            const uint32_t acc = tmem + lane_base + buf * C::kAccStride;
            if (MODE == 0) {
                // lanes i (gate) and i ^ 8 (up) share an intermediate row; per column pair the
                // gate lane finishes the even column and the up lane the odd one
                const bool is_up = (lane & 8) != 0;
                const int orow = mt * 64 + gu_row(quarter, lane);
                for (int tb = 0; tb < ntok; tb += 16) {
                    uint32_t v[16];
                    ld_acc(acc + tb, v);
#pragma unroll
                    for (int c = 0; c < 16; c += 2) {
                        const float mine_e = __uint_as_float(v[c]), mine_o = __uint_as_float(v[c + 1]);
                        const float other = __shfl_xor_sync(0xffffffffu, is_up ? mine_e : mine_o, 8);
                        const float g = is_up ? other : mine_e, u = is_up ? mine_o : other;
                        const int col = tb + c + (is_up ? 1 : 0);
                        if (col < ntok)
                            // SwiGLU with the hardware exp: the value is rounded to fp16 next, and the
                            // bit-exact libm exp (silu_mul) halved the gate/up kernel's speed (one
                            // epilogue warpgroup per SM: cfg4 466 -> 230 us, cfg2 111 -> 90 us) at the
                            // same layer rel-L2 (5.53e-4 both on cfg2)
                            act_out[(size_t)(p0 + col) * out_ld + kperm(orow)] =
                                __float2half_rn(g / (1.f + __expf(-g)) * u);
                    }
                }
            } else {
                // down: fp32 rows into y_out, or (act_out given) fp16 rows into act_out
                const int orow = mt * 128 + quarter * 32 + lane;
                for (int tb = 0; tb < ntok; tb += 16) {
                    uint32_t v[16];
                    ld_acc(acc + tb, v);
                    const int nt = min(16, ntok - tb);
                    if (act_out) {
                        __half* dst = act_out + (size_t)(p0 + tb) * out_ld + orow;
#pragma unroll
                        for (int t = 0; t < 16; t++)
                            if (t < nt) dst[(size_t)t * out_ld] = __float2half_rn(__uint_as_float(v[t]));
                    } else {
                        float* dst = y_out + (size_t)(p0 + tb) * out_ld + orow;
#pragma unroll
                        for (int t = 0; t < 16; t++)
                            if (t < nt) dst[(size_t)t * out_ld] = __uint_as_float(v[t]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
            st.stop(kStEpiWork);
        }
    }
    if (warp == kMmaWarp) st.total(kStMmaTotal, t_begin);   // the first issuer only
    if (lane == 0) st.flush(stats);
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------- helpers
// items of one dense matrix triple over T token rows (a shared expert): tile-major, row tiles inner
__global__ void dense_items_kernel(int T, int nt, int mt_gu, int mt_dn, int4* __restrict__ gu, int* __restrict__ n_gu,
                                   int4* __restrict__ dn, int* __restrict__ n_dn) {
    const int tiles = (T + nt - 1) / nt;
    for (int j = threadIdx.x; j < tiles * mt_gu; j += blockDim.x) {
        const int t = j / mt_gu;
        gu[j] = make_int4(0, j % mt_gu, t * nt, min(nt, T - t * nt));
    }
    for (int j = threadIdx.x; j < tiles * mt_dn; j += blockDim.x) {
        const int t = j / mt_dn;
        dn[j] = make_int4(0, j % mt_dn, t * nt, min(nt, T - t * nt));
    }
    if (threadIdx.x == 0) {
        *n_gu = tiles * mt_gu;
        *n_dn = tiles * mt_dn;
    }
}

// fp16 copy of the token rows in expert-sorted order: Xs[p] = X[ilist[p] / tok_div]
// rows [0, n) with n = *n_valid when given (the assignments the dispatch placed; routing entries
// that name no expert of the table leave the tail of ilist unwritten), else P
__global__ void gather_half_kernel(const float* __restrict__ X, const int* __restrict__ ilist,
                                   const int* __restrict__ n_valid, int tok_div, int P, int H,
                                   __half* __restrict__ Xs) {
    const int per_row = H / 8;
    const int n = n_valid ? min(*n_valid, P) : P;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < (long)n * per_row;
         i += (long)gridDim.x * blockDim.x) {
        const int p = (int)(i / per_row), c8 = (int)(i % per_row) * 8;
        const int t = ilist ? ilist[p] / tok_div : p;
        const float4 a = *reinterpret_cast<const float4*>(X + (size_t)t * H + c8);
        const float4 b = *reinterpret_cast<const float4*>(X + (size_t)t * H + c8 + 4);
        uint4 o;   // kperm order: positions 1 and 2 of each group of 4 swapped
        o.x = pack2(a.x, a.z);
        o.y = pack2(a.y, a.w);
        o.z = pack2(b.x, b.z);
        o.w = pack2(b.y, b.w);
        *reinterpret_cast<uint4*>(Xs + (size_t)p * H + c8) = o;
    }
}

// The same rows written token by token: each fp32 token row is read once and its fp16 copy
// stored to the slots of its valid assignments (pos_of[t*K + k], placed by the dispatch for
// 0 <= order < E), instead of re-reading the row once per assignment.
__global__ void gather_tokens_kernel(const float* __restrict__ X, const int* __restrict__ order,
                                     const int* __restrict__ pos_of, int T, int K, int E, int H,
                                     __half* __restrict__ Xs) {
    const int per_row = H / 8;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < (long)T * per_row;
         i += (long)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_row), c8 = (int)(i % per_row) * 8;
        const float4 a = *reinterpret_cast<const float4*>(X + (size_t)t * H + c8);
        const float4 b = *reinterpret_cast<const float4*>(X + (size_t)t * H + c8 + 4);
        uint4 o;   // kperm order: positions 1 and 2 of each group of 4 swapped
        o.x = pack2(a.x, a.z);
        o.y = pack2(a.y, a.w);
        o.z = pack2(b.x, b.z);
        o.w = pack2(b.y, b.w);
        for (int k = 0; k < K; k++) {
            const int e = order[(size_t)t * K + k];
            if (e >= 0 && e < E) *reinterpret_cast<uint4*>(Xs + (size_t)pos_of[(size_t)t * K + k] * H + c8) = o;
        }
    }
}

// the same from token rows that are already fp16
__global__ void gather_rows16_kernel(const __half* __restrict__ X, const int* __restrict__ ilist,
                                     const int* __restrict__ n_valid, int tok_div, int P, int H,
                                     __half* __restrict__ Xs) {
    const int per_row = H / 8;
    const int n = n_valid ? min(*n_valid, P) : P;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < (long)n * per_row;
         i += (long)gridDim.x * blockDim.x) {
        const int p = (int)(i / per_row), c8 = (int)(i % per_row) * 8;
        const int t = ilist ? ilist[p] / tok_div : p;
        const uint4 a = *reinterpret_cast<const uint4*>(X + (size_t)t * H + c8);
        uint4 o;   // kperm order
        o.x = __byte_perm(a.x, a.y, 0x5410);
        o.y = __byte_perm(a.x, a.y, 0x7632);
        o.z = __byte_perm(a.z, a.w, 0x5410);
        o.w = __byte_perm(a.z, a.w, 0x7632);
        *reinterpret_cast<uint4*>(Xs + (size_t)p * H + c8) = o;
    }
}

}  // namespace tc

// ------------------------------------------------------------------------------ host side
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool get_encode() {
    if (g_encode) return true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
        return false;
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    return true;
}

// weights [rows_total][row_bytes] viewed as uint32 elements, box = one superblock column x 64 rows
bool map_weights(CUtensorMap* m, const void* base, size_t rows_total, size_t row_bytes_, int bb) {
    const cuuint64_t dims[2] = {row_bytes_ / 4, rows_total};
    const cuuint64_t strides[1] = {row_bytes_};
    const cuuint32_t box[2] = {(cuuint32_t)(bb / 4), 64};
    const cuuint32_t es[2] = {1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// activations [P][K] fp16 as {64 halves, P rows, K/64 chunks}; box {64, 16 (i + 1), 2},
// 128-byte swizzle (the UMMA K-major SW128 layout)
bool map_acts(tc::ActMaps* m, const void* base, size_t P, size_t K) {
    const cuuint64_t dims[3] = {64, P, K / 64};
    const cuuint64_t strides[2] = {K * 2, 128};
    const cuuint32_t es[3] = {1, 1, 1};
    for (int i = 0; i < 8; i++) {
        const cuuint32_t box[3] = {64, (cuuint32_t)(16 * (i + 1)), 2};
        if (g_encode(&m->m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}
// encoded maps of the last few (buffer, rows, K), shared by all calls of the process
bool cached_act_maps(tc::ActMaps* out, const void* base, size_t P, size_t K) {
    struct Entry {
        const void* base;
        size_t P, K;
        tc::ActMaps maps;
    };
    static std::mutex mu;
    static Entry cache[4];
    static int next = 0;
    std::lock_guard<std::mutex> lk(mu);
    for (const Entry& e : cache)
        if (e.base == base && e.P == P && e.K == K) {
            *out = e.maps;
            return true;
        }
    Entry& e = cache[next];
    if (!map_acts(&e.maps, base, P, K)) {
        e.base = nullptr;
        return false;
    }
    e.base = base;
    e.P = P;
    e.K = K;
    next = (next + 1) % 4;
    *out = e.maps;
    return true;
}

template <int MODE, int CODE, int NT, bool STATS>
cudaError_t launch_tc_k(const CUtensorMap& a0, const CUtensorMap& a1, const tc::ActMaps& b, const int4* items,
                        const int* n_items, int grid, int rows_per_expert, int K, int out_ld, __half* act, float* y,
                        int* err, unsigned long long* stats, cudaStream_t s) {
    using C = tc::Cfg<MODE, CODE, NT>;
    auto kern = tc::moe_tc_kernel<MODE, CODE, NT, STATS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    kern<<<grid, C::kThreads, C::kSmem, s>>>(a0, a1, b, items, n_items, rows_per_expert, K, out_ld, act, y, err,
                                              stats);
    return cudaGetLastError();
}
template <int MODE, int CODE>
cudaError_t launch_tc(const CUtensorMap& a0, const CUtensorMap& a1, const tc::ActMaps& b, const int4* items,
                      const int* n_items, int grid, int nt, int rows_per_expert, int K, int out_ld, __half* act,
                      float* y, int* err, unsigned long long* stats, cudaStream_t s) {
    if (nt == 64)
        return stats ? launch_tc_k<MODE, CODE, 64, true>(a0, a1, b, items, n_items, grid, rows_per_expert, K, out_ld,
                                                         act, y, err, stats, s)
                     : launch_tc_k<MODE, CODE, 64, false>(a0, a1, b, items, n_items, grid, rows_per_expert, K, out_ld,
                                                          act, y, err, nullptr, s);
    return stats ? launch_tc_k<MODE, CODE, 128, true>(a0, a1, b, items, n_items, grid, rows_per_expert, K, out_ld, act,
                                                      y, err, stats, s)
                 : launch_tc_k<MODE, CODE, 128, false>(a0, a1, b, items, n_items, grid, rows_per_expert, K, out_ld,
                                                       act, y, err, nullptr, s);
}

}  // namespace

bool tc_supported(int cg, int cu, int cd, int inter, int n_in, int n_out) {
    auto ok = [](int c) { return c == DRACO_CODE_Q4_K || c == DRACO_CODE_Q6_K; };
    return ok(cg) && cg == cu && ok(cd) && inter % 256 == 0 && n_in % 256 == 0 && inter % 128 == 0 &&
           n_out % 128 == 0 && get_encode();
}

int tc_make_weight_maps(TcMaps* maps, const uint8_t* gate, const uint8_t* up, const uint8_t* down, int n_exp, int cg,
                        int cd, int inter, int n_in, int n_out) {
    if (!get_encode()) return -1;
    const int bbg = cg == DRACO_CODE_Q4_K ? 144 : kQ6Padded, bbd = cd == DRACO_CODE_Q4_K ? 144 : kQ6Padded;
    const size_t rg = (size_t)(n_in / 256) * bbg, rd = (size_t)(inter / 256) * bbd;
    if (!map_weights(&maps->gate, gate, (size_t)n_exp * inter, rg, bbg)) return -2;
    if (!map_weights(&maps->up, up, (size_t)n_exp * inter, rg, bbg)) return -2;
    if (!map_weights(&maps->down, down, (size_t)n_exp * n_out, rd, bbd)) return -2;
    return 0;
}

int tc_prepare(TcCall* call, int cg, int cd, int n_exp, int inter, int n_in, int n_out, int P, __half* Xs,
               __half* act_h) {
    call->cg = cg;
    call->cd = cd;
    call->n_exp = n_exp;
    call->inter = inter;
    call->n_in = n_in;
    call->n_out = n_out;
    call->P = P;
    call->nt = tc_token_tile(P, n_exp);
    if (P <= 0) return 0;
    if (!cached_act_maps(&call->mx, Xs, (size_t)P, (size_t)n_in) ||
        !cached_act_maps(&call->ma, act_h, (size_t)P, (size_t)inter))
        return -2;
    return 0;
}

void tc_dense_items(const TcCall& c, int4* items_gu, int* n_gu, int4* items_dn, int* n_dn, cudaStream_t s) {
    tc::dense_items_kernel<<<1, 256, 0, s>>>(c.P, c.nt, tc_tiles_gateup(c.inter), tc_tiles_down(c.n_out), items_gu,
                                             n_gu, items_dn, n_dn);
}

void tc_gather_tokens(const TcCall& c, const float* X, const int* order, const int* pos_of, int T, int K, int E,
                      __half* Xs, cudaStream_t s) {
    if (c.P <= 0 || T <= 0) return;
    tc::gather_tokens_kernel<<<148 * 8, 256, 0, s>>>(X, order, pos_of, T, K, E, c.n_in, Xs);
}

void tc_gather(const TcCall& c, const void* X, bool x_half, const int* ilist, const int* n_valid, int tok_div,
               __half* Xs, cudaStream_t s) {
    if (c.P <= 0) return;
    if (x_half)
        tc::gather_rows16_kernel<<<148 * 8, 256, 0, s>>>(static_cast<const __half*>(X), ilist, n_valid, tok_div, c.P,
                                                         c.n_in, Xs);
    else
        tc::gather_half_kernel<<<148 * 8, 256, 0, s>>>(static_cast<const float*>(X), ilist, n_valid, tok_div, c.P,
                                                       c.n_in, Xs);
}

int tc_gateup(const TcCall& c, const TcMaps& maps, const int4* items, const int* n_items, __half* act_h, int* err,
              unsigned long long* stats, cudaStream_t s) {
    if (c.P <= 0) return 0;
    cudaError_t e;
    if (c.cg == DRACO_CODE_Q4_K)
        e = launch_tc<0, DRACO_CODE_Q4_K>(maps.gate, maps.up, c.mx, items, n_items, 148, c.nt, c.inter, c.n_in, c.inter,
                                          act_h, nullptr, err, stats, s);
    else
        e = launch_tc<0, DRACO_CODE_Q6_K>(maps.gate, maps.up, c.mx, items, n_items, 148, c.nt, c.inter, c.n_in, c.inter,
                                          act_h, nullptr, err, stats, s);
    return e == cudaSuccess ? 0 : -3;
}

int tc_down(const TcCall& c, const TcMaps& maps, const int4* items, const int* n_items, void* y, bool half_out,
            int* err, unsigned long long* stats, cudaStream_t s) {
    if (c.P <= 0) return 0;
    cudaError_t e;
    __half* yh = half_out ? static_cast<__half*>(y) : nullptr;
    float* yf = half_out ? nullptr : static_cast<float*>(y);
    if (c.cd == DRACO_CODE_Q4_K)
        e = launch_tc<1, DRACO_CODE_Q4_K>(maps.down, maps.down, c.ma, items, n_items, 148, c.nt, c.n_out, c.inter,
                                          c.n_out, yh, yf, err, stats, s);
    else
        e = launch_tc<1, DRACO_CODE_Q6_K>(maps.down, maps.down, c.ma, items, n_items, 148, c.nt, c.n_out, c.inter,
                                          c.n_out, yh, yf, err, stats, s);
    return e == cudaSuccess ? 0 : -3;
}

}  // namespace draco
