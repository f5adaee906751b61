// Shared device helpers for the B200 MoE FFN kernels: GGUF superblock decoding, the
// exp used by the routers, and launch/error plumbing.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define DRACO_CODE_Q8_0 0
#define DRACO_CODE_Q6_K 4
#define DRACO_CODE_Q4_K 5
#define DRACO_CODE_F32 9

namespace draco {

// ------------------------------------------------------------------------------------------
// Formats (byte layouts of the reference's decoders, src/m5_kern_scalar.c:58-142)
// ------------------------------------------------------------------------------------------
__host__ __device__ inline int block_bytes(int code) {
    return code == DRACO_CODE_Q4_K ? 144 : code == DRACO_CODE_Q6_K ? 210 : code == DRACO_CODE_Q8_0 ? 34 : 0;
}
__host__ __device__ inline int block_values(int code) {
    return code == DRACO_CODE_Q8_0 ? 32 : 256;
}
// Q6_K superblocks are 210 B in GGUF files; copies held by the library's weight registry pad
// them to 224 B so every superblock starts on a 16-byte boundary (TMA-addressable).
constexpr int kQ6File = 210;
constexpr int kQ6Padded = 224;
// bytes of one row of n values; q6s = Q6_K superblock stride of the buffer (210 or 224)
__host__ __device__ inline size_t row_bytes(int code, int n, int q6s = kQ6File) {
    if (code == DRACO_CODE_Q6_K) return (size_t)(n / 256) * (size_t)q6s;
    const int bv = block_values(code);
    return (size_t)(n / bv) * (size_t)block_bytes(code);
}
__host__ inline bool code_supported(int code) {
    return code == DRACO_CODE_Q4_K || code == DRACO_CODE_Q6_K || code == DRACO_CODE_Q8_0;
}

// fp16 bits -> fp32, subnormals included (same values as src/m5_kern_scalar.c:9-21; the
// hardware conversion is exact for every fp16 input).
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Q4_K packed 6-bit scale and min of sub-block j from the 12 scale bytes
// (src/m5_kern_scalar.c:39-46).
__device__ __forceinline__ void q4k_sm(const uint8_t* s, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// ------------------------------------------------------------------------------------------
// expf with the exact results of the host C library the reference links (glibc >= 2.27 on
// x86-64, FMA code path).  Method: the table-driven exp of ARM's optimized-routines
// (Szabolcs Nagy, 2017), which glibc adopted: z = x * 32/ln2 in double, k = round(z),
// r = z - k (fused), 2^(k/32) from a 32-entry table of 2^(i/32) with the exponent folded
// into the integer bits, 2^(r/32) by a cubic in double, one final rounding to float.
// Checked against the host expf for all 2^32 float inputs during development; the tests
// compare the routers that use it bit-for-bit with the reference's C.
// ------------------------------------------------------------------------------------------
__constant__ uint64_t kExp2Tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

// the table-driven part for |x| < 88: 2^(k/32) from `lookup(k & 31)` (the 64-bit table entry)
template <typename Lookup>
__device__ __forceinline__ float host_expf_core(float x, Lookup lookup) {
    const double kInvLn2N = 0x1.71547652b82fep+0 * 32.0;
    const double kShift = 0x1.8p+52;
    const double kC0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    const double kC1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    const double kC2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = (double)x;
    const double z = __dmul_rn(kInvLn2N, xd);
    double kd = __dadd_rn(z, kShift);
    const uint64_t ki = (uint64_t)__double_as_longlong(kd);
    kd = __dsub_rn(kd, kShift);
    const double r = __fma_rn(kInvLn2N, xd, -kd);
    uint64_t t = lookup((int)(ki & 31));
    t += ki << 47;
    const double s = __longlong_as_double((long long)t);
    const double zz = __fma_rn(kC0, r, kC1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(kC2, r, 1.0);
    y = __fma_rn(zz, r2, y);
    y = __dmul_rn(y, s);
    return __double2float_rn(y);
}
// |x| >= 88, inf, nan: sets *res and returns true
__device__ __forceinline__ bool host_expf_special(float x, float* res) {
    const uint32_t ux = __float_as_uint(x);
    const uint32_t abstop = (ux >> 20) & 0x7ff;
    if (abstop < 0x42b) return false;               // |x| < 88 (top 12 bits of 88.0f)
    if (ux == 0xff800000u) *res = 0.0f;             // -inf
    else if (abstop >= 0x7f8) *res = x + x;         // nan / +inf
    else if (x > 0x1.62e42ep6f) *res = __int_as_float(0x7f800000);   // overflow
    else if (x < -0x1.9fe368p6f) *res = 0.0f;       // underflow
    else return false;
    return true;
}

__device__ __forceinline__ float host_expf(float x) {
    float sp;
    if (host_expf_special(x, &sp)) return sp;
    return host_expf_core(x, [](int i) { return kExp2Tab[i]; });
}

// The same for a whole converged warp: lane i holds table entry i (tab_lo, tab_hi: its low and
// high words, from exp_table_lane()), and each lane fetches its entry by shuffle instead of an
// indexed constant-memory read, which serialises over the lanes' distinct indices.  Every lane
// takes the shuffles; the special cases are selected afterwards.
__device__ __forceinline__ void exp_table_lane(uint32_t& tab_lo, uint32_t& tab_hi) {
    const uint64_t v = kExp2Tab[threadIdx.x & 31];
    tab_lo = (uint32_t)v;
    tab_hi = (uint32_t)(v >> 32);
}
__device__ __forceinline__ float host_expf_warp(float x, uint32_t tab_lo, uint32_t tab_hi) {
    const float y = host_expf_core(x, [&](int i) {
        return ((uint64_t)__shfl_sync(0xffffffffu, tab_hi, i) << 32) | __shfl_sync(0xffffffffu, tab_lo, i);
    });
    float sp;
    return host_expf_special(x, &sp) ? sp : y;
}

// g / (1 + e^-g) * u in the reference's operation order (src/m6_layer.c:733-736)
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, host_expf(-g))), u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace draco
