// Decode-sized grouped GEMV (few tokens per expert) on CUDA cores, fp32 activations.
//
// One block per (active expert, tile of rt weight rows): one thread bulk-copies the tile's rows
// of gate and up (or down), which are contiguous in the stacked expert tensor, from HBM into
// shared memory (cp.async.bulk on an mbarrier), so every resident block keeps its tile's bytes in
// flight independently of the arithmetic.  Four warps then take rt / 4 rows each: per 256-value
// superblock a lane decodes 8 values from aligned words of the staged bytes and multiplies them
// into per-token fp32 partial sums that a warp reduction finishes.  Decoding uses the byte-
// permute float trick: a 6-bit code q placed under exponent byte 0x40 is the float 2 + q/64, and
// one fma with (64 * scale, offset) gives scale * q - offset.
//
// Values are the reference's (src/m5_kern_scalar.c:69-142); the sums run in a different order
// (lane partials + tree), so results match the reference to rounding, not bit for bit.
#include "kernels.cuh"
#include "mbar.cuh"

namespace draco {
namespace {

constexpr int kDecWarps = 4;

__device__ __forceinline__ float code_float(uint32_t bytes4, int i) {   // 2 + byte_i / 64
    return __uint_as_float(__byte_perm(bytes4, 0x40000000u, 0x7044u | ((uint32_t)i << 8)));
}

// Q4_K 6-bit scale/min of sub-block j from the 12 scale bytes in three words (src/m5_kern_scalar.c:39-46)
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, int& sc, int& mn) {
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

// Lane layouts (8 values per lane per superblock, the lane's x positions as two float4):
//   Q4_K: qs word `lane`; low nibbles -> p = 64g + 4j + k (sub-block 2g), high -> p + 32,
//         g = lane >> 3, j = lane & 7
//   Q6_K: h = lane >> 4, i = lane & 15; ql word 64h + 4i, qh word 128 + 32h + 4(i & 7);
//         low nibbles -> p = 128h + 4i + k, high -> p + 64
template <int CODE>
__device__ __forceinline__ int x_pos(int lane) {
    if (CODE == DRACO_CODE_Q4_K) return 64 * (lane >> 3) + 4 * (lane & 7);
    return 128 * (lane >> 4) + 4 * (lane & 15);
}
template <int CODE>
__host__ __device__ constexpr int x_gap() {   // distance of the lane's second float4
    return CODE == DRACO_CODE_Q4_K ? 32 : 64;
}

// scale groups per superblock and their (64 * scale, -offset) pairs: Q4_K 8 sub-blocks of 32
// (a = 64 d sc_j, b = -(128 d sc_j + dmin m_j)), Q6_K 16 groups of 16 (a = 64 d sc, b = -160 d sc)
template <int CODE>
__host__ __device__ constexpr int scale_groups() {
    return CODE == DRACO_CODE_Q4_K ? 8 : 16;
}
template <int CODE>
__device__ __forceinline__ void superblock_scales(const uint8_t* blk, float2* out) {
    if (CODE == DRACO_CODE_Q4_K) {
        const uint4 hd = *reinterpret_cast<const uint4*>(blk);
        const float d = h2f((uint16_t)(hd.x & 0xffff)), dmin = h2f((uint16_t)(hd.x >> 16));
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int sc, mn;
            q4k_scale_min(hd.y, hd.z, hd.w, j, sc, mn);
            const float ds = d * (float)sc, dm = dmin * (float)mn;
            out[j] = make_float2(64.f * ds, -(128.f * ds + dm));
        }
    } else {
        const float d = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const float ds = d * (float)sc[j];
            out[j] = make_float2(64.f * ds, -160.f * ds);
        }
    }
}

// the lane's 8 weights of one superblock from its staged bytes and its row's scale table
template <int CODE>
__device__ __forceinline__ void decode8(const uint8_t* blk, const float2* tab, int lane, float w[8]) {
    if (CODE == DRACO_CODE_Q4_K) {
        const uint32_t qs = *reinterpret_cast<const uint32_t*>(blk + 16 + 4 * lane);
        const float4 ab = *reinterpret_cast<const float4*>(tab + 2 * (lane >> 3));   // sub-blocks 2g, 2g+1
        const uint32_t lo = qs & 0x0F0F0F0Fu, hi = (qs >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            w[k] = fmaf(code_float(lo, k), ab.x, ab.y);
            w[4 + k] = fmaf(code_float(hi, k), ab.z, ab.w);
        }
    } else {
        const int h = lane >> 4, i = lane & 15;
        const uint32_t ql = *reinterpret_cast<const uint32_t*>(blk + 64 * h + 4 * i);
        const uint32_t qh = *reinterpret_cast<const uint32_t*>(blk + 128 + 32 * h + 4 * (i & 7));
        const float2 sl = tab[8 * h + (i >> 2)], sh = tab[8 * h + 4 + (i >> 2)];
        const int s0 = 2 * (i >> 3);
        const uint32_t q_lo = (ql & 0x0F0F0F0Fu) | (((qh >> s0) & 0x03030303u) << 4);
        const uint32_t q_hi = ((ql >> 4) & 0x0F0F0F0Fu) | (((qh >> (s0 + 4)) & 0x03030303u) << 4);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            w[k] = fmaf(code_float(q_lo, k), sl.x, sl.y);
            w[4 + k] = fmaf(code_float(q_hi, k), sh.x, sh.y);
        }
    }
}

template <int CODE>
__device__ __forceinline__ void load_x8(const float* __restrict__ x, int sb, int lane, float v[8]) {
    const float* b = x + sb * 256 + x_pos<CODE>(lane);
    const float4 a = *reinterpret_cast<const float4*>(b);
    const float4 c = *reinterpret_cast<const float4*>(b + x_gap<CODE>());
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
}

__host__ __device__ __forceinline__ int superblock_bytes(int code, int q6s) {
    return code == DRACO_CODE_Q4_K ? 144 : q6s;
}
__host__ __device__ __forceinline__ int groups_of(int code) { return code == DRACO_CODE_Q4_K ? 8 : 16; }

// stage `bytes` of each of n matrices' tiles; returns false (after a second bounded wait for
// the copies) when the copy did not complete in time
__device__ __forceinline__ bool stage(uint64_t* bar, uint8_t* dst0, const uint8_t* src0, uint8_t* dst1,
                                      const uint8_t* src1, uint32_t bytes0, uint32_t bytes1, int* status) {
    if (threadIdx.x == 0) {
        sync::mbar_init(bar, 1);
        sync::fence_init();
        sync::mbar_expect_tx(bar, bytes0 + bytes1);
        sync::bulk_load(dst0, src0, bytes0, bar);
        if (bytes1) sync::bulk_load(dst1, src1, bytes1, bar);
    }
    __syncthreads();
    if (sync::mbar_wait(bar, 0)) return true;
    if (threadIdx.x == 0) atomicOr(status, 0x200);
    sync::mbar_wait(bar, 0);   // the copies must land before the block's shared memory goes away
    return false;
}

// scale tables of a staged tile: tab[(row * nb + sb) * G + j]
template <int CODE>
__device__ __forceinline__ void build_scales(const uint8_t* tile, int rows, int nb, int bb, float2* tab) {
    for (int idx = threadIdx.x; idx < rows * nb; idx += blockDim.x)
        superblock_scales<CODE>(tile + (size_t)idx * bb, tab + (size_t)idx * scale_groups<CODE>());
}

// dot products of the warp's rpw rows (of up to two matrices) with NT token rows
template <int CG, int CU, bool TWO, int NT>
__device__ __forceinline__ void rows_dot(const uint8_t* sg, const float2* tg, const uint8_t* su, const float2* tu,
                                         uint32_t rbg, uint32_t rbu, int bg, int bu, int nb, int r0, int rpw,
                                         const float* const (&xr)[2], int lane, float (&ag)[4][2], float (&au)[4][2]) {
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
        for (int j = 0; j < 2; j++) ag[r][j] = au[r][j] = 0.f;
    for (int sb = 0; sb < nb; sb++) {
        float xg[NT][8], xu[NT][8];
#pragma unroll
        for (int j = 0; j < NT; j++) {
            load_x8<CG>(xr[j], sb, lane, xg[j]);
            if (TWO && CG != CU) load_x8<CU>(xr[j], sb, lane, xu[j]);
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            if (r < rpw) {
                float w[8];
                const int rs = (r0 + r) * nb + sb;
                decode8<CG>(sg + (size_t)(r0 + r) * rbg + sb * bg, tg + (size_t)rs * scale_groups<CG>(), lane, w);
#pragma unroll
                for (int j = 0; j < NT; j++)
#pragma unroll
                    for (int i = 0; i < 8; i++) ag[r][j] = fmaf(w[i], xg[j][i], ag[r][j]);
                if (TWO) {
                    decode8<CU>(su + (size_t)(r0 + r) * rbu + sb * bu, tu + (size_t)rs * scale_groups<CU>(), lane, w);
#pragma unroll
                    for (int j = 0; j < NT; j++)
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            au[r][j] = fmaf(w[i], CG != CU ? xu[j][i] : xg[j][i], au[r][j]);
                }
            }
        }
    }
}

// gate/up + SwiGLU for the tokens of one expert: act[p][r] = silu(gate_e[r] . x_t) * (up_e[r] . x_t)
template <int CG, int CU>
__global__ void __launch_bounds__(32 * kDecWarps) dec_gateup_kernel(ExpertTable tab, const int* __restrict__ active,
                                                                   const int* __restrict__ n_active_p,
                                                                   const int* __restrict__ off,
                                                                   const int* __restrict__ ilist, int tok_div,
                                                                   const float* __restrict__ X, int inter, int n_in,
                                                                   int rt, float* __restrict__ act, int q6s,
                                                                   int* __restrict__ status) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t bar;
    const int ntile = inter / rt;
    const int item = blockIdx.x;
    if (item >= *n_active_p * ntile) return;
    const int e = active[item / ntile], tile = item % ntile;
    const int nb = n_in / 256;
    const int bg = superblock_bytes(CG, q6s), bu = superblock_bytes(CU, q6s);
    const uint32_t rbg = (uint32_t)(nb * bg), rbu = (uint32_t)(nb * bu);
    uint8_t* sg = dsm;
    uint8_t* su = dsm + rt * rbg;
    float2* tg = reinterpret_cast<float2*>(dsm + rt * (rbg + rbu));
    float2* tu = tg + rt * nb * scale_groups<CG>();
    if (!stage(&bar, sg, tab.w[3 * e] + (size_t)tile * rt * rbg, su, tab.w[3 * e + 1] + (size_t)tile * rt * rbu,
               rt * rbg, rt * rbu, status))
        return;
    build_scales<CG>(sg, rt, nb, bg, tg);
    build_scales<CU>(su, rt, nb, bu, tu);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rpw = rt / kDecWarps, r0 = warp * rpw;
    const int p0 = off[e], c = off[e + 1] - p0;
    for (int tc = 0; tc < c; tc += 2) {
        const int nt = min(2, c - tc);
        const float* xr[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int pj = p0 + tc + min(j, nt - 1);
            xr[j] = X + (size_t)(ilist ? ilist[pj] / tok_div : pj) * n_in;
        }
        float ag[4][2], au[4][2];
        if (nt == 2) rows_dot<CG, CU, true, 2>(sg, tg, su, tu, rbg, rbu, bg, bu, nb, r0, rpw, xr, lane, ag, au);
        else rows_dot<CG, CU, true, 1>(sg, tg, su, tu, rbg, rbu, bg, bu, nb, r0, rpw, xr, lane, ag, au);
#pragma unroll
        for (int r = 0; r < 4; r++) {
            if (r < rpw) {
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    if (j < nt) {
                        const float g = warp_sum(ag[r][j]), u = warp_sum(au[r][j]);
                        if (lane == 0) act[(size_t)(p0 + tc + j) * inter + tile * rt + r0 + r] = silu_mul(g, u);
                    }
                }
            }
        }
    }
}

// down: y[p][r] = down_e[r] . act[p] for the assignments p of one expert
template <int CD>
__global__ void __launch_bounds__(32 * kDecWarps) dec_down_kernel(ExpertTable tab, const int* __restrict__ active,
                                                                 const int* __restrict__ n_active_p,
                                                                 const int* __restrict__ off,
                                                                 const float* __restrict__ act, int inter, int n_out,
                                                                 int rt, float* __restrict__ y, int q6s,
                                                                 int* __restrict__ status) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t bar;
    const int ntile = n_out / rt;
    const int item = blockIdx.x;
    if (item >= *n_active_p * ntile) return;
    const int e = active[item / ntile], tile = item % ntile;
    const int nb = inter / 256;
    const int bd = superblock_bytes(CD, q6s);
    const uint32_t rbd = (uint32_t)(nb * bd);
    float2* td = reinterpret_cast<float2*>(dsm + rt * rbd);
    if (!stage(&bar, dsm, tab.w[3 * e + 2] + (size_t)tile * rt * rbd, nullptr, nullptr, rt * rbd, 0, status)) return;
    build_scales<CD>(dsm, rt, nb, bd, td);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rpw = rt / kDecWarps, r0 = warp * rpw;
    const int p0 = off[e], c = off[e + 1] - p0;
    for (int tc = 0; tc < c; tc += 2) {
        const int nt = min(2, c - tc);
        const float* xr[2] = {act + (size_t)(p0 + tc) * inter, act + (size_t)(p0 + tc + nt - 1) * inter};
        float ad[4][2], unused[4][2];
        if (nt == 2)
            rows_dot<CD, CD, false, 2>(dsm, td, nullptr, nullptr, rbd, 0, bd, 0, nb, r0, rpw, xr, lane, ad, unused);
        else
            rows_dot<CD, CD, false, 1>(dsm, td, nullptr, nullptr, rbd, 0, bd, 0, nb, r0, rpw, xr, lane, ad, unused);
#pragma unroll
        for (int r = 0; r < 4; r++) {
            if (r < rpw) {
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    if (j < nt) {
                        const float v = warp_sum(ad[r][j]);
                        if (lane == 0) y[(size_t)(p0 + tc + j) * n_out + tile * rt + r0 + r] = v;
                    }
                }
            }
        }
    }
}

// rows per tile: about 24 KB of each matrix, 4..16 rows, a multiple of 4 dividing `rows`
int tile_rows(int rows, uint32_t row_bytes_) {
    int rt = (int)(24576 / row_bytes_);
    rt = rt < 4 ? 4 : rt > 16 ? 16 : rt;
    rt &= ~3;
    while (rt > 4 && rows % rt) rt -= 4;
    return rows % rt ? 0 : rt;
}

}  // namespace

bool dec_supported(int cg, int cu, int cd, int inter, int n_in, int n_out, int q6s) {
    auto ok = [](int c) { return c == DRACO_CODE_Q4_K || c == DRACO_CODE_Q6_K; };
    auto rb = [&](int c, int n) { return (uint32_t)((n / 256) * superblock_bytes(c, q6s)); };
    return ok(cg) && ok(cu) && ok(cd) && (q6s == kQ6Padded || (cg != DRACO_CODE_Q6_K && cu != DRACO_CODE_Q6_K &&
                                                                cd != DRACO_CODE_Q6_K)) &&
           n_in % 256 == 0 && inter % 256 == 0 && tile_rows(inter, rb(cg, n_in) > rb(cu, n_in) ? rb(cg, n_in) : rb(cu, n_in)) &&
           tile_rows(n_out, rb(cd, inter));
}

int launch_dec_gateup(const ExpertTable& tab, int cg, int cu, const int* active, const int* n_active, int n_active_max,
                      const int* off, const int* ilist, int tok_div, const float* X, int inter, int n_in, float* act,
                      int q6s, int* status, cudaStream_t s) {
    const uint32_t rbg = (uint32_t)((n_in / 256) * superblock_bytes(cg, q6s));
    const uint32_t rbu = (uint32_t)((n_in / 256) * superblock_bytes(cu, q6s));
    const int rt = tile_rows(inter, rbg > rbu ? rbg : rbu);
    if (!rt) return -1;
    const size_t smem = (size_t)rt * (rbg + rbu) +
                        (size_t)rt * (n_in / 256) * (groups_of(cg) + groups_of(cu)) * sizeof(float2);
    const int grid = n_active_max * (inter / rt);
    if (grid <= 0) return 0;
#define DRACO_DEC_GU(A, B)                                                                                       \
    do {                                                                                                         \
        cudaFuncSetAttribute(dec_gateup_kernel<A, B>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);  \
        dec_gateup_kernel<A, B><<<grid, 32 * kDecWarps, smem, s>>>(tab, active, n_active, off, ilist, tok_div, X, \
                                                                    inter, n_in, rt, act, q6s, status);         \
    } while (0)
    constexpr int A = DRACO_CODE_Q4_K, B = DRACO_CODE_Q6_K;
    if (cg == A && cu == A) DRACO_DEC_GU(A, A);
    else if (cg == B && cu == B) DRACO_DEC_GU(B, B);
    else if (cg == A) DRACO_DEC_GU(A, B);
    else DRACO_DEC_GU(B, A);
#undef DRACO_DEC_GU
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_dec_down(const ExpertTable& tab, int cd, const int* active, const int* n_active, int n_active_max,
                    const int* off, const float* act, int inter, int n_out, float* y, int q6s, int* status,
                    cudaStream_t s) {
    const uint32_t rbd = (uint32_t)((inter / 256) * superblock_bytes(cd, q6s));
    const int rt = tile_rows(n_out, rbd);
    if (!rt) return -1;
    const size_t smem = (size_t)rt * rbd + (size_t)rt * (inter / 256) * groups_of(cd) * sizeof(float2);
    const int grid = n_active_max * (n_out / rt);
    if (grid <= 0) return 0;
    if (cd == DRACO_CODE_Q4_K) {
        cudaFuncSetAttribute(dec_down_kernel<DRACO_CODE_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        dec_down_kernel<DRACO_CODE_Q4_K><<<grid, 32 * kDecWarps, smem, s>>>(tab, active, n_active, off, act, inter,
                                                                          n_out, rt, y, q6s, status);
    } else {
        cudaFuncSetAttribute(dec_down_kernel<DRACO_CODE_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        dec_down_kernel<DRACO_CODE_Q6_K><<<grid, 32 * kDecWarps, smem, s>>>(tab, active, n_active, off, act, inter,
                                                                          n_out, rt, y, q6s, status);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace draco
