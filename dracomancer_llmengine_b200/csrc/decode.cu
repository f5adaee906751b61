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
#include "select.cuh"

#include <algorithm>
#include <vector>

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

// L2ONLY: the rows were written by other blocks of the same launch: load through L2 only
template <int CODE, bool L2ONLY = false>
__device__ __forceinline__ void load_x8(const float* __restrict__ x, int sb, int lane, float v[8]) {
    const float* b = x + sb * 256 + x_pos<CODE>(lane);
    const float4 a = L2ONLY ? __ldcg(reinterpret_cast<const float4*>(b)) : *reinterpret_cast<const float4*>(b);
    const float4 c = L2ONLY ? __ldcg(reinterpret_cast<const float4*>(b + x_gap<CODE>()))
                            : *reinterpret_cast<const float4*>(b + x_gap<CODE>());
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
template <int CG, int CU, bool TWO, int NT, bool L2ONLY = false>
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
            load_x8<CG, L2ONLY>(xr[j], sb, lane, xg[j]);
            if (TWO && CG != CU) load_x8<CU, L2ONLY>(xr[j], sb, lane, xu[j]);
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

// One staged weight row (nb superblocks of bb bytes, shared memory) with nt <= 2 token rows, the
// superblock scales computed cooperatively: for a group of superblocks (4 of Q4_K, 2 of Q6_K)
// every lane works out ONE (64 d sc, offset) pair -- lane L: Q4_K superblock L / 8, sub-block
// L % 8; Q6_K superblock L / 16, scale L % 16 -- and the lanes that decode with it fetch it by
// shuffle, instead of each lane unpacking its own scales for every superblock.  The pairs, the
// decoded weights and the sums are those of decode8 (same expressions, same order), so the
// results equal the other decode paths bit for bit.
template <int CODE>
__device__ __forceinline__ float2 coop_scale(const uint8_t* row, int nb, int bb, int sb0, int lane) {
    if constexpr (CODE == DRACO_CODE_Q4_K) {
        const int sb = sb0 + (lane >> 3), j = lane & 7;
        if (sb >= nb) return make_float2(0.f, 0.f);
        const uint4 hd = *reinterpret_cast<const uint4*>(row + (size_t)sb * bb);
        const float d = h2f((uint16_t)(hd.x & 0xffff)), dmin = h2f((uint16_t)(hd.x >> 16));
        const int t = 8 * (j & 3);
        const int sc_lo = (hd.y >> t) & 63, m_lo = (hd.z >> t) & 63;
        const int e2 = (hd.w >> t) & 0xff;
        const int sc_hi = (e2 & 15) | (((hd.y >> (t + 6)) & 3) << 4);
        const int m_hi = (e2 >> 4) | (((hd.z >> (t + 6)) & 3) << 4);
        const int sc = j < 4 ? sc_lo : sc_hi, mn = j < 4 ? m_lo : m_hi;
        const float ds = d * (float)sc, dm = dmin * (float)mn;
        return make_float2(64.f * ds, -(128.f * ds + dm));
    } else {
        const int sb = sb0 + (lane >> 4);
        if (sb >= nb) return make_float2(0.f, 0.f);
        const uint8_t* blk = row + (size_t)sb * bb;
        const float d = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
        const float ds = d * (float)reinterpret_cast<const int8_t*>(blk + 192)[lane & 15];
        return make_float2(64.f * ds, -160.f * ds);
    }
}

// R staged weight rows at once (independent sums that the scheduler interleaves), row r with
// the token rows xr[r] (SAME_X: every row with xr[0], loaded once)
template <int CODE, int NT, int R, bool SAME_X, bool L2ONLY = false>
__device__ __forceinline__ void rows_dot_smem(const uint8_t* const (&rows)[R], int nb, int bb,
                                              const float* const (&xr)[R][2], int lane, float (&acc)[R][2]) {
    constexpr int G = CODE == DRACO_CODE_Q4_K ? 4 : 2;   // superblocks per scale group
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int j = 0; j < 2; j++) acc[r][j] = 0.f;
    // the lanes holding this lane's two pairs (superblock offset u adds u * 32 / G)
    const int src_lo = CODE == DRACO_CODE_Q4_K ? 2 * (lane >> 3) : 8 * (lane >> 4) + ((lane & 15) >> 2);
    const int src_hi = CODE == DRACO_CODE_Q4_K ? src_lo + 1 : src_lo + 4;
    for (int sb0 = 0; sb0 < nb; sb0 += G) {
        float2 ab[R];
#pragma unroll
        for (int r = 0; r < R; r++) ab[r] = coop_scale<CODE>(rows[r], nb, bb, sb0, lane);
#pragma unroll
        for (int u = 0; u < G; u++) {
            const int sb = sb0 + u;
            float2 sl[R], sh[R];
#pragma unroll
            for (int r = 0; r < R; r++) {
                sl[r] = make_float2(__shfl_sync(0xffffffffu, ab[r].x, src_lo + u * (32 / G)),
                                    __shfl_sync(0xffffffffu, ab[r].y, src_lo + u * (32 / G)));
                sh[r] = make_float2(__shfl_sync(0xffffffffu, ab[r].x, src_hi + u * (32 / G)),
                                    __shfl_sync(0xffffffffu, ab[r].y, src_hi + u * (32 / G)));
            }
            if (sb < nb) {
                float xs0[NT][8];
                if (SAME_X) {
#pragma unroll
                    for (int j = 0; j < NT; j++) load_x8<CODE, L2ONLY>(xr[0][j], sb, lane, xs0[j]);
                }
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const uint8_t* blk = rows[r] + (size_t)sb * bb;
                    uint32_t q_lo, q_hi;
                    if constexpr (CODE == DRACO_CODE_Q4_K) {
                        const uint32_t qs = *reinterpret_cast<const uint32_t*>(blk + 16 + 4 * lane);
                        q_lo = qs & 0x0F0F0F0Fu;
                        q_hi = (qs >> 4) & 0x0F0F0F0Fu;
                    } else {
                        const int h = lane >> 4, i = lane & 15;
                        const uint32_t ql = *reinterpret_cast<const uint32_t*>(blk + 64 * h + 4 * i);
                        const uint32_t qh = *reinterpret_cast<const uint32_t*>(blk + 128 + 32 * h + 4 * (i & 7));
                        const int s0 = 2 * (i >> 3);
                        q_lo = (ql & 0x0F0F0F0Fu) | (((qh >> s0) & 0x03030303u) << 4);
                        q_hi = ((ql >> 4) & 0x0F0F0F0Fu) | (((qh >> (s0 + 4)) & 0x03030303u) << 4);
                    }
                    float w[8];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        w[k] = fmaf(code_float(q_lo, k), sl[r].x, sl[r].y);
                        w[4 + k] = fmaf(code_float(q_hi, k), sh[r].x, sh[r].y);
                    }
#pragma unroll
                    for (int j = 0; j < NT; j++) {
                        float xv[8];
                        if (SAME_X) {
#pragma unroll
                            for (int k = 0; k < 8; k++) xv[k] = xs0[j][k];
                        } else {
                            load_x8<CODE, L2ONLY>(xr[r][j], sb, lane, xv);
                        }
#pragma unroll
                        for (int k = 0; k < 8; k++) acc[r][j] = fmaf(w[k], xv[k], acc[r][j]);
                    }
                }
            }
        }
    }
}

// 16-byte asynchronous global -> shared copies of one thread (the load/store unit path, not the
// tensor-memory-access unit: every lane issues its own share of a row), grouped per piece
__device__ __forceinline__ void fd_cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void fd_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void fd_cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// wait until at most n of this thread's newest copy groups are still in flight
__device__ __forceinline__ void fd_cp_wait_n(int n) {
    switch (n) {
        case 7: fd_cp_wait<7>(); break;
        case 6: fd_cp_wait<6>(); break;
        case 5: fd_cp_wait<5>(); break;
        case 4: fd_cp_wait<4>(); break;
        case 3: fd_cp_wait<3>(); break;
        case 2: fd_cp_wait<2>(); break;
        case 1: fd_cp_wait<1>(); break;
        default: fd_cp_wait<0>(); break;
    }
}

// ------------------------------------------------------------------------------------------
// Fused decode layer: the whole MoE layer of a small token batch (T <= 8, T*K <= 64) in ONE
// cooperative launch of one block per SM:
//   phase A  router logits: the T*E exact-order chains (k ascending, rounded product then
//            rounded add, src/m6_layer.c:775-783) spread over the blocks, one lane per chain,
//            router rows and token rows streamed by a producer warp through a shared-memory
//            ring of bulk copies;
//   -- grid barrier 1 --
//   phase S  every block selects the routing of all T tokens itself from the logits (the
//            router's warp-level selection, bit-exact) and builds the active expert list;
//   phase B  warp tasks: one (active expert or shared expert, intermediate row) gate+up row
//            pair, all tokens routed to that expert, SwiGLU;
//   -- grid barrier 2 --
//   phase C  warp tasks: one output row over every active expert (and the shared expert),
//            then the k-ascending fused combine (+ shared expert) of that row.
// Each compute warp streams the weight rows of its own tasks through a private ring of
// asynchronous copies (cp.async, every lane its share), phase C's rows included as soon as there
// is room (they do not depend on the activations), so the weights of the whole layer are in
// flight while phase B computes.  Per row the arithmetic and its order are those of the
// separate dec_* kernels.
// Every wait is bounded: an mbarrier wait gives up after 2 s, a grid barrier after 1 s; a block
// that gives up raises a status bit (0x200 copy, 0x1000 grid barrier, 0x2000 a weight row that is
// not a whole aligned row), stops, and waits for its own copies in flight before it exits.
// ------------------------------------------------------------------------------------------
constexpr int kFdMaxTokens = 8;
constexpr int kFdMaxAssign = 64;
constexpr int kFdCompute = 16;            // compute warps (the producer warp is warp 16)
constexpr int kFdThreads = 32 * (kFdCompute + 1);
constexpr int kFdMaxSlots = 16;              // router chunk slots (all chunks at once when they fit)
constexpr int kFdMaxStg = 8;              // per-warp weight-row ring stages
constexpr uint64_t kFdGridWaitNs = 1000000000ull;
constexpr int kFdStampStride = 128;       // DRACO_B200_FD_STATS words per block

__device__ __forceinline__ void fd_compute_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kFdCompute) : "memory"); }

// grid barrier over all blocks (called by one thread); false on timeout
__device__ __forceinline__ bool fd_grid_arrive_wait(unsigned* ctr, unsigned target) {
    __threadfence();
    atomicAdd(ctr, 1u);
    const uint64_t t0 = sync::global_ns();
    for (uint32_t i = 0;; i++) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if (v >= target) break;
        if ((i & 15) == 15 && sync::global_ns() - t0 > kFdGridWaitNs) return false;
    }
    __threadfence();
    return true;
}

template <int CODE>
__device__ __forceinline__ void fd_scales(const uint8_t* tile, int rows, int nb, int bb, float2* tab, int tid,
                                          int nth) {
    for (int idx = tid; idx < rows * nb; idx += nth)
        superblock_scales<CODE>(tile + (size_t)idx * bb, tab + (size_t)idx * scale_groups<CODE>());
}

// rows of n floats from global memory into shared memory by the compute threads (float4 loads
// through L2: the rows may have been written by other blocks of this launch)
__device__ __forceinline__ void fd_stage_rows(float* dst, const float* src, size_t n, int tid) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (size_t i = tid; i < n / 4; i += 32 * kFdCompute) d4[i] = __ldcg(s4 + i);
}

// optional phase timestamps (DRACO_B200_FD_STATS): thread 0 of each block
__device__ __forceinline__ void fd_stamp(const FusedDecodeArgs& a, int i) {
    if (a.stamps && threadIdx.x == 0) a.stamps[(size_t)blockIdx.x * kFdStampStride + i] = sync::global_ns();
}

template <int CG, int CU, int CD, int NS>
__global__ void __launch_bounds__(kFdThreads) fused_decode_kernel(FusedDecodeArgs a) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t full[kFdMaxSlots], empty[kFdMaxSlots];
    // s_cabort: written by compute threads (and thread 0 at the grid barriers) and read by them
    // only after a barrier, so their decisions stay uniform; s_pabort: the producer's own
    __shared__ volatile int s_cabort, s_pabort;
    __shared__ int s_n_act, s_qc;
    __shared__ int s_first[kFdMaxAssign];
    __shared__ const uint8_t* s_wp[3 * kFdMaxAssign];   // gate, up, down of each active expert
    const int E = a.rp.n_exp, K = a.rp.n_used, H = a.rp.n_in, T = a.T, F = a.F;
    const int NA = T * K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int S = a.n_slots;
    const bool sh = a.sh_ff > 0;
    uint8_t* ring = dsm;
    // the router's slots and (after barrier 1) the compute warps' weight-row rings share the front
    const size_t ring_bytes = max((size_t)S * a.slot_bytes, (size_t)kFdCompute * a.n_stg * a.stg_bytes);
    float* xs = reinterpret_cast<float*>(dsm + ring_bytes);                     // [xs_cap] token / act rows
    const int ES = (E + 3) & ~3;                                                // 16-byte aligned rows
    float* V = xs + a.xs_cap;                                                   // [8][ES] selection scratch
    float* gsm = V + kFdMaxTokens * ES;                                         // [8][64]
    int* s_order = reinterpret_cast<int*>(gsm + kFdMaxTokens * 64);              // [64]
    float* s_wtop = reinterpret_cast<float*>(s_order + kFdMaxAssign);            // [64]
    int* act_e = reinterpret_cast<int*>(s_wtop + kFdMaxAssign);                  // [64]
    int* act_cnt = act_e + kFdMaxAssign;                                         // [64]
    int* act_asg = act_cnt + kFdMaxAssign;                                       // [64][8]
    float* ys = reinterpret_cast<float*>(act_asg + kFdMaxAssign * kFdMaxTokens);  // [16][64+8] expert outputs
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            sync::mbar_init(&full[i], 1);
            sync::mbar_init(&empty[i], 1);
        }
        sync::fence_init();
        s_cabort = 0;
        s_pabort = 0;
        s_qc = 0;
    }
    // token rows in shared memory when they fit (read in phase B; the router reads its own copies)
    if (warp < kFdCompute && (size_t)T * H <= (size_t)a.xs_cap) fd_stage_rows(xs, a.X, (size_t)T * H, threadIdx.x);
    __syncthreads();
    fd_stamp(a, 0);
    const bool producer = warp == kFdCompute;
    const int ctid = threadIdx.x;   // compute thread id (warps 0..3)
    uint32_t q = 0;                 // jobs issued (producer lane 0) / consumed (compute threads)

    // producer (lane 0 of the producer warp): the next slot, nullptr after a failed wait or
    // when the compute warps stopped
    auto claim = [&]() -> uint8_t* {
        const int sl = q % S;
        if (s_cabort || s_pabort) return nullptr;
        if (q >= (uint32_t)S && !sync::mbar_wait(&empty[sl], ((q / S) & 1) ^ 1)) {
            atomicOr(a.status, 0x200);
            s_pabort = 1;
            return nullptr;
        }
        return ring + (size_t)sl * a.slot_bytes;
    };
    // compute threads: job q's slot, nullptr (uniformly) after a failed wait
    auto take = [&]() -> uint8_t* {
        const int sl = q % S;
        if (!sync::mbar_wait(&full[sl], (q / S) & 1)) {
            atomicOr(a.status, 0x200);
            s_cabort = 1;
        }
        fd_compute_sync();
        if (s_cabort) return nullptr;
        return ring + (size_t)sl * a.slot_bytes;
    };
    auto release = [&]() {
        fd_compute_sync();
        if (ctid == 0)
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sync::smem_addr(&empty[q % S])) : "memory");
        q++;
    };

    // ---------------------------------------------------------------- phase A: router logits
    const int C = T * E;
    const int nch = (a.W && b < C) ? (C - 1 - b) / G + 1 : 0;
    const int KC = a.kc, RS = a.kc + 4;
    const int n_chunks = H / KC;
    // all k-chunks fit the slots at once: the copy warp issues them all up front and warp 0 alone
    // walks its chains as each chunk lands (no per-chunk block synchronisation); else the ring
    const bool all_at_once = n_chunks <= S;
    auto chain_chunk = [&](const uint8_t* src, float& acc, int ct) {
        const float4* w4 = reinterpret_cast<const float4*>(src + (size_t)lane * RS * 4);
        const float4* x4 = reinterpret_cast<const float4*>(src + (size_t)(nch + ct) * RS * 4);
#pragma unroll 8
        for (int k = 0; k < KC / 4; k++) {
            const float4 w = w4[k], x = x4[k];
            acc = __fadd_rn(acc, __fmul_rn(x.x, w.x));
            acc = __fadd_rn(acc, __fmul_rn(x.y, w.y));
            acc = __fadd_rn(acc, __fmul_rn(x.z, w.z));
            acc = __fadd_rn(acc, __fmul_rn(x.w, w.w));
        }
    };
    if (nch > 0) {
        if (producer) {
            if (lane == 0)
                for (int ch = 0; ch < n_chunks; ch++) {
                    uint8_t* dst = all_at_once ? ring + (size_t)ch * a.slot_bytes : claim();
                    if (!dst) break;
                    const int sl = q % S;
                    sync::mbar_expect_tx(&full[sl], (uint32_t)(nch + T) * KC * 4);
                    for (int i = 0; i < nch; i++) {
                        const int e = (b + G * i) % E;
                        sync::bulk_load(dst + (size_t)i * RS * 4, a.W + (size_t)e * H + (size_t)ch * KC, KC * 4,
                                        &full[sl]);
                    }
                    for (int t = 0; t < T; t++)
                        sync::bulk_load(dst + (size_t)(nch + t) * RS * 4, a.X + (size_t)t * H + (size_t)ch * KC,
                                        KC * 4, &full[sl]);
                    q++;
                }
        } else if (all_at_once) {
            if (warp == 0) {
                float acc = 0.f;
                const int c = b + G * lane;
                const int ct = c / E;
                bool done = true;
                for (int ch = 0; ch < n_chunks; ch++) {
                    if (!sync::mbar_wait(&full[ch], 0)) {
                        if (lane == 0) atomicOr(a.status, 0x200);
                        s_cabort = 1;
                        done = false;
                        break;
                    }
                    if (lane < nch) chain_chunk(ring + (size_t)ch * a.slot_bytes, acc, ct);
                    q++;
                }
                if (done && lane < nch) a.logits[(size_t)ct * E + c % E] = acc;
            }
        } else {
            float acc = 0.f;
            const int c = b + G * lane;
            const int ct = c / E;
            bool done = true;
            for (int ch = 0; ch < n_chunks; ch++) {
                const uint8_t* src = take();
                if (!src) {
                    done = false;
                    break;
                }
                if (warp == 0 && lane < nch) chain_chunk(src, acc, ct);
                release();
            }
            if (done && warp == 0 && lane < nch) a.logits[(size_t)ct * E + c % E] = acc;
        }
    }
    if (ctid == 0) s_qc = (int)q;   // router jobs the compute warps consumed
    // ---------------------------------------------------------------- grid barrier 1
    __syncthreads();
    fd_stamp(a, 1);
    if (a.W && threadIdx.x == 0) {
        if (s_cabort || s_pabort || !fd_grid_arrive_wait(a.bar, (unsigned)(G + a.bar_extra))) {
            if (!s_cabort && !s_pabort) atomicOr(a.status, 0x1000);
            s_cabort = 1;
        }
    }
    __syncthreads();
    bool ok = !s_cabort && !s_pabort;   // uniform over the block from here
    fd_stamp(a, 2);
    // ---------------------------------------------------------------- phase S: routing
    if (ok) {
        if (a.W) {
            for (int t = warp; t < T && warp < kFdMaxTokens; t += kFdMaxTokens) {
                float* Vw = V + (size_t)warp * ES;
                for (int e = lane; e < E; e += 32) Vw[e] = __ldcg(a.logits + (size_t)t * E + e);
                __syncwarp();
                if (t == 0) fd_stamp(a, 66);
                select_token<NS>(a.rp, Vw, s_order + t * K, s_wtop + t * K, a.route_err, Vw, gsm + warp * 64);
                __syncwarp();
            }
        } else {
            for (int i = threadIdx.x; i < NA; i += blockDim.x) {
                s_order[i] = a.order[i];
                s_wtop[i] = a.wtop[i];
            }
        }
    }
    fd_stamp(a, 64);
    __syncthreads();
    if (ok && a.W && b == 0)
        for (int i = threadIdx.x; i < NA; i += blockDim.x) {
            a.order[i] = s_order[i];
            a.wtop[i] = s_wtop[i];
        }
    // active experts ascending; per active expert its assignments in order (token ascending)
    if (threadIdx.x < NA) {
        const int i = threadIdx.x, e = ok ? s_order[i] : -1;
        bool first = e >= 0 && e < E;
        for (int j = 0; j < i && first; j++) first = s_order[j] != e;
        s_first[i] = first;
    }
    __syncthreads();
    if (threadIdx.x < NA && ok) {
        const int i = threadIdx.x, e = s_order[i];
        if (e >= 0 && e < E) {
            int rank = 0, pos = 0, cnt = 0;
            for (int j = 0; j < NA; j++) {
                const int ej = s_order[j];
                if (s_first[j] && ej < e) rank++;
                if (ej == e) {
                    cnt++;
                    if (j < i) pos++;
                }
            }
            if (s_first[i]) {
                act_e[rank] = e;
                act_cnt[rank] = cnt;
            }
            act_asg[rank * kFdMaxTokens + pos] = i;
        }
    }
    if (threadIdx.x == 0) {
        int n = 0;
        for (int i = 0; i < NA; i++) n += s_first[i];
        s_n_act = n;
    }
    __syncthreads();
    fd_stamp(a, 65);
    if (ok && threadIdx.x < 3 * s_n_act) s_wp[threadIdx.x] = a.tab.w[3 * act_e[threadIdx.x / 3] + threadIdx.x % 3];
    __syncthreads();
    fd_stamp(a, 3);
    const int n_act = ok ? s_n_act : 0;
    // ---------------------------------------------------------------- phases B and C
    // Warp tasks: phase B = one (expert or shared expert, intermediate row) pair of gate and up
    // rows, phase C = one output row over every active expert (and the shared expert), combined
    // in k order right away.  Each compute warp streams the weight rows of its own tasks, in task
    // order, through a private ring of n_stg stages: every lane copies its 16-byte share of a row
    // with cp.async, one copy group per row (a single thread issuing bulk copies per row is held to
    // the copy engine's per-copy rate, ~70 cycles a copy per SM, a ceiling for rows of ~1 KB);
    // phase C's rows do not depend on the activations, so they are issued as soon as phase B's
    // leave room, before grid barrier 2.  The ring aliases the router's slots (all of them
    // consumed before barrier 1).
    const int nb = H / 256, nbd = F / 256, nbds = sh ? a.sh_ff / 256 : 0;
    const int bg = superblock_bytes(CG, a.q6s), bd = superblock_bytes(CD, a.q6s);
    const uint32_t rbg = (uint32_t)nb * bg, rbd = (uint32_t)nbd * bd, rbds = (uint32_t)nbds * bd;
    const int tasks_b = ok ? n_act * F + (sh ? a.sh_ff : 0) : 0;
    const int tasks_c = ok ? a.n_out : 0;
    const int gw = b * kFdCompute + warp, GW = G * kFdCompute;   // this warp's global index, all warps
    const int NST = a.n_stg;
    const int per_c = n_act + (sh ? 1 : 0);   // pieces of a phase C task
    if (!producer) {
        uint8_t* wring = ring + (size_t)warp * NST * a.stg_bytes;
        // producer cursor (uniform over the warp; lane 0 issues): the next piece's phase, task, part
        // (phase C has no pieces when no expert is active and there is no shared expert: every
        // routing entry of the batch named no expert of the table)
        int p_ph = 0, p_task = gw, p_sub = 0;
        if (p_task >= tasks_b) {
            p_ph = 1;
            if (p_task >= tasks_c || per_c == 0) p_ph = 2;
        }
        uint32_t n_iss = 0, n_con = 0;   // pieces issued / consumed
        bool wok = ok;
        // (a stage is only ever read by this warp's generic loads before the copy that rewrites
        // it, and those loads completed before the __syncwarp of release_pieces)
        auto issue = [&]() {
            while (wok && p_ph < 2 && n_iss < n_con + a.ahead) {
                const uint8_t* src;
                uint32_t bytes;
                if (p_ph == 0) {
                    const bool shx = p_task >= n_act * F;
                    const int ax = shx ? 0 : p_task / F, row = shx ? p_task - n_act * F : p_task % F;
                    const uint8_t* base = shx ? (p_sub ? a.sh_u : a.sh_g) : s_wp[3 * ax + p_sub];
                    src = base + (size_t)row * rbg;
                    bytes = rbg;
                    if (++p_sub == 2) {
                        p_sub = 0;
                        p_task += GW;
                        if (p_task >= tasks_b) {
                            p_ph = 1;
                            p_task = gw;
                            if (p_task >= tasks_c || per_c == 0) p_ph = 2;
                        }
                    }
                } else {
                    const bool shx = p_sub == n_act;
                    src = shx ? a.sh_d + (size_t)p_task * rbds : s_wp[3 * p_sub + 2] + (size_t)p_task * rbd;
                    bytes = shx ? rbds : rbd;
                    if (++p_sub == per_c) {
                        p_sub = 0;
                        p_task += GW;
                        if (p_task >= tasks_c) p_ph = 2;
                    }
                }
                // a piece must be a whole, aligned row that fits a stage (status 0x2000 otherwise:
                // the warp stops instead of copying)
                if (src == nullptr || bytes == 0 || bytes > (uint32_t)a.stg_bytes || ((uintptr_t)src & 15u)) {
                    if (lane == 0) atomicOr(a.status, 0x2000);
                    wok = false;
                    break;
                }
                const int st = n_iss % NST;
                uint8_t* dst = wring + (size_t)st * a.stg_bytes;
                for (uint32_t off = 16u * lane; off < bytes; off += 512u) fd_cp16(dst + off, src + off);
                fd_cp_commit();   // one group per piece on every lane
                n_iss++;
            }
        };
        // the next piece in shared memory (nullptr after a failed wait)
        unsigned long long t_acc[4] = {0, 0, 0, 0};   // DRACO_B200_FD_STATS: wait/compute ns, B and C
        int t_ph = 0;
        auto take_piece = [&]() -> const uint8_t* {
            const unsigned long long tw0 = a.stamps ? sync::global_ns() : 0;
            const int st = n_con % NST;
            fd_cp_wait_n((int)(n_iss - n_con) - 1);   // this piece's group has landed (own copies)
            __syncwarp();                             // and the other lanes' shares are visible
            wok = __all_sync(0xffffffffu, wok);
            if (a.stamps) t_acc[2 * t_ph] += sync::global_ns() - tw0;
            if (a.stamps && lane == 0 && n_con == 0) a.stamps[(size_t)blockIdx.x * kFdStampStride + 8 + warp] = sync::global_ns();
            return wok ? wring + (size_t)st * a.stg_bytes : nullptr;
        };
        auto release_pieces = [&](int n) {
            __syncwarp();
            n_con += n;
            issue();
        };
        issue();
        if (a.stamps && lane == 0) a.stamps[(size_t)blockIdx.x * kFdStampStride + 68 + warp] = sync::global_ns();
        const bool x_in_smem = (size_t)T * H <= (size_t)a.xs_cap;   // staged at the start
        const float* xbase = x_in_smem ? xs : a.X;
        for (int task = gw; wok && task < tasks_b; task += GW) {
            const bool shx = task >= n_act * F;
            const int ax = shx ? 0 : task / F;
            const int row = shx ? task - n_act * F : task % F;
            const int cnt = shx ? T : act_cnt[ax];
            const uint8_t* grow = take_piece();
            n_con++;
            const uint8_t* urow = wok ? take_piece() : nullptr;
            n_con--;
            if (!wok) break;
            for (int tc = 0; tc < cnt; tc += 2) {
                const int nt = min(2, cnt - tc);
                const float* xr[2];
                int slot[2];
#pragma unroll
                for (int jj = 0; jj < 2; jj++) {
                    const int m = tc + min(jj, nt - 1);
                    const int i = shx ? m : act_asg[ax * kFdMaxTokens + m];
                    slot[jj] = i;
                    xr[jj] = xbase + (size_t)(shx ? i : i / K) * H;
                }
                float acc[2][2];
                const uint8_t* const gu[2] = {grow, urow};
                const float* const xx[2][2] = {{xr[0], xr[1]}, {xr[0], xr[1]}};
                const unsigned long long tc0 = a.stamps ? sync::global_ns() : 0;
                static_assert(CG == CU, "the fused kernel runs gate and up of one format");
                if (nt == 2) rows_dot_smem<CG, 2, 2, true>(gu, nb, bg, xx, lane, acc);
                else rows_dot_smem<CG, 1, 2, true>(gu, nb, bg, xx, lane, acc);
                if (a.stamps) t_acc[1] += sync::global_ns() - tc0;
                const float (&ag)[2] = acc[0];
                const float (&au)[2] = acc[1];
#pragma unroll
                for (int jj = 0; jj < 2; jj++) {
                    if (jj < nt) {
                        const float gv = warp_sum(ag[jj]), uv = warp_sum(au[jj]);
                        if (lane == 0) {
                            if (shx) a.act_sh[(size_t)slot[jj] * a.sh_ff + row] = silu_mul(gv, uv);
                            else a.act[(size_t)slot[jj] * F + row] = silu_mul(gv, uv);
                        }
                    }
                }
            }
            release_pieces(2);
        }
        if (!wok) s_cabort = 1;
        if (a.stamps && lane == 0) a.stamps[(size_t)blockIdx.x * kFdStampStride + 24 + warp] = sync::global_ns();
        // ------------------------------------------------------------ grid barrier 2
        fd_compute_sync();
        fd_stamp(a, 4);
        if (ctid == 0) {
            if (!ok || s_cabort || !fd_grid_arrive_wait(a.bar + 1, (unsigned)(G + a.bar_extra))) {
                if (ok && !s_cabort) atomicOr(a.status, 0x1000);
                s_cabort = 1;
            }
        }
        fd_compute_sync();
        fd_stamp(a, 5);
        ok = !s_cabort;
        wok = wok && ok;
        // the activation rows of every assignment (and the shared expert's) in shared memory
        const size_t act_n = (size_t)NA * F + (sh ? (size_t)T * a.sh_ff : 0);
        const bool a_in_smem = act_n <= (size_t)a.xs_cap;
        if (ok && a_in_smem) {
            fd_stage_rows(xs, a.act, (size_t)NA * F, ctid);
            if (sh) fd_stage_rows(xs + (size_t)NA * F, a.act_sh, (size_t)T * a.sh_ff, ctid);
        }
        fd_compute_sync();
        const float* abase = a_in_smem ? xs : a.act;
        const float* sbase = a_in_smem ? xs + (size_t)NA * F : a.act_sh;
        float* yw = ys + (size_t)warp * (kFdMaxAssign + kFdMaxTokens);   // this warp's expert outputs
        t_ph = 1;
        for (int r = gw; wok && r < tasks_c; r += GW) {
            for (int x = 0; x < per_c; x++) {
                const bool shx = x == n_act;
                const int cnt = shx ? T : act_cnt[x];
                const int nbx = shx ? nbds : nbd;
                if (!shx && x + 1 < n_act && cnt == 1 && act_cnt[x + 1] == 1) {
                    // two experts with one assignment each: both rows at once
                    const uint8_t* d0 = take_piece();
                    n_con++;
                    const uint8_t* d1 = wok ? take_piece() : nullptr;
                    n_con--;
                    if (!wok) break;
                    const int i0 = act_asg[x * kFdMaxTokens], i1 = act_asg[(x + 1) * kFdMaxTokens];
                    const uint8_t* const dd[2] = {d0, d1};
                    const float* const xx[2][2] = {{abase + (size_t)i0 * F, abase + (size_t)i0 * F},
                                                   {abase + (size_t)i1 * F, abase + (size_t)i1 * F}};
                    float ad[2][2];
                    const unsigned long long tc0 = a.stamps ? sync::global_ns() : 0;
                    if (a_in_smem) rows_dot_smem<CD, 1, 2, false>(dd, nbx, bd, xx, lane, ad);
                    else rows_dot_smem<CD, 1, 2, false, true>(dd, nbx, bd, xx, lane, ad);
                    if (a.stamps) t_acc[3] += sync::global_ns() - tc0;
                    const float v0 = warp_sum(ad[0][0]), v1 = warp_sum(ad[1][0]);
                    if (lane == 0) {
                        yw[i0] = v0;
                        yw[i1] = v1;
                    }
                    release_pieces(2);
                    x++;
                    continue;
                }
                const uint8_t* drow = take_piece();
                if (!drow) break;
                for (int tc = 0; tc < cnt; tc += 2) {
                    const int nt = min(2, cnt - tc);
                    const float* xr[1][2];
                    int slot[2];
#pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
                        const int m = tc + min(jj, nt - 1);
                        const int i = shx ? m : act_asg[x * kFdMaxTokens + m];
                        slot[jj] = shx ? NA + i : i;
                        xr[0][jj] = shx ? sbase + (size_t)i * a.sh_ff : abase + (size_t)i * F;
                    }
                    const uint8_t* const dd[1] = {drow};
                    float ad[1][2];
                    const unsigned long long tc0 = a.stamps ? sync::global_ns() : 0;
                    if (a_in_smem) {
                        if (nt == 2) rows_dot_smem<CD, 2, 1, true>(dd, nbx, bd, xr, lane, ad);
                        else rows_dot_smem<CD, 1, 1, true>(dd, nbx, bd, xr, lane, ad);
                    } else {
                        // rows written by other blocks of this launch: L2 loads
                        if (nt == 2) rows_dot_smem<CD, 2, 1, true, true>(dd, nbx, bd, xr, lane, ad);
                        else rows_dot_smem<CD, 1, 1, true, true>(dd, nbx, bd, xr, lane, ad);
                    }
                    if (a.stamps) t_acc[3] += sync::global_ns() - tc0;
#pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
                        if (jj < nt) {
                            const float v = warp_sum(ad[0][jj]);
                            if (lane == 0) yw[slot[jj]] = v;
                        }
                    }
                }
                release_pieces(1);
            }
            if (!wok) break;
            __syncwarp();
            // combine: k ascending fused multiply-adds, then the shared expert
            if (lane < T) {
                const int t = lane;
                float acc = 0.f;
                for (int k = 0; k < K; k++) {
                    const int i = t * K + k, e = s_order[i];
                    if (e >= 0 && e < E) acc = fmaf(s_wtop[i], yw[i], acc);
                }
                if (sh) acc = __fadd_rn(acc, yw[NA + t]);
                a.out[(size_t)t * a.n_out + r] = acc;
            }
            __syncwarp();
        }
        if (a.stamps && lane == 0) {
            a.stamps[(size_t)blockIdx.x * kFdStampStride + 40 + warp] = sync::global_ns();
            if (warp == 0 || warp == 15)
                for (int i = 0; i < 4; i++) a.stamps[(size_t)blockIdx.x * kFdStampStride + 56 + (warp ? 4 : 0) + i] = t_acc[i];
        }
        // copies issued but not consumed (after a failure) land before the warp exits
        fd_cp_wait<0>();
        __syncwarp();
        fd_stamp(a, 6);
    }
    __syncthreads();
    // router copies issued but not consumed (after a failure) land before the block exits
    if (producer && lane == 0)
        for (uint32_t r = (uint32_t)s_qc; r < q; r++) sync::mbar_wait(&full[r % S], (r / S) & 1);
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


int launch_fused_decode(FusedDecodeArgs a, int cg, int cu, int cd, cudaStream_t s) {
    const int E = a.rp.n_exp, K = a.rp.n_used, H = a.rp.n_in, T = a.T;
    if (T < 1 || T > kFdMaxTokens || T * K > kFdMaxAssign || E > 512 || cg != cu) return 1;
    if (H % 256 || a.F % 256 || (a.sh_ff && a.sh_ff % 256) || a.n_out % 4) return 1;
    auto ok_code = [](int c) { return c == DRACO_CODE_Q4_K || c == DRACO_CODE_Q6_K; };
    if (!ok_code(cg) || !ok_code(cd)) return 1;
    if (a.q6s != kQ6Padded && (cg == DRACO_CODE_Q6_K || cd == DRACO_CODE_Q6_K)) return 1;
    // per device: SM count and cooperative-launch support; per (kernel, shared memory bytes): the
    // attribute set and the occupancy check passed (queried once, not on every decode call)
    struct DevInfo {
        int sms = -1, coop = 0;
        std::vector<std::pair<const void*, size_t>> ready;   // (kernel, bytes) checked
        std::vector<std::pair<const void*, size_t>> attr;    // (kernel, largest bytes set)
    };
    static DevInfo info[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 1;
    }
    DevInfo& di = info[dev];
    if (di.sms < 0) {
        if (cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev) ||
            cudaDeviceGetAttribute(&di.coop, cudaDevAttrCooperativeLaunch, dev)) {
            cudaGetLastError();
            di.sms = -1;
            return 1;
        }
    }
    const int sms = di.sms;
    if (!di.coop) return 1;
    const int G = sms;   // one block per SM
    // router chunk: the longest of 512 / 256 / 128 values whose ring stage stays within 64 KB
    const int nch_max = (T * E + G - 1) / G;
    if (nch_max > 32) return 1;
    auto stage_a = [&](int kc) { return (size_t)(nch_max + T) * (kc + 4) * 4; };
    int kc = 128;
    for (int c : {512, 256})
        if (H % c == 0 && stage_a(c) <= 64u * 1024) {
            kc = c;
            break;
        }
    const size_t slot = (stage_a(kc) + 127) / 128 * 128;
    // token rows (phase B) / activation rows (phase C) staged in shared memory up to 32 KB
    const size_t rows_b = (size_t)T * H, rows_c = (size_t)T * K * a.F + (size_t)T * a.sh_ff;
    const int xs_cap = (int)std::min<size_t>(8192, std::max(rows_b, rows_c));
    const size_t extra = (size_t)xs_cap * 4 + ((size_t)kFdMaxTokens * ((E + 3) & ~3) + kFdMaxTokens * 64) * 4 +
                         2 * kFdMaxAssign * 4 + (2 * kFdMaxAssign + kFdMaxAssign * kFdMaxTokens) * 4 +
                         (size_t)(kFdMaxAssign + kFdMaxTokens) * kFdCompute * 4 + 256;
    // per-warp weight-row ring: stages of the longest row, as many as fit (at least 2: a gate/up
    // task holds two)
    const int bg = superblock_bytes(cg, a.q6s), bd = superblock_bytes(cd, a.q6s);
    const size_t stg = std::max({(size_t)(H / 256) * bg, (size_t)(a.F / 256) * bd, (size_t)(a.sh_ff / 256) * bd});
    constexpr size_t kSmemMax = 220u * 1024;
    if (extra + 2 * kFdCompute * stg > kSmemMax) return 1;
    const int n_stg = (int)std::min<size_t>(kFdMaxStg, (kSmemMax - extra) / (kFdCompute * stg));
    const size_t wring = (size_t)kFdCompute * n_stg * stg;
    // router chunk slots: every chunk of the row at once when they fit next to the weight rings'
    // share of shared memory (they alias it), else a ring of 4
    const int n_chunks = H / kc;
    int slots = 4;
    if (n_chunks <= kFdMaxSlots && n_chunks * slot <= std::max(wring, kSmemMax - extra)) slots = std::max(4, n_chunks);
    while (slots > 2 && slots * slot > std::max(wring, kSmemMax - extra)) slots--;
    const size_t total = std::max(slots * slot, wring) + extra;
    if (total > kSmemMax) return 1;
    const void* kern = nullptr;
    const int ns = E <= 128 ? 4 : E <= 256 ? 8 : 16;
    constexpr int Q4 = DRACO_CODE_Q4_K, Q6 = DRACO_CODE_Q6_K;
#define DRACO_FD_PICK(A, D)                                                                  \
    if (cg == A && cd == D)                                                                  \
        kern = ns == 4   ? (const void*)fused_decode_kernel<A, A, D, 4>                      \
               : ns == 8 ? (const void*)fused_decode_kernel<A, A, D, 8>                      \
                         : (const void*)fused_decode_kernel<A, A, D, 16>;
    DRACO_FD_PICK(Q4, Q6)
    DRACO_FD_PICK(Q4, Q4)
    DRACO_FD_PICK(Q6, Q6)
    DRACO_FD_PICK(Q6, Q4)
#undef DRACO_FD_PICK
    if (!kern) return 1;
    // the kernel's dynamic shared memory limit only grows: a smaller request after a larger one
    // keeps the larger setting, which covers both
    auto at = std::find_if(di.attr.begin(), di.attr.end(), [&](const auto& p) { return p.first == kern; });
    if (at == di.attr.end() || at->second < total) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)total) != cudaSuccess) {
            cudaGetLastError();
            return 1;
        }
        if (at == di.attr.end()) di.attr.emplace_back(kern, total);
        else at->second = total;
    }
    const std::pair<const void*, size_t> key(kern, total);
    if (std::find(di.ready.begin(), di.ready.end(), key) == di.ready.end()) {
        int occ = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kFdThreads, total) != cudaSuccess || occ < 1) {
            cudaGetLastError();
            return 1;
        }
        di.ready.push_back(key);
    }
    a.slot_bytes = (int)slot;
    a.n_slots = slots;
    a.stg_bytes = (int)stg;
    a.n_stg = n_stg;
    // rows in flight per warp (DRACO_B200_FD_AHEAD, default all stages); at least 2: a gate/up
    // task holds two
    static const int ahead_env = [] {
        const char* e = getenv("DRACO_B200_FD_AHEAD");
        return e ? atoi(e) : 0;
    }();
    a.ahead = ahead_env >= 2 ? std::min(ahead_env, n_stg) : n_stg;
    a.kc = kc;
    a.xs_cap = xs_cap;
    void* args[] = {&a};
    const cudaError_t e = cudaLaunchCooperativeKernel(kern, G, kFdThreads, args, total, s);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return e == cudaErrorCooperativeLaunchTooLarge ? 1 : -3;
    }
    return 0;
}

}  // namespace draco
