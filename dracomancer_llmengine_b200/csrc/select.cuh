// Token routing selection (softmax, or sigmoid + bias + group limit; stable top-k; weights) as
// a warp-level device routine, shared by the router's select kernel (route.cu) and the fused
// decode kernel (fused_decode.cu).  Semantics: src/m6_layer.c:771-796 and :823-866.
#pragma once
#include "kernels.cuh"

namespace draco {

constexpr int kMaxExperts = 512;   // the reference's fixed arrays (src/m6_layer.c:774,791)
constexpr int kMaxUsed = 64;       // (src/m6_layer.c:860-862)
constexpr int kMaxGroups = 64;     // (src/m6_layer.c:843,852)
constexpr int kSelWarps = 4;

// (v2, i2) beats (v1, i1): larger value, or equal value at a lower valid index.  Invalid
// candidates carry i = -1 and never beat a valid one.
__device__ __forceinline__ bool beats(float v2, int i2, float v1, int i1) {
    if (i2 < 0) return false;
    if (i1 < 0) return true;
    return v2 > v1 || (v2 == v1 && i2 < i1);
}

// Sum of n <= 64 values v_j (lane j & 31 holds v_j in v0 for j < 32, in v1 above) in numpy's
// float32 pairwise order for arrays of at most 128 elements: n < 8 sequentially from 0; else 8
// running sums r_i = v_i + v_{i+8} + ... over the first n - n % 8 values, combined as
// ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)), then the remaining values in order.
// Every lane returns the sum.
__device__ __forceinline__ float pairwise_sum_warp(float v0, float v1, int n) {
    const int lane = threadIdx.x & 31;
    auto elem = [&](int j) { return __shfl_sync(0xffffffffu, j < 32 ? v0 : v1, j & 31); };
    if (n < 8) {
        float s = 0.f;
        for (int j = 0; j < n; j++) s = __fadd_rn(s, elem(j));
        return s;
    }
    const int n8 = n - n % 8;
    float r = 0.f;
    for (int j = 0; j < n8; j += 8) {
        const int src = (j + (lane & 7)) & 31;
        const float a = __shfl_sync(0xffffffffu, v0, src), b = __shfl_sync(0xffffffffu, v1, src);
        const float v = j + (lane & 7) < 32 ? a : b;
        r = j == 0 ? v : __fadd_rn(r, v);
    }
    float q[8];
#pragma unroll
    for (int i = 0; i < 8; i++) q[i] = __shfl_sync(0xffffffffu, r, i);
    float s = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3])),
                        __fadd_rn(__fadd_rn(q[4], q[5]), __fadd_rn(q[6], q[7])));
    for (int j = n8; j < n; j++) s = __fadd_rn(s, elem(j));
    return s;
}

// One warp per token.  Lane l holds experts l + 32 j (j < NS) in registers with a bitmask of
// those still selectable; each of the K rounds takes every lane's best candidate and a 5-step
// shuffle max over a (score, expert) key, then fetches the winner's probability.  The order of
// comparisons gives exactly the reference's scan (src/m6_layer.c:860-870): the largest score
// wins, the lowest expert index among equal scores, and only scores above the -1e30 floor count
// (NaN never does).  The softmax denominator and the weight sum are taken sequentially in the
// reference's order.
template <int NS>
__device__ __forceinline__ void select_token(const RouterParams& p, const float* __restrict__ lg, int* order_row,
                                             float* wtop_row, int* err, float* V, float* gs) {
    const int lane = threadIdx.x & 31;
    const int E = p.n_exp, K = p.n_used;
    float S[NS], P[NS];
    uint32_t tab_lo, tab_hi;   // this lane's entry of the exp table (host_expf_warp)
    exp_table_lane(tab_lo, tab_hi);
    if (p.scoring == 0) {
        // max-subtracted softmax (src/m6_layer.c:784-789)
        float mx = -1e30f;
#pragma unroll
        for (int j = 0; j < NS; j++) {
            const int e = lane + 32 * j;
            S[j] = e < E ? lg[e] : 0.f;
            if (e < E && S[j] > mx) mx = S[j];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, mx, o);
            mx = ov > mx ? ov : mx;
        }
#pragma unroll
        for (int j = 0; j < NS; j++) {
            const int e = lane + 32 * j;
            P[j] = host_expf_warp(__fsub_rn(S[j], mx), tab_lo, tab_hi);
            if (e < E) V[e] = P[j];
        }
        __syncwarp();
        float s = 0.f;
        if (lane == 0) {
            int e = 0;
            for (; e + 4 <= E; e += 4) {
                const float4 q = *reinterpret_cast<const float4*>(V + e);
                s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, q.x), q.y), q.z), q.w);
            }
            for (; e < E; e++) s = __fadd_rn(s, V[e]);
        }
        s = __shfl_sync(0xffffffffu, s, 0);
        const float inv = __fdiv_rn(1.0f, s);
#pragma unroll
        for (int j = 0; j < NS; j++) {
            P[j] = __fmul_rn(P[j], inv);
            S[j] = P[j];
        }
    } else {
        // sigmoid scores; bias only steers the selection (src/m6_layer.c:833-840)
#pragma unroll
        for (int j = 0; j < NS; j++) {
            const int e = lane + 32 * j;
            const float l = e < E ? lg[e] : 0.f;
            P[j] = __fdiv_rn(1.0f, __fadd_rn(1.0f, host_expf_warp(-l, tab_lo, tab_hi)));
            S[j] = __fadd_rn(P[j], p.probs_b && e < E ? p.probs_b[e] : 0.0f);
        }
        if (p.n_group > 1) {
            // group score = sum of the group's two largest (src/m6_layer.c:841-859), then the
            // n_group_used best groups by the same strict-greater scan
#pragma unroll
            for (int j = 0; j < NS; j++)
                if (lane + 32 * j < E) V[lane + 32 * j] = S[j];
            __syncwarp();
            const int per = E / p.n_group;
            for (int g = lane; g < p.n_group; g += 32) {
                float m1 = -1e30f, m2 = -1e30f;
                for (int i = 0; i < per; i++) {
                    const float v = V[g * per + i];
                    if (v > m1) {
                        m2 = m1;
                        m1 = v;
                    } else if (v > m2) {
                        m2 = v;
                    }
                }
                gs[g] = __fadd_rn(m1, m2);
            }
            __syncwarp();
            uint32_t gavail = 0, gsel = 0;   // groups lane, lane + 32
            float G[2];
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int g = lane + 32 * j;
                G[j] = g < p.n_group ? gs[g] : 0.f;
                if (g < p.n_group) gavail |= 1u << j;
            }
            for (int r = 0; r < p.n_group_used; r++) {
                float bv = -1e30f;
                int bi = -1;
#pragma unroll
                for (int j = 0; j < 2; j++)
                    if ((gavail >> j & 1) && G[j] > bv) {
                        bv = G[j];
                        bi = lane + 32 * j;
                    }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (beats(ov, oi, bv, bi)) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (bi < 0) {
                    if (lane == 0) atomicOr(err, 1);
                    break;
                }
                if ((bi & 31) == lane) {
                    gavail &= ~(1u << (bi >> 5));
                    gsel |= 1u << (bi >> 5);
                }
            }
            // every lane learns the chosen groups
            const unsigned long long chosen =
                (unsigned long long)__ballot_sync(0xffffffffu, gsel & 1) |
                ((unsigned long long)__ballot_sync(0xffffffffu, gsel >> 1 & 1) << 32);
#pragma unroll
            for (int j = 0; j < NS; j++) {
                const int e = lane + 32 * j;
                if (e < E && !(chosen >> (e / per) & 1)) S[j] = -1e30f;
            }
        }
    }
    uint32_t avail = 0;
#pragma unroll
    for (int j = 0; j < NS; j++)
        if (lane + 32 * j < E) avail |= 1u << j;
    // lane l keeps result l (and l + 32 when K > 32)
    static_assert(kMaxUsed <= 64, "two results per lane");
    int my_i0 = -1, my_i1 = -1;
    float my_p0 = 0.f, my_p1 = 0.f;
    for (int r = 0; r < K; r++) {
        float bv = -1e30f, bp = 0.f;
        int bi = -1;
#pragma unroll
        for (int j = 0; j < NS; j++)
            if ((avail >> j & 1) && S[j] > bv) {
                bv = S[j];
                bp = P[j];
                bi = lane + 32 * j;
            }
        // warp argmax as one 64-bit key max: the score in order-preserving bits above the
        // complemented index, so a larger key is a larger score or, at an equal score, the lower
        // index (the strict-greater scan's tie rule); no candidate (bi = -1) is key 0, below all.
        // Scores here are above -1e30, never NaN and never -0, so equal keys are equal scores.
        const uint32_t ub = __float_as_uint(bv);
        const uint32_t ord = (ub & 0x80000000u) ? ~ub : (ub | 0x80000000u);
        unsigned long long key = bi < 0 ? 0ull : ((unsigned long long)ord << 32) | (0xffffffffu - (uint32_t)bi);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long ok = __shfl_xor_sync(0xffffffffu, key, o);
            key = ok > key ? ok : key;
        }
        bi = key ? (int)(0xffffffffu - (uint32_t)(key & 0xffffffffu)) : -1;
        bp = __shfl_sync(0xffffffffu, bp, bi >= 0 ? (bi & 31) : 0);   // the winner's probability
        if (bi < 0) {
            if (lane == 0) atomicOr(err, 2);
        } else if ((bi & 31) == lane) {
            avail &= ~(1u << (bi >> 5));
        }
        if ((r & 31) == lane) {
            if (r < 32) {
                my_i0 = bi;
                my_p0 = bi >= 0 ? bp : 0.f;
            } else {
                my_i1 = bi;
                my_p1 = bi >= 0 ? bp : 0.f;
            }
        }
    }
    // weights (src/m6_layer.c:871-880): sum in selection order, then per-lane division
    float s = 0.f;
    const bool renorm = p.scoring == 0 || p.norm_w;
    if (p.scoring != 0 && p.norm_w == 2) {
        // the numpy drivers' renormalisation (src/k2_engine.py:506-507, src/k2_prefill.py:
        // 125-126): no clamp, the sum in numpy's pairwise float32 order
        s = pairwise_sum_warp(my_p0, my_p1, K);
    } else {
        for (int j = 0; j < K; j++) s = __fadd_rn(s, __shfl_sync(0xffffffffu, j < 32 ? my_p0 : my_p1, j & 31));
        if (s < 6.103515625e-5f) s = 6.103515625e-5f;
    }
    const bool scale = p.scoring != 0 && p.w_scale != 0.f && p.w_scale != 1.f;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int j = lane + 32 * h;
        if (j < K) {
            float wl = h ? my_p1 : my_p0;
            if (renorm) wl = __fdiv_rn(wl, s);
            if (scale) wl = __fmul_rn(wl, p.w_scale);
            order_row[j] = h ? my_i1 : my_i0;
            wtop_row[j] = wl;
        }
    }
}


}  // namespace draco
