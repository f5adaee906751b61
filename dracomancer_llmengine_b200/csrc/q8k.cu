// Q8_K activation mode: activations quantised per 256 values to int8 with one fp32 scale and
// int16 group sums (the block_q8_K format of ggml), multiplied with Q4_K / Q6_K weights in
// integer arithmetic.  The reference engine keeps fp32 activations throughout; this mode is
// an optional fast decode path, bit-exact with its CPU restatement in the test checker:
// integer superblock sums are exact, and their float combination runs per row in
// superblock order on one lane.
#include "kernels.cuh"

namespace draco {

// one warp per 256-value block: d = amax/127, q = rint(x * 127/amax) in [-127, 127]
__global__ void q8k_quantize_kernel(const float* __restrict__ x, int nblk, float* __restrict__ d,
                                    int8_t* __restrict__ q, int16_t* __restrict__ bsums) {
    const int lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < nblk; b += nw) {
        const float* xb = x + (size_t)b * 256 + lane * 8;
        const float4 a0 = *reinterpret_cast<const float4*>(xb);
        const float4 a1 = *reinterpret_cast<const float4*>(xb + 4);
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) amax = fabsf(v[i]) > amax ? fabsf(v[i]) : amax;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, amax, o);
            amax = ov > amax ? ov : amax;
        }
        int s = 0;
        uint32_t packed[2] = {0u, 0u};
        if (amax != 0.f) {
            const float iscale = __fdiv_rn(127.f, amax);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                int qi = (int)rintf(__fmul_rn(iscale, v[i]));
                qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
                s += qi;
                packed[i >> 2] |= ((uint32_t)(qi & 0xff)) << (8 * (i & 3));
            }
            if (lane == 0) d[b] = __fdiv_rn(1.f, iscale);
        } else if (lane == 0) {
            d[b] = 0.f;
        }
        *reinterpret_cast<uint2*>(q + (size_t)b * 256 + lane * 8) = make_uint2(packed[0], packed[1]);
        s += __shfl_xor_sync(0xffffffffu, s, 1);     // 16-value groups = lane pairs
        if ((lane & 1) == 0) bsums[(size_t)b * 16 + (lane >> 1)] = (int16_t)s;
    }
}

void launch_q8k_quantize(const float* x, int rows, int n, float* d, int8_t* q, int16_t* bsums, cudaStream_t s) {
    const int nblk = rows * (n / 256);
    q8k_quantize_kernel<<<max(1, min(148 * 8, (nblk + 7) / 8)), 256, 0, s>>>(x, nblk, d, q, bsums);
}

__device__ __forceinline__ int warp_isum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Integer dots of superblock sb of a Q4_K row with a Q8_K vector, complete on every lane.
//   isc = sum_j sc_j * sum_{k in sub-block j} q4*q8,  imn = sum_j m_j * bsum_j
__device__ __forceinline__ void q4k_q8k_sb(const uint8_t* __restrict__ row, int sb, int lane,
                                           const int8_t* __restrict__ q8, const int16_t* __restrict__ bs,
                                           int& isc, int& imn) {
    const uint8_t* blk = row + (size_t)sb * 144;
    uint8_t s12[12];
    {
        const uint32_t s0 = __ldg(reinterpret_cast<const unsigned int*>(blk + 4));
        const uint32_t s1 = __ldg(reinterpret_cast<const unsigned int*>(blk + 8));
        const uint32_t s2 = __ldg(reinterpret_cast<const unsigned int*>(blk + 12));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            s12[i] = (uint8_t)(s0 >> (8 * i));
            s12[4 + i] = (uint8_t)(s1 >> (8 * i));
            s12[8 + i] = (uint8_t)(s2 >> (8 * i));
        }
    }
    const int g = lane >> 3, kk = (lane & 7) * 4;
    const uint32_t qs = __ldg(reinterpret_cast<const unsigned int*>(blk + 16 + 4 * lane));
    const int* qv = reinterpret_cast<const int*>(q8 + (size_t)sb * 256 + 64 * g + kk);
    const int lo = __dp4a((int)(qs & 0x0F0F0F0Fu), qv[0], 0);
    const int hi = __dp4a((int)((qs >> 4) & 0x0F0F0F0Fu), qv[8], 0);
    int sc0, m0, sc1, m1;
    q4k_sm(s12, 2 * g, sc0, m0);
    q4k_sm(s12, 2 * g + 1, sc1, m1);
    isc = warp_isum(sc0 * lo + sc1 * hi);
    int mterm = 0;
    if (lane < 8) {
        int scj, mj;
        q4k_sm(s12, lane, scj, mj);
        mterm = mj * ((int)bs[sb * 16 + 2 * lane] + (int)bs[sb * 16 + 2 * lane + 1]);
    }
    imn = warp_isum(mterm);
}

// isum = sum_g sc_g * sum_{k in 16-group g} (q6 - 32) * q8 for superblock sb of a Q6_K row
__device__ __forceinline__ int q6k_q8k_sb(const uint8_t* __restrict__ row, int sb, int lane,
                                          const int8_t* __restrict__ q8, int q6s) {
    const uint8_t* blk = row + (size_t)sb * q6s;
    const int h = lane >> 4, kk = 2 * (lane & 15);
    const uint32_t qlA = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(blk + h * 64 + kk));
    const uint32_t qlB = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(blk + h * 64 + 32 + kk));
    const uint32_t qh = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(blk + 128 + h * 32 + kk));
    const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
    const int8_t* qb = q8 + (size_t)sb * 256 + h * 128 + kk;
    int acc = 0;
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const uint32_t ql = (s & 1) ? qlB : qlA;
        int part = 0;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int lo = (ql >> (8 * i + 4 * (s >> 1))) & 15;
            const int hi = (qh >> (8 * i + 2 * s)) & 3;
            part += ((lo | (hi << 4)) - 32) * (int)qb[32 * s + i];
        }
        acc += (int)__ldg(sc + h * 8 + 2 * s + (kk >> 4)) * part;
    }
    return warp_isum(acc);
}

__global__ void q8k_block_dots_kernel(int code, const uint8_t* __restrict__ W, int rows, int n_in,
                                      const int8_t* __restrict__ q, const int16_t* __restrict__ bs,
                                      int32_t* __restrict__ out2, int q6s) {
    const int lane = threadIdx.x & 31;
    const int nb = n_in / 256;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const size_t rb = row_bytes(code, n_in, q6s);
    for (int it = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < rows * nb; it += nw) {
        const int r = it / nb, sb = it % nb;
        int a, m = 0;
        if (code == DRACO_CODE_Q4_K) q4k_q8k_sb(W + rb * r, sb, lane, q, bs, a, m);
        else a = q6k_q8k_sb(W + rb * r, sb, lane, q, q6s);
        if (lane == 0) {
            out2[(size_t)it * 2] = a;
            out2[(size_t)it * 2 + 1] = m;
        }
    }
}

void launch_q8k_block_dots(int code, const uint8_t* W, int rows, int n_in, const int8_t* q, const int16_t* bsums,
                           int32_t* out2, cudaStream_t s, int q6s) {
    const int items = rows * (n_in / 256);
    q8k_block_dots_kernel<<<max(1, min(148 * 8, (items + 7) / 8)), 256, 0, s>>>(code, W, rows, n_in, q, bsums, out2,
                                                                                q6s);
}

// row dot in Q8_K mode, float combination in superblock order (the order of orc_gemv_q8k)
template <int CODE>
__device__ __forceinline__ float q8k_row_dot(const uint8_t* __restrict__ row, int nb, int lane,
                                             const int8_t* __restrict__ q, const float* __restrict__ d8,
                                             const int16_t* __restrict__ bs, int q6s) {
    float dot = 0.f;
    for (int sb = 0; sb < nb; sb++) {
        if (CODE == DRACO_CODE_Q4_K) {
            int isc, imn;
            q4k_q8k_sb(row, sb, lane, q, bs, isc, imn);
            const uint32_t hd = __ldg(reinterpret_cast<const unsigned int*>(row + (size_t)sb * 144));
            const float d = h2f((uint16_t)(hd & 0xffff)), dmin = h2f((uint16_t)(hd >> 16));
            const float v = fmaf(d, (float)isc, -__fmul_rn(dmin, (float)imn));
            dot = fmaf(d8[sb], v, dot);
        } else {
            const int is = q6k_q8k_sb(row, sb, lane, q, q6s);
            const float d6 = h2f(__ldg(reinterpret_cast<const unsigned short*>(row + (size_t)sb * q6s + 208)));
            dot = fmaf(__fmul_rn(d8[sb], d6), (float)is, dot);
        }
    }
    return dot;
}

template <int CODE>
__global__ void gemv_q8k_kernel(const uint8_t* __restrict__ W, int rows, int n_in, const int8_t* __restrict__ q,
                                const float* __restrict__ d, const int16_t* __restrict__ bs, float* __restrict__ y,
                                int q6s) {
    const int lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    const size_t rb = row_bytes(CODE, n_in, q6s);
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += nw) {
        const float v = q8k_row_dot<CODE>(W + rb * r, n_in / 256, lane, q, d, bs, q6s);
        if (lane == 0) y[r] = v;
    }
}

void launch_gemv_q8k(int code, const uint8_t* W, int rows, int n_in, const int8_t* q, const float* d,
                     const int16_t* bsums, float* y, cudaStream_t s, int q6s) {
    const int grid = max(1, min(148 * 8, (rows + 7) / 8));
    if (code == DRACO_CODE_Q4_K)
        gemv_q8k_kernel<DRACO_CODE_Q4_K><<<grid, 256, 0, s>>>(W, rows, n_in, q, d, bsums, y, q6s);
    else
        gemv_q8k_kernel<DRACO_CODE_Q6_K><<<grid, 256, 0, s>>>(W, rows, n_in, q, d, bsums, y, q6s);
}

// grouped gate/up + SwiGLU with Q8_K activations of the assignment's token
template <int CG, int CU>
__global__ void gateup_q8k_kernel(ExpertTable tab, const int* __restrict__ active, const int* __restrict__ n_active_p,
                                  const int* __restrict__ off, const int* __restrict__ ilist, int tok_div,
                                  const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                  const int16_t* __restrict__ xbs, int inter, int n_in, float* __restrict__ act,
                                  int q6s) {
    const int n_active = *n_active_p;
    constexpr int kRows = 8;   // one warp per row, 8 warps per item
    const int nrb = (inter + kRows - 1) / kRows;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = n_in / 256;
    const size_t rbg = row_bytes(CG, n_in, q6s), rbu = row_bytes(CU, n_in, q6s);
    for (int item = blockIdx.x; item < n_active * nrb; item += gridDim.x) {
        const int a = item / nrb, rbi = item % nrb;
        const int e = active[a];
        const int p0 = off[e], c = off[e + 1] - p0;
        const int row = rbi * kRows + warp;
        if (row >= inter) continue;
        const uint8_t* G = tab.w[3 * e] + rbg * row;
        const uint8_t* U = tab.w[3 * e + 1] + rbu * row;
        for (int j = 0; j < c; j++) {
            const int t = ilist ? ilist[p0 + j] / tok_div : p0 + j;
            const int8_t* q = xq + (size_t)t * n_in;
            const float* d = xd + (size_t)t * nb;
            const int16_t* bs = xbs + (size_t)t * nb * 16;
            const float g = q8k_row_dot<CG>(G, nb, lane, q, d, bs, q6s);
            const float u = q8k_row_dot<CU>(U, nb, lane, q, d, bs, q6s);
            if (lane == 0) act[(size_t)(p0 + j) * inter + row] = silu_mul(g, u);
        }
    }
}

void launch_gateup_q8k(const ExpertTable& tab, int cg, const int* active, const int* n_active, int n_active_max,
                       const int* off, const int* ilist, int tok_div, const int8_t* xq, const float* xd,
                       const int16_t* xbs, int inter, int n_in, float* act, cudaStream_t s, int q6s) {
    const int grid = max(1, min(148 * 8, n_active_max * ((inter + 7) / 8)));
    if (cg == DRACO_CODE_Q4_K)
        gateup_q8k_kernel<DRACO_CODE_Q4_K, DRACO_CODE_Q4_K><<<grid, 256, 0, s>>>(tab, active, n_active, off, ilist,
                                                                                 tok_div, xq, xd, xbs, inter, n_in, act, q6s);
    else
        gateup_q8k_kernel<DRACO_CODE_Q6_K, DRACO_CODE_Q6_K><<<grid, 256, 0, s>>>(tab, active, n_active, off, ilist,
                                                                                 tok_div, xq, xd, xbs, inter, n_in, act, q6s);
}

}  // namespace draco
