// Grouped dequant-GEMV / small-batch GEMM on CUDA cores, fp32 activations.
//
// Lane layout: a warp walks a weight row one 256-value superblock at a time; each lane owns
// 8 values of the superblock and loads exactly the bytes they live in (Q4_K: one aligned u32
// of nibbles; Q6_K: three u16 (two ql pairs + one qh pair); Q8_0: four u16), so a warp's
// loads of one superblock are contiguous.  Values are decoded to fp32 as the reference does
// (src/m5_kern_scalar.c:69-142) and multiplied into per-lane fp32 partial sums that a warp
// reduction finishes.  Rows are taken RPW at a time per warp so the x fragment loaded for a
// superblock is reused by every row.
#include "kernels.cuh"

#include <algorithm>

namespace draco {

// value position p (0..255 within the superblock) of the lane's j-th value
template <int CODE>
__device__ __forceinline__ int lane_pos(int lane, int j);

template <>
__device__ __forceinline__ int lane_pos<DRACO_CODE_Q4_K>(int lane, int j) {
    // qs bytes 4*lane..+3: low nibbles -> sub-block 2g, high nibbles -> 2g+1, g = lane/8
    return ((lane >> 3) * 2 + (j >> 2)) * 32 + (lane & 7) * 4 + (j & 3);
}
template <>
__device__ __forceinline__ int lane_pos<DRACO_CODE_Q6_K>(int lane, int j) {
    // qh pair 2*(lane%16) of half lane/16; j = 2*s + i  ->  p = h*128 + 32*s + kk + i
    return (lane >> 4) * 128 + 32 * (j >> 1) + 2 * (lane & 15) + (j & 1);
}
template <>
__device__ __forceinline__ int lane_pos<DRACO_CODE_Q8_0>(int lane, int j) {
    return (lane >> 2) * 32 + (lane & 3) * 8 + j;
}

// the lane's 8 fp32 x values of superblock sb (x already offset to the row of x)
template <int CODE>
__device__ __forceinline__ void lane_x(const float* __restrict__ x, int sb, int lane, float v[8]) {
    const float* b = x + sb * 256;
    if (CODE == DRACO_CODE_Q4_K) {
        const float4 a = *reinterpret_cast<const float4*>(b + lane_pos<CODE>(lane, 0));
        const float4 c = *reinterpret_cast<const float4*>(b + lane_pos<CODE>(lane, 4));
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    } else if (CODE == DRACO_CODE_Q6_K) {
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const float2 a = *reinterpret_cast<const float2*>(b + lane_pos<CODE>(lane, 2 * s));
            v[2 * s] = a.x;
            v[2 * s + 1] = a.y;
        }
    } else {
        const float4 a = *reinterpret_cast<const float4*>(b + lane_pos<CODE>(lane, 0));
        const float4 c = *reinterpret_cast<const float4*>(b + lane_pos<CODE>(lane, 4));
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    }
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
    return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p));
}

// the lane's 8 dequantised weights of superblock sb of `row`
template <int CODE>
__device__ __forceinline__ void lane_w(const uint8_t* __restrict__ row, int sb, int lane, float w[8], int q6s) {
    if (CODE == DRACO_CODE_Q4_K) {
        const uint8_t* blk = row + (size_t)sb * 144;
        const uint32_t hd = __ldg(reinterpret_cast<const unsigned int*>(blk));
        const uint32_t s0 = __ldg(reinterpret_cast<const unsigned int*>(blk + 4));
        const uint32_t s1 = __ldg(reinterpret_cast<const unsigned int*>(blk + 8));
        const uint32_t s2 = __ldg(reinterpret_cast<const unsigned int*>(blk + 12));
        const uint32_t qs = __ldg(reinterpret_cast<const unsigned int*>(blk + 16 + 4 * lane));
        const float d = h2f((uint16_t)(hd & 0xffff)), dmin = h2f((uint16_t)(hd >> 16));
        uint8_t sb12[12];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            sb12[i] = (uint8_t)(s0 >> (8 * i));
            sb12[4 + i] = (uint8_t)(s1 >> (8 * i));
            sb12[8 + i] = (uint8_t)(s2 >> (8 * i));
        }
        const int g = lane >> 3;
        int sc0, m0, sc1, m1;
        q4k_sm(sb12, 2 * g, sc0, m0);
        q4k_sm(sb12, 2 * g + 1, sc1, m1);
        const float ds0 = d * (float)sc0, dm0 = dmin * (float)m0;
        const float ds1 = d * (float)sc1, dm1 = dmin * (float)m1;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[i] = fmaf(ds0, (float)((qs >> (8 * i)) & 15), -dm0);
            w[4 + i] = fmaf(ds1, (float)((qs >> (8 * i + 4)) & 15), -dm1);
        }
    } else if (CODE == DRACO_CODE_Q6_K) {
        const uint8_t* blk = row + (size_t)sb * q6s;
        const int h = lane >> 4, kk = 2 * (lane & 15);
        const uint32_t qlA = ld_u16(blk + h * 64 + kk);
        const uint32_t qlB = ld_u16(blk + h * 64 + 32 + kk);
        const uint32_t qh = ld_u16(blk + 128 + h * 32 + kk);
        const float d = h2f((uint16_t)ld_u16(blk + 208));
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const uint32_t ql = (s & 1) ? qlB : qlA;
            const float dsc = d * (float)__ldg(sc + h * 8 + 2 * s + (kk >> 4));
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int lo = (ql >> (8 * i + 4 * (s >> 1))) & 15;
                const int hi = (qh >> (8 * i + 2 * s)) & 3;
                w[2 * s + i] = dsc * (float)((lo | (hi << 4)) - 32);
            }
        }
    } else {
        const uint8_t* blk = row + (size_t)(sb * 8 + (lane >> 2)) * 34;
        const float d = h2f((uint16_t)ld_u16(blk));
        const uint8_t* q = blk + 2 + (lane & 3) * 8;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t v = ld_u16(q + 2 * i);
            w[2 * i] = d * (float)(int8_t)(v & 0xff);
            w[2 * i + 1] = d * (float)(int8_t)(v >> 8);
        }
    }
}

// number of superblock steps of a row and whether a lane's step is in range (Q8_0 rows may
// end inside a 256-value step)
__device__ __forceinline__ int n_steps(int n_in) { return (n_in + 255) / 256; }
template <int CODE>
__device__ __forceinline__ bool lane_live(int sb, int lane, int n_in) {
    if (CODE == DRACO_CODE_Q8_0) return (sb * 8 + (lane >> 2)) * 32 < n_in;
    return true;
}

constexpr int kRPW = 4;     // rows per warp
constexpr int kCT = 4;      // tokens per pass
constexpr int kWarps = 4;   // warps per block
constexpr int kRowsPerItem = kRPW * kWarps;

// ------------------------------------------------------------------------------------------
// gate/up + SwiGLU: act[p][r] = silu(gate_e[r] . x_t) * (up_e[r] . x_t) for the tokens of each
// active expert; p is the sorted position of the assignment, t = ilist[p] / tok_div.
// ------------------------------------------------------------------------------------------
template <int CG, int CU>
__global__ void __launch_bounds__(32 * kWarps) gateup_kernel(ExpertTable tab, const int* __restrict__ active,
                                                            const int* __restrict__ n_active_p,
                                                            const int* __restrict__ off,
                                                            const int* __restrict__ ilist, int tok_div,
                                                            const float* __restrict__ X, int inter, int n_in,
                                                            float* __restrict__ act, int q6s) {
    const int n_active = *n_active_p;
    const int nrb = (inter + kRowsPerItem - 1) / kRowsPerItem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t rbg = row_bytes(CG, n_in, q6s), rbu = row_bytes(CU, n_in, q6s);
    const int steps = n_steps(n_in);
    for (int item = blockIdx.x; item < n_active * nrb; item += gridDim.x) {
        const int a = item / nrb, rb = item % nrb;
        const int e = active[a];
        const int p0 = off[e], c = off[e + 1] - p0;
        const uint8_t* G = tab.w[3 * e];
        const uint8_t* U = tab.w[3 * e + 1];
        const int r0 = rb * kRowsPerItem + warp * kRPW;
        for (int tc = 0; tc < c; tc += kCT) {
            const int nt = min(kCT, c - tc);
            const float* xr[kCT];
#pragma unroll
            for (int j = 0; j < kCT; j++) {
                const int pj = p0 + tc + min(j, nt - 1);
                const int t = ilist ? ilist[pj] / tok_div : pj;
                xr[j] = X + (size_t)t * n_in;
            }
            float ag[kRPW][kCT], au[kRPW][kCT];
#pragma unroll
            for (int r = 0; r < kRPW; r++)
#pragma unroll
                for (int j = 0; j < kCT; j++) ag[r][j] = au[r][j] = 0.f;
            for (int sb = 0; sb < steps; sb++) {
                float xv[kCT][8];
#pragma unroll
                for (int j = 0; j < kCT; j++) {
                    if (CG == CU && lane_live<CG>(sb, lane, n_in)) lane_x<CG>(xr[j], sb, lane, xv[j]);
                }
#pragma unroll
                for (int r = 0; r < kRPW; r++) {
                    const int row = r0 + r;
                    if (row >= inter) break;
                    float w[8];
                    if (lane_live<CG>(sb, lane, n_in)) {
                        if (CG != CU) {
#pragma unroll
                            for (int j = 0; j < kCT; j++) lane_x<CG>(xr[j], sb, lane, xv[j]);
                        }
                        lane_w<CG>(G + rbg * row, sb, lane, w, q6s);
#pragma unroll
                        for (int j = 0; j < kCT; j++)
#pragma unroll
                            for (int i = 0; i < 8; i++) ag[r][j] = fmaf(w[i], xv[j][i], ag[r][j]);
                    }
                    if (lane_live<CU>(sb, lane, n_in)) {
                        if (CG != CU) {
#pragma unroll
                            for (int j = 0; j < kCT; j++) lane_x<CU>(xr[j], sb, lane, xv[j]);
                        }
                        lane_w<CU>(U + rbu * row, sb, lane, w, q6s);
#pragma unroll
                        for (int j = 0; j < kCT; j++)
#pragma unroll
                            for (int i = 0; i < 8; i++) au[r][j] = fmaf(w[i], xv[j][i], au[r][j]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < kRPW; r++)
#pragma unroll
                for (int j = 0; j < kCT; j++) {
                    const float g = warp_sum(ag[r][j]);
                    const float u = warp_sum(au[r][j]);
                    const int row = r0 + r;
                    if (lane == 0 && row < inter && j < nt)
                        act[(size_t)(p0 + tc + j) * inter + row] = silu_mul(g, u);
                }
        }
    }
}

// ------------------------------------------------------------------------------------------
// down: y[p][r] = down_e[r] . act[p] for every sorted assignment p of each active expert
// ------------------------------------------------------------------------------------------
template <int CD>
__global__ void __launch_bounds__(32 * kWarps) down_kernel(ExpertTable tab, const int* __restrict__ active,
                                                          const int* __restrict__ n_active_p,
                                                          const int* __restrict__ off,
                                                          const float* __restrict__ act, int inter,
                                                          int n_out, float* __restrict__ y, int q6s) {
    const int n_active = *n_active_p;
    const int nrb = (n_out + kRowsPerItem - 1) / kRowsPerItem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t rbd = row_bytes(CD, inter, q6s);
    const int steps = n_steps(inter);
    for (int item = blockIdx.x; item < n_active * nrb; item += gridDim.x) {
        const int a = item / nrb, rb = item % nrb;
        const int e = active[a];
        const int p0 = off[e], c = off[e + 1] - p0;
        const uint8_t* D = tab.w[3 * e + 2];
        const int r0 = rb * kRowsPerItem + warp * kRPW;
        for (int tc = 0; tc < c; tc += kCT) {
            const int nt = min(kCT, c - tc);
            float ad[kRPW][kCT];
#pragma unroll
            for (int r = 0; r < kRPW; r++)
#pragma unroll
                for (int j = 0; j < kCT; j++) ad[r][j] = 0.f;
            for (int sb = 0; sb < steps; sb++) {
                if (!lane_live<CD>(sb, lane, inter)) continue;
                float xv[kCT][8];
#pragma unroll
                for (int j = 0; j < kCT; j++)
                    lane_x<CD>(act + (size_t)(p0 + tc + min(j, nt - 1)) * inter, sb, lane, xv[j]);
#pragma unroll
                for (int r = 0; r < kRPW; r++) {
                    const int row = r0 + r;
                    if (row >= n_out) break;
                    float w[8];
                    lane_w<CD>(D + rbd * row, sb, lane, w, q6s);
#pragma unroll
                    for (int j = 0; j < kCT; j++)
#pragma unroll
                        for (int i = 0; i < 8; i++) ad[r][j] = fmaf(w[i], xv[j][i], ad[r][j]);
                }
            }
#pragma unroll
            for (int r = 0; r < kRPW; r++)
#pragma unroll
                for (int j = 0; j < kCT; j++) {
                    const float v = warp_sum(ad[r][j]);
                    const int row = r0 + r;
                    if (lane == 0 && row < n_out && j < nt) y[(size_t)(p0 + tc + j) * n_out + row] = v;
                }
        }
    }
}

static int grid_for(int items) { return max(1, min(items, 148 * 8)); }

#define DRACO_GU(A, B)                                                                           \
    gateup_kernel<A, B><<<grid, 32 * kWarps, 0, s>>>(tab, active, n_active, off, ilist, tok_div, X, \
                                                      inter, n_in, act, q6s)

void launch_gateup_codes(const ExpertTable& tab, int cg, int cu, const int* active, const int* n_active,
                         int n_active_max, const int* off, const int* ilist, int tok_div, const float* X,
                         int inter, int n_in, float* act, cudaStream_t s, int q6s) {
    const int grid = grid_for(n_active_max * ((inter + kRowsPerItem - 1) / kRowsPerItem));
    constexpr int A = DRACO_CODE_Q4_K, B = DRACO_CODE_Q6_K, C = DRACO_CODE_Q8_0;
    if (cg == A && cu == A) DRACO_GU(A, A);
    else if (cg == B && cu == B) DRACO_GU(B, B);
    else if (cg == C && cu == C) DRACO_GU(C, C);
    else if (cg == A && cu == B) DRACO_GU(A, B);
    else if (cg == A && cu == C) DRACO_GU(A, C);
    else if (cg == B && cu == A) DRACO_GU(B, A);
    else if (cg == B && cu == C) DRACO_GU(B, C);
    else if (cg == C && cu == A) DRACO_GU(C, A);
    else DRACO_GU(C, B);
}

void launch_down_code(const ExpertTable& tab, int cd, const int* active, const int* n_active,
                      int n_active_max, const int* off, const float* act, int inter, int n_out, float* y,
                      cudaStream_t s, int q6s) {
    const int grid = grid_for(n_active_max * ((n_out + kRowsPerItem - 1) / kRowsPerItem));
    if (cd == DRACO_CODE_Q4_K)
        down_kernel<DRACO_CODE_Q4_K><<<grid, 32 * kWarps, 0, s>>>(tab, active, n_active, off, act, inter, n_out, y, q6s);
    else if (cd == DRACO_CODE_Q6_K)
        down_kernel<DRACO_CODE_Q6_K><<<grid, 32 * kWarps, 0, s>>>(tab, active, n_active, off, act, inter, n_out, y, q6s);
    else
        down_kernel<DRACO_CODE_Q8_0><<<grid, 32 * kWarps, 0, s>>>(tab, active, n_active, off, act, inter, n_out, y, q6s);
}

// ------------------------------------------------------------------------------------------
// plain row dot products over a dense batch: Y[t][r] = W[r] . X[t]
// ------------------------------------------------------------------------------------------
template <int CODE>
__global__ void __launch_bounds__(32 * kWarps) dense_kernel(const uint8_t* __restrict__ W,
                                                           const float* __restrict__ X, int T, int n_out,
                                                           int n_in, long x_stride, int o0,
                                                           float* __restrict__ Y, long y_stride, int q6s) {
    const int nrb = (n_out - o0 + kRowsPerItem - 1) / kRowsPerItem;
    const int ntc = (T + kCT - 1) / kCT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t rb = row_bytes(CODE, n_in, q6s);
    const int steps = n_steps(n_in);
    for (int item = blockIdx.x; item < nrb * ntc; item += gridDim.x) {
        const int rbi = item % nrb, tc = (item / nrb) * kCT;
        const int nt = min(kCT, T - tc);
        const int r0 = o0 + rbi * kRowsPerItem + warp * kRPW;
        float acc[kRPW][kCT];
#pragma unroll
        for (int r = 0; r < kRPW; r++)
#pragma unroll
            for (int j = 0; j < kCT; j++) acc[r][j] = 0.f;
        for (int sb = 0; sb < steps; sb++) {
            if (!lane_live<CODE>(sb, lane, n_in)) continue;
            float xv[kCT][8];
#pragma unroll
            for (int j = 0; j < kCT; j++) lane_x<CODE>(X + (size_t)(tc + min(j, nt - 1)) * x_stride, sb, lane, xv[j]);
#pragma unroll
            for (int r = 0; r < kRPW; r++) {
                const int row = r0 + r;
                if (row >= n_out) break;
                float w[8];
                lane_w<CODE>(W + rb * row, sb, lane, w, q6s);
#pragma unroll
                for (int j = 0; j < kCT; j++)
#pragma unroll
                    for (int i = 0; i < 8; i++) acc[r][j] = fmaf(w[i], xv[j][i], acc[r][j]);
            }
        }
#pragma unroll
        for (int r = 0; r < kRPW; r++)
#pragma unroll
            for (int j = 0; j < kCT; j++) {
                const float v = warp_sum(acc[r][j]);
                const int row = r0 + r;
                if (lane == 0 && row < n_out && j < nt) Y[(size_t)(tc + j) * y_stride + row] = v;
            }
    }
}

static void dense_launch(int code, const uint8_t* W, const float* X, int T, int n_out, int n_in, long x_stride,
                         int o0, float* Y, long y_stride, cudaStream_t s, int q6s) {
    const int items = ((n_out - o0 + kRowsPerItem - 1) / kRowsPerItem) * ((T + kCT - 1) / kCT);
    const int grid = grid_for(items);
    if (code == DRACO_CODE_Q4_K)
        dense_kernel<DRACO_CODE_Q4_K><<<grid, 32 * kWarps, 0, s>>>(W, X, T, n_out, n_in, x_stride, o0, Y, y_stride, q6s);
    else if (code == DRACO_CODE_Q6_K)
        dense_kernel<DRACO_CODE_Q6_K><<<grid, 32 * kWarps, 0, s>>>(W, X, T, n_out, n_in, x_stride, o0, Y, y_stride, q6s);
    else
        dense_kernel<DRACO_CODE_Q8_0><<<grid, 32 * kWarps, 0, s>>>(W, X, T, n_out, n_in, x_stride, o0, Y, y_stride, q6s);
}

void launch_gemv_rows(int code, const uint8_t* W, const float* x, int n_in, int o0, int o1, float* y,
                      cudaStream_t s, int q6s) {
    if (o1 > o0) dense_launch(code, W, x, 1, o1, n_in, n_in, o0, y, o1, s, q6s);
}

void launch_gemm_dense(int code, const uint8_t* W, const float* X, int T, int n_out, int n_in, float* Y,
                       cudaStream_t s, int q6s) {
    dense_launch(code, W, X, T, n_out, n_in, n_in, 0, Y, n_out, s, q6s);
}

// ------------------------------------------------------------------------------------------
// dequantise rows to fp32
// ------------------------------------------------------------------------------------------
template <int CODE>
__global__ void dequant_kernel(const uint8_t* __restrict__ W, int rows, int n_in, float* __restrict__ out, int q6s) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const size_t rb = row_bytes(CODE, n_in, q6s);
    const int steps = n_steps(n_in);
    for (int it = warp; it < rows * steps; it += nwarps) {
        const int r = it / steps, sb = it % steps;
        if (!lane_live<CODE>(sb, lane, n_in)) continue;
        float w[8];
        lane_w<CODE>(W + rb * r, sb, lane, w, q6s);
#pragma unroll
        for (int j = 0; j < 8; j++) out[(size_t)r * n_in + sb * 256 + lane_pos<CODE>(lane, j)] = w[j];
    }
}

void launch_dequant(int code, const uint8_t* W, int rows, int n_in, float* out, cudaStream_t s, int q6s) {
    const int grid = max(1, min(148 * 4, (rows * ((n_in + 255) / 256) + 7) / 8));
    if (code == DRACO_CODE_Q4_K) dequant_kernel<DRACO_CODE_Q4_K><<<grid, 256, 0, s>>>(W, rows, n_in, out, q6s);
    else if (code == DRACO_CODE_Q6_K) dequant_kernel<DRACO_CODE_Q6_K><<<grid, 256, 0, s>>>(W, rows, n_in, out, q6s);
    else dequant_kernel<DRACO_CODE_Q8_0><<<grid, 256, 0, s>>>(W, rows, n_in, out, q6s);
}

// ------------------------------------------------------------------------------------------
// combine: out[t][r] = fma(w[t,K-1], y, ... fma(w[t,0], y, 0)) (+ shared[t][r])
// (src/m6_moe_tok.c:148-159; the ungated shared expert is added after, src/m6_engine.c:348)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __half* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

template <typename Y>
__global__ void combine_kernel(const Y* __restrict__ y, const int* __restrict__ order,
                               const float* __restrict__ wtop, const int* __restrict__ pos_of, int T, int K,
                               int E, int n_out, const float* __restrict__ shared, float* __restrict__ out) {
    const int t = blockIdx.y;
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n_out; r += gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int k = 0; k < K; k++) {
            const int i = t * K + k;
            const int e = order[i];
            if (e < 0 || e >= E) continue;
            acc = fmaf(wtop[i], to_f(y[(size_t)pos_of[i] * n_out + r]), acc);
        }
        if (shared) acc = __fadd_rn(acc, shared[(size_t)t * n_out + r]);
        out[(size_t)t * n_out + r] = acc;
    }
}

// The same sums for n_out % 4 == 0, one block per token row: warp 0 stages the row's valid
// (weight, y row) pairs in k order in shared memory, then every thread runs the identical fma
// chain over float4 columns with the y loads of four assignments issued ahead of their fmas.
// out_blk != nullptr: row t goes to out_blk[t / blk] + (t % blk) * n_out instead (the row blocks
// of other GPUs' buffers, peer stores), a row without a valid assignment is not written, and
// every thread fences its stores at system scope before it ends, so a flag barrier that follows
// publishes them.
constexpr int kCombineMaxK = 64;
constexpr int kCombineThreads = 128;
__device__ __forceinline__ void fma4(float4& a, float w, const float4& v) {
    a.x = fmaf(w, v.x, a.x);
    a.y = fmaf(w, v.y, a.y);
    a.z = fmaf(w, v.z, a.z);
    a.w = fmaf(w, v.w, a.w);
}
template <typename Y>
__global__ void __launch_bounds__(kCombineThreads) combine_rows_kernel(
    const Y* __restrict__ y, const int* __restrict__ order, const float* __restrict__ wtop,
    const int* __restrict__ pos_of, int K, int E, int n_out, int cpb, const float* __restrict__ shared,
    float* __restrict__ out, float* const* __restrict__ out_blk, int blk) {
    __shared__ float sw[kCombineMaxK];
    __shared__ const Y* sy[kCombineMaxK];
    __shared__ int sn;
    const int t = blockIdx.x;
    const int n4 = n_out / 4;
    const int c0 = blockIdx.y * cpb, c1 = min(n4, c0 + cpb);   // this block's float4 columns
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int base = 0;
        for (int k0 = 0; k0 < K; k0 += 32) {
            const int k = k0 + lane;
            bool v = false;
            int p = 0;
            float w = 0.f;
            if (k < K) {
                const int e = order[(size_t)t * K + k];
                v = e >= 0 && e < E;
                if (v) {
                    p = pos_of[(size_t)t * K + k];
                    w = wtop[(size_t)t * K + k];
                }
            }
            const unsigned m = __ballot_sync(0xffffffffu, v);
            if (v) {
                const int j = base + __popc(m & ((1u << lane) - 1u));
                sw[j] = w;
                sy[j] = y + (size_t)p * n_out;
            }
            base += __popc(m);
        }
        if (lane == 0) sn = base;
    }
    __syncthreads();
    const int n = sn;
    if (out_blk && n == 0) return;   // a padding row: nothing of this slice to send
    const float4* sh = shared ? reinterpret_cast<const float4*>(shared + (size_t)t * n_out) : nullptr;
    float4* o = reinterpret_cast<float4*>(out_blk ? out_blk[t / blk] + (size_t)(t % blk) * n_out
                                                  : out + (size_t)t * n_out);
    for (int c = c0 + threadIdx.x; c < c1; c += kCombineThreads) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        int j = 0;
        for (; j + 4 <= n; j += 4) {
            const float4 v0 = load4(sy[j] + 4 * c), v1 = load4(sy[j + 1] + 4 * c), v2 = load4(sy[j + 2] + 4 * c),
                         v3 = load4(sy[j + 3] + 4 * c);
            fma4(acc, sw[j], v0);
            fma4(acc, sw[j + 1], v1);
            fma4(acc, sw[j + 2], v2);
            fma4(acc, sw[j + 3], v3);
        }
        for (; j < n; j++) fma4(acc, sw[j], load4(sy[j] + 4 * c));
        if (sh) {
            const float4 v = sh[c];
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        o[c] = acc;
    }
    if (out_blk) __threadfence_system();
}

__global__ void half_to_float_kernel(const __half* __restrict__ x, float* __restrict__ y, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __half2float(x[i]);
}
void launch_half_to_float(const __half* x, float* y, size_t n, cudaStream_t s) {
    const int blocks = (int)std::max<size_t>(1, std::min<size_t>(148 * 8, (n + 255) / 256));
    half_to_float_kernel<<<blocks, 256, 0, s>>>(x, y, n);
}

__global__ void set_pair_kernel(int* d, int a, int b) {
    d[0] = a;
    d[1] = b;
}
void launch_set_pair(int* d, int a, int b, cudaStream_t s) { set_pair_kernel<<<1, 1, 0, s>>>(d, a, b); }

template <typename Y>
static void combine_typed(const Y* y, const int* order, const float* wtop, const int* pos_of, int T, int K, int E,
                          int n_out, const float* shared, float* out, float* const* out_blk, int blk,
                          cudaStream_t s) {
    const bool vec = n_out % 4 == 0 && K <= kCombineMaxK && !((uintptr_t)y & 15) && !((uintptr_t)out & 15) &&
                     !((uintptr_t)shared & 15);
    if (vec || out_blk) {   // row blocks: the caller checked n_out % 4 == 0, K <= kCombineMaxK
        // few rows: each row split over blocks of one float4 column a thread, so small batches
        // still spread over the SMs
        const int n4 = n_out / 4;
        const int cpb = T >= 148 ? n4 : kCombineThreads;
        dim3 grid(T, (n4 + cpb - 1) / cpb);
        if (T > 0)
            combine_rows_kernel<<<grid, kCombineThreads, 0, s>>>(y, order, wtop, pos_of, K, E, n_out, cpb, shared, out,
                                                                 out_blk, blk);
        return;
    }
    dim3 grid((n_out + 255) / 256, T);
    combine_kernel<<<grid, 256, 0, s>>>(y, order, wtop, pos_of, T, K, E, n_out, shared, out);
}

void launch_combine(const float* y, const int* order, const float* wtop, const int* pos_of, int T, int K, int E,
                    int n_out, const float* shared, float* out, cudaStream_t s, float* const* out_blk, int blk) {
    combine_typed(y, order, wtop, pos_of, T, K, E, n_out, shared, out, out_blk, blk, s);
}
void launch_combine_half(const __half* y, const int* order, const float* wtop, const int* pos_of, int T, int K, int E,
                         int n_out, const float* shared, float* out, cudaStream_t s, float* const* out_blk, int blk) {
    combine_typed(y, order, wtop, pos_of, T, K, E, n_out, shared, out, out_blk, blk, s);
}

// ------------------------------------------------------------------------------------------
// scalar-gated shared expert (src/m6_engine.c:1113-1127): out = y * sigmoid(gw . x)
// ------------------------------------------------------------------------------------------
__global__ void shexp_gate_kernel(const float* __restrict__ x, const float* __restrict__ gw, int h,
                                  const float* __restrict__ y, float* __restrict__ sg, float* __restrict__ out) {
    const int t = blockIdx.x;
    __shared__ float s_gate;
    if (threadIdx.x < 32) {
        float acc = 0.f;
        for (int i = threadIdx.x; i < h; i += 32) acc = fmaf(gw[i], x[(size_t)t * h + i], acc);
        acc = warp_sum(acc);
        if (threadIdx.x == 0) {
            sg[t] = acc;
            s_gate = __fdiv_rn(1.0f, __fadd_rn(1.0f, host_expf(-acc)));
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < h; i += blockDim.x) out[(size_t)t * h + i] = y[(size_t)t * h + i] * s_gate;
}

void launch_shexp_gate(const float* x, const float* gw, int h, const float* y, float* sg, float* out, int T,
                       cudaStream_t s) {
    shexp_gate_kernel<<<T, 256, 0, s>>>(x, gw, h, y, sg, out);
}

// ------------------------------------------------------------------------------------------
// Q6_K copies with 224-byte superblocks: src holds n_mats matrices of rows x nb superblocks of
// 210 B (src_per bytes apart); dst gets them densely with every superblock padded to 224 B
// (pad bytes zero).  One warp per superblock, u16 copies (GGUF superblocks are 2-aligned).
// ------------------------------------------------------------------------------------------
__global__ void q6_pad_kernel(const uint8_t* __restrict__ src, size_t src_per, int n_mats, int rows, int nb,
                              uint8_t* __restrict__ dst) {
    const int lane = threadIdx.x & 31;
    const long total = (long)n_mats * rows * nb;
    const long nw = ((long)gridDim.x * blockDim.x) >> 5;
    for (long b = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < total; b += nw) {
        const long mat = b / ((long)rows * nb), rem = b % ((long)rows * nb);
        const unsigned short* s16 =
            reinterpret_cast<const unsigned short*>(src + (size_t)mat * src_per + (size_t)rem * kQ6File);
        unsigned short* d16 = reinterpret_cast<unsigned short*>(dst + (size_t)b * kQ6Padded);
        for (int i = lane; i < kQ6Padded / 2; i += 32) d16[i] = i < kQ6File / 2 ? s16[i] : (unsigned short)0;
    }
}

void launch_q6_pad(const uint8_t* src, size_t src_per, int n_mats, int rows, int nb, uint8_t* dst, cudaStream_t s) {
    const long total = (long)n_mats * rows * nb;
    const int grid = (int)std::min<long>(148L * 16, (total + 7) / 8);
    q6_pad_kernel<<<grid > 0 ? grid : 1, 256, 0, s>>>(src, src_per, n_mats, rows, nb, dst);
}

}  // namespace draco
