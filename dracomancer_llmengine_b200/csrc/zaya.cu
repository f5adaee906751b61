// Router MLP of the top-1 MoE op with a learned router (m6_zaya_moe_op, src/m6_engine.c:795-835):
//   rh  = W_down . x + b_down (+ rh_state * eda_scale); rh_state <- rh
//   t1  = rms_norm(rh) * rnorm                     (eps 1e-5, src/m6_engine.c:31-37)
//   rh  = gelu_erf(W_fc1 . t1 + b_fc1); t1 = gelu_erf(W_fc2 . rh + b_fc2)
//   lg  = W_out . t1; p = softmax(lg); best = argmax(p + bal) (first index among equals)
//   routing of the one token: expert `best` with weight p[best], or none when best >= n_exp
//   or best == iskip (the layer output is then zero)
// The router matrices are F32 (code 9) or F16 (code 7) rows.  The expert GEMVs run on the
// library's grouped kernels with this routing.
#include "kernels.cuh"

namespace draco {
namespace {

__device__ __forceinline__ float row_dot(int code, const void* W, int r, int n, const float* x, int lane) {
    float acc = 0.f;
    if (code == 9) {
        const float* w = reinterpret_cast<const float*>(W) + (size_t)r * n;
        for (int i = lane; i < n; i += 32) acc = fmaf(w[i], x[i], acc);
    } else {
        const __half* w = reinterpret_cast<const __half*>(W) + (size_t)r * n;
        for (int i = lane; i < n; i += 32) acc = fmaf(__half2float(w[i]), x[i], acc);
    }
    return warp_sum(acc);
}

__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

// rh[r] for r < RH: one warp per row
__global__ void zaya_down_kernel(ZayaRouterArgs a) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= a.RH) return;
    float v = row_dot(a.cdown, a.wdown, warp, a.H, a.x, lane) + a.bdown[warp];
    if (a.eda_scale) v = fmaf(a.state_in[warp], a.eda_scale[warp], v);
    if (lane == 0) {
        a.rh[warp] = v;
        a.state_out[warp] = v;
    }
}

// the rest of the router, one block
__global__ void zaya_mlp_kernel(ZayaRouterArgs a) {
    extern __shared__ float sm[];
    float* t1 = sm;              // [RH]
    float* t2 = t1 + a.RH;       // [RH]
    float* lg = t2 + a.RH;       // [nclass]
    __shared__ float red[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float ss = 0.f;
    for (int i = tid; i < a.RH; i += blockDim.x) {
        const float v = a.rh[i];
        t2[i] = v;
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float s = 0.f;
        for (int w = 0; w < nw; w++) s += red[w];
        red[0] = 1.f / sqrtf(s / (float)a.RH + 1e-5f);
    }
    __syncthreads();
    const float inv = red[0];
    for (int i = tid; i < a.RH; i += blockDim.x) t1[i] = t2[i] * inv * a.rnorm[i];
    __syncthreads();
    for (int r = warp; r < a.RH; r += nw) {
        const float v = row_dot(a.cfc1, a.wfc1, r, a.RH, t1, lane);
        if (lane == 0) t2[r] = gelu_erf(v + a.bfc1[r]);
    }
    __syncthreads();
    for (int r = warp; r < a.RH; r += nw) {
        const float v = row_dot(a.cfc2, a.wfc2, r, a.RH, t2, lane);
        if (lane == 0) t1[r] = gelu_erf(v + a.bfc2[r]);
    }
    __syncthreads();
    for (int r = warp; r < a.nclass; r += nw) {
        const float v = row_dot(a.cout, a.wout, r, a.RH, t1, lane);
        if (lane == 0) lg[r] = v;
    }
    __syncthreads();
    if (tid == 0) {
        float mx = -1e30f;
        for (int i = 0; i < a.nclass; i++) mx = lg[i] > mx ? lg[i] : mx;
        float sum = 0.f;
        for (int i = 0; i < a.nclass; i++) {
            lg[i] = host_expf(lg[i] - mx);
            sum += lg[i];
        }
        const float invs = 1.f / sum;
        int best = 0;
        float bv = -1e30f;
        for (int i = 0; i < a.nclass; i++) {
            const float v = lg[i] * invs + a.bal[i];
            if (v > bv) {
                bv = v;
                best = i;
            }
        }
        const bool skip = best >= a.nexp || best == a.iskip;
        a.order[0] = skip ? -1 : best;
        a.wtop[0] = lg[best] * invs;
    }
}

}  // namespace

int launch_zaya_router(const ZayaRouterArgs& a, cudaStream_t s) {
    if (a.RH <= 0 || a.RH > 4096 || a.nclass <= 0 || a.nclass > 1024) return -1;
    const int threads = 256;
    const int blocks = (a.RH * 32 + threads - 1) / threads;
    zaya_down_kernel<<<blocks, threads, 0, s>>>(a);
    const size_t smem = sizeof(float) * (2 * (size_t)a.RH + a.nclass);
    zaya_mlp_kernel<<<1, 512, smem, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace draco
