// Router, top-k selection and expert dispatch (sorting assignments by expert).
//
// Bit-exact with the reference's C routers (src/m6_layer.c:771-796 softmax, :823-866 sigmoid
// with bias and groups, top-k :808-821): logits are sums of individually rounded products in
// index order (the reference's build vectorises the products and adds them one by one), the
// exp is the host C library's (common.cuh), sums run sequentially in expert order, ties go
// to the lower expert index.
#include "kernels.cuh"

namespace draco {

// ------------------------------------------------------------------------------------------
// logits[t][e] = (((x[t][0]*w[e][0]) + x[t][1]*w[e][1]) + ...), every product rounded.
// Tiled like an SGEMM without split-K: each thread owns RT tokens of one expert and walks k
// upward, so every output is the reference's exact sequence of roundings.
// ------------------------------------------------------------------------------------------
template <int TY, int RT>
__global__ void __launch_bounds__(32 * TY) router_logits_kernel(const float* __restrict__ X,
                                                               const float* __restrict__ W, int T,
                                                               int E, int H,
                                                               float* __restrict__ logits) {
    constexpr int KC = 32;
    __shared__ float ws[32][KC + 1];
    __shared__ float xs[TY * RT][KC + 1];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int tid = ty * 32 + tx;
    const int e0 = blockIdx.x * 32;
    const int t0 = blockIdx.y * (TY * RT);
    float acc[RT];
#pragma unroll
    for (int r = 0; r < RT; r++) acc[r] = 0.f;
    for (int k0 = 0; k0 < H; k0 += KC) {
        for (int i = tid; i < 32 * KC; i += 32 * TY) {
            const int ee = i / KC, kk = i % KC;
            const int e = e0 + ee, k = k0 + kk;
            ws[ee][kk] = (e < E && k < H) ? W[(size_t)e * H + k] : 0.f;
        }
        for (int i = tid; i < TY * RT * KC; i += 32 * TY) {
            const int tt = i / KC, kk = i % KC;
            const int t = t0 + tt, k = k0 + kk;
            xs[tt][kk] = (t < T && k < H) ? X[(size_t)t * H + k] : 0.f;
        }
        __syncthreads();
        const int kn = min(KC, H - k0);
        for (int kk = 0; kk < kn; kk++) {
            const float w = ws[tx][kk];
#pragma unroll
            for (int r = 0; r < RT; r++) acc[r] = __fadd_rn(acc[r], __fmul_rn(xs[ty + TY * r][kk], w));
        }
        __syncthreads();
    }
    const int e = e0 + tx;
    if (e < E) {
#pragma unroll
        for (int r = 0; r < RT; r++) {
            const int t = t0 + ty + TY * r;
            if (t < T) logits[(size_t)t * E + e] = acc[r];
        }
    }
}

// Many-warp variant: one output per thread, a 8-token x 32-expert tile per 256-thread block
// (small shared footprint, so several blocks share an SM and hide each other's loads), k-chunks
// of 64 staged in shared memory and read as float4 (4 consecutive k of one row); each thread
// still walks k upward one rounded product at a time.  Rows are padded to 68 floats so the
// expert rows a warp reads at one k fall in distinct bank groups.
__global__ void __launch_bounds__(256) router_logits_v2(const float* __restrict__ X, const float* __restrict__ W,
                                                        int T, int E, int H, float* __restrict__ logits) {
    constexpr int KC = 64, LD = KC + 4, TT = 8, TE = 32;
    constexpr int NV = (TT + TE) * (KC / 4);            // float4 slots per chunk
    constexpr int PER = (NV + 255) / 256;               // per thread
    __shared__ __align__(16) float xs[TT][LD];
    __shared__ __align__(16) float ws[TE][LD];
    const int tid = threadIdx.x, ty = tid >> 5, tx = tid & 31;
    const int t0 = blockIdx.x * TT, e0 = blockIdx.y * TE;
    // the next chunk is fetched into registers while the current one is consumed
    float4 pre[PER];
    auto fetch = [&](int k0) {
        const int kn = min(KC, H - k0);
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int i = tid + 256 * j;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < NV) {
                const int rr = i / (KC / 4), k4 = (i % (KC / 4)) * 4;
                const bool is_x = rr < TT;
                const int row = is_x ? t0 + rr : e0 + rr - TT;
                if ((is_x ? row < T : row < E) && k4 < kn) {
                    const float* src = (is_x ? X : W) + (size_t)row * H + k0 + k4;
                    if (k4 + 4 <= kn) v = *reinterpret_cast<const float4*>(src);
                    else {
                        v.x = src[0];
                        if (k4 + 1 < kn) v.y = src[1];
                        if (k4 + 2 < kn) v.z = src[2];
                    }
                }
            }
            pre[j] = v;
        }
    };
    auto stash = [&]() {
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int i = tid + 256 * j;
            if (i < NV) {
                const int rr = i / (KC / 4), k4 = (i % (KC / 4)) * 4;
                float* dst = rr < TT ? &xs[rr][k4] : &ws[rr - TT][k4];
                *reinterpret_cast<float4*>(dst) = pre[j];
            }
        }
    };
    float acc = 0.f;
    fetch(0);
    for (int k0 = 0; k0 < H; k0 += KC) {
        const int kn = min(KC, H - k0);
        stash();
        __syncthreads();
        if (k0 + KC < H) fetch(k0 + KC);
        const int kq = kn / 4;
        for (int q = 0; q < kq; q++) {
            const float4 xv = *reinterpret_cast<const float4*>(&xs[ty][4 * q]);
            const float4 wv = *reinterpret_cast<const float4*>(&ws[tx][4 * q]);
            acc = __fadd_rn(acc, __fmul_rn(xv.x, wv.x));
            acc = __fadd_rn(acc, __fmul_rn(xv.y, wv.y));
            acc = __fadd_rn(acc, __fmul_rn(xv.z, wv.z));
            acc = __fadd_rn(acc, __fmul_rn(xv.w, wv.w));
        }
        for (int k = 4 * kq; k < kn; k++) acc = __fadd_rn(acc, __fmul_rn(xs[ty][k], ws[tx][k]));
        __syncthreads();
    }
    const int t = t0 + ty, e = e0 + tx;
    if (t < T && e < E) logits[(size_t)t * E + e] = acc;
}

void launch_router_logits(const float* X, const float* W, int T, int E, int H, float* logits,
                          cudaStream_t s) {
    const bool vec_ok = H % 4 == 0 && ((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0;
    if (T <= 4 || !vec_ok) {
        dim3 grid((E + 31) / 32, (T + 3) / 4);
        router_logits_kernel<4, 1><<<grid, dim3(32, 4), 0, s>>>(X, W, T, E, H, logits);
    } else {
        dim3 grid((T + 7) / 8, (E + 31) / 32);
        router_logits_v2<<<grid, 256, 0, s>>>(X, W, T, E, H, logits);
    }
}

// ------------------------------------------------------------------------------------------
// Selection: one warp per token.
// ------------------------------------------------------------------------------------------
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

// strict-greater argmax over unused entries with the reference's -1e30 floor
__device__ int warp_argmax(const float* v, const unsigned char* used, int n, int lane) {
    float bv = -1e30f;
    int bi = -1;
    for (int i = lane; i < n; i += 32)
        if (!used[i] && v[i] > bv) {
            bv = v[i];
            bi = i;
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
    return bi;
}

__global__ void __launch_bounds__(32 * kSelWarps) router_select_kernel(RouterParams p, int T,
                                                                      const float* __restrict__ logits,
                                                                      int* __restrict__ order,
                                                                      float* __restrict__ wtop,
                                                                      int* __restrict__ err) {
    __shared__ float s_p[kSelWarps][kMaxExperts];
    __shared__ float s_sel[kSelWarps][kMaxExperts];
    __shared__ unsigned char s_used[kSelWarps][kMaxExperts];
    __shared__ float s_gs[kSelWarps][kMaxGroups];
    __shared__ unsigned char s_gused[kSelWarps][kMaxGroups];
    __shared__ int s_idx[kSelWarps][kMaxUsed];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kSelWarps + w;
    if (t >= T) return;
    const int E = p.n_exp, K = p.n_used;
    const float* lg = logits + (size_t)t * E;
    float* P = s_p[w];
    float* S = s_sel[w];
    unsigned char* used = s_used[w];
    if (p.scoring == 0) {
        // max-subtracted softmax (src/m6_layer.c:784-789)
        float mx = -1e30f;
        for (int e = lane; e < E; e += 32) {
            const float v = lg[e];
            P[e] = v;
            mx = v > mx ? v : mx;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, mx, o);
            mx = ov > mx ? ov : mx;
        }
        for (int e = lane; e < E; e += 32) P[e] = host_expf(__fsub_rn(P[e], mx));
        __syncwarp();
        float s = 0.f;
        if (lane == 0)
            for (int e = 0; e < E; e++) s = __fadd_rn(s, P[e]);
        s = __shfl_sync(0xffffffffu, s, 0);
        const float inv = __fdiv_rn(1.0f, s);
        for (int e = lane; e < E; e += 32) {
            P[e] = __fmul_rn(P[e], inv);
            S[e] = P[e];
            used[e] = 0;
        }
    } else {
        // sigmoid scores; bias only steers the selection (src/m6_layer.c:833-840)
        for (int e = lane; e < E; e += 32) {
            const float pe = __fdiv_rn(1.0f, __fadd_rn(1.0f, host_expf(-lg[e])));
            P[e] = pe;
            S[e] = __fadd_rn(pe, p.probs_b ? p.probs_b[e] : 0.0f);
            used[e] = 0;
        }
        __syncwarp();
        if (p.n_group > 1) {
            // group score = sum of the group's two largest (src/m6_layer.c:841-859)
            const int per = E / p.n_group;
            for (int g = lane; g < p.n_group; g += 32) {
                float m1 = -1e30f, m2 = -1e30f;
                for (int i = 0; i < per; i++) {
                    const float v = S[g * per + i];
                    if (v > m1) {
                        m2 = m1;
                        m1 = v;
                    } else if (v > m2) {
                        m2 = v;
                    }
                }
                s_gs[w][g] = __fadd_rn(m1, m2);
                s_gused[w][g] = 0;
            }
            __syncwarp();
            for (int j = 0; j < p.n_group_used; j++) {
                const int bg = warp_argmax(s_gs[w], s_gused[w], p.n_group, lane);
                if (bg < 0) {
                    if (lane == 0) atomicOr(err, 1);
                    break;
                }
                if (lane == 0) s_gused[w][bg] = 1;
                __syncwarp();
            }
            __syncwarp();
            for (int e = lane; e < E; e += 32)
                if (!s_gused[w][e / per]) S[e] = -1e30f;
        }
    }
    __syncwarp();
    for (int j = 0; j < K; j++) {
        const int bi = warp_argmax(S, used, E, lane);
        if (lane == 0) {
            s_idx[w][j] = bi;
            if (bi >= 0) used[bi] = 1;
            else atomicOr(err, 2);
        }
        __syncwarp();
    }
    if (lane == 0) {
        float wl[kMaxUsed];
        float s = 0.f;
        for (int j = 0; j < K; j++) {
            const int i = s_idx[w][j];
            wl[j] = i >= 0 ? P[i] : 0.f;
            s = __fadd_rn(s, wl[j]);
        }
        if (p.scoring == 0 || p.norm_w) {
            if (s < 6.103515625e-5f) s = 6.103515625e-5f;
            for (int j = 0; j < K; j++) wl[j] = __fdiv_rn(wl[j], s);
        }
        if (p.scoring != 0 && p.w_scale != 0.f && p.w_scale != 1.f)
            for (int j = 0; j < K; j++) wl[j] = __fmul_rn(wl[j], p.w_scale);
        for (int j = 0; j < K; j++) {
            order[(size_t)t * K + j] = s_idx[w][j];
            wtop[(size_t)t * K + j] = wl[j];
        }
    }
}

void launch_router_select(const RouterParams& p, int T, RouteBufs& b, cudaStream_t s) {
    router_select_kernel<<<(T + kSelWarps - 1) / kSelWarps, 32 * kSelWarps, 0, s>>>(
        p, T, b.logits, b.order, b.wtop, b.err);
}

// ------------------------------------------------------------------------------------------
// Dispatch: stable counting sort of assignments i = t*K + k by expert (the order of
// src/m6_moe_tok.c:53-70), in three passes over chunks of 1024 assignments: per-chunk expert
// counts; per-expert prefix over chunks plus expert offsets; placement, where a chunk's warps
// take turns and each ranks its lanes among equal experts with a match mask, so every
// expert's list is in increasing i.
// ------------------------------------------------------------------------------------------
constexpr int kChunk = 1024;

__global__ void __launch_bounds__(kChunk) dispatch_count_kernel(const int* __restrict__ order, int n, int E,
                                                               int* __restrict__ chunk_counts) {
    __shared__ int sc[kMaxExperts];
    for (int e = threadIdx.x; e < E; e += blockDim.x) sc[e] = 0;
    __syncthreads();
    const int i = blockIdx.x * kChunk + threadIdx.x;
    if (i < n) {
        const int e = order[i];
        if (e >= 0 && e < E) atomicAdd(&sc[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[(size_t)blockIdx.x * E + e] = sc[e];
}

__global__ void __launch_bounds__(kMaxExperts) dispatch_scan_kernel(int* __restrict__ chunk_counts, int n_chunks,
                                                                   int E, int* __restrict__ counts,
                                                                   int* __restrict__ off, int* __restrict__ active,
                                                                   int* __restrict__ n_active) {
    __shared__ int sv[kMaxExperts];
    __shared__ int sa[kMaxExperts];
    const int e = threadIdx.x;
    // per expert: exclusive prefix over chunks (in place), total
    int c = 0;
    if (e < E)
        for (int k = 0; k < n_chunks; k++) {
            const int v = chunk_counts[(size_t)k * E + e];
            chunk_counts[(size_t)k * E + e] = c;
            c += v;
        }
    if (e < E) counts[e] = c;
    sv[e] = c;
    sa[e] = c > 0 ? 1 : 0;
    __syncthreads();
    for (int o = 1; o < kMaxExperts; o <<= 1) {   // inclusive scans over experts
        const int v = e >= o ? sv[e - o] : 0;
        const int a = e >= o ? sa[e - o] : 0;
        __syncthreads();
        sv[e] += v;
        sa[e] += a;
        __syncthreads();
    }
    const int base = sv[e] - c;   // exclusive offset of expert e
    if (e < E) {
        off[e + 1] = sv[e];
        if (c > 0) active[sa[e] - 1] = e;
        for (int k = 0; k < n_chunks; k++) chunk_counts[(size_t)k * E + e] += base;
    }
    if (e == 0) {
        off[0] = 0;
        *n_active = sa[kMaxExperts - 1];
    }
}

__global__ void __launch_bounds__(kChunk) dispatch_place_kernel(const int* __restrict__ order, int n, int E,
                                                               const int* __restrict__ chunk_base,
                                                               int* __restrict__ ilist, int* __restrict__ pos_of) {
    __shared__ int cursor[kMaxExperts];
    for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = chunk_base[(size_t)blockIdx.x * E + e];
    __syncthreads();
    const int i = blockIdx.x * kChunk + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int e = i < n ? order[i] : -1;
    if (e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const bool leader = rank == 0;
    for (int w = 0; w < kChunk / 32; w++) {
        if (warp == w && e >= 0) {
            const int p = cursor[e] + rank;
            ilist[p] = i;
            pos_of[i] = p;
        }
        __syncwarp();
        if (warp == w && e >= 0 && leader) cursor[e] += __popc(peers);
        __syncthreads();
    }
}

void launch_dispatch(int T, int K, int E, RouteBufs& b, cudaStream_t s) {
    const int n = T * K;
    const int n_chunks = max(1, (n + kChunk - 1) / kChunk);
    dispatch_count_kernel<<<n_chunks, kChunk, 0, s>>>(b.order, n, E, b.chunk_counts);
    dispatch_scan_kernel<<<1, kMaxExperts, 0, s>>>(b.chunk_counts, n_chunks, E, b.counts, b.off, b.active,
                                                   b.n_active);
    dispatch_place_kernel<<<n_chunks, kChunk, 0, s>>>(b.order, n, E, b.chunk_counts, b.ilist, b.pos_of);
}

// host expf replica over an array (test hook)
__global__ void expf_kernel(const float* x, float* y, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        y[i] = host_expf(x[i]);
}
void launch_expf(const float* x, float* y, long n, cudaStream_t s) {
    expf_kernel<<<148 * 8, 256, 0, s>>>(x, y, n);
}

}  // namespace draco
