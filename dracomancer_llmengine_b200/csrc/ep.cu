// Expert-parallel token exchange: the per-rank send plan, the row packing and the home-side
// combine.  Experts are split contiguously over G ranks (rank r owns [r*E/G, (r+1)*E/G)); a
// token sends its row once to every rank that owns at least one of its K experts, with its full
// routing row (K global expert ids, K weights) beside it.  The owner computes the weighted sum of
// its own experts for that row; the home rank adds the G partial rows in rank order.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "kernels.cuh"

namespace draco {

namespace {

constexpr int kPlanThreads = 1024;

// inclusive warp scan
__device__ __forceinline__ int warp_incl(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

// bit r set when one of the token's K experts lives on rank r
__device__ __forceinline__ unsigned token_mask(const int* order, int t, int K, int E, int e_loc) {
    unsigned m = 0;
    for (int k = 0; k < K; k++) {
        const int e = order[(size_t)t * K + k];
        if (e >= 0 && e < E) m |= 1u << (e / e_loc);
    }
    return m;
}

// One block.  Thread i owns tokens [i*chunk, (i+1)*chunk); rows are rank-major and, within a
// rank, in token order.  counts[r] = rows for rank r; row_of[t*G + r] = row or -1;
// src_tok[row] = t.  block == 0: rank r's rows follow rank r-1's (compact); block > 0: rank r's
// rows start at r*block (fixed-size blocks, block >= T).  MAXG >= G bounds the per-thread rank
// counters (registers).
template <int MAXG>
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const int* __restrict__ order, int T, int K, int E,
                                                               int G, int block, int* __restrict__ counts,
                                                               int* __restrict__ row_of, int* __restrict__ src_tok) {
    __shared__ int warp_tot[MAXG][kPlanThreads / 32];
    __shared__ int rank_base[MAXG + 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int e_loc = E / G;
    const int chunk = (T + kPlanThreads - 1) / kPlanThreads;
    const int t0 = min(T, tid * chunk), t1 = min(T, t0 + chunk);
    int c[MAXG];
#pragma unroll
    for (int r = 0; r < MAXG; r++) c[r] = 0;
    for (int t = t0; t < t1; t++) {
        const unsigned m = token_mask(order, t, K, E, e_loc);
#pragma unroll
        for (int r = 0; r < MAXG; r++) c[r] += (m >> r) & 1u;
    }
    // exclusive prefix over threads, per rank
    int ex[MAXG];
#pragma unroll
    for (int r = 0; r < MAXG; r++) {
        const int inc = warp_incl(c[r]);
        ex[r] = inc - c[r];
        if (lane == 31) warp_tot[r][warp] = inc;
    }
    __syncthreads();
    if (warp == 0) {
        for (int r = 0; r < G; r++) {
            const int v = warp_tot[r][lane];
            const int inc = warp_incl(v);
            warp_tot[r][lane] = inc - v;   // exclusive over warps
            if (lane == 31) rank_base[r + 1] = inc;   // rank total for now
        }
    }
    __syncthreads();
    if (tid == 0) {
        rank_base[0] = 0;
        for (int r = 0; r < G; r++) {
            const int n = rank_base[r + 1];
            counts[r] = n;
            rank_base[r + 1] = block ? (r + 1) * block : rank_base[r] + n;
        }
    }
    __syncthreads();
    int pos[MAXG];
#pragma unroll
    for (int r = 0; r < MAXG; r++) pos[r] = r < G ? rank_base[r] + warp_tot[r][warp] + ex[r] : 0;
    for (int t = t0; t < t1; t++) {
        const unsigned m = token_mask(order, t, K, E, e_loc);
#pragma unroll
        for (int r = 0; r < MAXG; r++) {
            if (r >= G) break;
            int row = -1;
            if ((m >> r) & 1u) {
                row = pos[r]++;
                src_tok[row] = t;
            }
            row_of[(size_t)t * G + r] = row;
        }
    }
}

// One warp per send row: the token's activations and its routing row (K ids, K weight bits).
// Compact (block == 0): rows [0, min(sum counts, cap)).  Fixed blocks: all G*block rows, the
// unused tail of each block gets routing ids -1 (no expert) and no activations.
__global__ void ep_pack_kernel(const float* __restrict__ X, const int* __restrict__ order,
                               const float* __restrict__ wtop, const int* __restrict__ counts, int G,
                               const int* __restrict__ src_tok, int block, int cap, int K, int H,
                               float* __restrict__ send_x, int* __restrict__ send_meta) {
    int S = 0;
    if (block) {
        S = G * block;
    } else {
        for (int r = 0; r < G; r++) S += counts[r];
    }
    S = min(S, cap);
    const int lane = threadIdx.x & 31;
    const int wpb = blockDim.x >> 5;
    for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < S; row += gridDim.x * wpb) {
        if (block && row % block >= counts[row / block]) {
            for (int k = lane; k < K; k += 32) {
                send_meta[(size_t)row * 2 * K + k] = -1;
                send_meta[(size_t)row * 2 * K + K + k] = 0;
            }
            continue;
        }
        const int t = src_tok[row];
        const float4* src = reinterpret_cast<const float4*>(X + (size_t)t * H);
        float4* dst = reinterpret_cast<float4*>(send_x + (size_t)row * H);
        for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
        for (int k = lane; k < K; k += 32) {
            send_meta[(size_t)row * 2 * K + k] = order[(size_t)t * K + k];
            send_meta[(size_t)row * 2 * K + K + k] = __float_as_int(wtop[(size_t)t * K + k]);
        }
    }
}

// Home-side combine: out[t] = sum over r ascending of back[row_of[t][r]] (+ shared[t]), one
// thread per 4 outputs, all of a thread's (at most MAXG) loads issued before the first add.
template <int MAXG>
__global__ void ep_combine_kernel(const float* __restrict__ back, const int* __restrict__ row_of, int T, int G,
                                  int H, const float* __restrict__ shared, float* __restrict__ out) {
    const int H4 = H / 4;
    const size_t n = (size_t)T * H4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / H4), c = (int)(i % H4);
        float4 v[MAXG];
        bool has[MAXG];
#pragma unroll
        for (int r = 0; r < MAXG; r++) {
            const int row = r < G ? __ldg(row_of + (size_t)t * G + r) : -1;
            has[r] = row >= 0;
            if (has[r]) v[r] = reinterpret_cast<const float4*>(back + (size_t)row * H)[c];
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < MAXG; r++) {
            if (!has[r]) continue;
            acc.x = __fadd_rn(acc.x, v[r].x);
            acc.y = __fadd_rn(acc.y, v[r].y);
            acc.z = __fadd_rn(acc.z, v[r].z);
            acc.w = __fadd_rn(acc.w, v[r].w);
        }
        if (shared) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(shared + (size_t)t * H) + c);
            acc.x = __fadd_rn(acc.x, u.x);
            acc.y = __fadd_rn(acc.y, u.y);
            acc.z = __fadd_rn(acc.z, u.z);
            acc.w = __fadd_rn(acc.w, u.w);
        }
        reinterpret_cast<float4*>(out + (size_t)t * H)[c] = acc;
    }
}

// given routing into the layer's buffers: strided rows, expert ids shifted to the local range
// (may run in place: each element is read and written by the same thread)
__global__ void route_in_kernel(const int* order, const float* wtop, int ld, int e_base, int T, int K, int* o_order,
                                float* o_wtop) {
    const int n = T * K;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int t = i / K, k = i % K;
        const int e = order[(size_t)t * ld + k];
        const float w = wtop[(size_t)t * ld + k];
        o_order[i] = e < 0 ? -1 : e - e_base;
        o_wtop[i] = w;
    }
}

// ---- peer-memory exchange (CUDA IPC mappings of the other ranks' buffers, plain loads/stores) ----

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Dispatch by stores into the owners' receive buffers: the row for (token t, rank d) goes to
// row rank*block + j of rank d's buffer (j = its place among the rows this rank sends to d), and
// the unused rows of that block get routing ids -1.  Every thread fences its stores at system
// scope before the kernel ends, so the barrier that follows publishes them.
__global__ void ep_push_kernel(const float* __restrict__ X, const int* __restrict__ order,
                               const float* __restrict__ wtop, const int* __restrict__ counts, int G, int rank,
                               const int* __restrict__ src_tok, int block, int K, int H, void* const* dst_x,
                               int x16, int* const* dst_meta) {
    const int lane = threadIdx.x & 31;
    const int wpb = blockDim.x >> 5;
    const int S = G * block;
    for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < S; row += gridDim.x * wpb) {
        const int d = row / block, j = row - d * block;
        const size_t drow = (size_t)rank * block + j;
        int* meta = dst_meta[d] + drow * 2 * K;
        if (j >= counts[d]) {
            for (int k = lane; k < K; k += 32) {
                meta[k] = -1;
                meta[K + k] = 0;
            }
            continue;
        }
        const int t = src_tok[row];
        const float4* src = reinterpret_cast<const float4*>(X + (size_t)t * H);
        if (x16) {   // fp16 rows: half the bytes over the links; the owner's GEMM rounds to fp16 anyway
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(dst_x[d]) + drow * H);
            for (int i = lane; i < H / 8; i += 32) {
                const float4 a = src[2 * i], b = src[2 * i + 1];
                const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
                const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
                uint4 o;
                o.x = *reinterpret_cast<const uint32_t*>(&h0);
                o.y = *reinterpret_cast<const uint32_t*>(&h1);
                o.z = *reinterpret_cast<const uint32_t*>(&h2);
                o.w = *reinterpret_cast<const uint32_t*>(&h3);
                dst[i] = o;
            }
        } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(dst_x[d]) + drow * H);
            for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
        }
        for (int k = lane; k < K; k += 32) {
            meta[k] = order[(size_t)t * K + k];
            meta[K + k] = __float_as_int(wtop[(size_t)t * K + k]);
        }
    }
    __threadfence_system();
}

// All ranks meet: rank r's flag word `rank` is set to this barrier's epoch in every peer's flag
// array (release, system scope), then each rank waits until all G words of its own array reach
// the epoch (acquire).  The epoch counter lives in device memory, so a captured graph replays
// correctly.  The wait gives up after kWaitNs and sets 0x400 in *status.
constexpr uint64_t kWaitNs = 2000000000ull;
__global__ void ep_barrier_kernel(unsigned* const* peer_flags, unsigned* my_flags, unsigned* epoch_ctr, int G,
                                  int rank, int* status) {
    __shared__ unsigned e;
    if (threadIdx.x == 0) {
        e = *epoch_ctr + 1;
        *epoch_ctr = e;
    }
    __syncthreads();
    __threadfence_system();
    const int r = threadIdx.x;
    if (r < G) {
        st_release_sys(peer_flags[r] + rank, e);
        const uint64_t t0 = global_ns();
        for (unsigned i = 0; ld_acquire_sys(my_flags + r) - e > 0x7fffffffu; i++) {   // flag < e (wrapping)
            if ((i & 255) == 255 && global_ns() - t0 > kWaitNs) {
                atomicOr(status, 0x400);
                break;
            }
        }
    }
    __syncthreads();
}

// Combine by loads from the owners' partial buffers: out[t] = sum over r ascending of
// partial_r[rank*block + j_r(t)] (+ shared[t]), j_r(t) = row_of[t][r] - r*block.  One thread per
// 4 outputs; all of a thread's (at most MAXG) loads are issued before the first add.
template <int MAXG>
__global__ void ep_pull_combine_kernel(const float* const* src_partial, const int* __restrict__ row_of, int T,
                                       int G, int rank, int block, int H, const float* __restrict__ shared,
                                       float* __restrict__ out) {
    const int H4 = H / 4;
    const size_t n = (size_t)T * H4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / H4), c = (int)(i % H4);
        float4 v[MAXG];
        bool has[MAXG];
#pragma unroll
        for (int r = 0; r < MAXG; r++) {
            const int row = r < G ? __ldg(row_of + (size_t)t * G + r) : -1;
            has[r] = row >= 0;
            if (has[r]) {
                const size_t srow = (size_t)rank * block + (row - r * block);
                v[r] = reinterpret_cast<const float4*>(src_partial[r] + srow * H)[c];
            }
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < MAXG; r++) {
            if (!has[r]) continue;
            acc.x = __fadd_rn(acc.x, v[r].x);
            acc.y = __fadd_rn(acc.y, v[r].y);
            acc.z = __fadd_rn(acc.z, v[r].z);
            acc.w = __fadd_rn(acc.w, v[r].w);
        }
        if (shared) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(shared + (size_t)t * H) + c);
            acc.x = __fadd_rn(acc.x, u.x);
            acc.y = __fadd_rn(acc.y, u.y);
            acc.z = __fadd_rn(acc.z, u.z);
            acc.w = __fadd_rn(acc.w, u.w);
        }
        reinterpret_cast<float4*>(out + (size_t)t * H)[c] = acc;
    }
}

}  // namespace

void launch_ep_push(const float* X, const int* order, const float* wtop, const int* counts, int G, int rank,
                    const int* src_tok, int block, int K, int H, void* const* dst_x, int x16, int* const* dst_meta,
                    cudaStream_t s) {
    const int rows = G * block;
    const int blocks = std::max(1, std::min(148 * 4, (rows + 7) / 8));
    ep_push_kernel<<<blocks, 256, 0, s>>>(X, order, wtop, counts, G, rank, src_tok, block, K, H, dst_x, x16,
                                          dst_meta);
}

void launch_ep_barrier(unsigned* const* peer_flags, unsigned* my_flags, unsigned* epoch_ctr, int G, int rank,
                       int* status, cudaStream_t s) {
    ep_barrier_kernel<<<1, 32, 0, s>>>(peer_flags, my_flags, epoch_ctr, G, rank, status);
}

void launch_ep_pull_combine(const float* const* src_partial, const int* row_of, int T, int G, int rank, int block,
                            int H, const float* shared, float* out, cudaStream_t s) {
    const size_t n = (size_t)T * (H / 4);
    const int blocks = (int)std::max<size_t>(1, std::min<size_t>(148 * 8, (n + 255) / 256));
    if (G <= 2)
        ep_pull_combine_kernel<2><<<blocks, 256, 0, s>>>(src_partial, row_of, T, G, rank, block, H, shared, out);
    else if (G <= 4)
        ep_pull_combine_kernel<4><<<blocks, 256, 0, s>>>(src_partial, row_of, T, G, rank, block, H, shared, out);
    else if (G <= 8)
        ep_pull_combine_kernel<8><<<blocks, 256, 0, s>>>(src_partial, row_of, T, G, rank, block, H, shared, out);
    else
        ep_pull_combine_kernel<kEpMaxRanks><<<blocks, 256, 0, s>>>(src_partial, row_of, T, G, rank, block, H, shared,
                                                                  out);
}

void launch_ep_plan(const int* order, int T, int K, int E, int G, int block, int* counts, int* row_of,
                    int* src_tok, cudaStream_t s) {
    if (G <= 2)
        ep_plan_kernel<2><<<1, kPlanThreads, 0, s>>>(order, T, K, E, G, block, counts, row_of, src_tok);
    else if (G <= 4)
        ep_plan_kernel<4><<<1, kPlanThreads, 0, s>>>(order, T, K, E, G, block, counts, row_of, src_tok);
    else if (G <= 8)
        ep_plan_kernel<8><<<1, kPlanThreads, 0, s>>>(order, T, K, E, G, block, counts, row_of, src_tok);
    else
        ep_plan_kernel<kEpMaxRanks><<<1, kPlanThreads, 0, s>>>(order, T, K, E, G, block, counts, row_of, src_tok);
}

void launch_ep_pack(const float* X, const int* order, const float* wtop, const int* counts, int G, const int* src_tok,
                    int block, int cap, int K, int H, float* send_x, int* send_meta, cudaStream_t s) {
    const int blocks = std::max(1, std::min(148 * 4, (cap + 7) / 8));
    ep_pack_kernel<<<blocks, 256, 0, s>>>(X, order, wtop, counts, G, src_tok, block, cap, K, H, send_x, send_meta);
}

void launch_ep_combine(const float* back, const int* row_of, int T, int G, int H, const float* shared, float* out,
                       cudaStream_t s) {
    const size_t n = (size_t)T * (H / 4);
    const int blocks = (int)std::max<size_t>(1, std::min<size_t>(148 * 8, (n + 255) / 256));
    if (G <= 2)
        ep_combine_kernel<2><<<blocks, 256, 0, s>>>(back, row_of, T, G, H, shared, out);
    else if (G <= 4)
        ep_combine_kernel<4><<<blocks, 256, 0, s>>>(back, row_of, T, G, H, shared, out);
    else if (G <= 8)
        ep_combine_kernel<8><<<blocks, 256, 0, s>>>(back, row_of, T, G, H, shared, out);
    else
        ep_combine_kernel<kEpMaxRanks><<<blocks, 256, 0, s>>>(back, row_of, T, G, H, shared, out);
}

void launch_route_in(const int* order, const float* wtop, int ld, int e_base, int T, int K, int* o_order,
                     float* o_wtop, cudaStream_t s) {
    const int n = T * K;
    const int blocks = std::max(1, std::min(148 * 4, (n + 255) / 256));
    route_in_kernel<<<blocks, 256, 0, s>>>(order, wtop, ld, e_base, T, K, o_order, o_wtop);
}

}  // namespace draco
