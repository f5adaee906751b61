// Router, top-k selection and expert dispatch (sorting assignments by expert).
//
// Bit-exact with the reference's C routers (src/m6_layer.c:771-796 softmax, :823-866 sigmoid
// with bias and groups, top-k :808-821): logits are sums of individually rounded products in
// index order (the reference's build vectorises the products and adds them one by one), the
// exp is the host C library's (common.cuh), sums run sequentially in expert order, ties go
// to the lower expert index.
#include "kernels.cuh"
#include "select.cuh"

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
                                                               float* __restrict__ logits,
                                                               int* __restrict__ zero_err) {
    if (zero_err && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && threadIdx.y == 0) *zero_err = 0;
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

// Tiled variant: an 8-token x 32-expert block of 4 warps; warp w owns experts 8w..8w+7 and
// lane l the token l & 7 with the expert pair 2 (l >> 3), +1, so one float4 of a token row
// serves two dot products and shared-memory reads stay near one wavefront per operand row
// group.  k-chunks of 128 stream into a 3-stage shared-memory ring with cp.async (two chunks in
// flight while one is consumed), read as float4 (4 consecutive k of one row) with the next
// float4s fetched ahead; each dot product still walks k upward one rounded product at a time.
// Rows are padded to 132 floats so the rows a warp reads at one k fall in distinct bank
// groups.  Needs H % 4 == 0 and 16-byte aligned X and W.
namespace rl {
constexpr int KC = 128, LD = KC + 4, TT = 8;
// NW warps per block cover TE = 8 NW experts
template <int NW>
struct Shape {
    static constexpr int TE = 8 * NW, NTH = 32 * NW;
    static constexpr int NV = (TT + TE) * (KC / 4);   // 16-byte copies per chunk
    static constexpr int PER = NV / NTH;
    static_assert(NV % NTH == 0, "copies per thread");
};
// ring depth: 3 chunks when each chunk carries enough work (many tokens), 8 for decode-sized
// batches, where a chunk is only ~512 cycles of add chain against ~2 us of cold HBM latency
template <int NS, int NW>
constexpr int smem_bytes() {
    return NS * (TT + Shape<NW>::TE) * LD * 4;
}
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(src_bytes)
                 : "memory");
}
template <int NS, int NW>
__global__ void __launch_bounds__(32 * NW) router_logits_v2(const float* __restrict__ X, const float* __restrict__ W,
                                                            int T, int E, int H, float* __restrict__ logits,
                                                            int* __restrict__ zero_err) {
    using namespace rl;
    constexpr int TE = Shape<NW>::TE, NTH = Shape<NW>::NTH, PER = Shape<NW>::PER;
    if (zero_err && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *zero_err = 0;
    extern __shared__ __align__(16) float rl_smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ti = lane & 7, ep = 8 * warp + 2 * (lane >> 3);   // token row, first expert row (tile-relative)
    const int t0 = blockIdx.x * TT, e0 = blockIdx.y * TE;
    const int nc = (H + KC - 1) / KC;
    // this thread's copies: chunk-relative source rows and stage offsets, fixed for all chunks
    const float* src[PER];
    int dst[PER];
    bool valid[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int i = tid + NTH * j;
        const int rr = i / (KC / 4), k4 = (i % (KC / 4)) * 4;
        const bool is_x = rr < TT;
        const int row = is_x ? t0 + rr : e0 + rr - TT;
        valid[j] = is_x ? row < T : row < E;
        src[j] = valid[j] ? (is_x ? X : W) + (size_t)row * H + k4 : X;
        dst[j] = rr * LD + k4;
    }
    auto issue = [&](int c) {
        if (c < nc) {
            float* st = rl_smem + (c % NS) * (TT + TE) * LD;
            const int k0 = c * KC;
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const bool in = valid[j] && k0 + dst[j] % LD < H;
                cp_async16(st + dst[j], in ? src[j] + k0 : X, in ? 16 : 0);   // zero-fill outside
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
#pragma unroll
    for (int c = 0; c < NS - 1; c++) issue(c);
    float a0 = 0.f, a1 = 0.f;
    for (int c = 0; c < nc; c++) {
        issue(c + NS - 1);
        asm volatile("cp.async.wait_group %0;" ::"n"(NS - 1) : "memory");
        __syncthreads();
        const float* st = rl_smem + (c % NS) * (TT + TE) * LD;
        const float4* xr = reinterpret_cast<const float4*>(st + ti * LD);
        const float4* w0r = reinterpret_cast<const float4*>(st + (TT + ep) * LD);
        const float4* w1r = reinterpret_cast<const float4*>(st + (TT + ep + 1) * LD);
        const int kq = min(KC, H - c * KC) / 4;   // H is a multiple of 4
        auto step = [&](const float4& xv, const float4& u, const float4& v) {
            a0 = __fadd_rn(a0, __fmul_rn(xv.x, u.x));
            a1 = __fadd_rn(a1, __fmul_rn(xv.x, v.x));
            a0 = __fadd_rn(a0, __fmul_rn(xv.y, u.y));
            a1 = __fadd_rn(a1, __fmul_rn(xv.y, v.y));
            a0 = __fadd_rn(a0, __fmul_rn(xv.z, u.z));
            a1 = __fadd_rn(a1, __fmul_rn(xv.z, v.z));
            a0 = __fadd_rn(a0, __fmul_rn(xv.w, u.w));
            a1 = __fadd_rn(a1, __fmul_rn(xv.w, v.w));
        };
        if (kq == KC / 4) {
            // full chunk, fully unrolled, loads issued two steps ahead of the two add chains
            float4 x0 = xr[0], u0 = w0r[0], v0 = w1r[0];
            float4 x1 = xr[1], u1 = w0r[1], v1 = w1r[1];
#pragma unroll
            for (int q = 0; q < KC / 4; q += 2) {
                float4 x2 = x0, u2 = u0, v2 = v0, x3 = x1, u3 = u1, v3 = v1;
                if (q + 2 < KC / 4) {
                    x2 = xr[q + 2];
                    u2 = w0r[q + 2];
                    v2 = w1r[q + 2];
                    x3 = xr[q + 3];
                    u3 = w0r[q + 3];
                    v3 = w1r[q + 3];
                }
                step(x0, u0, v0);
                step(x1, u1, v1);
                x0 = x2;
                u0 = u2;
                v0 = v2;
                x1 = x3;
                u1 = u3;
                v1 = v3;
            }
        } else {
            for (int q = 0; q < kq; q++) step(xr[q], w0r[q], w1r[q]);
        }
        __syncthreads();   // stage c % NS is refilled by the next iteration's issue(c + NS)
    }
    const int t = t0 + ti, e = e0 + ep;
    if (t < T) {
        if (e < E) logits[(size_t)t * E + e] = a0;
        if (e + 1 < E) logits[(size_t)t * E + e + 1] = a1;
    }
}

// Register-tiled variant: a block of NW warps shares one tile of TE = 32*EPL experts; warp w owns
// TPW token rows (read as warp-wide broadcasts of 4 consecutive k) and lane l the experts
// l + 32 j (rows 68 floats apart, so one 128-bit read per expert is conflict-free).  Per 4 k a
// lane reads TPW + EPL float4 and updates TPW*EPL chains, each still one rounded product and
// one rounded add per k in ascending order.  k-chunks of 64 stream into an NS-stage cp.async
// ring.  Needs H % 4 == 0 and 16-byte aligned X and W.
namespace rt {
constexpr int KC = 64, LD = KC + 4;
template <int TPW, int EPL, int NW, int NS>
constexpr int smem_bytes() {
    return NS * (TPW * NW + 32 * EPL) * LD * 4;
}
}  // namespace rt
template <int TPW, int EPL, int NW, int NS>
__global__ void __launch_bounds__(32 * NW) router_tile_kernel(const float* __restrict__ X, const float* __restrict__ W,
                                                              int T, int E, int H, float* __restrict__ logits,
                                                              int* __restrict__ zero_err) {
    using namespace rt;
    constexpr int TT = TPW * NW, TE = 32 * EPL, NTH = 32 * NW, ROWS = TT + TE, NV = ROWS * (KC / 4);
    extern __shared__ __align__(16) float rt_smem[];
    if (zero_err && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *zero_err = 0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * TT, e0 = blockIdx.y * TE;
    const int nc = (H + KC - 1) / KC;
    auto issue = [&](int c) {
        if (c < nc) {
            float* st = rt_smem + (c % NS) * ROWS * LD;
            const int k0 = c * KC;
            for (int i = tid; i < NV; i += NTH) {
                const int rr = i / (KC / 4), k4 = (i % (KC / 4)) * 4;
                const bool is_x = rr < TT;
                const int row = is_x ? t0 + rr : e0 + rr - TT;
                const bool in = (is_x ? row < T : row < E) && k0 + k4 < H;
                const float* src = in ? (is_x ? X : W) + (size_t)row * H + k0 + k4 : X;
                cp_async16(st + rr * LD + k4, src, in ? 16 : 0);   // zero-fill outside
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
#pragma unroll
    for (int c = 0; c < NS - 1; c++) issue(c);
    float acc[TPW][EPL];
#pragma unroll
    for (int i = 0; i < TPW; i++)
#pragma unroll
        for (int j = 0; j < EPL; j++) acc[i][j] = 0.f;
    auto step = [&](const float4 (&xv)[TPW], const float4 (&wv)[EPL]) {
#pragma unroll
        for (int i = 0; i < TPW; i++)
#pragma unroll
            for (int j = 0; j < EPL; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xv[i].x, wv[j].x));
#pragma unroll
        for (int i = 0; i < TPW; i++)
#pragma unroll
            for (int j = 0; j < EPL; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xv[i].y, wv[j].y));
#pragma unroll
        for (int i = 0; i < TPW; i++)
#pragma unroll
            for (int j = 0; j < EPL; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xv[i].z, wv[j].z));
#pragma unroll
        for (int i = 0; i < TPW; i++)
#pragma unroll
            for (int j = 0; j < EPL; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xv[i].w, wv[j].w));
    };
    for (int c = 0; c < nc; c++) {
        issue(c + NS - 1);
        asm volatile("cp.async.wait_group %0;" ::"n"(NS - 1) : "memory");
        __syncthreads();
        const float* st = rt_smem + (c % NS) * ROWS * LD;
        const float4* xr = reinterpret_cast<const float4*>(st + warp * TPW * LD);
        const float4* wr = reinterpret_cast<const float4*>(st + (TT + lane) * LD);
        const int kq = min(KC, H - c * KC) / 4;   // H is a multiple of 4
        auto load = [&](int q, float4 (&xv)[TPW], float4 (&wv)[EPL]) {
#pragma unroll
            for (int j = 0; j < EPL; j++) wv[j] = wr[j * 32 * (LD / 4) + q];
#pragma unroll
            for (int i = 0; i < TPW; i++) xv[i] = xr[i * (LD / 4) + q];
        };
        if (kq == KC / 4) {
            float4 xa[TPW], wa[EPL], xb[TPW], wb[EPL];
            load(0, xa, wa);
#pragma unroll
            for (int q = 0; q < KC / 4; q += 2) {
                load(q + 1, xb, wb);
                step(xa, wa);
                if (q + 2 < KC / 4) load(q + 2, xa, wa);
                step(xb, wb);
            }
        } else {
            for (int q = 0; q < kq; q++) {
                float4 xa[TPW], wa[EPL];
                load(q, xa, wa);
                step(xa, wa);
            }
        }
        __syncthreads();   // stage c % NS is refilled by the next iteration's issue(c + NS)
    }
#pragma unroll
    for (int i = 0; i < TPW; i++) {
        const int t = t0 + warp * TPW + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < EPL; j++) {
            const int e = e0 + lane + 32 * j;
            if (e < E) logits[(size_t)t * E + e] = acc[i][j];
        }
    }
}

template <int TPW, int EPL, int NW, int NS>
static void launch_router_tile(const float* X, const float* W, int T, int E, int H, float* logits, cudaStream_t s,
                               int* zero_err) {
    constexpr int sm = rt::smem_bytes<TPW, EPL, NW, NS>();
    cudaFuncSetAttribute(router_tile_kernel<TPW, EPL, NW, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    dim3 grid((T + TPW * NW - 1) / (TPW * NW), (E + 32 * EPL - 1) / (32 * EPL));
    router_tile_kernel<TPW, EPL, NW, NS><<<grid, 32 * NW, sm, s>>>(X, W, T, E, H, logits, zero_err);
}

static int router_tiles(int T, int E, int tt, int te) { return ((T + tt - 1) / tt) * ((E + te - 1) / te); }

void launch_router_logits(const float* X, const float* W, int T, int E, int H, float* logits,
                          cudaStream_t s, int* zero_err) {
    const bool vec_ok = H % 4 == 0 && ((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0;
    if (vec_ok) {
        if (router_tiles(T, E, 40, 64) >= 148) {   // enough 40..64 x 64 tiles for every SM: 10-16 chains a lane
            // token rows per warp (8 warps a block): the one that minimises the busiest SM's
            // work, (blocks on that SM) x (rows per warp); the full 8-row tiles of cfg4 (256 blocks
            // on 148 SMs) left 40 SMs with one block while the others ran two
            int best = 8;
            long best_cost = -1;
            for (int tpw = 8; tpw >= 5; tpw--) {
                const long blocks = (long)((T + 8 * tpw - 1) / (8 * tpw)) * ((E + 63) / 64);
                const long cost = (blocks + 147) / 148 * tpw;
                if (best_cost < 0 || cost < best_cost) {
                    best_cost = cost;
                    best = tpw;
                }
            }
            switch (best) {
                case 5: launch_router_tile<5, 2, 8, 3>(X, W, T, E, H, logits, s, zero_err); break;
                case 6: launch_router_tile<6, 2, 8, 3>(X, W, T, E, H, logits, s, zero_err); break;
                case 7: launch_router_tile<7, 2, 8, 3>(X, W, T, E, H, logits, s, zero_err); break;
                default: launch_router_tile<8, 2, 8, 3>(X, W, T, E, H, logits, s, zero_err); break;
            }
            return;
        }
        if (T <= 16) {
            dim3 grid((T + 7) / 8, (E + 31) / 32);
            constexpr int sm = rl::smem_bytes<8, 4>();
            cudaFuncSetAttribute(router_logits_v2<8, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
            router_logits_v2<8, 4><<<grid, 128, sm, s>>>(X, W, T, E, H, logits, zero_err);
        } else {
            // 8 tokens x 16 experts a block: twice the blocks of 32-expert tiles, so mid-sized
            // batches (a few hundred tokens) put more warps on each SM
            dim3 grid((T + 7) / 8, (E + 15) / 16);
            constexpr int sm = rl::smem_bytes<3, 2>();
            cudaFuncSetAttribute(router_logits_v2<3, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
            router_logits_v2<3, 2><<<grid, 64, sm, s>>>(X, W, T, E, H, logits, zero_err);
        }
        return;
    }
    dim3 grid((E + 31) / 32, (T + 3) / 4);
    router_logits_kernel<4, 1><<<grid, dim3(32, 4), 0, s>>>(X, W, T, E, H, logits, zero_err);
}

// ------------------------------------------------------------------------------------------
// Selection: one warp per token.
// ------------------------------------------------------------------------------------------
template <int NS>
__global__ void __launch_bounds__(32 * kSelWarps) router_select_kernel(RouterParams p, int T,
                                                                      const float* __restrict__ logits,
                                                                      int* __restrict__ order,
                                                                      float* __restrict__ wtop,
                                                                      int* __restrict__ err) {
    __shared__ __align__(16) float s_v[kSelWarps][kMaxExperts];
    __shared__ float s_gs[kSelWarps][kMaxGroups];
    const int w = threadIdx.x >> 5;
    const int t = blockIdx.x * kSelWarps + w;
    if (t >= T) return;
    select_token<NS>(p, logits + (size_t)t * p.n_exp, order + (size_t)t * p.n_used, wtop + (size_t)t * p.n_used, err,
                     s_v[w], s_gs[w]);
}

void launch_router_select(const RouterParams& p, int T, RouteBufs& b, cudaStream_t s) {
    const int grid = (T + kSelWarps - 1) / kSelWarps, nth = 32 * kSelWarps;
    const int ns = (p.n_exp + 31) / 32;
    if (ns <= 1) router_select_kernel<1><<<grid, nth, 0, s>>>(p, T, b.logits, b.order, b.wtop, b.err);
    else if (ns <= 2) router_select_kernel<2><<<grid, nth, 0, s>>>(p, T, b.logits, b.order, b.wtop, b.err);
    else if (ns <= 4) router_select_kernel<4><<<grid, nth, 0, s>>>(p, T, b.logits, b.order, b.wtop, b.err);
    else if (ns <= 8) router_select_kernel<8><<<grid, nth, 0, s>>>(p, T, b.logits, b.order, b.wtop, b.err);
    else router_select_kernel<16><<<grid, nth, 0, s>>>(p, T, b.logits, b.order, b.wtop, b.err);
}

// ------------------------------------------------------------------------------------------
// Dispatch: counting sort of assignments i = t*K + k by expert (the grouping of
// src/m6_moe_tok.c:53-70), in three passes over chunks of 1024 assignments: per-chunk expert
// counts; per-expert prefix over chunks plus expert offsets; placement by warp-aggregated
// shared-memory atomics.  Chunks keep increasing i from one to the next; inside a chunk the
// slot order of one expert's assignments follows the atomics, which no result depends on
// (every later step works per slot and each output row reads its own slots).
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
                                                                   int* __restrict__ n_active, ItemLists il) {
    __shared__ int sv[kMaxExperts];
    __shared__ int sa[kMaxExperts];
    __shared__ int st[kMaxExperts];
    const int e = threadIdx.x;
    // per expert: exclusive prefix over chunks (in place), total
    int c = 0;
    if (e < E) {   // eight independent loads in flight, then the in-place exclusive prefix
        int k = 0;
        for (; k + 8 <= n_chunks; k += 8) {
            int v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = chunk_counts[(size_t)(k + u) * E + e];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                chunk_counts[(size_t)(k + u) * E + e] = c;
                c += v[u];
            }
        }
        for (; k < n_chunks; k++) {
            const int v = chunk_counts[(size_t)k * E + e];
            chunk_counts[(size_t)k * E + e] = c;
            c += v;
        }
    }
    if (e < E) counts[e] = c;
    const int tiles = (c + il.nt - 1) / il.nt;
    sv[e] = c;
    sa[e] = c > 0 ? 1 : 0;
    st[e] = tiles;
    __syncthreads();
    for (int o = 1; o < kMaxExperts; o <<= 1) {   // inclusive scans over experts
        const int v = e >= o ? sv[e - o] : 0;
        const int a = e >= o ? sa[e - o] : 0;
        const int u = e >= o ? st[e - o] : 0;
        __syncthreads();
        sv[e] += v;
        sa[e] += a;
        st[e] += u;
        __syncthreads();
    }
    if (e < E) {
        off[e + 1] = sv[e];
        if (c > 0) active[sa[e] - 1] = e;
    }
    // (the place kernel adds off[e] to the per-chunk prefix left in chunk_counts)
    if (e == 0) {
        off[0] = 0;
        *n_active = sa[kMaxExperts - 1];
    }
    if (e == 0 && il.zero) *il.zero = 0;
    if (!il.gu) return;
    // tensor-core items, one per (token tile, row tile): tile j belongs to the expert whose
    // inclusive tile prefix first exceeds j
    const int n_tiles = st[kMaxExperts - 1];
    if (e == 0) {
        *il.n_gu = n_tiles * il.mt_gu;
        *il.n_dn = n_tiles * il.mt_dn;
    }
    if (e < E) il.tiles[e] = st[e];   // inclusive token-tile prefix, for dispatch_items_kernel
}

// Tensor-core items, one per (token tile, row tile), built in parallel: tile j belongs to the
// expert whose inclusive tile prefix first exceeds j (binary search over tiles[]).
__global__ void dispatch_items_kernel(ItemLists il, const int* __restrict__ off, int E) {
    const int n_tiles = il.tiles[E - 1];
    const int mt_sum = il.mt_gu + il.mt_dn;
    const int total = n_tiles * mt_sum;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < total; j += gridDim.x * blockDim.x) {
        const int tile = j / mt_sum, r = j % mt_sum;
        int lo = 0, hi = E - 1;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (il.tiles[mid] > tile) hi = mid;
            else lo = mid + 1;
        }
        const int x = lo;
        const int cx = off[x + 1] - off[x];
        const int first_tile = il.tiles[x] - (cx + il.nt - 1) / il.nt;
        const int t0 = (tile - first_tile) * il.nt;
        const int4 item = make_int4(x, r < il.mt_gu ? r : r - il.mt_gu, off[x] + t0, min(il.nt, cx - t0));
        if (r < il.mt_gu) il.gu[tile * il.mt_gu + r] = item;
        else il.dn[tile * il.mt_dn + r - il.mt_gu] = item;
    }
}

// Placement: a chunk's assignments of expert e take the slots off[e] + (the expert's count in
// earlier chunks) + (a per-chunk shared-memory counter).  Within a chunk the slot order follows
// the atomics, not i: every consumer of the sorted order works per slot (an assignment's row of
// Xs, act and y), so which slot an assignment gets does not change any result.
__global__ void __launch_bounds__(kChunk) dispatch_place_kernel(const int* __restrict__ order, int n, int E,
                                                               const int* __restrict__ chunk_base,
                                                               const int* __restrict__ off,
                                                               int* __restrict__ ilist, int* __restrict__ pos_of) {
    __shared__ int cursor[kMaxExperts];
    for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = off[e] + chunk_base[(size_t)blockIdx.x * E + e];
    __syncthreads();
    const int i = blockIdx.x * kChunk + threadIdx.x;
    int e = i < n ? order[i] : -1;
    if (e >= E) e = -1;
    const int lane = threadIdx.x & 31;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (e >= 0 && lane == leader) base = atomicAdd(&cursor[e], __popc(peers));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (e >= 0) {
        const int p = base + __popc(peers & ((1u << lane) - 1u));
        ilist[p] = i;
        pos_of[i] = p;
    }
}

// All three passes in one block when the assignments fit one chunk (decode-sized batches).
__global__ void __launch_bounds__(kChunk) dispatch_single_kernel(const int* __restrict__ order, int n, int E,
                                                                int* __restrict__ counts, int* __restrict__ off,
                                                                int* __restrict__ active, int* __restrict__ n_active,
                                                                int* __restrict__ ilist, int* __restrict__ pos_of,
                                                                int* __restrict__ zero) {
    __shared__ int cnt[kMaxExperts];
    if (zero && threadIdx.x == 0) *zero = 0;
    __shared__ int sv[kMaxExperts];
    __shared__ int sa[kMaxExperts];
    const int tid = threadIdx.x;
    if (tid < kMaxExperts) cnt[tid] = 0;
    __syncthreads();
    int e = tid < n ? order[tid] : -1;
    if (e >= E) e = -1;
    if (e >= 0) atomicAdd(&cnt[e], 1);
    __syncthreads();
    if (tid < kMaxExperts) {
        sv[tid] = cnt[tid];
        sa[tid] = cnt[tid] > 0 ? 1 : 0;
    }
    __syncthreads();
    for (int o = 1; o < kMaxExperts; o <<= 1) {   // inclusive scans over experts
        int v = 0, a = 0;
        if (tid < kMaxExperts && tid >= o) {
            v = sv[tid - o];
            a = sa[tid - o];
        }
        __syncthreads();
        if (tid < kMaxExperts) {
            sv[tid] += v;
            sa[tid] += a;
        }
        __syncthreads();
    }
    if (tid < E) {
        const int c = cnt[tid];
        counts[tid] = c;
        off[tid + 1] = sv[tid];
        if (c > 0) active[sa[tid] - 1] = tid;
    }
    if (tid == 0) {
        off[0] = 0;
        *n_active = sa[kMaxExperts - 1];
    }
    // placement as in dispatch_place_kernel (slot order within an expert follows the atomics)
    __shared__ int cursor[kMaxExperts];
    if (tid < kMaxExperts) cursor[tid] = sv[tid] - cnt[tid];
    __syncthreads();
    const int lane = tid & 31;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (e >= 0 && lane == leader) base = atomicAdd(&cursor[e], __popc(peers));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (e >= 0) {
        const int p = base + __popc(peers & ((1u << lane) - 1u));
        ilist[p] = tid;
        pos_of[tid] = p;
    }
}

int launch_dispatch(int T, int K, int E, RouteBufs& b, cudaStream_t s, const ItemLists& items) {
    const int n = T * K;
    const int n_chunks = max(1, (n + kChunk - 1) / kChunk);
    if (n_chunks == 1 && !items.gu) {   // one chunk: count, scan and place in one block
        dispatch_single_kernel<<<1, kChunk, 0, s>>>(b.order, n, E, b.counts, b.off, b.active, b.n_active, b.ilist,
                                                    b.pos_of, items.zero);
        return 1;
    }
    dispatch_count_kernel<<<n_chunks, kChunk, 0, s>>>(b.order, n, E, b.chunk_counts);
    dispatch_scan_kernel<<<1, kMaxExperts, 0, s>>>(b.chunk_counts, n_chunks, E, b.counts, b.off, b.active,
                                                   b.n_active, items);
    dispatch_place_kernel<<<n_chunks, kChunk, 0, s>>>(b.order, n, E, b.chunk_counts, b.off, b.ilist, b.pos_of);
    if (!items.gu) return 3;
    dispatch_items_kernel<<<148 * 2, 256, 0, s>>>(items, b.off, E);
    return 4;
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
