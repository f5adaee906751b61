// Kernel entry points of the B200 MoE FFN path, launched by the C-ABI layer (abi.cu).
#pragma once
#include "common.cuh"

namespace draco {

// Router/dispatch scratch for one call, all device memory.
struct RouteBufs {
    float* logits;      // [T][E]
    int* order;         // [T][K]    selected experts, selection order
    float* wtop;        // [T][K]    gate weights
    int* counts;        // [E]
    int* off;           // [E+1]     exclusive prefix of counts
    int* ilist;         // [T*K]     assignment ids i = t*K + k sorted by (expert, i)
    int* pos_of;        // [T*K]     sorted position of assignment i
    int* active;        // [E]       experts with count > 0, ascending
    int* n_active;      // [1]
    int* err;           // [1]       nonzero: routing produced an invalid selection
    int* chunk_counts;  // [ceil(T*K/1024)][E] dispatch scratch
};

// dispatch scratch ints for n assignments over E experts
inline size_t dispatch_chunk_ints(int n, int E) { return (size_t)((n + 1023) / 1024 + 1) * (size_t)E; }

// Router parameters (semantics of src/m6_layer.c:771-796 and :823-866).
struct RouterParams {
    int scoring;        // 0 softmax + renorm (granite), 1 sigmoid (+bias, groups) (bailing)
    int n_exp, n_used, n_in;
    int n_group, n_group_used, norm_w;
    float w_scale;
    const float* probs_b;   // device [E] or nullptr
};

// Weight table: 3 device pointers per expert (gate, up, down) and their format codes.
struct ExpertTable {
    const uint8_t* const* w;   // device array [3 * n_exp] of device pointers (gate, up, down)
};

// logits[t][e] = sum_k X[t][k] * gate_inp[e][k] (k ascending, rounded products); also sets
// *zero_err = 0 when given (the routing status word the select kernel then raises)
void launch_router_logits(const float* X, const float* gate_inp, int T, int E, int H, float* logits,
                          cudaStream_t s, int* zero_err = nullptr);
void launch_router_select(const RouterParams& p, int T, RouteBufs& b, cudaStream_t s);
// Work items of the tensor-core grouped GEMM (int4 {expert, row tile, first sorted position,
// tokens}): per active expert in increasing order, its token tiles of <= nt, each times the
// row tiles of the matrix.  Built by the dispatch scan when `gu` is set.  The dispatch also
// zeroes *zero when given (the expert GEMMs' status word).
struct ItemLists {
    int4* gu = nullptr;
    int* n_gu = nullptr;
    int mt_gu = 0;
    int4* dn = nullptr;
    int* n_dn = nullptr;
    int mt_dn = 0;
    int nt = 128;
    int* zero = nullptr;
    int* tiles = nullptr;   // [E] scratch: inclusive token-tile prefix per expert
};
// returns the number of kernels launched
int launch_dispatch(int T, int K, int E, RouteBufs& b, cudaStream_t s, const ItemLists& items = ItemLists());
// Decode-sized grouped GEMV with bulk-copy staged weight tiles (decode.cu): Q4_K/Q6_K only,
// 16-byte aligned rows (Q6_K in the registry's 224-byte layout).  status gets 0x200 if a staged
// copy did not complete in time.
bool dec_supported(int cg, int cu, int cd, int inter, int n_in, int n_out, int q6s);
int launch_dec_gateup(const ExpertTable& tab, int cg, int cu, const int* active, const int* n_active, int n_active_max,
                      const int* off, const int* ilist, int tok_div, const float* X, int inter, int n_in, float* act,
                      int q6s, int* status, cudaStream_t s);
int launch_dec_down(const ExpertTable& tab, int cd, const int* active, const int* n_active, int n_active_max,
                    const int* off, const float* act, int inter, int n_out, float* y, int q6s, int* status,
                    cudaStream_t s);
// The whole decode layer of a small batch (T <= 8 tokens, T*K <= 64) in one cooperative
// launch (decode.cu): router logits (exact order), selection, gate/up + SwiGLU, down, combine,
// shared expert.  Device pointers throughout; `bar` (2 words) must be zero at launch.
struct FusedDecodeArgs {
    ExpertTable tab;
    const uint8_t* sh_g;        // shared expert matrices (same formats as the routed ones) or null
    const uint8_t* sh_u;
    const uint8_t* sh_d;
    int sh_ff;                  // 0: no shared expert
    const float* W;             // router [E][n_in]; nullptr: routing given in order/wtop
    RouterParams rp;
    const float* X;             // [T][n_in]
    int T, F, n_out;
    float* out;                 // [T][n_out]
    int* order;                 // [T][K]: written (router) or read (given routing)
    float* wtop;
    float* logits;              // [T][E] scratch
    float* act;                 // [T*K][F] scratch
    float* act_sh;              // [T][sh_ff] scratch
    unsigned* bar;              // [2] grid barrier counters
    int* status;                // 0x200 staged copy wait ran out, 0x1000 grid barrier wait ran out
    int* route_err;             // the routing status word (select)
    int q6s;
    int bar_extra;              // test hook: arrivals awaited beyond the grid (0 in use)
    unsigned long long* stamps; // optional [grid][8] %globaltimer at the phase boundaries (or null)
    int slot_bytes, n_slots;    // set by the launcher: router ring slots
    int stg_bytes, n_stg;       // per-warp weight-row ring: stage bytes, stages
    int ahead;                  // weight rows a warp keeps in flight (<= n_stg)
    int kc, xs_cap;             // router k-chunk, staged-row floats
};
// 0 launched; 1 not applicable (the caller runs the separate kernels); -3 launch error
int launch_fused_decode(FusedDecodeArgs a, int cg, int cu, int cd, cudaStream_t s);

// Router MLP of the top-1 learned-router MoE op (zaya.cu, src/m6_engine.c:795-835): device
// pointers; router matrices F32 (code 9) or F16 (7); writes the routing of the one token
// (order[0] = expert or -1, wtop[0]) and the new recurrent state.
struct ZayaRouterArgs {
    const void *wdown, *wfc1, *wfc2, *wout;
    int cdown, cfc1, cfc2, cout;
    const float *bdown, *bfc1, *bfc2, *rnorm, *eda_scale, *bal;
    const float* x;             // [H]
    const float* state_in;      // [RH] (read when eda_scale is given)
    float* state_out;           // [RH]
    float* rh;                  // [RH] scratch
    int H, RH, nclass, nexp, iskip;
    int* order;
    float* wtop;
};
int launch_zaya_router(const ZayaRouterArgs& a, cudaStream_t s);

// d[0] = a, d[1] = b (small device-side constants, stream ordered and graph capturable)
void launch_set_pair(int* d, int a, int b, cudaStream_t s);

// gate/up (+SwiGLU) over grouped assignments.  Token of sorted position p is
// ilist[p] / tok_div (ilist == nullptr: identity).  act is [positions][inter] in sorted order.
// cg/cu: uniform format codes of the gate and up matrices.
void launch_gateup_codes(const ExpertTable& tab, int cg, int cu, const int* active, const int* n_active,
                         int n_active_max, const int* off, const int* ilist, int tok_div, const float* X,
                         int inter, int n_in, float* act, cudaStream_t s, int q6s);
// down over grouped assignments: y[p][r] = dot(down_e row r, act[p])
void launch_down_code(const ExpertTable& tab, int cd, const int* active, const int* n_active,
                      int n_active_max, const int* off, const float* act, int inter, int n_out, float* y,
                      cudaStream_t s, int q6s);
// out[t][r] = sum_k w[t,k] * y[pos_of[t*K+k]][r] (k ascending, fused multiply-add),
// then + shared[t][r] when shared != nullptr.  out_blk != nullptr (n_out % 4 == 0, K <= 64):
// row t goes to out_blk[t / blk] + (t % blk) * n_out, rows without a valid assignment are not
// written, and the stores are fenced at system scope (peer buffers)
void launch_combine(const float* y, const int* order, const float* wtop, const int* pos_of, int T,
                    int K, int E, int n_out, const float* shared, float* out, cudaStream_t s,
                    float* const* out_blk = nullptr, int blk = 0);
void launch_half_to_float(const __half* x, float* y, size_t n, cudaStream_t s);
// the same with fp16 expert output rows (the tensor-core path)
void launch_combine_half(const __half* y, const int* order, const float* wtop, const int* pos_of, int T,
                         int K, int E, int n_out, const float* shared, float* out, cudaStream_t s,
                         float* const* out_blk = nullptr, int blk = 0);
// rows y[r] = dot(W row r, x) for r in [o0, o1), any supported code, one vector
void launch_gemv_rows(int code, const uint8_t* W, const float* x, int n_in, int o0, int o1, float* y,
                      cudaStream_t s, int q6s);
// Y[t][r] = dot(W row r, X[t]) for a dense token batch (m5_gemm semantics)
void launch_gemm_dense(int code, const uint8_t* W, const float* X, int T, int n_out, int n_in,
                       float* Y, cudaStream_t s, int q6s);
// dequantise rows to fp32
void launch_dequant(int code, const uint8_t* W, int rows, int n_in, float* out, cudaStream_t s, int q6s);
// repack Q6_K matrices from 210-byte to 224-byte superblocks (registry copies)
void launch_q6_pad(const uint8_t* src, size_t src_per, int n_mats, int rows, int nb, uint8_t* dst,
                   cudaStream_t s);
// out[i] = y[i] * sigmoid(dot(gw, x)) for the scalar-gated shared expert; writes the gate
// logit to sg
void launch_shexp_gate(const float* x, const float* gw, int h, const float* y, float* sg, float* out,
                       int T, cudaStream_t s);
// host expf replica over an array (test hook)
void launch_expf(const float* x, float* y, long n, cudaStream_t s);

// ---- expert parallelism: token exchange over G ranks (experts split contiguously) ----
constexpr int kEpMaxRanks = 16;
// per-rank send plan of one rank's tokens: counts[G], row_of[T*G] (row or -1), src_tok[rows];
// block > 0 places rank r's rows from r*block on
void launch_ep_plan(const int* order, int T, int K, int E, int G, int block, int* counts, int* row_of,
                    int* src_tok, cudaStream_t s);
// send rows: X[src_tok[row]] and the routing row (K ids, K weight bits) for every planned row
void launch_ep_pack(const float* X, const int* order, const float* wtop, const int* counts, int G,
                    const int* src_tok, int block, int cap, int K, int H, float* send_x, int* send_meta,
                    cudaStream_t s);
// out[t] = sum over ranks (ascending) of back[row_of[t*G + r]] + shared[t]
void launch_ep_combine(const float* back, const int* row_of, int T, int G, int H, const float* shared,
                       float* out, cudaStream_t s);
// peer-memory exchange: dispatch stores into the owners' buffers (dst_x/dst_meta: device arrays
// of G peer pointers), a flag barrier over G ranks (bounded wait, 0x400 in *status), combine
// loads from the owners' partial buffers
void launch_ep_push(const float* X, const int* order, const float* wtop, const int* counts, int G, int rank,
                    const int* src_tok, int block, int K, int H, void* const* dst_x, int x16, int* const* dst_meta,
                    cudaStream_t s);
void launch_ep_barrier(unsigned* const* peer_flags, unsigned* my_flags, unsigned* epoch_ctr, int G, int rank,
                       int* status, cudaStream_t s);
void launch_ep_pull_combine(const float* const* src_partial, const int* row_of, int T, int G, int rank,
                            int block, int H, const float* shared, float* out, cudaStream_t s);
// given routing rows (row stride ld) into contiguous [T][K] buffers, ids minus e_base
void launch_route_in(const int* order, const float* wtop, int ld, int e_base, int T, int K, int* o_order,
                     float* o_wtop, cudaStream_t s);

// ---- Q8_K activation mode ----
void launch_q8k_quantize(const float* x, int rows, int n, float* d, int8_t* q, int16_t* bsums,
                         cudaStream_t s);
// integer superblock dots of W rows with one Q8_K vector: Q4_K -> (isc, imn) pairs,
// Q6_K -> isum (second entry 0)
void launch_q8k_block_dots(int code, const uint8_t* W, int rows, int n_in, const int8_t* q,
                           const int16_t* bsums, int32_t* out2, cudaStream_t s, int q6s);
// gate/up over grouped assignments with Q8_K activations (xq/xd/xbs: per token row)
void launch_gateup_q8k(const ExpertTable& tab, int cg, const int* active, const int* n_active,
                       int n_active_max, const int* off, const int* ilist, int tok_div,
                       const int8_t* xq, const float* xd, const int16_t* xbs, int inter, int n_in,
                       float* act, cudaStream_t s, int q6s);
void launch_gemv_q8k(int code, const uint8_t* W, int rows, int n_in, const int8_t* q, const float* d,
                     const int16_t* bsums, float* y, cudaStream_t s, int q6s);

}  // namespace draco
