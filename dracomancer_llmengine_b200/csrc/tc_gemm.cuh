// Host interface of the tensor-core grouped expert GEMM (tc_gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace draco {

// TMA descriptors of one layer's stacked expert matrices (device copies, Q6_K padded)
struct TcMaps {
    CUtensorMap gate, up, down;
};

// activation tensor maps, one per token-tile height R = 16 (i + 1): 3D view
// {64 halves, rows, K / 64 chunks} with box {64, R, 2}
struct TcActMaps {
    CUtensorMap m[8];
};

// one call's operands: the fp16 activation maps of Xs and act_h and the sizes
struct TcCall {
    TcActMaps mx, ma;
    int cg = 0, cd = 0, n_exp = 0, inter = 0, n_in = 0, n_out = 0, P = 0, nt = 128;
};

// formats/shapes the tensor-core path handles
bool tc_supported(int cg, int cu, int cd, int inter, int n_in, int n_out);
// describe stacked weights: gate/up [n_exp*inter rows][n_in values], down [n_exp*n_out][inter]
int tc_make_weight_maps(TcMaps* maps, const uint8_t* gate, const uint8_t* up, const uint8_t* down, int n_exp,
                        int cg, int cd, int inter, int n_in, int n_out);
// The three launches of one call, for P sorted assignments (the item lists were built by the
// dispatch scan with tc_token_tile / tc_tiles_*):
//   tc_gather: Xs[p] = fp16(X[ilist[p] / tok_div]) for p < *n_valid (all P when n_valid is null);
//              X fp32 rows, or fp16 rows (x_half) copied as they are
//   tc_gateup: act_h = fp16(silu(gate . Xs) * (up . Xs)) per item
//   tc_down:   y = down . act_h per item (fp32)
// err (device int) is nonzero after a bounded wait ran out; stats optionally collects wait
// cycles (kTcStatSites per kernel).
int tc_prepare(TcCall* call, int cg, int cd, int n_exp, int inter, int n_in, int n_out, int P, __half* Xs,
               __half* act_h);
void tc_gather(const TcCall& call, const void* X, bool x_half, const int* ilist, const int* n_valid, int tok_div,
               __half* Xs, cudaStream_t s);
// the same for fp32 token rows read once each: row t goes to the slots pos_of[t*K + k] of its
// assignments with 0 <= order[t*K + k] < E
void tc_gather_tokens(const TcCall& c, const float* X, const int* order, const int* pos_of, int T, int K, int E,
                      __half* Xs, cudaStream_t s);
// item lists of a dense (shared-expert) call: one expert, call.P token rows in order
void tc_dense_items(const TcCall& call, int4* items_gu, int* n_gu, int4* items_dn, int* n_dn, cudaStream_t s);
int tc_gateup(const TcCall& call, const TcMaps& maps, const int4* items, const int* n_items, __half* act_h, int* err,
              unsigned long long* stats, cudaStream_t s);
// y: fp32 rows, or fp16 rows when half_out
int tc_down(const TcCall& call, const TcMaps& maps, const int4* items, const int* n_items, void* y, bool half_out,
            int* err, unsigned long long* stats, cudaStream_t s);
// wait-statistics sites per kernel (stats holds 2 * kTcStatSites counters: gate/up, down)
constexpr int kTcStatSites = 15;
// weight-row tiles per expert: gate/up tiles hold 64 rows of each matrix, down tiles 128 rows
inline int tc_tiles_gateup(int inter) { return inter / 64; }
inline int tc_tiles_down(int n_out) { return n_out / 128; }
// tokens per item for P assignments over n_exp experts: tiles of <= 64 (eight activation
// stages, two MMA issuers) when experts average <= 40 tokens, else <= 128 (four stages, one
// issuer)
inline int tc_token_tile(int P, int n_exp) { return P <= 40 * n_exp ? 64 : 128; }
// item-list capacity for P assignments over at most n_active_max experts (token tiles of 64 or
// more tokens)
inline size_t tc_items_capacity(int P, int n_active_max, int row_tiles) {
    return ((size_t)P / 64 + (size_t)n_active_max + 1) * (size_t)row_tiles;
}

}  // namespace draco
