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

// formats/shapes the tensor-core path handles
bool tc_supported(int cg, int cu, int cd, int inter, int n_in, int n_out);
// describe stacked weights: gate/up [n_exp*inter rows][n_in values], down [n_exp*n_out][inter]
int tc_make_weight_maps(TcMaps* maps, const uint8_t* gate, const uint8_t* up, const uint8_t* down, int n_exp,
                        int cg, int cd, int inter, int n_in, int n_out);
// gather (fp16) -> gate/up GEMM (+SwiGLU, fp16 act) -> down GEMM (fp32 y), for the sorted
// assignments described by off/active/ilist; the item lists were built by the dispatch scan
// (ItemLists with tc_token_tile / tc_tiles_*).  Scratch: Xs [P][n_in] and act_h [P][inter]
// fp16, items buffers (see tc_items_capacity), err (device int, nonzero after a timeout).
int tc_run(const TcMaps& maps, int cg, int cd, int n_exp, int inter, int n_in, int n_out, const float* X,
           const int* ilist, int tok_div, int P, const int* off, const int* active, const int* n_active,
           __half* Xs, __half* act_h, float* y, int4* items_gu, int* n_items_gu, int4* items_dn, int* n_items_dn,
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
