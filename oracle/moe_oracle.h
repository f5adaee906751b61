/* CPU restatement of the reference's quantized MoE FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker the CUDA path is compared with
 * (tests, __graft_entry__.smoke, and the cpu_baseline leg of bench.py); nothing in the
 * product links, loads or calls it.
 *
 * Every function restates the algorithm of one reference function (file:line given below,
 * paths inside the reference project) in this file's own code.  Pinned in the CPU test
 * suite against the reference's C compiled unmodified into oracle/_ref: routers, gemv rows
 * and the decode layer are bit-identical; the chunked-prefill layer agrees to fp32 rounding
 * (the reference's fused GEMM sums 16 lanes at a time).
 */
#ifndef DRACO_MOE_ORACLE_H
#define DRACO_MOE_ORACLE_H
#include <stdint.h>
#include <stddef.h>
#ifdef __cplusplus
extern "C" {
#endif

/* fp16 -> fp32 incl. subnormals                        (src/m5_kern_scalar.c:9-21) */
float orc_f16_to_f32(uint16_t h);
/* bytes of one row of n_in values for format code      (src/m6_engine.c:40-54) */
size_t orc_row_bytes(int code, int n_in);
/* y[r] = dot(row r, x) for r in [o0, o1); codes 0 Q8_0, 4 Q6_K, 5 Q4_K
 *                                                       (src/m5_kern_scalar.c:48-165) */
int orc_gemv_range(int code, const float* x, const uint8_t* W, int n_out, int n_in, float* y,
                   int o0, int o1);
/* one row dequantised to fp32                          (src/m5/m5_gemm.c:55-235) */
int orc_dequant_row(int code, const uint8_t* row, int n_in, float* out);

/* softmax router: logits, max-subtracted softmax, stable top-k, renormalised with the
 * 2^-14 clamp                                          (src/m6_layer.c:771-796) */
void orc_route_softmax(const float* x, const float* gate_inp, int n_exp, int n_used, int n_in,
                       int* idx, float* w, float* probs_out);
/* sigmoid router: +bias for selection, group-limited top-k, weights from the unbiased
 * sigmoid, optional renorm (clamp) and scale           (src/m6_layer.c:823-866)
 * norm_w == 2: the numpy drivers' renormalisation instead (src/k2_engine.py:506-507): no clamp,
 * numpy's pairwise sum order */
void orc_route_sigmoid(const float* x, const float* gate_inp, const float* probs_b, int n_exp,
                       int n_used, int n_group, int n_group_used, int norm_w, float w_scale,
                       int n_in, int* idx, float* w, float* probs_out);
/* the two routers over T token rows [T][n_in] (one OpenMP thread per token); scoring 0 softmax,
 * 1 sigmoid; idx/w [T][n_used] */
void orc_route_batch(int scoring, const float* X, int T, const float* gate_inp, const float* probs_b,
                     int n_exp, int n_used, int n_group, int n_group_used, int norm_w, float w_scale,
                     int n_in, int* idx, float* w);
/* numpy's float32 pairwise sum of n <= 128 contiguous values */
float orc_pairwise_sum(const float* a, int n);
/* stable top-k (ties -> lower index)                   (src/m6_layer.c:808-821) */
void orc_topk(const float* v, int n, int k, int* out);

/* gate/up gemv -> SwiGLU -> down gemv -> out = sum_j w_j y_j (j ascending)
 *                                                       (src/m6_layer.c:699-764) */
void orc_moe_experts(const float* x, const uint64_t* p3, const int* c3, const float* wtop,
                     int n_used, int inter, int n_in, int n_out, float* out);
/* full decode layers                                    (src/m6_layer.c:771-802, 823-873) */
void orc_granite_moe(const float* x, const uint64_t* ptrs, const int* codes, const float* gate_inp,
                     int n_exp, int n_used, int inter, int n_in, int n_out, float* out);
void orc_bailing_moe(const float* x, const uint64_t* ptrs, const int* codes, const float* gate_inp,
                     const float* probs_b, int n_exp, int n_used, int n_group, int n_group_used,
                     int norm_w, float w_scale, int inter, int n_in, int n_out, float* out);
/* shared experts: scalar sigmoid-gated (src/m6_engine.c:1113-1127) and ungated added to out
 * (src/m6_engine.c:324-348) */
void orc_granite_shexp(const float* x, const uint64_t* shp, const int* shc, int shi, int h,
                       float* out);
void orc_shared_add(const float* x, const uint8_t* g, const uint8_t* u, const uint8_t* d,
                    int cg, int cu, int cd, int sh_ff, int n_in, int n_out, float* out);

/* orc_shared_add over T token rows (one OpenMP thread per token) */
void orc_shared_add_batch(const float* X, int T, const uint8_t* g, const uint8_t* u, const uint8_t* d,
                          int cg, int cu, int cd, int sh_ff, int n_in, int n_out, float* out);

/* chunked prefill: stable counting sort by expert, per-expert gate/up/SwiGLU/down, per-token
 * combine in k order                                    (src/m6_moe_tok.c:44-161) */
void orc_moe_tok(const float* X, const int* order, const float* wtop, const uint64_t* ep,
                 const int* ec, int T, int n_used, int inter, int n_in, int n_out, int n_exp,
                 float* out);

/* ---- Q8_K activations (not in the reference; format of ggml's block_q8_K) ----
 * per 256 values: d = amax/127 (fp32), q = rint(x * 127/amax) clamped to [-127, 127],
 * bsums[16] = sums of q over 16-value groups.  amax == 0 -> d = 0, q = 0. */
void orc_q8k_quantize(const float* x, int n, float* d, int8_t* q, int16_t* bsums);
/* integer superblock dot of one Q4_K superblock with one Q8_K block:
 * isc = sum_j sc_j * sum_{k in sub-block j} q4*q8,  imn = sum_j m_j * (q8 sum of sub-block j) */
void orc_q4k_q8k_block(const uint8_t* blk, const int8_t* q8, const int16_t* bsums,
                       int32_t* isc, int32_t* imn);
/* integer superblock dot of one Q6_K superblock with one Q8_K block:
 * isum = sum_{g=0..15} sc_g * sum_{k in 16-group g} (q6-32)*q8 */
void orc_q6k_q8k_block(const uint8_t* blk, const int8_t* q8, int32_t* isum);
/* row dot products in Q8K mode: per superblock b (ascending)
 *   Q4_K: dot += d8_b * (d4_b * isc_b - dmin4_b * imn_b);  Q6_K: dot += d8_b * d6_b * isum_b */
void orc_gemv_q8k(int code, const float* d8, const int8_t* q8, const int16_t* bsums,
                  const uint8_t* W, int n_out, int n_in, float* y);

/* the host C library's expf over an array (checker for the device replica of it) */
void orc_expf_array(const float* x, float* y, long n);

#ifdef __cplusplus
}
#endif
#endif
