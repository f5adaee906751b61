/* draco_moe_b200.h -- C ABI of the B200 MoE FFN library (libdraco_moe_b200.so).
 *
 * Part 1 re-exports the reference engine's MoE entry points with their exact signatures and
 * argument meaning, so the reference's numpy/ctypes drivers bind this library instead of the
 * CPU one.  Each declaration cites the reference interface it replaces (paths inside the
 * reference project).  Part 2 adds entry points the reference has no counterpart for.
 *
 * Common behaviour:
 *   - Weights are addressed by the caller's pointers, as in the reference (host virtual
 *     addresses into a GGUF mmap or numpy buffer).  The first call that sees a weight range
 *     copies it to device memory once; later calls reuse the copy.  Device addresses are
 *     accepted as well and used in place.  Registered host weights must stay unchanged while
 *     registered (draco_b200_forget / draco_b200_reset drop copies).
 *   - Activations/outputs may be host or device memory; host calls are synchronous, like the
 *     reference.
 *   - The `void` entry points keep the reference's signature, which has no error path: on an
 *     error they print one line to stderr, fill the output with NaN and record the message for
 *     draco_b200_last_error().  DRACO_B200_STRICT=1 aborts the process instead.
 *   - Format codes: 0 Q8_0, 4 Q6_K, 5 Q4_K (9 F32 for the shared-expert gate row).
 */
#ifndef DRACO_MOE_B200_H
#define DRACO_MOE_B200_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ============================ Part 1: reference entry points ============================ */

/* softmax router (max-subtracted, stable top-k, renormalised, clamp 2^-14) + experts
 * replaces src/m6_layer.c:771-802 (m6_granite_moe); `scratch` is accepted and unused */
void m6_granite_moe(const float* x0, const uint64_t* ptrs, const int* codes, const float* gate_inp,
                    int n_exp, int n_used, int inter, int n_in, int n_out, float* scratch, float* out);

/* sigmoid router (+probs_b for selection, n_group/n_group_used group limit, optional renorm,
 * w_scale) + experts.  replaces src/m6_layer.c:823-873 (m6_bailing_moe) */
void m6_bailing_moe(const float* x0, const uint64_t* ptrs, const int* codes, const float* gate_inp,
                    const float* probs_b, int n_exp, int n_used, int n_group, int n_group_used,
                    int norm_w, float w_scale, int inter, int n_in, int n_out, float* scratch,
                    float* out);

/* op-pointer MoE with ungated shared expert; field order of src/m6_engine.c:306-316 */
typedef struct M6MoeP {
    const uint64_t* exp_ptrs;
    const int* exp_codes;
    const float *gate_inp, *probs_b;
    int n_exp, n_used, n_group, n_group_used, norm_w;
    float w_scale;
    int inter, n_in, n_out;
    const uint8_t *sh_g, *sh_u, *sh_d;
    int csg, csu, csd, sh_ff;
    float* scratch;
} M6MoeP;
/* replaces src/m6_engine.c:318-349 (m6_moe_op) */
void m6_moe_op(const float* xn, void* pv, float* out);

/* scalar sigmoid-gated shared expert: out = down(silu(gate x) * up x) * sigmoid(gate_inp . x);
 * shp/shc = [gate, up, down, gate_inp(F32)].  sg[0] receives the gate logit and shg the
 * ungated expert output; sh is accepted and unused.
 * replaces src/m6_engine.c:1113-1127 (m6_granite_shexp) */
void m6_granite_shexp(const float* x, const uint64_t* shp, const int* shc, float* sg, float* sh,
                      float* shg, float* out, int shi, int h);

/* chunked-prefill MoE over T tokens with caller-made routing (order/wtop [T][n_used]);
 * out[t] = sum_k wtop[t,k] * expert_{order[t,k]}(X[t]), k ascending.  DQ, GA, gwbuf, work
 * and iwork are accepted and unused (the device path is self-contained).
 * replaces src/m6_moe_tok.c:44-161 (m6_moe_tok) */
typedef int (*m6_dequant_fn)(int, const uint8_t*, int, float*);
typedef int (*m6_gemm_auto_fn)(int, const float*, const uint8_t*, int, int, int, float*);
void m6_moe_tok(m6_dequant_fn DQ, m6_gemm_auto_fn GA, float* gwbuf, const float* X,
                const int* order, const float* wtop, const uint64_t* ep, const int* ec, int T,
                int n_used, int inter, int n_in, int n_out, int n_exp, float* out, float* work,
                int* iwork);

/* caller-routed experts of one token: the table ptrs/codes holds exactly the n_exp (<= 64)
 * selected experts (gate, up, down each), wtop their weights; out = sum_j wtop[j] * expert_j(x0),
 * j ascending.  m6_moe_batch/2 have the fixed shape inter 512, hidden 2048; m6_moe_batch2 adds
 * sigmoid(x0 . sh_gate_inp) * shared expert (sh_ptrs/sh_codes: gate, up, down; no gate row:
 * nothing added, as the reference's gate is then 0); scratch is accepted and unused.
 * replaces src/m6_layer.c:522-537 (m6_moe_batch), :547-604 (m6_moe_batch2),
 *          :606-634 (m6_moe_batch3), :656-690 (m6_moe_batch4) */
void m6_moe_batch(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp,
                  float* out);
void m6_moe_batch2(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp,
                   const uint64_t* sh_ptrs, const int* sh_codes, const float* sh_gate_inp, float* scratch,
                   float* out);
void m6_moe_batch3(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp,
                   int inter, int n_in, int n_out, float* out);
void m6_moe_batch4(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp,
                   int inter, int n_in, int n_out, float* scratch, float* out);

/* top-1 MoE with a learned router MLP (2-layer GELU MLP over a recurrent state, softmax over
 * nclass classes + balancing biases; classes >= nexp or == iskip mean "no expert", output 0).
 * Router matrices F32 (9) or F16 (7); experts: exp_gp[e] a fused [2*inter][hidden] gate|up
 * matrix, exp_dp[e] the down matrix.  rh_state (host, [hidden2]) is read (with eda_scale) and
 * overwritten with the new state, as in the reference.  Field order of src/m6_engine.c:781-793.
 * replaces src/m6_engine.c:795-835 (m6_zaya_moe_op) */
typedef struct M6ZayaMoeP {
    const uint8_t *wdown, *wfc1, *wfc2, *wout;
    int cdown, cfc1, cfc2, cout;
    const float *bdown, *bfc1, *bfc2;
    const float* rnorm;
    const float* eda_scale;
    const float* bal;
    const uint64_t *exp_gp, *exp_dp;
    const int *exp_cg, *exp_cd;
    int nexp, nclass, inter, hidden, hidden2, iskip;
    float* rh_state;
    float* scratch;
} M6ZayaMoeP;
void m6_zaya_moe_op(const float* xn, void* pv, float* out);

/* N selected experts' GEMV: y[e][o] = sum_i x_e[i] * W[idx[e]][o][i], x_e = x + e*x_stride.
 * Returns 0, -1 (shape), -3 (device error).
 * replaces src/m5/m5_batch8_k.c:80-114 (m5_gemvn_q4k) and :170-183 (m5_gemvn_q6k) */
int m5_gemvn_q4k(const float* x, long x_stride, const uint8_t* W, const int* idx, long per,
                 int n_out_e, int n_in, int n_exp, float* y);
int m5_gemvn_q6k(const float* x, long x_stride, const uint8_t* W, const int* idx, long per,
                 int n_out_e, int n_in, int n_exp, float* y);

/* row GEMV for codes 0/4/5; returns 0 or -1 (unsupported code)
 * replaces src/m5_kern_scalar.c:146-165 (m5_scalar_supported, m5_gemv, m5_gemv_range) */
int m5_scalar_supported(int code);
int m5_gemv(int code, const float* x, const uint8_t* W, int n_out, int n_in, float* y);
int m5_gemv_range(int code, const float* x, const uint8_t* W, int n_out, int n_in, float* y,
                  int o0, int o1);

/* dense prefill projections Y[T][n_out] = X[T][n_in] . W^T and row dequantisation
 * replaces src/m5/m5_gemm.c:55-235 (m5_dequant_row), :249-272 (m5_gemm),
 *          src/m5/m5_gemm_fused.c:211-241 (m5_gemm_q80/q6k/q4k, m5_gemm_auto) */
int m5_dequant_row(int code, const uint8_t* row, int n_in, float* out);
int m5_gemm(int code, const float* X, const uint8_t* W, int T, int n_out, int n_in, float* Y,
            float* wbuf);
int m5_gemm_auto(int code, const float* X, const uint8_t* W, int c, int n_out, int n_in, float* Y);
void m5_gemm_q80(const float* X, const uint8_t* W, int c, int n_out, int n_in, float* Y);
void m5_gemm_q6k(const float* X, const uint8_t* W, int c, int n_out, int n_in, float* Y);
void m5_gemm_q4k(const float* X, const uint8_t* W, int c, int n_out, int n_in, float* Y);

/* kernel-library loading is a no-op here (returns 0); chunk width is recorded only.
 * replaces src/m6_layer.c:123-140 (m6_init_dl), :46 (m6_set_moe_chunk) */
int m6_init_dl(const char* p012, const char* p3, const char* p4, const char* p56, const char* ps);
int m6_set_moe_chunk(int v);

/* host wall time of each synchronous MoE layer call accumulates in slot 23 (the reference's
 * "experts total" slot); per-phase device times come from draco_b200_profile_read.
 * replaces src/m6_layer.c:18-27 */
extern double m6_prof_t[24];
extern long m6_prof_n[24];
void m6_prof_reset(void);
double m6_prof_get(int i);
long m6_prof_cnt(int i);

/* bytes of one row of n_in values; replaces src/m6_engine.c:40-54 (m6_rowbytes) */
size_t m6_rowbytes(int code, int n_in);

/* ============================ Part 2: extensions ============================ */

/* Last error message of this thread's most recent failing call ("" if none). */
const char* draco_b200_last_error(void);
/* Library version string. */
const char* draco_b200_version(void);
/* Number of visible CUDA devices (0 if none). */
int draco_b200_device_count(void);

/* Whole MoE layer on T tokens: routing (softmax or sigmoid/groups as in m6_granite_moe /
 * m6_bailing_moe, bit-identical selection and weights), grouped experts, combine in k order,
 * optional ungated shared expert (sh_ff > 0).  X/out may be host or device memory; with
 * device pointers and a non-null stream the call is asynchronous on that stream.
 * order_out/wtop_out (optional, [T][n_used], same memory kind as X) receive the routing. */
typedef struct DracoMoeLayer {
    int n_exp, n_used, inter, n_in, n_out;
    const uint64_t* exp_ptrs;   /* [3*n_exp] gate, up, down (host array of host or device addresses) */
    const int* exp_codes;       /* [3*n_exp] */
    const float* gate_inp;      /* [n_exp][n_in] fp32 */
    const float* probs_b;       /* [n_exp] or NULL (sigmoid scoring only) */
    int scoring;                /* 0 softmax (granite), 1 sigmoid (bailing) */
    int n_group, n_group_used, norm_w;
    float w_scale;
    const void *sh_gate, *sh_up, *sh_down;  /* shared expert or NULL */
    int sh_code_g, sh_code_u, sh_code_d, sh_ff;
} DracoMoeLayer;
int draco_b200_moe_forward(const DracoMoeLayer* L, const float* X, int T, float* out,
                           int* order_out, float* wtop_out, void* stream);

/* Routing only: order/wtop [T][n_used] (host or device, like X). */
int draco_b200_route(const DracoMoeLayer* L, const float* X, int T, int* order, float* wtop,
                     void* stream);

/* Routed experts on caller-given routing (no reference counterpart; the expert-parallel
 * building block).  L describes a contiguous slice of a larger expert set: routing ids e with
 * first_expert <= e < first_expert + L->n_exp select L's expert e - first_expert, all other ids
 * (other slices, negative) are skipped.  Rows of order/wtop are ld entries apart (0: n_used);
 * the first n_used of each row are used.
 *   out[t] = sum over k ascending of wtop[t][k] * expert(X[t])   (+ the shared expert when
 *            with_shared != 0 and L has one)
 * order == NULL: no routed experts, out = shared expert (L must have one).  Pointers are all
 * host (synchronous) or all device (asynchronous on stream when given).  gate_inp/probs_b of L
 * are not used.  x_fp16 != 0: X holds fp16 rows (device memory only); the tensor-core path
 * reads them as they are (it rounds its activations to fp16 in any case), the CUDA-core paths
 * widen them to fp32 first. */
int draco_b200_experts_forward(const DracoMoeLayer* L, const void* X, int T, const int* order,
                               const float* wtop, int ld, int first_expert, float* out,
                               int with_shared, int x_fp16, void* stream);

/* The routed part of draco_b200_experts_forward for an expert-parallel owner whose results go
 * straight to the ranks that sent the rows: row q of the result (the weighted sum, k ascending,
 * of row q's experts in [first_expert, first_expert + n_exp)) is stored to
 * out_blocks[q / block] + (q % block) * n_out, out_blocks being a device array of row-block
 * addresses (other GPUs' buffers mapped into this process, or this GPU's own).  Rows without an
 * expert in the slice are not written.  The stores are fenced at system scope before the call's
 * last kernel ends, so a flag barrier enqueued after it publishes them.  Device pointers only
 * (asynchronous on stream when given); needs n_out % 4 == 0 and n_used <= 64; no shared expert.  Replaces nothing in the
 * reference (single-process there); per rank it is src/m6_moe_tok.c:44-161 on the rank's slice. */
int draco_b200_experts_forward_to_ranks(const DracoMoeLayer* L, const void* X, int T,
                                        const int* order, const float* wtop, int ld,
                                        int first_expert, float* const* out_blocks, int block,
                                        int x_fp16, void* stream);

/* Expert-parallel token exchange over n_ranks ranks that split n_exp experts contiguously
 * (rank r owns [r*n_exp/n_ranks, (r+1)*n_exp/n_ranks)).  Device pointers, 16-byte aligned,
 * asynchronous on stream.
 *  ep_plan: for T local tokens with routing order[T][K]: counts[r] = rows sent to rank r (a token
 *    sends one row to each rank owning any of its experts); row_of[t*n_ranks + r] = that row's
 *    index in the rank-major send buffer or -1; src_tok[row] = t.  block == 0: compact rows
 *    (rank r's rows follow rank r-1's; capacity T*min(K, n_ranks)); block >= T: rank r's rows
 *    start at r*block (capacity n_ranks*block), the layout of an equal-split all-to-all.
 *  ep_pack: send_x[row] = X[src_tok[row]] (H floats), send_meta[row] = {order[t][0..K),
 *    bits of wtop[t][0..K)} (2K ints) for the first min(rows, cap) rows; with block > 0 the
 *    unused rows of each block get ids -1 (no expert) and their activations are left as is.
 *  ep_combine: out[t] = sum over r ascending of back[row_of[t*n_ranks + r]] (+ shared[t]);
 *    back holds the owners' partial rows in send order. */
int draco_b200_ep_plan(const int* order, int T, int K, int n_exp, int n_ranks, int block, int* counts,
                       int* row_of, int* src_tok, void* stream);
int draco_b200_ep_pack(const float* X, const int* order, const float* wtop, const int* counts, int n_ranks,
                       const int* src_tok, int block, int cap, int K, int H, float* send_x, int* send_meta,
                       void* stream);
int draco_b200_ep_combine(const float* back, const int* row_of, int T, int n_ranks, int H,
                          const float* shared, float* out, void* stream);

/* Peer-memory exchange (one process per GPU of one node; replaces the all-to-alls).
 *  ep_mem_alloc: zeroed device buffer plus its CUDA IPC handle (64 bytes) for the other ranks;
 *    ep_mem_open/close map/unmap a peer's buffer from its handle; ep_mem_free releases.
 *  ep_push: the dispatch of ep_pack with block > 0, written straight into the owners' receive
 *    buffers: row j of the block for rank d lands at row rank*block + j of dst_x[d] (H floats)
 *    and dst_meta[d] (2K ints); unused rows of the block get ids -1.  dst_x/dst_meta are device
 *    arrays of n_ranks pointers (this rank's own buffers at index rank).  x_fp16 != 0: the rows
 *    are stored as fp16 (H % 8 == 0).
 *  ep_barrier: every rank sets its word in each peer's flag array (peer_flags: device array of
 *    n_ranks pointers to the ranks' flag arrays of n_ranks words) to the next epoch (*epoch, a
 *    device counter) and waits until its own array my_flags holds that epoch from all ranks.
 *    The wait is bounded (2 s), after which 0x400 is set in *status and the kernel returns.
 *  ep_pull_combine: ep_combine reading the owners' partial rows in place: out[t] = sum over r
 *    ascending of src_partial[r][rank*block + row_of[t][r] - r*block] (+ shared[t]). */
int draco_b200_ep_mem_alloc(size_t bytes, void** ptr, void* handle);
int draco_b200_ep_mem_open(const void* handle, void** ptr);
int draco_b200_ep_mem_close(void* ptr);
int draco_b200_ep_mem_free(void* ptr);
int draco_b200_ep_push(const float* X, const int* order, const float* wtop, const int* counts, int n_ranks,
                       int rank, const int* src_tok, int block, int K, int H, void* const* dst_x,
                       int x_fp16, int* const* dst_meta, void* stream);
int draco_b200_ep_barrier(unsigned* const* peer_flags, unsigned* my_flags, unsigned* epoch, int n_ranks,
                          int rank, int* status, void* stream);
int draco_b200_ep_pull_combine(const float* const* src_partial, const int* row_of, int T, int n_ranks,
                               int rank, int block, int H, const float* shared, float* out, void* stream);

/* Allocation-free m6_moe_tok, for callers that cannot let a library allocate device memory
 * (an engine that reserves HBM for weights and KV cache up front and forbids allocations
 * outside its pool; a decode loop that cannot take cudaMalloc's implicit synchronisation).
 * No counterpart in the reference.  All pointers are device memory except ep_dev (a host array
 * of 3*n_exp DEVICE addresses of the gate, up and down matrices) and ec (host codes).  Scratch
 * is a fixed 32 MiB device array inside the library, held by every GPU that loads it until the
 * process exits: calls needing more (T*n_used*(inter+n_out)*4 bytes plus small lists) return -4
 * without running.  All calls share that array and it keeps the last call's contents; calls that
 * overlap on the GPU race on it.  The first call on a device looks up the array's address.
 * Asynchronous on `stream`.  Returns 0, -1 (shape or arguments, including a null weight address
 * or one not aligned for its format: Q4_K 16 bytes, the others 2), -3 (CUDA error), -4 (exceeds
 * the scratch maximum); messages go to stderr. */
int draco_b200_moe_tok_noalloc(const float* X, const int* order, const float* wtop,
                               const uint64_t* ep_dev, const int* ec, int T, int n_used, int inter,
                               int n_in, int n_out, int n_exp, float* out, void* stream);

/* Grouped expert GEMM path: 0 automatic (tensor cores from DRACO_B200_TC_MIN_P = 128
 * token-expert assignments per call, when the formats and shapes allow), 1 CUDA cores,
 * 2 tensor cores whenever supported.  DRACO_B200_GEMM sets the initial value.  Returns the
 * previous mode. */
int draco_b200_set_gemm_path(int mode);

/* Fused decode layer on (1, the default) or off (0): batches of at most 8 tokens and 64
 * token-expert assignments run the whole layer (router logits, selection, gate/up, down, combine,
 * shared expert) as one cooperative kernel instead of separate launches.  DRACO_B200_FUSED_DECODE
 * sets the initial value.  Returns the previous setting. */
int draco_b200_set_fused_decode(int on);
/* Test hook: the fused decode kernel's grid barriers wait for n arrivals beyond its own blocks
 * (n > 0 models a block that never arrives: the bounded waits run out after about a second, the
 * kernel reports code 0x1000 and the call returns -5).  Returns the previous value; 0 in use. */
int draco_b200_test_fused_barrier_extra(int n);

/* Activation mode for gate/up: 0 fp32 (reference semantics, default), 1 Q8_K (int8
 * activations, integer superblock dots).  Returns the previous mode. */
int draco_b200_set_act_mode(int mode);

/* Per-phase device timing with CUDA events on the launching stream (enable != 0 turns it on
 * and clears the totals).  profile_read fills ms[i] (total milliseconds) and counts[i] for
 * phases 0 route, 1 dispatch, 2 gate/up, 3 down, 4 shared expert, 5 combine, 6 gather of the
 * fp16 token rows (tensor-core path), 7 the fused single-launch decode layer (batches of at most
 * 8 tokens and 64 token-expert assignments: routing through combine in one kernel); returns
 * the number of phases. */
int draco_b200_profile(int enable);
int draco_b200_profile_read(double* ms, long* counts, int n);
/* Number of kernels this library has launched since it was loaded. */
long draco_b200_launch_count(void);

/* Copy a host weight range to device memory now (otherwise done on first use). */
int draco_b200_register(const void* host, size_t bytes);
/* Drop the device copy of the range starting at `host`; 0 if found. */
int draco_b200_forget(const void* host);
/* Drop every device copy, cached table and workspace of the current device. */
void draco_b200_reset(void);
/* Bytes of device memory held for weight copies on the current device. */
size_t draco_b200_registered_bytes(void);

/* Test hooks (device arrays or host arrays, synchronous). */
int draco_b200_expf(const float* x, float* y, long n);
/* logits[t][e] = sum over k ascending of rounded x[t][k]*W[e][k] (router logits alone) */
int draco_b200_router_logits(const float* X, const float* W, int T, int E, int H, float* logits);
int draco_b200_q8k_quantize(const float* x, int n, float* d, int8_t* q, int16_t* bsums);
int draco_b200_q8k_block_dots(int code, const uint8_t* W, int rows, int n_in, const int8_t* q,
                              const int16_t* bsums, int32_t* out2);
int draco_b200_gemv_q8k(int code, const uint8_t* W, int rows, int n_in, const int8_t* q,
                        const float* d, const int16_t* bsums, float* y);

#ifdef __cplusplus
}
#endif
#endif
