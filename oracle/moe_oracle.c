/* CPU restatement of the reference's quantized MoE FFN path (see moe_oracle.h).
 * TEST INFRASTRUCTURE ONLY — the checker, never the thing measured or shipped.
 *
 * Arithmetic follows the reference's operation order.  This file is compiled with
 * -ffp-contract=off and spells out fmaf() exactly where gcc fuses the reference's
 * `acc += a * b` into one rounding (Q4_K rows, the weighted combines); where the reference's
 * build keeps the product rounded on its own (router logits, whose products gcc vectorises
 * first; Q6_K and Q8_0 rows) this file writes a plain multiply and add.  The results are
 * bit-identical to the reference built with -O3 and FMA enabled.
 */
#include "moe_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

float orc_f16_to_f32(uint16_t h) {
    /* sign | exponent rebias | mantissa; subnormals as man * 2^-24 (src/m5_kern_scalar.c:9-21) */
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            float v = (float)m * 0x1p-24f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float ld_f16(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_f16_to_f32(h);
}

size_t orc_row_bytes(int code, int n_in) {
    switch (code) {
        case 0: return (size_t)(n_in / 32) * 34;
        case 4: return (size_t)(n_in / 256) * 210;
        case 5: return (size_t)(n_in / 256) * 144;
        default: return 0;
    }
}

/* Q4_K 6-bit (scale, min) of sub-block j                    (src/m5_kern_scalar.c:39-46) */
static inline void q4k_scale_min(const uint8_t* s, int j, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* one row dot product in the scalar kernel's order          (src/m5_kern_scalar.c:48-144) */
static float row_dot(int code, const uint8_t* row, const float* x, int n_in) {
    float dot = 0.f;
    if (code == 0) {
        for (int b = 0; b < n_in / 32; b++) {
            const uint8_t* p = row + (size_t)b * 34;
            const float d = ld_f16(p);
            float acc = 0.f;
            for (int i = 0; i < 32; i++) acc += (float)(int8_t)p[2 + i] * x[b * 32 + i];
            dot += d * acc;
        }
    } else if (code == 5) {
        for (int b = 0; b < n_in / 256; b++) {
            const uint8_t* p = row + (size_t)b * 144;
            const float d = ld_f16(p), dmin = ld_f16(p + 2);
            for (int j = 0; j < 8; j++) {
                int sc, mn;
                q4k_scale_min(p + 4, j, &sc, &mn);
                const float dsc = d * (float)sc, dm = dmin * (float)mn;
                const uint8_t* qb = p + 16 + (j >> 1) * 32;
                float acc = 0.f;
                for (int k = 0; k < 32; k++) {
                    const int q = (j & 1) ? (qb[k] >> 4) : (qb[k] & 15);
                    const float w = fmaf(dsc, (float)q, -dm);
                    acc = fmaf(w, x[b * 256 + j * 32 + k], acc);
                }
                dot += acc;
            }
        }
    } else if (code == 4) {
        for (int b = 0; b < n_in / 256; b++) {
            const uint8_t* p = row + (size_t)b * 210;
            const uint8_t* ql = p;
            const uint8_t* qh = p + 128;
            const int8_t* sc = (const int8_t*)(p + 192);
            const float d = ld_f16(p + 208);
            for (int r = 0; r < 8; r++) {             /* 32-value row r of the superblock */
                const int half = r & 1, nib_hi = (r >> 1) & 1, grp = r >> 2;
                const int shift = (r & 3) * 2;
                for (int g = 0; g < 2; g++) {         /* two 16-value scale groups */
                    const float dsc = d * (float)sc[r * 2 + g];
                    float acc = 0.f;
                    for (int k = 0; k < 16; k++) {
                        const int kk = g * 16 + k;
                        const int lo = (ql[grp * 64 + half * 32 + kk] >> (nib_hi * 4)) & 15;
                        const int hi = (qh[grp * 32 + kk] >> shift) & 3;
                        acc += (float)((lo | (hi << 4)) - 32) * x[b * 256 + r * 32 + kk];
                    }
                    dot += dsc * acc;
                }
            }
        }
    }
    return dot;
}

int orc_gemv_range(int code, const float* x, const uint8_t* W, int n_out, int n_in, float* y,
                   int o0, int o1) {
    (void)n_out;
    const size_t rb = orc_row_bytes(code, n_in);
    if (rb == 0) return -1;
    #pragma omp parallel for schedule(static) if (o1 - o0 >= 256)
    for (int r = o0; r < o1; r++) y[r] = row_dot(code, W + rb * (size_t)r, x, n_in);
    return 0;
}

int orc_dequant_row(int code, const uint8_t* row, int n_in, float* out) {
    /* value map of src/m5/m5_gemm.c:56-68 (Q8_0), :142-170 (Q4_K), :193-211 (Q6_K) */
    if (code == 0) {
        for (int b = 0; b < n_in / 32; b++) {
            const uint8_t* p = row + (size_t)b * 34;
            const float d = ld_f16(p);
            for (int i = 0; i < 32; i++) out[b * 32 + i] = d * (float)(int8_t)p[2 + i];
        }
        return 0;
    }
    if (code == 5) {
        for (int b = 0; b < n_in / 256; b++) {
            const uint8_t* p = row + (size_t)b * 144;
            const float d = ld_f16(p), dmin = ld_f16(p + 2);
            for (int j = 0; j < 8; j++) {
                int sc, mn;
                q4k_scale_min(p + 4, j, &sc, &mn);
                const float dsc = d * (float)sc, dm = dmin * (float)mn;
                const uint8_t* qb = p + 16 + (j >> 1) * 32;
                for (int k = 0; k < 32; k++) {
                    const int q = (j & 1) ? (qb[k] >> 4) : (qb[k] & 15);
                    out[b * 256 + j * 32 + k] = dsc * (float)q - dm;
                }
            }
        }
        return 0;
    }
    if (code == 4) {
        for (int b = 0; b < n_in / 256; b++) {
            const uint8_t* p = row + (size_t)b * 210;
            const int8_t* sc = (const int8_t*)(p + 192);
            const float d = ld_f16(p + 208);
            for (int e = 0; e < 256; e++) {
                const uint8_t l = p[(e >> 7) * 64 + (e & 63)];
                const int lo = ((e >> 6) & 1) ? (l >> 4) : (l & 15);
                const int hi = (p[128 + (e >> 7) * 32 + (e & 31)] >> (((e >> 5) & 3) * 2)) & 3;
                out[b * 256 + e] = d * (float)sc[e >> 4] * (float)((lo | (hi << 4)) - 32);
            }
        }
        return 0;
    }
    return -1;
}

void orc_topk(const float* v, int n, int k, int* out) {
    /* k passes of strict-greater argmax over the unused entries (src/m6_layer.c:808-821) */
    char* used = (char*)calloc((size_t)n, 1);
    for (int t = 0; t < k; t++) {
        int best = -1;
        float bv = -1e30f;
        for (int i = 0; i < n; i++)
            if (!used[i] && v[i] > bv) {
                bv = v[i];
                best = i;
            }
        out[t] = best;
        if (best >= 0) used[best] = 1;
    }
    free(used);
}

static float router_logit(const float* x, const float* w, int n_in) {
    float acc = 0.f;
    for (int i = 0; i < n_in; i++) acc += x[i] * w[i];    /* each product rounded, summed in order */
    return acc;
}

void orc_route_softmax(const float* x, const float* gate_inp, int n_exp, int n_used, int n_in,
                       int* idx, float* w, float* probs_out) {
    float* p = (float*)malloc(sizeof(float) * (size_t)n_exp);
    for (int e = 0; e < n_exp; e++) p[e] = router_logit(x, gate_inp + (size_t)e * n_in, n_in);
    float mx = -1e30f;
    for (int e = 0; e < n_exp; e++) mx = p[e] > mx ? p[e] : mx;
    float s = 0.f;
    for (int e = 0; e < n_exp; e++) {
        p[e] = expf(p[e] - mx);
        s += p[e];
    }
    const float inv = 1.f / s;
    for (int e = 0; e < n_exp; e++) p[e] *= inv;
    orc_topk(p, n_exp, n_used, idx);
    float ws = 0.f;
    for (int j = 0; j < n_used; j++) {
        w[j] = p[idx[j]];
        ws += w[j];
    }
    if (ws < 6.103515625e-5f) ws = 6.103515625e-5f;
    for (int j = 0; j < n_used; j++) w[j] /= ws;
    if (probs_out) memcpy(probs_out, p, sizeof(float) * (size_t)n_exp);
    free(p);
}

float orc_pairwise_sum(const float* a, int n) {
    /* numpy's float32 add.reduce over a contiguous run of n <= 128 values */
    if (n < 8) {
        float r = 0.f;
        for (int i = 0; i < n; i++) r += a[i];
        return r;
    }
    float r[8];
    for (int j = 0; j < 8; j++) r[j] = a[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8)
        for (int j = 0; j < 8; j++) r[j] += a[i + j];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; i++) res += a[i];
    return res;
}

void orc_route_sigmoid(const float* x, const float* gate_inp, const float* probs_b, int n_exp,
                       int n_used, int n_group, int n_group_used, int norm_w, float w_scale,
                       int n_in, int* idx, float* w, float* probs_out) {
    float* p = (float*)malloc(sizeof(float) * (size_t)n_exp);
    float* sel = (float*)malloc(sizeof(float) * (size_t)n_exp);
    for (int e = 0; e < n_exp; e++) {
        const float acc = router_logit(x, gate_inp + (size_t)e * n_in, n_in);
        p[e] = 1.f / (1.f + expf(-acc));
        sel[e] = p[e] + (probs_b ? probs_b[e] : 0.f);
    }
    if (n_group > 1) {
        const int per = n_exp / n_group;
        float* gs = (float*)malloc(sizeof(float) * (size_t)n_group);
        int* gt = (int*)malloc(sizeof(int) * (size_t)n_group);
        char* keep = (char*)calloc((size_t)n_group, 1);
        for (int g = 0; g < n_group; g++) {     /* group score = sum of the group's top two */
            float a = -1e30f, b = -1e30f;
            for (int i = 0; i < per; i++) {
                const float v = sel[g * per + i];
                if (v > a) {
                    b = a;
                    a = v;
                } else if (v > b) {
                    b = v;
                }
            }
            gs[g] = a + b;
        }
        orc_topk(gs, n_group, n_group_used, gt);
        for (int i = 0; i < n_group_used; i++) keep[gt[i]] = 1;
        for (int g = 0; g < n_group; g++)
            if (!keep[g])
                for (int i = 0; i < per; i++) sel[g * per + i] = -1e30f;
        free(gs);
        free(gt);
        free(keep);
    }
    orc_topk(sel, n_exp, n_used, idx);
    float s = 0.f;
    for (int j = 0; j < n_used; j++) {
        w[j] = p[idx[j]];
        s += w[j];
    }
    if (norm_w == 2) {
        /* the numpy drivers (src/k2_engine.py:506-507): rw / rw.sum() * scale, no clamp, the sum
         * in numpy's float32 pairwise order (8 running sums for n >= 8) */
        s = orc_pairwise_sum(w, n_used);
        for (int j = 0; j < n_used; j++) w[j] /= s;
    } else if (norm_w) {
        if (s < 6.103515625e-5f) s = 6.103515625e-5f;
        for (int j = 0; j < n_used; j++) w[j] /= s;
    }
    if (w_scale != 0.f && w_scale != 1.f)
        for (int j = 0; j < n_used; j++) w[j] *= w_scale;
    if (probs_out) memcpy(probs_out, p, sizeof(float) * (size_t)n_exp);
    free(p);
    free(sel);
}

/* Routing of T token rows at once: the per-token routers above, one token per OpenMP thread
 * (each token's routing is independent, so the threads change nothing in the results).
 * scoring 0 = orc_route_softmax, 1 = orc_route_sigmoid. */
void orc_route_batch(int scoring, const float* X, int T, const float* gate_inp, const float* probs_b,
                     int n_exp, int n_used, int n_group, int n_group_used, int norm_w, float w_scale,
                     int n_in, int* idx, float* w) {
    #pragma omp parallel for schedule(dynamic, 4)
    for (int t = 0; t < T; t++) {
        const float* x = X + (size_t)t * n_in;
        if (scoring == 0)
            orc_route_softmax(x, gate_inp, n_exp, n_used, n_in, idx + (size_t)t * n_used,
                              w + (size_t)t * n_used, NULL);
        else
            orc_route_sigmoid(x, gate_inp, probs_b, n_exp, n_used, n_group, n_group_used, norm_w,
                              w_scale, n_in, idx + (size_t)t * n_used, w + (size_t)t * n_used, NULL);
    }
}

static inline float silu_mul(float g, float u) { return (g / (1.f + expf(-g))) * u; }

void orc_moe_experts(const float* x, const uint64_t* p3, const int* c3, const float* wtop,
                     int n_used, int inter, int n_in, int n_out, float* out) {
    float* act = (float*)malloc(sizeof(float) * (size_t)n_used * inter);
    float* u = (float*)malloc(sizeof(float) * (size_t)inter);
    float* yd = (float*)malloc(sizeof(float) * (size_t)n_used * n_out);
    for (int j = 0; j < n_used; j++) {
        float* a = act + (size_t)j * inter;
        orc_gemv_range(c3[3 * j], x, (const uint8_t*)(uintptr_t)p3[3 * j], inter, n_in, a, 0, inter);
        orc_gemv_range(c3[3 * j + 1], x, (const uint8_t*)(uintptr_t)p3[3 * j + 1], inter, n_in, u, 0, inter);
        for (int i = 0; i < inter; i++) a[i] = silu_mul(a[i], u[i]);
        orc_gemv_range(c3[3 * j + 2], a, (const uint8_t*)(uintptr_t)p3[3 * j + 2], n_out, inter,
                       yd + (size_t)j * n_out, 0, n_out);
    }
    for (int i = 0; i < n_out; i++) {
        float s = 0.f;
        /* the reference's build vectorises this j loop 4 wide (products rounded, summed in
         * order) and finishes the remainder with fused multiply-adds */
        const int jv = n_used & ~3;
        for (int j = 0; j < jv; j++) s += wtop[j] * yd[(size_t)j * n_out + i];
        for (int j = jv; j < n_used; j++) s = fmaf(wtop[j], yd[(size_t)j * n_out + i], s);
        out[i] = s;
    }
    free(act);
    free(u);
    free(yd);
}

static void gather_selected(const uint64_t* ptrs, const int* codes, const int* idx, int n_used,
                            uint64_t* p3, int* c3) {
    for (int j = 0; j < n_used; j++)
        for (int t = 0; t < 3; t++) {
            p3[3 * j + t] = ptrs[3 * idx[j] + t];
            c3[3 * j + t] = codes[3 * idx[j] + t];
        }
}

void orc_granite_moe(const float* x, const uint64_t* ptrs, const int* codes, const float* gate_inp,
                     int n_exp, int n_used, int inter, int n_in, int n_out, float* out) {
    int* idx = (int*)malloc(sizeof(int) * (size_t)n_used);
    float* w = (float*)malloc(sizeof(float) * (size_t)n_used);
    uint64_t* p3 = (uint64_t*)malloc(sizeof(uint64_t) * 3 * (size_t)n_used);
    int* c3 = (int*)malloc(sizeof(int) * 3 * (size_t)n_used);
    orc_route_softmax(x, gate_inp, n_exp, n_used, n_in, idx, w, NULL);
    gather_selected(ptrs, codes, idx, n_used, p3, c3);
    orc_moe_experts(x, p3, c3, w, n_used, inter, n_in, n_out, out);
    free(idx);
    free(w);
    free(p3);
    free(c3);
}

void orc_bailing_moe(const float* x, const uint64_t* ptrs, const int* codes, const float* gate_inp,
                     const float* probs_b, int n_exp, int n_used, int n_group, int n_group_used,
                     int norm_w, float w_scale, int inter, int n_in, int n_out, float* out) {
    int* idx = (int*)malloc(sizeof(int) * (size_t)n_used);
    float* w = (float*)malloc(sizeof(float) * (size_t)n_used);
    uint64_t* p3 = (uint64_t*)malloc(sizeof(uint64_t) * 3 * (size_t)n_used);
    int* c3 = (int*)malloc(sizeof(int) * 3 * (size_t)n_used);
    orc_route_sigmoid(x, gate_inp, probs_b, n_exp, n_used, n_group, n_group_used, norm_w, w_scale,
                      n_in, idx, w, NULL);
    gather_selected(ptrs, codes, idx, n_used, p3, c3);
    orc_moe_experts(x, p3, c3, w, n_used, inter, n_in, n_out, out);
    free(idx);
    free(w);
    free(p3);
    free(c3);
}

void orc_granite_shexp(const float* x, const uint64_t* shp, const int* shc, int shi, int h,
                       float* out) {
    float sg;
    float* g = (float*)malloc(sizeof(float) * (size_t)shi);
    float* u = (float*)malloc(sizeof(float) * (size_t)shi);
    float* y = (float*)malloc(sizeof(float) * (size_t)h);
    /* the scalar gate row is F32 (code 9) in the reference's drivers: plain fp32 dot */
    {
        const float* gw = (const float*)(uintptr_t)shp[3];
        float acc = 0.f;
        for (int i = 0; i < h; i++) acc = fmaf(gw[i], x[i], acc);
        sg = acc;
    }
    orc_gemv_range(shc[0], x, (const uint8_t*)(uintptr_t)shp[0], shi, h, g, 0, shi);
    orc_gemv_range(shc[1], x, (const uint8_t*)(uintptr_t)shp[1], shi, h, u, 0, shi);
    for (int i = 0; i < shi; i++) g[i] = silu_mul(g[i], u[i]);
    orc_gemv_range(shc[2], g, (const uint8_t*)(uintptr_t)shp[2], h, shi, y, 0, h);
    const float gate = 1.f / (1.f + expf(-sg));
    for (int i = 0; i < h; i++) out[i] = y[i] * gate;
    free(g);
    free(u);
    free(y);
}

void orc_shared_add(const float* x, const uint8_t* gw, const uint8_t* uw, const uint8_t* dw,
                    int cg, int cu, int cd, int sh_ff, int n_in, int n_out, float* out) {
    float* g = (float*)malloc(sizeof(float) * (size_t)sh_ff);
    float* u = (float*)malloc(sizeof(float) * (size_t)sh_ff);
    float* y = (float*)malloc(sizeof(float) * (size_t)n_out);
    orc_gemv_range(cg, x, gw, sh_ff, n_in, g, 0, sh_ff);
    orc_gemv_range(cu, x, uw, sh_ff, n_in, u, 0, sh_ff);
    for (int i = 0; i < sh_ff; i++) g[i] = silu_mul(g[i], u[i]);
    orc_gemv_range(cd, g, dw, n_out, sh_ff, y, 0, n_out);
    for (int i = 0; i < n_out; i++) out[i] += y[i];
    free(g);
    free(u);
    free(y);
}

/* orc_shared_add for T token rows (one OpenMP thread per token; rows are independent) */
void orc_shared_add_batch(const float* X, int T, const uint8_t* gw, const uint8_t* uw, const uint8_t* dw,
                          int cg, int cu, int cd, int sh_ff, int n_in, int n_out, float* out) {
    #pragma omp parallel for schedule(dynamic, 1)
    for (int t = 0; t < T; t++)
        orc_shared_add(X + (size_t)t * n_in, gw, uw, dw, cg, cu, cd, sh_ff, n_in, n_out, out + (size_t)t * n_out);
}

void orc_moe_tok(const float* X, const int* order, const float* wtop, const uint64_t* ep,
                 const int* ec, int T, int n_used, int inter, int n_in, int n_out, int n_exp,
                 float* out) {
    const int n = T * n_used;
    int* off = (int*)calloc((size_t)n_exp + 1, sizeof(int));
    int* slot = (int*)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
    int* ilist = (int*)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
    int* cur = (int*)malloc(sizeof(int) * (size_t)n_exp);
    /* stable counting sort of assignments i = t*n_used + k by expert (src/m6_moe_tok.c:53-70) */
    for (int i = 0; i < n; i++)
        if (order[i] >= 0 && order[i] < n_exp) off[order[i] + 1]++;
    for (int e = 0; e < n_exp; e++) off[e + 1] += off[e];
    for (int e = 0; e < n_exp; e++) cur[e] = off[e];
    for (int i = 0; i < n; i++) {
        const int e = order[i];
        if (e < 0 || e >= n_exp) continue;
        slot[i] = cur[e] - off[e];
        ilist[cur[e]++] = i;
    }
    float* yd = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * n_out);
    /* per expert: gate/up -> SwiGLU -> down for each of its tokens (src/m6_moe_tok.c:96-146) */
    #pragma omp parallel for schedule(dynamic, 1)
    for (int e = 0; e < n_exp; e++) {
        const int c = off[e + 1] - off[e];
        if (c <= 0) continue;
        float* g = (float*)malloc(sizeof(float) * (size_t)inter);
        float* u = (float*)malloc(sizeof(float) * (size_t)inter);
        for (int j = 0; j < c; j++) {
            const float* xt = X + (size_t)(ilist[off[e] + j] / n_used) * n_in;
            orc_gemv_range(ec[3 * e], xt, (const uint8_t*)(uintptr_t)ep[3 * e], inter, n_in, g, 0, inter);
            orc_gemv_range(ec[3 * e + 1], xt, (const uint8_t*)(uintptr_t)ep[3 * e + 1], inter, n_in, u, 0, inter);
            for (int r = 0; r < inter; r++) g[r] = silu_mul(g[r], u[r]);
            orc_gemv_range(ec[3 * e + 2], g, (const uint8_t*)(uintptr_t)ep[3 * e + 2], n_out, inter,
                           yd + (size_t)(off[e] + j) * n_out, 0, n_out);
        }
        free(g);
        free(u);
    }
    /* per-token combine in k order (src/m6_moe_tok.c:148-159) */
    memset(out, 0, sizeof(float) * (size_t)T * n_out);
    for (int t = 0; t < T; t++) {
        float* o = out + (size_t)t * n_out;
        for (int k = 0; k < n_used; k++) {
            const int i = t * n_used + k, e = order[i];
            if (e < 0 || e >= n_exp) continue;
            const float* y = yd + ((size_t)off[e] + slot[i]) * n_out;
            for (int r = 0; r < n_out; r++) o[r] = fmaf(wtop[i], y[r], o[r]);
        }
    }
    free(off);
    free(slot);
    free(ilist);
    free(cur);
    free(yd);
}

/* ------------------------------- Q8_K activation mode ------------------------------- */

void orc_q8k_quantize(const float* x, int n, float* d, int8_t* q, int16_t* bsums) {
    for (int b = 0; b < n / 256; b++) {
        const float* xb = x + (size_t)b * 256;
        float amax = 0.f;
        for (int i = 0; i < 256; i++) amax = fabsf(xb[i]) > amax ? fabsf(xb[i]) : amax;
        int8_t* qb = q + (size_t)b * 256;
        if (amax == 0.f) {
            d[b] = 0.f;
            memset(qb, 0, 256);
            for (int g = 0; g < 16; g++) bsums[b * 16 + g] = 0;
            continue;
        }
        const float iscale = 127.f / amax;
        for (int i = 0; i < 256; i++) {
            int v = (int)rintf(iscale * xb[i]);
            qb[i] = (int8_t)(v > 127 ? 127 : (v < -127 ? -127 : v));
        }
        d[b] = 1.f / iscale;
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += qb[g * 16 + i];
            bsums[b * 16 + g] = (int16_t)s;
        }
    }
}

void orc_q4k_q8k_block(const uint8_t* blk, const int8_t* q8, const int16_t* bsums,
                       int32_t* isc, int32_t* imn) {
    int32_t a = 0, m = 0;
    for (int j = 0; j < 8; j++) {
        int sc, mn;
        q4k_scale_min(blk + 4, j, &sc, &mn);
        const uint8_t* qb = blk + 16 + (j >> 1) * 32;
        int32_t s = 0;
        for (int k = 0; k < 32; k++) s += ((j & 1) ? (qb[k] >> 4) : (qb[k] & 15)) * (int32_t)q8[j * 32 + k];
        a += sc * s;
        m += mn * ((int32_t)bsums[2 * j] + (int32_t)bsums[2 * j + 1]);
    }
    *isc = a;
    *imn = m;
}

void orc_q6k_q8k_block(const uint8_t* blk, const int8_t* q8, int32_t* isum) {
    const int8_t* sc = (const int8_t*)(blk + 192);
    int32_t acc = 0;
    for (int g = 0; g < 16; g++) {
        int32_t s = 0;
        for (int k = 0; k < 16; k++) {
            const int e = g * 16 + k;
            const uint8_t l = blk[(e >> 7) * 64 + (e & 63)];
            const int lo = ((e >> 6) & 1) ? (l >> 4) : (l & 15);
            const int hi = (blk[128 + (e >> 7) * 32 + (e & 31)] >> (((e >> 5) & 3) * 2)) & 3;
            s += ((lo | (hi << 4)) - 32) * (int32_t)q8[e];
        }
        acc += sc[g] * s;
    }
    *isum = acc;
}

void orc_gemv_q8k(int code, const float* d8, const int8_t* q8, const int16_t* bsums,
                  const uint8_t* W, int n_out, int n_in, float* y) {
    const int nb = n_in / 256;
    const size_t rb = orc_row_bytes(code, n_in);
    #pragma omp parallel for schedule(static) if (n_out >= 256)
    for (int r = 0; r < n_out; r++) {
        float dot = 0.f;
        for (int b = 0; b < nb; b++) {
            if (code == 5) {
                const uint8_t* blk = W + rb * (size_t)r + (size_t)b * 144;
                int32_t isc, imn;
                orc_q4k_q8k_block(blk, q8 + (size_t)b * 256, bsums + b * 16, &isc, &imn);
                const float v = fmaf(ld_f16(blk), (float)isc, -ld_f16(blk + 2) * (float)imn);
                dot = fmaf(d8[b], v, dot);
            } else {
                const uint8_t* blk = W + rb * (size_t)r + (size_t)b * 210;
                int32_t is;
                orc_q6k_q8k_block(blk, q8 + (size_t)b * 256, &is);
                dot = fmaf(d8[b] * ld_f16(blk + 208), (float)is, dot);
            }
        }
        y[r] = dot;
    }
}

/* the host C library's expf over an array (checker for the device replica) */
void orc_expf_array(const float* x, float* y, long n) {
    for (long i = 0; i < n; i++) y[i] = expf(x[i]);
}
