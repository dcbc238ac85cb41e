/* vireo_oracle.c — CPU restatement of vireo's MoE FFN hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker: it is loaded by
 * tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline leg, and
 * never by the product library (vireo_b200/), which must fail loudly when its
 * CUDA build is missing instead of falling back to anything here.
 *
 * It restates the reference algorithm step for step, with the same rounding
 * steps as the reference's AVX2 build (the reference compiles with -std=c11,
 * so plain C expressions are not contracted into FMAs, while its AVX2
 * intrinsics are explicit FMAs).  Reference citations (vireo, src/):
 *   half -> float                 gguf_compute.c:17-36
 *   Q4_K scale/min unpack         gguf_compute.c:45-51
 *   Q4_K / Q5_0 / Q6_K dequant    gguf_compute.c:52-66 / 68-82 / 83-103
 *   gguf_dequant_row              gguf_compute.c:105-124
 *   hsum256, dot_block_q8_0, dot_f32 (8-lane FMA order)  gguf_compute.c:127-157
 *   gguf_matmul                   gguf_compute.c:159-214
 *   block sizes                   gguf.c:27-38
 *   softmax_n                     gguf_run.c:181-182
 *   moe_ffn (router, top-k, renorm, SwiGLU experts, combine, residual)
 *                                 gguf_run.c:185-214
 * Pinned bit-for-bit against the compiled reference by tests/test_oracle.py
 * (golden fixtures in tests/golden/, produced by tests/golden/gen_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ggml wire type ids (gguf.h:20-23 subset). */
enum { OT_F32 = 0, OT_F16 = 1, OT_Q5_0 = 6, OT_Q8_0 = 8, OT_Q4_K = 12, OT_Q6_K = 14 };

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* IEEE binary16 -> binary32, exact for every input (zeros, subnormals, inf,
 * NaN payloads kept in the top mantissa bits). */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 31u) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e == 0u) {
        /* zero or subnormal: value is m * 2^-24, exactly representable */
        float f = (float)m * 0x1p-24f;
        memcpy(&bits, &f, 4);
        bits |= sign;
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float ldh(const uint8_t *p) { uint16_t h; memcpy(&h, p, 2); return orc_f16_to_f32(h); }

/* bytes per block / elements per block (gguf.c:27-38) */
int orc_type_block(uint32_t t, int *be, int *bb) {
    switch (t) {
    case OT_F32: *be = 1; *bb = 4; return 0;
    case OT_F16: *be = 1; *bb = 2; return 0;
    case OT_Q8_0: *be = 32; *bb = 34; return 0;
    case OT_Q5_0: *be = 32; *bb = 22; return 0;
    case OT_Q4_K: *be = 256; *bb = 144; return 0;
    case OT_Q6_K: *be = 256; *bb = 210; return 0;
    default: return -1;
    }
}

/* ---- dequantisation ---------------------------------------------------- */

/* Q4_K super-block (144 B): d f16 @0, dmin f16 @2, 12 packed 6-bit
 * (scale, min) pairs @4, 128 nibble bytes @16.  Sub-block j of 32 values:
 * value = (d*sc_j)*q - (dmin*m_j).  Pairs 0..3 sit in the low 6 bits of
 * bytes 0..3 (scales) and 4..7 (mins); pairs 4..7 take their low nibble from
 * bytes 8..11 and their top two bits from the top bits of bytes 0..7. */
static void q4k_pair(const uint8_t *s, int j, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void deq_q4k(const uint8_t *blk, float *y, int n) {
    for (int b = 0; b < n / 256; b++, blk += 144) {
        float d = ldh(blk), dm = ldh(blk + 2);
        const uint8_t *sc = blk + 4, *qs = blk + 16;
        for (int c = 0; c < 4; c++) { /* 64-value chunk: low nibbles, then high */
            int s0, m0, s1, m1;
            q4k_pair(sc, 2 * c, &s0, &m0);
            q4k_pair(sc, 2 * c + 1, &s1, &m1);
            float dl = d * (float)s0, ml = dm * (float)m0;
            float dh = d * (float)s1, mh = dm * (float)m1;
            for (int l = 0; l < 32; l++) { float t = dl * (float)(qs[32 * c + l] & 15); y[l] = t - ml; }
            for (int l = 0; l < 32; l++) { float t = dh * (float)(qs[32 * c + l] >> 4); y[32 + l] = t - mh; }
            y += 64;
        }
    }
}

/* Q5_0 block (22 B): d f16, 32 high bits (little-endian u32), 16 nibble bytes;
 * value = d * (q5 - 16); element j (<16) low nibble, j+16 high nibble. */
static void deq_q5_0(const uint8_t *blk, float *y, int n) {
    for (int b = 0; b < n / 32; b++, blk += 22, y += 32) {
        float d = ldh(blk);
        uint32_t hi;
        memcpy(&hi, blk + 2, 4);
        const uint8_t *qs = blk + 6;
        for (int j = 0; j < 16; j++) {
            int q0 = (int)((qs[j] & 15) | (((hi >> j) & 1u) << 4)) - 16;
            int q1 = (int)((qs[j] >> 4) | (((hi >> (j + 16)) & 1u) << 4)) - 16;
            y[j] = (float)q0 * d;
            y[j + 16] = (float)q1 * d;
        }
    }
}

/* Q6_K super-block (210 B): 128 low-nibble bytes @0, 64 two-bit bytes @128,
 * 16 int8 scales @192, d f16 @208.  Each 128-value half h uses ql[64h..],
 * qh[32h..], scales[8h..]; within it four 32-value streams s=0..3 take the
 * low/high nibble of ql[l] or ql[l+32] and bit pair s of qh[l]; value =
 * (d*scale)*(q6-32) with one scale per 16 values. */
static void deq_q6k(const uint8_t *blk, float *y, int n) {
    for (int b = 0; b < n / 256; b++, blk += 210) {
        float d = ldh(blk + 208);
        for (int h = 0; h < 2; h++) {
            const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
            const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h);
            for (int l = 0; l < 32; l++) {
                int g = l / 16;
                int q0 = (int)((ql[l] & 15) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q1 = (int)((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q2 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q3 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                float t;
                t = d * (float)sc[g + 0]; y[l] = t * (float)q0;
                t = d * (float)sc[g + 2]; y[l + 32] = t * (float)q1;
                t = d * (float)sc[g + 4]; y[l + 64] = t * (float)q2;
                t = d * (float)sc[g + 6]; y[l + 96] = t * (float)q3;
            }
            y += 128;
        }
    }
}

/* Returns 0 when the type is one the reference dequantises, -1 otherwise
 * (the reference leaves dst untouched in that case). */
int orc_dequant_row(uint32_t type, const void *src, float *dst, int n) {
    const uint8_t *p = (const uint8_t *)src;
    switch (type) {
    case OT_F32: memcpy(dst, src, (size_t)n * 4); return 0;
    case OT_F16:
        for (int i = 0; i < n; i++) dst[i] = ldh(p + 2 * i);
        return 0;
    case OT_Q8_0:
        for (int b = 0; b < n / 32; b++) {
            float d = ldh(p + 34 * b);
            const int8_t *q = (const int8_t *)(p + 34 * b + 2);
            for (int i = 0; i < 32; i++) dst[32 * b + i] = (float)q[i] * d;
        }
        return 0;
    case OT_Q5_0: deq_q5_0(p, dst, n); return 0;
    case OT_Q4_K: deq_q4k(p, dst, n); return 0;
    case OT_Q6_K: deq_q6k(p, dst, n); return 0;
    default: return -1;
    }
}

/* ---- dot products in the reference's 8-lane AVX2 order ----------------- */

/* horizontal sum of 8 lanes: fold the upper four onto the lower four, then
 * (l0+l1)+(l2+l3) — the reduction tree of the reference's hsum256 */
static inline float hsum8(const float v[8]) {
    float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
    float s01 = a0 + a1, s23 = a2 + a3;
    return s01 + s23;
}

static inline float dot_q8_block(const int8_t *q, const float *x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < 4; k++)
        for (int l = 0; l < 8; l++) acc[l] = fmaf((float)q[8 * k + l], x[8 * k + l], acc[l]);
    return hsum8(acc);
}

static inline float dot_lanes(const float *a, const float *b, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s = hsum8(acc);
    for (; i < n; i++) { float t = a[i] * b[i]; s = s + t; }
    return s;
}

/* y[o] = sum_i W[o,i] * x[i] for o < d; W row-major, d rows of n values in
 * the given block format.  Returns -1 for an unsupported type (y untouched). */
int orc_matmul(float *y, const float *x, uint32_t type, const void *data, int n, int d) {
    const uint8_t *base = (const uint8_t *)data;
    int be, bb;
    if (orc_type_block(type, &be, &bb)) return -1;
    size_t row_bytes = (size_t)(n / be) * bb;
    if (type == OT_Q8_0) {
#pragma omp parallel for schedule(static) if ((long)n * (long)d > (1L << 20))
        for (int o = 0; o < d; o++) {
            const uint8_t *row = base + (size_t)o * row_bytes;
            float acc = 0.0f;
            for (int j = 0; j < n / 32; j++) {
                float ds = ldh(row + 34 * j);
                float t = dot_q8_block((const int8_t *)(row + 34 * j + 2), x + 32 * j) * ds;
                acc = acc + t;
            }
            y[o] = acc;
        }
        return 0;
    }
    if (type == OT_F32 || type == OT_F16) {
#pragma omp parallel for schedule(static) if ((long)n * (long)d > (1L << 20))
        for (int o = 0; o < d; o++) {
            const uint8_t *row = base + (size_t)o * row_bytes;
            float acc = 0.0f;
            for (int i = 0; i < n; i++) {
                float w;
                if (type == OT_F32) memcpy(&w, row + 4 * i, 4);
                else w = ldh(row + 2 * i);
                float t = w * x[i];
                acc = acc + t;
            }
            y[o] = acc;
        }
        return 0;
    }
    /* block-quantised: dequantise the row, then the 8-lane dot */
#pragma omp parallel for schedule(static) if ((long)n * (long)d > (1L << 20))
    for (int o = 0; o < d; o++) {
        float *tmp = (float *)malloc((size_t)n * sizeof(float));
        orc_dequant_row(type, base + (size_t)o * row_bytes, tmp, n);
        y[o] = dot_lanes(tmp, x, n);
        free(tmp);
    }
    return 0;
}

/* ---- MoE FFN block ------------------------------------------------------ */

typedef struct {
    int dim, ffn_exp, n_experts, n_used, topk_renorm;
    uint32_t router_type, gate_type, up_type, down_type;
    const void *router;            /* [n_experts][dim] */
    const void *gate, *up, *down;  /* 3-D expert tensors, expert outermost */
    uint64_t gate_nbytes, up_nbytes, down_nbytes;
} orc_moe_layer;

/* softmax over n values in place: running max, exp, sequential sum, divide */
static void softmax_inplace(float *v, int n) {
    float m = v[0];
    for (int i = 1; i < n; i++) if (v[i] > m) m = v[i];
    float s = 0.0f;
    for (int i = 0; i < n; i++) { v[i] = expf(v[i] - m); s = s + v[i]; }
    for (int i = 0; i < n; i++) v[i] = v[i] / s;
}

/* One expert's FFN for one token (gguf_run.c:202-208): gate and up mat-vecs,
 * SwiGLU h = g / (1 + expf(-g)) * u, down mat-vec into dn [dim].  g and u
 * are [ffn_exp] work buffers (g ends holding h). */
static void expert_ffn(const orc_moe_layer *L, int e, const float *hb, float *g, float *u, float *dn) {
    int d = L->dim, fe = L->ffn_exp, ne = L->n_experts;
    uint64_t gs = L->gate_nbytes / (uint64_t)ne, us = L->up_nbytes / (uint64_t)ne,
             ds = L->down_nbytes / (uint64_t)ne;
    orc_matmul(g, hb, L->gate_type, (const uint8_t *)L->gate + (uint64_t)e * gs, d, fe);
    orc_matmul(u, hb, L->up_type, (const uint8_t *)L->up + (uint64_t)e * us, d, fe);
    for (int i = 0; i < fe; i++) {
        float gi = g[i];
        float den = 1.0f + expf(-gi);
        float s = gi / den;
        g[i] = s * u[i];
    }
    orc_matmul(dn, g, L->down_type, (const uint8_t *)L->down + (uint64_t)e * ds, fe, d);
}

/* expert_ffn for callers (the expert-parallel dataflow tests run one expert
 * at a time on the rank that holds it); returns -1 for a bad expert id. */
int orc_expert_ffn(const orc_moe_layer *L, int e, const float *hb, float *dn) {
    if (e < 0 || e >= L->n_experts) return -1;
    float *g = (float *)malloc(sizeof(float) * (size_t)L->ffn_exp);
    float *u = (float *)malloc(sizeof(float) * (size_t)L->ffn_exp);
    expert_ffn(L, e, hb, g, u, dn);
    free(g); free(u);
    return 0;
}

/* One token through the MoE FFN.  hb: normalised hidden [dim]; x: residual
 * [dim], updated in place (x += sum_t w_t * expert_t(hb)).  ids/wts receive
 * the selected experts in rank order and their gate weights (after renorm).
 * probs (optional, [n_experts]) receives the softmax probabilities.
 * Returns the number of experts used (min(n_used, 64)). */
int orc_moe_ffn_bias(const orc_moe_layer *L, const float *hb, float *x, int32_t *ids, float *wts,
                     float *probs, const float *bias);
int orc_moe_ffn(const orc_moe_layer *L, const float *hb, float *x, int32_t *ids, float *wts,
                float *probs) {
    return orc_moe_ffn_bias(L, hb, x, ids, wts, probs, NULL);
}

/* The same with a per-expert bias added to the router logits before the
 * softmax (the imbalanced-routing configuration adds it in its harness; the
 * reference has no bias, and bias == NULL is exactly orc_moe_ffn). */
/* Routing of one token (gguf_run.c:187-192): router mat-vec, optional
 * per-expert bias, softmax, greedy top-k (k passes of a strict '>' argmax
 * over the unused experts, starting from -1, so ties go to the lowest id),
 * optional renormalisation by the sequential sum of the selected weights.
 * idx/w receive min(n_used, 64) entries; probs (optional) the softmax. */
static int route_token(const orc_moe_layer *L, const float *hb, const float *bias, int *idx, float *w,
                       float *probs) {
    int d = L->dim, ne = L->n_experts, k = L->n_used;
    int kk = k < 64 ? k : 64;
    float *rl = (float *)malloc(sizeof(float) * (size_t)ne);
    orc_matmul(rl, hb, L->router_type, L->router, d, ne);
    if (bias) for (int e = 0; e < ne; e++) rl[e] = rl[e] + bias[e];
    softmax_inplace(rl, ne);
    if (probs) memcpy(probs, rl, sizeof(float) * (size_t)ne);
    for (int t = 0; t < kk; t++) {
        int best = -1;
        float bv = -1.0f;
        for (int e = 0; e < ne; e++) {
            int used = 0;
            for (int j = 0; j < t; j++) if (idx[j] == e) { used = 1; break; }
            if (!used && rl[e] > bv) { bv = rl[e]; best = e; }
        }
        idx[t] = best;
        w[t] = bv;
    }
    if (L->topk_renorm) {
        float ws = 0.0f;
        for (int t = 0; t < kk; t++) ws = ws + w[t];
        if (ws > 0) for (int t = 0; t < kk; t++) w[t] = w[t] / ws;
    }
    free(rl);
    return kk;
}

int orc_moe_ffn_bias(const orc_moe_layer *L, const float *hb, float *x, int32_t *ids, float *wts,
                     float *probs, const float *bias) {
    int d = L->dim, fe = L->ffn_exp;
    float *g = (float *)malloc(sizeof(float) * (size_t)fe);
    float *u = (float *)malloc(sizeof(float) * (size_t)fe);
    float *dn = (float *)malloc(sizeof(float) * (size_t)d);
    float *acc = (float *)calloc((size_t)d, sizeof(float));
    int idx[64];
    float w[64];
    int kk = route_token(L, hb, bias, idx, w, probs);
    for (int t = 0; t < kk; t++) {
        int e = idx[t];
        if (e < 0) continue;
        expert_ffn(L, e, hb, g, u, dn);
        for (int i = 0; i < d; i++) { float t2 = w[t] * dn[i]; acc[i] = acc[i] + t2; }
    }
    for (int i = 0; i < d; i++) x[i] = x[i] + acc[i];
    if (ids) for (int t = 0; t < kk; t++) ids[t] = idx[t];
    if (wts) for (int t = 0; t < kk; t++) wts[t] = w[t];
    free(g); free(u); free(dn); free(acc);
    return kk;
}

/* n_tok tokens, one after another (each independent, as separate decode
 * tokens through one layer).  hb: [n_tok][dim]; x: [n_tok][dim] in/out;
 * ids/wts: [n_tok][n_used] (may be NULL). */
int orc_moe_ffn_batch(const orc_moe_layer *L, int n_tok, const float *hb, float *x,
                      int32_t *ids, float *wts) {
    int kk = L->n_used < 64 ? L->n_used : 64;
    for (int t = 0; t < n_tok; t++)
        orc_moe_ffn(L, hb + (size_t)t * L->dim, x + (size_t)t * L->dim,
                    ids ? ids + (size_t)t * kk : NULL, wts ? wts + (size_t)t * kk : NULL, NULL);
    return kk;
}

/* orc_moe_ffn_batch with a router bias (NULL = none); tokens in parallel
 * (each token's computation is independent and sequential in itself, so the
 * results do not depend on the thread count). */
int orc_moe_ffn_batch_bias(const orc_moe_layer *L, int n_tok, const float *hb, float *x,
                           int32_t *ids, float *wts, const float *bias) {
    int kk = L->n_used < 64 ? L->n_used : 64;
    int saved = orc_max_threads();
    orc_set_threads(1);  /* one thread per token below; no nested parallel mat-vecs */
    #pragma omp parallel for schedule(dynamic, 1) num_threads(saved)
    for (int t = 0; t < n_tok; t++)
        orc_moe_ffn_bias(L, hb + (size_t)t * L->dim, x + (size_t)t * L->dim,
                         ids ? ids + (size_t)t * kk : NULL, wts ? wts + (size_t)t * kk : NULL, NULL, bias);
    orc_set_threads(saved);
    return kk;
}

/* Routing alone for n_tok tokens (route_token per token, tokens in
 * parallel; bias may be NULL): ids/wts [n_tok][min(n_used, 64)]. */
int orc_route_batch_bias(const orc_moe_layer *L, int n_tok, const float *hb, int32_t *ids, float *wts,
                         const float *bias) {
    int kk = L->n_used < 64 ? L->n_used : 64;
    int saved = orc_max_threads();
    orc_set_threads(1);
    #pragma omp parallel for schedule(dynamic, 16) num_threads(saved)
    for (int t = 0; t < n_tok; t++) {
        int idx[64];
        float w[64];
        route_token(L, hb + (size_t)t * L->dim, bias, idx, w, NULL);
        for (int j = 0; j < kk; j++) {
            ids[(size_t)t * kk + j] = idx[j];
            wts[(size_t)t * kk + j] = w[j];
        }
    }
    orc_set_threads(saved);
    return kk;
}
