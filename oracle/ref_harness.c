/* ref_harness.c — drives the reference's own CPU MoE path.
 *
 * TEST INFRASTRUCTURE ONLY (checker and CPU baseline; never product code).
 * Compiled by oracle/Makefile together with the reference's unmodified
 * sources (src/gguf.c, src/gguf_compute.c, src/expert_store.c and the KV
 * sources gguf_run.c links against) into oracle/_ref/libvireo_ref.so.
 *
 * The reference's MoE block, moe_ffn (src/gguf_run.c:185-214), is a static
 * function, so this file includes src/gguf_run.c with its main() renamed and
 * calls moe_ffn directly on a Model whose MoE fields are filled here.  The
 * expert weights are written to an anonymous file and registered with the
 * reference ExpertStore exactly as gguf_run.c:325-331 does (expert e of each
 * 3-D tensor at base + e * (nbytes / n_experts)), so every lookup, pread and
 * eviction is the reference's own.  expert_store_lookup is routed through a
 * recording hook (same signature, forwards to the real function) so the
 * selected expert ids can be read back in rank order.
 */
#define _GNU_SOURCE
#define main vireo_gguf_main
#define expert_store_lookup ref_hook_lookup
#include "gguf_run.c"
#undef expert_store_lookup
#undef main

#include <sys/mman.h>
#include <unistd.h>

int expert_store_lookup(ExpertStore *s, int layer, int expert, ExpertView *view);

static int g_rec_ids[64];
static int g_rec_n;

/* Routing margin of the decoder forward() in progress: at the first lookup
 * of each layer, m->rlog holds that layer's router softmax (gguf_run.c:
 * 187-188, the top-k scan :191 has just run); the smallest log-probability
 * gap among its n_used + 1 largest values is recorded.  A gap near zero is
 * a near-tie, where any other summation order may pick another expert. */
static Model *g_gap_model;
static int g_gap_layer;
static double g_gap_min;

static double topk_log_gap(const float *p, int ne, int k) {
    float top[65];
    int n = k + 1 < ne ? k + 1 : ne;
    if (n > 65) n = 65;
    for (int i = 0; i < n; i++) top[i] = -1.0f;
    for (int e = 0; e < ne; e++) {
        float v = p[e];
        for (int i = 0; i < n; i++)
            if (v > top[i]) { float t = top[i]; top[i] = v; v = t; }
    }
    double g = INFINITY;
    for (int i = 0; i + 1 < n; i++) {
        if (top[i + 1] <= 0.0f) break;
        double d = log((double)top[i]) - log((double)top[i + 1]);
        if (d < g) g = d;
    }
    return g;
}

int ref_hook_lookup(ExpertStore *s, int layer, int expert, ExpertView *view) {
    if (g_rec_n < 64) g_rec_ids[g_rec_n] = expert;
    g_rec_n++;
    if (g_gap_model && layer != g_gap_layer) {
        g_gap_layer = layer;
        double g = topk_log_gap(g_gap_model->rlog, g_gap_model->n_experts, g_gap_model->n_used);
        if (g < g_gap_min) g_gap_min = g;
    }
    return expert_store_lookup(s, layer, expert, view);
}

typedef struct {
    Model m;
    gguf_ctx g;
    Layer ly;
    gguf_tensor router, gate, up, down;
    int fd;
    void *anchor;
} RefMoe;

void ref_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int ref_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int write_all(int fd, const void *p, uint64_t n, uint64_t off) {
    const uint8_t *b = (const uint8_t *)p;
    while (n) {
        ssize_t w = pwrite(fd, b, n > (1u << 30) ? (1u << 30) : n, (off_t)off);
        if (w <= 0) return -1;
        b += w; n -= (uint64_t)w; off += (uint64_t)w;
    }
    return 0;
}

/* One MoE layer (layer index 0) with the given tensors.  cap_bytes is the
 * ExpertStore budget (0 = unbounded), as VIREO_EXPERT_CAP_MB sets it. */
RefMoe *ref_moe_create(int dim, int ffn_exp, int n_experts, int n_used, int renorm,
                       uint32_t router_type, const void *router, uint64_t router_nbytes,
                       uint32_t gate_type, const void *gate, uint64_t gate_nbytes,
                       uint32_t up_type, const void *up, uint64_t up_nbytes,
                       uint32_t down_type, const void *down, uint64_t down_nbytes,
                       uint64_t cap_bytes) {
    RefMoe *r = (RefMoe *)calloc(1, sizeof(RefMoe));
    if (!r) return NULL;
    r->fd = memfd_create("vireo_ref_experts", 0);
    if (r->fd < 0) { free(r); return NULL; }
    uint64_t off_g = 0, off_u = gate_nbytes, off_d = gate_nbytes + up_nbytes;
    if (write_all(r->fd, gate, gate_nbytes, off_g) || write_all(r->fd, up, up_nbytes, off_u) ||
        write_all(r->fd, down, down_nbytes, off_d)) {
        close(r->fd); free(r); return NULL;
    }
    /* tensors: data pointers only feed the (unused) base-offset arithmetic in
     * moe_ffn; expert bytes come from the ExpertStore. */
    r->anchor = malloc(16);
    r->g.map = r->anchor;
    r->router.data = router; r->router.ggml_type = router_type; r->router.nbytes = router_nbytes;
    r->gate.data = r->anchor; r->gate.ggml_type = gate_type; r->gate.nbytes = gate_nbytes;
    r->up.data = r->anchor; r->up.ggml_type = up_type; r->up.nbytes = up_nbytes;
    r->down.data = r->anchor; r->down.ggml_type = down_type; r->down.nbytes = down_nbytes;
    r->ly.router = &r->router; r->ly.gate_exps = &r->gate; r->ly.up_exps = &r->up; r->ly.down_exps = &r->down;
    Model *m = &r->m;
    m->g = &r->g;
    m->L = &r->ly;
    m->n_layers = 1;
    m->dim = dim; m->ffn_exp = ffn_exp; m->n_experts = n_experts; m->n_used = n_used;
    m->topk_renorm = renorm; m->is_moe = 1; m->exp_type = gate_type;
    m->rlog = (float *)malloc(sizeof(float) * (size_t)n_experts);
    m->gbuf = (float *)malloc(sizeof(float) * (size_t)ffn_exp);
    m->ubuf = (float *)malloc(sizeof(float) * (size_t)ffn_exp);
    m->dbuf = (float *)malloc(sizeof(float) * (size_t)dim);
    m->moe_acc = (float *)malloc(sizeof(float) * (size_t)dim);
    m->es = expert_store_create(r->fd, cap_bytes, 1, n_experts);
    uint32_t gs = (uint32_t)(gate_nbytes / (uint64_t)n_experts);
    uint32_t us = (uint32_t)(up_nbytes / (uint64_t)n_experts);
    uint32_t ds = (uint32_t)(down_nbytes / (uint64_t)n_experts);
    for (int e = 0; e < n_experts; e++) {
        ExpertSlices sl = {off_g + (uint64_t)e * gs, off_u + (uint64_t)e * us, off_d + (uint64_t)e * ds,
                           gs, us, ds};
        expert_store_register(m->es, 0, e, &sl);
    }
    return r;
}

/* Runs the reference moe_ffn for one token.  hb: normalised hidden [dim]
 * (not modified by the reference); x: residual [dim] in/out.  ids/wts get
 * the experts the reference looked up, in rank order, and their gate
 * weights (softmax probabilities, renormalised as moe_ffn does when
 * topk_renorm is set).  Returns the number of experts looked up. */
int ref_moe_ffn(RefMoe *r, const float *hb, float *x, int32_t *ids, float *wts) {
    Model *m = &r->m;
    float *hcopy = (float *)malloc(sizeof(float) * (size_t)m->dim);
    memcpy(hcopy, hb, sizeof(float) * (size_t)m->dim);
    m->x = x;
    g_rec_n = 0;
    moe_ffn(m, 0, hcopy);
    free(hcopy);
    int n = g_rec_n < 64 ? g_rec_n : 64;
    if (ids) for (int t = 0; t < n; t++) ids[t] = g_rec_ids[t];
    if (wts) {
        /* after moe_ffn, m->rlog holds the softmax probabilities */
        float ws = 0.0f;
        for (int t = 0; t < n; t++) { wts[t] = m->rlog[g_rec_ids[t]]; ws = ws + wts[t]; }
        if (m->topk_renorm && ws > 0) for (int t = 0; t < n; t++) wts[t] = wts[t] / ws;
    }
    return n;
}

/* n_tok independent tokens through the layer, one moe_ffn call each. */
int ref_moe_ffn_batch(RefMoe *r, int n_tok, const float *hb, float *x, int32_t *ids, float *wts) {
    int k = r->m.n_used < 64 ? r->m.n_used : 64;
    for (int t = 0; t < n_tok; t++)
        ref_moe_ffn(r, hb + (size_t)t * r->m.dim, x + (size_t)t * r->m.dim,
                    ids ? ids + (size_t)t * k : NULL, wts ? wts + (size_t)t * k : NULL);
    return k;
}

void ref_moe_stats(RefMoe *r, ExpertStats *st) { expert_store_stats(r->m.es, st); }

void ref_moe_destroy(RefMoe *r) {
    if (!r) return;
    Model *m = &r->m;
    expert_store_destroy(m->es);
    free(m->rlog); free(m->gbuf); free(m->ubuf); free(m->dbuf); free(m->moe_acc);
    free(r->anchor);
    close(r->fd);
    free(r);
}

/* gguf_matmul on a bare tensor (type + data), as moe_ffn builds them
 * (gguf_run.c:202-204). */
void ref_matmul(float *y, const float *x, uint32_t type, const void *data, int n, int d) {
    gguf_tensor t;
    memset(&t, 0, sizeof(t));
    t.data = data;
    t.ggml_type = type;
    gguf_matmul(y, x, &t, n, d);
}

/* ---- whole decode steps: the reference's forward() (gguf_run.c:216-252) ----
 * A Model built here from caller-owned tensors (the fields main() fills from
 * GGUF metadata, gguf_run.c:276-293, 297-333), with the reference's dense KV
 * store (exact attention, src/kvstore_dense.c) and its ExpertStore over an
 * anonymous file holding every layer's experts. */
typedef struct {
    uint32_t type;
    const void *data;
    uint64_t nbytes;
    uint64_t dim0;
} RefTensorIn;

enum { RT_ATTN_NORM, RT_WQ, RT_WK, RT_WV, RT_WO, RT_FFN_NORM, RT_Q_NORM, RT_K_NORM, RT_ROUTER, RT_GATE, RT_UP,
       RT_DOWN, RT_N };

typedef struct {
    Model m;
    gguf_ctx g;
    gguf_tensor tok_embd, out_norm, lm_head;
    gguf_tensor *lt;  /* [n_layers][RT_N] */
    int fd;
    void *anchor;
} RefDec;

static void ref_tensor(gguf_tensor *t, const RefTensorIn *in) {
    memset(t, 0, sizeof(*t));
    t->data = in->data;
    t->ggml_type = in->type;
    t->nbytes = in->nbytes;
    t->dims[0] = in->dim0;
    t->n_dims = 1;
}

RefDec *ref_decoder_create(int n_layers, int dim, int n_heads, int n_kv_heads, int head_size, int vocab, float eps,
                           float rope_base, int n_experts, int n_used, int ffn_exp, int topk_renorm,
                           const RefTensorIn *tok_embd, const RefTensorIn *out_norm, const RefTensorIn *lm_head,
                           const RefTensorIn *layers) {
    RefDec *r = (RefDec *)calloc(1, sizeof(RefDec));
    if (!r) return NULL;
    r->fd = memfd_create("vireo_ref_decoder_experts", 0);
    if (r->fd < 0) { free(r); return NULL; }
    r->anchor = malloc(16);
    r->g.map = r->anchor;
    r->lt = (gguf_tensor *)calloc((size_t)n_layers * RT_N, sizeof(gguf_tensor));
    Model *m = &r->m;
    m->g = &r->g;
    m->n_layers = n_layers; m->dim = dim; m->n_heads = n_heads; m->n_kv_heads = n_kv_heads;
    m->head_size = head_size; m->vocab = vocab; m->eps = eps; m->rope_base = rope_base; m->ffn = ffn_exp;
    m->is_moe = 1; m->n_experts = n_experts; m->n_used = n_used; m->ffn_exp = ffn_exp; m->topk_renorm = topk_renorm;
    ref_tensor(&r->tok_embd, tok_embd);
    ref_tensor(&r->out_norm, out_norm);
    ref_tensor(&r->lm_head, lm_head);
    m->tok_embd = &r->tok_embd; m->out_norm = &r->out_norm; m->lm_head = &r->lm_head;
    m->L = (Layer *)calloc((size_t)n_layers, sizeof(Layer));
    uint64_t off = 0;
    m->es = expert_store_create(r->fd, 0, n_layers, n_experts);
    for (int l = 0; l < n_layers; l++) {
        gguf_tensor *t = r->lt + (size_t)l * RT_N;
        const RefTensorIn *in = layers + (size_t)l * RT_N;
        for (int i = 0; i < RT_N; i++) ref_tensor(&t[i], &in[i]);
        Layer *ly = &m->L[l];
        ly->attn_norm = &t[RT_ATTN_NORM]; ly->wq = &t[RT_WQ]; ly->wk = &t[RT_WK]; ly->wv = &t[RT_WV];
        ly->wo = &t[RT_WO]; ly->ffn_norm = &t[RT_FFN_NORM];
        ly->q_norm = in[RT_Q_NORM].data ? &t[RT_Q_NORM] : NULL;
        ly->k_norm = in[RT_K_NORM].data ? &t[RT_K_NORM] : NULL;
        ly->router = &t[RT_ROUTER];
        /* expert tensors: bytes come from the ExpertStore; data only feeds
         * the (unused) base-offset arithmetic in moe_ffn */
        uint64_t og = off, ou = og + in[RT_GATE].nbytes, od = ou + in[RT_UP].nbytes;
        if (write_all(r->fd, in[RT_GATE].data, in[RT_GATE].nbytes, og) ||
            write_all(r->fd, in[RT_UP].data, in[RT_UP].nbytes, ou) ||
            write_all(r->fd, in[RT_DOWN].data, in[RT_DOWN].nbytes, od))
            return NULL;
        off = od + in[RT_DOWN].nbytes;
        t[RT_GATE].data = r->anchor; t[RT_UP].data = r->anchor; t[RT_DOWN].data = r->anchor;
        ly->gate_exps = &t[RT_GATE]; ly->up_exps = &t[RT_UP]; ly->down_exps = &t[RT_DOWN];
        uint32_t gs = (uint32_t)(in[RT_GATE].nbytes / (uint64_t)n_experts);
        uint32_t us = (uint32_t)(in[RT_UP].nbytes / (uint64_t)n_experts);
        uint32_t ds = (uint32_t)(in[RT_DOWN].nbytes / (uint64_t)n_experts);
        for (int e = 0; e < n_experts; e++) {
            ExpertSlices sl = {og + (uint64_t)e * gs, ou + (uint64_t)e * us, od + (uint64_t)e * ds, gs, us, ds};
            expert_store_register(m->es, l, e, &sl);
        }
    }
    m->exp_type = r->lt[RT_GATE].ggml_type;
    KVConfig cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.n_layers = n_layers * n_kv_heads;
    cfg.kv_dim = head_size;
    m->kv = kvstore_dense_create(cfg);
    m->x = malloc(dim * 4); m->xb = malloc(dim * 4);
    m->q = malloc((size_t)n_heads * head_size * 4); m->k = malloc((size_t)n_kv_heads * head_size * 4);
    m->v = malloc((size_t)n_kv_heads * head_size * 4); m->att_out = malloc((size_t)n_heads * head_size * 4);
    m->logits = malloc((size_t)vocab * 4);
    m->rlog = malloc((size_t)n_experts * 4); m->gbuf = malloc((size_t)ffn_exp * 4);
    m->ubuf = malloc((size_t)ffn_exp * 4); m->dbuf = malloc((size_t)dim * 4); m->moe_acc = malloc((size_t)dim * 4);
    return r;
}

/* forward(m, token, pos, want_logits); logits_out [vocab] (when want_logits)
 * and x_out [dim] (the residual stream) may be NULL. */
int ref_decoder_forward(RefDec *r, int token, int pos, int want_logits, float *logits_out, float *x_out) {
    Model *m = &r->m;
    g_gap_model = m;
    g_gap_layer = -1;
    g_gap_min = INFINITY;
    float *lg = forward(m, token, pos, want_logits);
    g_gap_model = NULL;
    if (lg && logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)m->vocab);
    if (x_out) memcpy(x_out, m->x, sizeof(float) * (size_t)m->dim);
    return lg ? argmax(lg, m->vocab) : -1;
}

/* Positions [0, n_pos) of every (layer, kv head) of the reference's dense KV
 * store filled through its own kv_append (src/kvstore.h:60-63) with seeded
 * vectors (each value the sum of four uniforms on [-0.5, 0.5), so about
 * N(0, 1/3)): the state a prompt of n_pos tokens leaves, for timing decode
 * steps at that context without running the prompt (CPU baseline only; the
 * values steer nothing but the softmax weights). */
void ref_decoder_fill_kv(RefDec *r, int n_pos, uint64_t seed) {
    Model *m = &r->m;
    int hs = m->head_size;
    float *k = (float *)malloc(sizeof(float) * (size_t)hs);
    float *v = (float *)malloc(sizeof(float) * (size_t)hs);
    uint64_t z = seed * 0x9E3779B97F4A7C15ull + 1;
    for (int l = 0; l < m->n_layers; l++)
        for (int kh = 0; kh < m->n_kv_heads; kh++)
            for (int pos = 0; pos < n_pos; pos++) {
                for (int i = 0; i < 2 * hs; i++) {
                    float a = 0.0f;
                    for (int j = 0; j < 4; j++) {
                        z = z * 6364136223846793005ull + 1442695040888963407ull;
                        a += (float)(z >> 40) * (1.0f / 16777216.0f) - 0.5f;
                    }
                    if (i < hs) k[i] = a; else v[i - hs] = a;
                }
                kv_append(m->kv, l * m->n_kv_heads + kh, pos, k, v);
            }
    free(k); free(v);
}

/* The smallest router log-probability gap among the top n_used + 1 experts
 * over every layer of the last ref_decoder_forward call. */
double ref_decoder_last_gap(void) { return g_gap_min; }

void ref_decoder_destroy(RefDec *r) {
    if (!r) return;
    Model *m = &r->m;
    kv_destroy(m->kv);
    expert_store_destroy(m->es);
    free(m->x); free(m->xb); free(m->q); free(m->k); free(m->v); free(m->att_out); free(m->logits);
    free(m->rlog); free(m->gbuf); free(m->ubuf); free(m->dbuf); free(m->moe_acc);
    free(m->L); free(r->lt); free(r->anchor);
    close(r->fd);
    free(r);
}
