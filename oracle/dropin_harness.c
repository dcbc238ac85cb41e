/* dropin_harness.c — the reference's decoder, opened from a GGUF file.
 *
 * TEST INFRASTRUCTURE ONLY (a checker; never product code).  oracle/
 * dropin.py compiles it twice against the reference's unmodified sources:
 *
 *   _ref/dropin_ref.so   src/gguf_run.c + gguf.c + gguf_compute.c +
 *                        expert_store.c + the KV sources: the reference as
 *                        it ships.
 *   _ref/dropin_b200.so  (VIREO_DROPIN) the same with gguf_compute.c and
 *                        expert_store.c dropped and libvireo_b200.so linked
 *                        in their place, and gguf_run.c given the one-line
 *                        hook at the top of moe_ffn that the integration
 *                        notes describe (added to a temporary copy of the
 *                        file at build time; the reference tree is not
 *                        modified): the MoE block of every layer runs as one
 *                        gguf_moe_ffn_host call.
 *
 * Both load a model as the runner's main() does (src/gguf_run.c:270-341:
 * gguf_open, the "<arch>.*" keys, the tensors by name, the ExpertStore over
 * the file's descriptor with one slice per expert), except that the KV
 * store is the dense one (src/kvstore_dense.c: exact attention, no block
 * selection), and expose forward() (src/gguf_run.c:216-252) one step at a
 * time.  gguf_run.c is included with its main() renamed.
 */
#define _GNU_SOURCE
#define main vireo_gguf_main
#include "gguf_run.c"
#undef main

#ifdef VIREO_DROPIN
#include "gguf_moe.h"
#include "gguf_compute.h"

int gguf_weights_register(const void *host, uint64_t nbytes);

static gguf_moe **g_moe;  /* one handle per layer, made at the layer's first token */
static long g_hook_calls;

/* The hook at the top of moe_ffn: the whole block on the GPU.  Returns 0
 * (the reference's own body runs) when the layer's shape is not on the
 * device path or a call fails. */
static int vireo_moe_hook(Model *m, int layer, float *hb) {
    if (!g_moe) g_moe = (gguf_moe **)calloc((size_t)m->n_layers, sizeof(*g_moe));
    if (!g_moe[layer]) {
        const Layer *ly = &m->L[layer];
        gguf_moe_desc d;
        memset(&d, 0, sizeof(d));
        d.dim = m->dim;
        d.ffn_exp = m->ffn_exp;
        d.n_experts = m->n_experts;
        d.n_used = m->n_used;
        d.topk_renorm = m->topk_renorm;
        d.router_type = ly->router->ggml_type;
        d.gate_type = ly->gate_exps->ggml_type;
        d.up_type = ly->up_exps->ggml_type;
        d.down_type = ly->down_exps->ggml_type;
        d.router = ly->router->data;
        d.gate_exps = ly->gate_exps->data;
        d.up_exps = ly->up_exps->data;
        d.down_exps = ly->down_exps->data;
        d.gate_nbytes = ly->gate_exps->nbytes;
        d.up_nbytes = ly->up_exps->nbytes;
        d.down_nbytes = ly->down_exps->nbytes;
        if (gguf_moe_create_host(&d, &g_moe[layer]) != VIREO_OK) return 0;
    }
    if (gguf_moe_ffn_host(g_moe[layer], hb, m->x, 1, NULL, NULL) != VIREO_OK) return 0;
    g_hook_calls++;
    return 1;
}
#endif

/* MoE blocks run through the hook so far (0 in the reference build). */
long dropin_hook_calls(void) {
#ifdef VIREO_DROPIN
    return g_hook_calls;
#else
    return 0;
#endif
}

typedef struct {
    Model m;
    gguf_ctx *g;
} DropIn;

static int read_u(const gguf_ctx *g, const char *arch, const char *suffix, int *out) {
    char key[160];
    uint64_t u;
    snprintf(key, sizeof(key), "%s.%s", arch, suffix);
    if (gguf_get_u64(g, key, &u)) return -1;
    *out = (int)u;
    return 0;
}

static void read_f(const gguf_ctx *g, const char *arch, const char *suffix, float *out) {
    char key[160];
    snprintf(key, sizeof(key), "%s.%s", arch, suffix);
    gguf_get_f32(g, key, out);
}

DropIn *dropin_open(const char *path) {
    gguf_ctx *g = gguf_open(path);
    if (!g) return NULL;
    DropIn *r = (DropIn *)calloc(1, sizeof(DropIn));
    Model *m = &r->m;
    r->g = g;
    m->g = g;
    char arch[64] = "qwen2";
    uint64_t alen;
    const char *a = gguf_get_str(g, "general.architecture", &alen);
    if (a) {
        size_t n = alen < 63 ? alen : 63;
        memcpy(arch, a, n);
        arch[n] = 0;
    }
    /* shapes (gguf_run.c:276-293) */
    read_u(g, arch, "block_count", &m->n_layers);
    read_u(g, arch, "embedding_length", &m->dim);
    read_u(g, arch, "feed_forward_length", &m->ffn);
    read_u(g, arch, "attention.head_count", &m->n_heads);
    read_u(g, arch, "attention.head_count_kv", &m->n_kv_heads);
    read_f(g, arch, "attention.layer_norm_rms_epsilon", &m->eps);
    m->rope_base = 10000.0f;
    read_f(g, arch, "rope.freq_base", &m->rope_base);
    m->head_size = m->dim / m->n_heads;
    read_u(g, arch, "attention.key_length", &m->head_size);
    int ne = 0;
    if (read_u(g, arch, "expert_count", &ne) == 0 && ne > 0) {
        m->is_moe = 1;
        m->n_experts = ne;
        m->n_used = 8;
        read_u(g, arch, "expert_used_count", &m->n_used);
        m->ffn_exp = m->ffn;
        read_u(g, arch, "expert_feed_forward_length", &m->ffn_exp);
        m->topk_renorm = strcmp(arch, "olmoe") != 0;
        read_u(g, arch, "expert_weights_norm", &m->topk_renorm);
    }
    /* tensors (gguf_run.c:294-315) */
    m->tok_embd = gguf_tensor_by_name(g, "token_embd.weight");
    m->out_norm = gguf_tensor_by_name(g, "output_norm.weight");
    m->lm_head = gguf_tensor_by_name(g, "output.weight");
    if (!m->tok_embd || !m->out_norm || !m->is_moe) {
        gguf_close(g);
        free(r);
        return NULL;
    }
    if (!m->lm_head) m->lm_head = m->tok_embd;
    m->vocab = (int)m->tok_embd->dims[1];
    m->L = (Layer *)calloc((size_t)m->n_layers, sizeof(Layer));
    for (int l = 0; l < m->n_layers; l++) {
        Layer *ly = &m->L[l];
        char nb[96];
        ly->attn_norm = T(g, "blk.%d.attn_norm.weight", l);
        ly->wq = T(g, "blk.%d.attn_q.weight", l);
        ly->wk = T(g, "blk.%d.attn_k.weight", l);
        ly->wv = T(g, "blk.%d.attn_v.weight", l);
        ly->wo = T(g, "blk.%d.attn_output.weight", l);
        ly->ffn_norm = T(g, "blk.%d.ffn_norm.weight", l);
        snprintf(nb, sizeof(nb), "blk.%d.attn_q.bias", l);
        ly->bq = gguf_tensor_by_name(g, nb);
        snprintf(nb, sizeof(nb), "blk.%d.attn_k.bias", l);
        ly->bk = gguf_tensor_by_name(g, nb);
        snprintf(nb, sizeof(nb), "blk.%d.attn_v.bias", l);
        ly->bv = gguf_tensor_by_name(g, nb);
        snprintf(nb, sizeof(nb), "blk.%d.attn_q_norm.weight", l);
        ly->q_norm = gguf_tensor_by_name(g, nb);
        snprintf(nb, sizeof(nb), "blk.%d.attn_k_norm.weight", l);
        ly->k_norm = gguf_tensor_by_name(g, nb);
        ly->router = T(g, "blk.%d.ffn_gate_inp.weight", l);
        ly->gate_exps = T(g, "blk.%d.ffn_gate_exps.weight", l);
        ly->up_exps = T(g, "blk.%d.ffn_up_exps.weight", l);
        ly->down_exps = T(g, "blk.%d.ffn_down_exps.weight", l);
    }
    /* experts through the ExpertStore over the file (gguf_run.c:317-331) */
    m->exp_type = m->L[0].gate_exps->ggml_type;
    m->es = expert_store_create(g->fd, 0, m->n_layers, m->n_experts);
    for (int l = 0; l < m->n_layers; l++) {
        const Layer *ly = &m->L[l];
        const uint8_t *base = (const uint8_t *)g->map;
        uint64_t og = (uint64_t)((const uint8_t *)ly->gate_exps->data - base);
        uint64_t ou = (uint64_t)((const uint8_t *)ly->up_exps->data - base);
        uint64_t od = (uint64_t)((const uint8_t *)ly->down_exps->data - base);
        uint32_t gs = (uint32_t)(ly->gate_exps->nbytes / (uint64_t)m->n_experts);
        uint32_t us = (uint32_t)(ly->up_exps->nbytes / (uint64_t)m->n_experts);
        uint32_t ds = (uint32_t)(ly->down_exps->nbytes / (uint64_t)m->n_experts);
        for (int e = 0; e < m->n_experts; e++) {
            ExpertSlices sl = {og + (uint64_t)e * gs, ou + (uint64_t)e * us, od + (uint64_t)e * ds, gs, us, ds};
            expert_store_register(m->es, l, e, &sl);
        }
    }
    /* the dense (exact) KV store */
    KVConfig cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.n_layers = m->n_layers * m->n_kv_heads;
    cfg.kv_dim = m->head_size;
    m->kv = kvstore_dense_create(cfg);
    m->x = malloc((size_t)m->dim * 4);
    m->xb = malloc((size_t)m->dim * 4);
    m->q = malloc((size_t)m->n_heads * m->head_size * 4);
    m->k = malloc((size_t)m->n_kv_heads * m->head_size * 4);
    m->v = malloc((size_t)m->n_kv_heads * m->head_size * 4);
    m->att_out = malloc((size_t)m->n_heads * m->head_size * 4);
    m->logits = malloc((size_t)m->vocab * 4);
    m->rlog = malloc((size_t)m->n_experts * 4);
    m->gbuf = malloc((size_t)m->ffn_exp * 4);
    m->ubuf = malloc((size_t)m->ffn_exp * 4);
    m->dbuf = malloc((size_t)m->dim * 4);
    m->moe_acc = malloc((size_t)m->dim * 4);
#ifdef VIREO_DROPIN
    /* the file's tensors resident in HBM for the host-pointer gguf_matmul */
    gguf_weights_register(g->data, (uint64_t)((const uint8_t *)g->map + g->size - g->data));
#endif
    return r;
}

int dropin_dim(const DropIn *r) { return r->m.dim; }
int dropin_vocab(const DropIn *r) { return r->m.vocab; }

/* forward(token, pos); logits_out [vocab] and x_out [dim] may be NULL.
 * Returns the argmax of the logits (want_logits) or -1. */
int dropin_forward(DropIn *r, int token, int pos, int want_logits, float *logits_out, float *x_out) {
    float *lg = forward(&r->m, token, pos, want_logits);
    if (lg && logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)r->m.vocab);
    if (x_out) memcpy(x_out, r->m.x, sizeof(float) * (size_t)r->m.dim);
    return lg ? argmax(lg, r->m.vocab) : -1;
}

void dropin_close(DropIn *r) {
    if (!r) return;
    Model *m = &r->m;
#ifdef VIREO_DROPIN
    if (g_moe) {
        for (int l = 0; l < m->n_layers; l++) gguf_moe_destroy(g_moe[l]);
        free(g_moe);
        g_moe = NULL;
    }
#endif
    kv_destroy(m->kv);
    expert_store_destroy(m->es);
    free(m->x); free(m->xb); free(m->q); free(m->k); free(m->v); free(m->att_out); free(m->logits);
    free(m->rlog); free(m->gbuf); free(m->ubuf); free(m->dbuf); free(m->moe_acc);
    free(m->L);
    gguf_close(r->g);
    free(r);
}
