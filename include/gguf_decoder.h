/* vireo-b200: the rest of the reference's decoder forward pass on the GPU,
 * around the MoE block, so that whole decode steps run on the device.
 *
 * Replaces forward() of the reference runner (vireo src/gguf_run.c:216-252)
 * for one token: embedding row dequantisation (:218), per layer RMSNorm
 * (:161-165, :222), Q/K/V mat-vecs with optional bias (:223-225, :166), QK
 * RMSNorm over the full width or per head (:226-229, :177-179), NEOX RoPE
 * (:168-173, :230-231), KV append and exact attention over every cached
 * position (the dense KV store with the shared online softmax,
 * src/kvstore_dense.c:39-49, src/kvstore.h:77-101), the output mat-vec and
 * residual add (:236-237), the FFN RMSNorm and the MoE block (:238-239,
 * gguf_moe.h), the final norm and the LM head (:249-251) and the greedy
 * argmax (:253, strict '>' so the lowest id wins ties).
 *
 * The reference has no device path; every call here is new and returns an
 * int status (vireo_status.h).  All pointers are DEVICE pointers. */
#ifndef VIREO_GGUF_DECODER_H
#define VIREO_GGUF_DECODER_H
#include <stdint.h>

#include "gguf_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Model-wide fields, as the reference reads them from GGUF metadata
 * (gguf_run.c:276-293). */
typedef struct {
    int n_layers, dim, n_heads, n_kv_heads, head_size, vocab;
    float eps, rope_base;
    int max_ctx;              /* KV cache positions to hold (at most 1,441,792) */
    int kv_f16;               /* 1: keys and values cached as f16; 0: f32 (the reference's) */
    uint32_t tok_embd_type;   /* any type gguf_dequant_row reads */
    const void *tok_embd;     /* [vocab] rows of dim */
    const float *out_norm;    /* [dim] F32 */
    uint32_t lm_head_type;
    const void *lm_head;      /* [vocab] rows of dim (the reference falls back to tok_embd) */
} gguf_decoder_desc;

/* One layer (gguf_run.c:141-145).  Norm weights and biases are F32; a NULL
 * bias or QK-norm is absent.  q_norm_len / k_norm_len: head_size (per-head
 * norm, Qwen3) or the full width (OLMoE).  moe: the layer's MoE block from
 * gguf_moe_create (the decoder does not own it). */
typedef struct {
    const float *attn_norm, *ffn_norm;
    uint32_t wq_type, wk_type, wv_type, wo_type;
    const void *wq, *wk, *wv, *wo;
    const float *bq, *bk, *bv;
    const float *q_norm, *k_norm;
    int q_norm_len, k_norm_len;
    gguf_moe *moe;
} gguf_decoder_layer;

typedef struct gguf_decoder gguf_decoder;

/* Validates the shapes and allocates the KV cache and the activations.
 * Supported: head_size 64 or 128, n_heads / n_kv_heads in
 * {1, 2, 4, 8}, dim <= 16384. */
int gguf_decoder_create(const gguf_decoder_desc *desc, const gguf_decoder_layer *layers, gguf_decoder **out);

/* One decode step (forward(m, token, pos, want_logits), gguf_run.c:216):
 * token at position pos (0 <= pos < max_ctx; positions are appended in order,
 * as the reference's KV store does).  logits: DEVICE [vocab] out, or NULL
 * (no LM head: a prompt step, as want_logits = 0); next: DEVICE int32 out
 * (the argmax of the logits), or NULL.  Stream-ordered; device failures
 * surface in gguf_decoder_sync. */
int gguf_decoder_step(gguf_decoder *dec, int token, int pos, float *logits, int32_t *next, void *stream);

/* The same with the token id read from DEVICE memory (e.g. the previous
 * step's `next`), so that greedy decoding chains steps with no host read.
 * An id outside [0, vocab) embeds zeros and is reported by
 * gguf_decoder_sync as VIREO_ERR_ARG. */
int gguf_decoder_step_dev(gguf_decoder *dec, const int32_t *token, int pos, float *logits, int32_t *next,
                          void *stream);

/* The residual stream x [dim] after the last step (DEVICE, owned by dec). */
const float *gguf_decoder_hidden(const gguf_decoder *dec);

int gguf_decoder_sync(gguf_decoder *dec, void *stream);
void gguf_decoder_destroy(gguf_decoder *dec);

#ifdef __cplusplus
}
#endif
#endif
