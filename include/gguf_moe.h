/* vireo-b200: the MoE FFN block on B200 (sm_100a).
 *
 * The reference computes the MoE FFN in moe_ffn (vireo src/gguf_run.c:185-214),
 * a static function inside its model runner: router matvec (:187), softmax
 * (:181-182), greedy top-k with ties to the lowest expert id (:190-191),
 * optional renormalisation (:192), and per selected expert gate/up matvec,
 * SwiGLU and down matvec with a rank-ordered weighted combine (:198-213),
 * adding the result into the residual x.  This header exports that block
 * as a C-ABI call so a host model loop can replace the body of moe_ffn with
 * one gguf_moe_ffn call per layer.
 *
 * One decode token runs as one kernel launch with one CTA per SM: router,
 * top-k, then each selected expert's gate/up + SwiGLU and down on its own
 * group of CTAs, and the rank-ordered combine, with the expert weights
 * streamed raw (GGUF blocks, no repacking) from HBM. */
#ifndef VIREO_GGUF_MOE_H
#define VIREO_GGUF_MOE_H
#include <stdint.h>

#include "gguf.h"
#include "expert_store.h"
#include "vireo_status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One MoE layer.  Mirrors the reference Model/Layer fields moe_ffn reads:
 * dim, ffn_exp, n_experts, n_used, topk_renorm (src/gguf_run.c:154) and the
 * tensors ffn_gate_inp / ffn_{gate,up,down}_exps (src/gguf_run.c:312-315).
 * All pointers are DEVICE pointers.  The expert tensors are the 3-D GGUF
 * tensors with the expert index outermost: expert e of gate_exps starts at
 * gate_exps + e * (gate_nbytes / n_experts), as gguf_run.c:326-331 slices
 * them. */
typedef struct {
    int dim, ffn_exp, n_experts, n_used, topk_renorm;
    uint32_t router_type, gate_type, up_type, down_type;
    const void *router;
    const void *gate_exps, *up_exps, *down_exps;
    uint64_t gate_nbytes, up_nbytes, down_nbytes;
} gguf_moe_desc;

typedef struct gguf_moe gguf_moe;

/* Validates the layer, picks the kernel and allocates its device scratch.
 * Fast path: router F32; gate/up (same type) and down in Q8_0/Q4_K/Q6_K;
 * dim % 512 == 0; ffn_exp % 256 == 0; n_experts <= 256; n_used <= 64 and
 * at most the GPU's SM count. */
int gguf_moe_create(const gguf_moe_desc *desc, gguf_moe **out);

/* The same layer with HOST pointers in desc (e.g. the tensors of an mmap'd
 * GGUF file, as the reference's loader finds them, src/gguf_run.c:312-315):
 * the layer is checked as gguf_moe_create checks it, then its router and
 * expert tensors are copied to device memory owned by the handle (freed by
 * gguf_moe_destroy).  Host memory is not needed after the call. */
int gguf_moe_create_host(const gguf_moe_desc *desc, gguf_moe **out);

/* n_tok independent tokens through the layer, one after another (decode).
 * hb: [n_tok][dim] normalised hidden; x: [n_tok][dim] residual, updated in
 * place (x += MoE(hb)); ids / wts: [n_tok][n_used] selected experts in rank
 * order and their gate weights, or NULL.  Device pointers, stream-ordered,
 * no host synchronisation; device-side failures surface in gguf_moe_sync.
 * Each token is one kernel launched with programmatic dependent launch: it
 * may read the router weights before the preceding kernel on the stream has
 * finished, so router weights must not be written by that kernel. */
int gguf_moe_ffn(gguf_moe *m, const float *hb, float *x, int n_tok, int32_t *ids, float *wts, void *stream);

/* No counterpart in the reference (its moe_ffn always routes with the
 * router, gguf_run.c:187-192): n_tok tokens through the layer with the route
 * given by the caller instead of the router -- a routing-override hook.
 * ids / wts: HOST arrays [n_tok][n_used], rank-order expert ids (-1 = unused
 * slot) and the gate weights the combine uses (final: no softmax, no
 * renormalisation); expert_ptrs: HOST array [n_tok][n_used][3] of DEVICE
 * addresses of each selected expert's gate, up and down slices (16-byte
 * aligned; NULL = unused slot).  The arrays are read during the call (each
 * token's route travels in its launch), so they may be reused at once.
 * hb / x as in gguf_moe_ffn; stream-ordered. */
int gguf_moe_ffn_routed(gguf_moe *m, const float *hb, float *x, int n_tok, const int32_t *ids, const float *wts,
                        const void *const *expert_ptrs, void *stream);

/* The reference's per-expert ExpertStore use in moe_ffn (gguf_run.c:199-210:
 * lookup, compute, release) for one token whose route is given on the host
 * (ids / wts: HOST arrays [n_used], as gguf_moe_ffn_routed): each selected
 * expert of `layer` is looked up asynchronously (misses are copied to the
 * device on the store's copy stream and `stream` waits for them), the routed
 * kernel runs on `stream`, and the leases end when it completes.  An expert
 * whose lookup fails is skipped, as the reference does. */
int gguf_moe_ffn_store(gguf_moe *m, ExpertStore *store, int layer, const float *hb, float *x, const int32_t *ids,
                       const float *wts, void *stream);

/* Batched (prefill) MoE FFN: n_tok tokens at once, the same function as
 * gguf_moe_ffn per token (the reference's moe_ffn, gguf_run.c:185-214), as
 * grouped GEMMs over the experts on the tensor cores.  hb_bf16: DEVICE
 * [n_tok][dim] bf16 hidden vectors; x: DEVICE [n_tok][dim] fp32 residual,
 * updated in place; router_bias: DEVICE [n_experts] added to the router
 * logits before the softmax, or NULL (the reference has none); ids / wts:
 * DEVICE [n_tok][n_used] selection out, or NULL.  Stream-ordered; device
 * failures surface in gguf_moe_sync.  Supported: router F32, gate/up Q4_K,
 * down Q6_K, dim % 256 == 0, ffn_exp % 256 == 0, n_experts <= 128,
 * n_used <= 8; other layers return VIREO_ERR_UNSUPPORTED.  Activations and
 * dequantised weights are f16 with fp32 accumulation: hidden values must lie
 * within f16 range. */
int gguf_moe_prefill(gguf_moe *m, const void *hb_bf16, float *x, int n_tok, const float *router_bias, int32_t *ids,
                     float *wts, void *stream);

/* Same with HOST buffers: copies in, runs, copies out, synchronises. */
int gguf_moe_ffn_host(gguf_moe *m, const float *hb, float *x, int n_tok, int32_t *ids, float *wts);

/* Waits for the layer's work on stream and returns its device status. */
int gguf_moe_sync(gguf_moe *m, void *stream);

/* Point expert e's gate/up/down weights at arbitrary device addresses
 * (arrays of n_experts pointers; a NULL array keeps the current pointers).
 * Used when an ExpertStore owns the expert slabs. */
int gguf_moe_set_expert_ptrs(gguf_moe *m, const void *const *gate, const void *const *up,
                             const void *const *down);

/* Phase tracing (diagnostics): when dev_buf is non-NULL, every later
 * launch writes 72 %globaltimer stamps (ns) per CTA into dev_buf
 * [gguf_moe_grid(m)][72]: kernel start, router partials written, all
 * partials visible, routing done, own gate/up units done, all gate/up units
 * done, down tables built, down units done (consumer side); first gate/up
 * issue, first down issue, last issue, copies drained (producer side);
 * then (stage ready, unit done) pairs for the CTA's first 24 units and 8
 * spare stamps.  The buffer must hold the full 72 stamps per CTA.  NULL
 * turns tracing off. */
int gguf_moe_set_trace(gguf_moe *m, unsigned long long *dev_buf);
int gguf_moe_grid(const gguf_moe *m);

void gguf_moe_destroy(gguf_moe *m);

/* ---- Expert parallelism (no counterpart in the reference, which runs on one
 * host): the batched MoE FFN of gguf_moe_prefill spread over the GPUs of one
 * node, one process per GPU.  Each rank routes its own slice of the tokens
 * and computes the experts placed on it (owner[e] == rank).  The kernels move
 * the rows themselves over NVLink peer memory (CUDA IPC mappings of every
 * rank's buffers): each (token, slot) row is stored straight into its
 * expert's GEMM operand on the owning rank, and the down GEMM stores each
 * output row straight back into the source rank's return buffer.  NCCL (run
 * time loaded, libnccl.so.2) carries only the per-expert counts and two
 * barriers per call.  The result on every rank is bit-identical to
 * gguf_moe_prefill on one GPU over the same tokens. */
typedef struct gguf_moe_ep gguf_moe_ep;

/* An NCCL unique id (128 bytes) for gguf_moe_ep_create: rank 0 makes it and
 * hands the same bytes to every rank by any side channel. */
int gguf_moe_ep_unique_id(void *id128);

/* Host only.  Expert placement by expected load: heaviest expert first onto
 * the least-loaded rank that still has room; every rank gets floor or ceil of
 * n_experts / world experts.  owner: [n_experts] out. */
int gguf_moe_ep_place(const double *expected_load, int n_experts, int world, int32_t *owner);

/* Host only.  Where `rank`'s rows land: counts[src * n_experts + e] = pairs
 * rank src routes to expert e.  Each owner lays out its experts' row ranges
 * in expert order, each range padded to the GEMM tile (128 rows), and within
 * an expert's range the sources in rank order.  dst_off: [n_experts] out,
 * the first row of `rank`'s pairs in expert e's range on owner[e];
 * rows_here: out (or NULL), the rows `rank` receives. */
int gguf_moe_ep_rows(const int32_t *counts, const int32_t *owner, int n_experts, int world, int rank,
                     int32_t *dst_off, int32_t *rows_here);

/* Collective (every rank calls it with the same id, owner, world and
 * max_tokens; the current CUDA device is this rank's GPU; world <= 8).
 * desc: the layer as for gguf_moe_create; only the slices of the experts
 * this rank owns are read.  max_tokens: the most local tokens a call may
 * pass (sizes the exchange buffers).  Supported layers: those of
 * gguf_moe_prefill with n_experts <= 128. */
int gguf_moe_ep_create(const gguf_moe_desc *desc, const int32_t *owner, int rank, int world, int max_tokens,
                       const void *id128, gguf_moe_ep **out);

/* Collective.  n_tok local tokens (may differ between ranks, may be 0, at
 * most max_tokens): arguments as gguf_moe_prefill, DEVICE pointers.
 * Stream-ordered with no host synchronisation (the row layout is computed on
 * the device from the all-gathered counts); device failures surface in
 * gguf_moe_ep_sync, whose wait is bounded: a peer that stops answering ends
 * it with VIREO_ERR_TIMEOUT and leaves the handle unusable. */
int gguf_moe_prefill_ep(gguf_moe_ep *ep, const void *hb_bf16, float *x, int n_tok, const float *router_bias,
                        int32_t *ids, float *wts, void *stream);
int gguf_moe_ep_sync(gguf_moe_ep *ep, void *stream);
/* The rank's layer handle (owned by ep; valid until gguf_moe_ep_destroy). */
gguf_moe *gguf_moe_ep_layer(gguf_moe_ep *ep);
/* Collective (unmaps the peers' buffers, destroys the communicator). */
void gguf_moe_ep_destroy(gguf_moe_ep *ep);

/* No counterpart in the reference: an extension for callers that may not
 * allocate device memory.  Same computation and arguments as gguf_moe_ffn,
 * with the layer given by its descriptor (device pointers, the rules of
 * gguf_moe_create) instead of a handle.  Allocates nothing: the kernel's
 * scratch is a fixed 256 KiB device array in the library (a layer needs
 * about 17 KiB plus 4 B per value of n_used * (dim + ffn_exp), 128 B per 16
 * rows of dim and 24 B per expert: 131 KiB for dim 2048, 64 experts top-8,
 * ffn_exp 1024); a layer needing more returns VIREO_ERR_NOMEM.  The first call on a device sets that device up (takes
 * the array's address, zeroes it) and must come before any stream capture.
 * Every call zeroes the launch's sync, status and counter words first.
 * Every call synchronises stream (NULL = the legacy default stream) before
 * it returns, also when a launch fails, and returns the kernel's status.  All calls on one device share the array: calls that
 * overlap on the GPU race. */
int gguf_moe_ffn_noalloc(const gguf_moe_desc *desc, const float *hb, float *x, int n_tok, int32_t *ids,
                         float *wts, void *stream);

/* Shared expert.  No counterpart in the reference's code (its roadmap names
 * shared-expert models, Qwen2-MoE and DeepSeek, as the next step): one
 * expert FFN that every token takes beside the routed ones.  Per token
 * x += s * down(silu(gate . hb) * (up . hb)), the reference's expert
 * arithmetic (gguf_run.c:202-208) on the shared tensors, with
 * s = sigmoid(gate_inp . hb) when gate_inp is given (Qwen2-MoE's
 * ffn_gate_inp_shexp) and s = 1 otherwise (DeepSeek).  Called after
 * gguf_moe_ffn with the same hb and x it completes such a layer:
 * x += MoE(hb), then x += s * E(hb).  Tensors as for gguf_moe_create
 * (DEVICE pointers, GGUF rows: gate and up [ffn][dim], down [dim][ffn];
 * Q8_0 / Q4_K / Q6_K / Q5_0; dim % 512 == 0, ffn % 256 == 0); gate_inp:
 * DEVICE [dim] fp32 or NULL. */
typedef struct {
    int dim, ffn;
    uint32_t gate_type, up_type, down_type;
    const void *gate, *up, *down;
    const float *gate_inp;
} gguf_moe_shexp_desc;

typedef struct gguf_moe_shexp gguf_moe_shexp;

int gguf_moe_shexp_create(const gguf_moe_shexp_desc *desc, gguf_moe_shexp **out);
/* n_tok tokens (hb, x: DEVICE [n_tok][dim]), one launch each, stream-ordered;
 * failures surface in gguf_moe_shexp_sync. */
int gguf_moe_shexp_ffn(gguf_moe_shexp *sh, const float *hb, float *x, int n_tok, void *stream);
int gguf_moe_shexp_sync(gguf_moe_shexp *sh, void *stream);
void gguf_moe_shexp_destroy(gguf_moe_shexp *sh);

#ifdef __cplusplus
}
#endif
#endif
