"""Whole decode steps on the device (gguf_decoder_*, through the C-ABI)
against the reference's own forward() (src/gguf_run.c:216-252, compiled from
the reference sources into oracle/_ref with its dense KV store and its
ExpertStore), teacher-forced on the same seeded token ids.

Tolerance on the logits: max |got - ref| / max |ref| <= 2e-3 with an f32 KV
cache (the reference's), 1e-2 with the f16 cache.  The greedy token must
agree wherever the reference's top-2 logit gap exceeds twice the largest
logit difference.

Routing margin: the hidden states of a decoder cannot be margin-filtered the
way the MoE-layer tests filter their tokens, so each case's seed is one on
which the reference's router never comes near a tie: at every step and layer
the log-probability gaps among the n_used + 1 most likely experts are at
least min_gap (1e-4; 5e-4 for the f16 cache, whose rounding moves the
router inputs more).  At a near-tie any other summation order may pick
another expert; the CPU test below checks the margins of every case, and
run_case asserts them again, so that a seed without one fails loudly instead
of comparing two different routings.
"""
import numpy as np
import pytest

from oracle import oracle as O
from vireo_b200 import synth as S

gpu = pytest.mark.gpu


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def tokens(seed, n, vocab):
    return (S.u64(seed, 77, n) % np.uint64(vocab)).astype(np.int64)


def gqa8_spec(head_size, qk_norm):
    return S.DecoderSpec(2, 512, 8, 1, head_size, 640, S.MoeLayerSpec(512, 256, 16, 4, 1, S.GGML_Q4_K, S.GGML_Q4_K,
                                                                      S.GGML_Q6_K), qk_norm=qk_norm)


def long_f16_spec():
    return S.DecoderSpec(2, 512, 8, 2, 128, 768, S.MoeLayerSpec(512, 256, 8, 2, 1, S.GGML_Q4_K, S.GGML_Q4_K,
                                                                S.GGML_Q6_K), qk_norm="head", eps=1e-6,
                         rope_base=1000000.0)


def qwen3_geometry_spec():
    """Config 3's geometry in one layer: dim 2048, 32 q / 4 kv heads x 128,
    per-head QK norm, 128 experts top-8 renormalised (ffn 768), and the
    151,936-row Q6_K LM head."""
    return S.DecoderSpec(1, 2048, 32, 4, 128, 151936, S.qwen3_layer(), qk_norm="head", eps=1e-6,
                         rope_base=1000000.0)


# (spec, seed, steps, min_gap) of every reference comparison below
MARGIN_CASES = [
    (qwen3_geometry_spec, 101, 320, 1e-4),
    (qwen3_geometry_spec, 171, 136, 5e-4),
    (S.tiny_olmoe_decoder, 31, 12, 1e-4),
    (S.tiny_qwen3_decoder, 32, 12, 1e-4),
    (long_f16_spec, 41, 260, 5e-4),
    (lambda: gqa8_spec(64, None), 32, 140, 1e-4),
    (lambda: gqa8_spec(128, "head"), 32, 140, 1e-4),
]


def reference_min_gap(spec, seed, steps):
    """Smallest router log-probability gap the reference's forward() meets
    over `steps` teacher-forced steps (CPU only)."""
    D = S.Decoder(spec, seed)
    R = O.RefDecoder(D)
    try:
        g = np.inf
        for pos, tok in enumerate(tokens(seed, steps, spec.vocab)):
            R.step(int(tok), pos, False)
            g = min(g, R.last_gap())
        return g
    finally:
        R.close()


@pytest.mark.parametrize("case", range(len(MARGIN_CASES)))
def test_reference_routing_margin_of_decoder_seeds(case):
    """The seeds of the device comparisons keep the reference's router away
    from near-ties for their whole runs (CPU, the reference alone)."""
    if not O.ref_available():
        pytest.skip("reference library not built")
    make, seed, steps, min_gap = MARGIN_CASES[case]
    assert reference_min_gap(make(), seed, steps) >= min_gap


def run_case(spec, seed, kv_f16, steps, check_from=0, min_gap=1e-4):
    import torch
    import vireo_b200 as V
    if not O.ref_available():
        pytest.skip("reference library not built")
    D = S.Decoder(spec, seed)
    toks = tokens(seed, steps, spec.vocab)
    # the reference's trajectory first, with its routing margins
    R = O.RefDecoder(D)
    try:
        ref = []
        for pos, tok in enumerate(toks):
            rl, _, ra = R.step(int(tok), pos, pos >= check_from)
            gap = R.last_gap()
            assert gap >= min_gap, f"seed {seed}: router near-tie (gap {gap:.2e}) at step {pos}; pick another seed"
            ref.append((rl, ra))
    finally:
        R.close()
    G = V.Decoder(D, max_ctx=steps + 8, kv_f16=kv_f16)
    try:
        lg = torch.zeros(spec.vocab, dtype=torch.float32, device="cuda")
        nx = torch.zeros(1, dtype=torch.int32, device="cuda")
        worst = 0.0
        for pos, tok in enumerate(toks):
            want = pos >= check_from
            G.step(int(tok), pos, logits=lg if want else None, next=nx if want else None)
            if not want:
                continue
            rl, ra = ref[pos]
            G.sync()
            got = lg.cpu().numpy()
            e = rel_err(got, rl)
            worst = max(worst, e)
            top = np.sort(rl)[::-1]
            if top[0] - top[1] > 2 * np.abs(got - rl).max():
                assert int(nx.item()) == ra, (pos, int(nx.item()), ra)
        return worst
    finally:
        G.close()


@gpu
@pytest.mark.parametrize("kind,seed", [("olmoe", 31), ("qwen3", 32)])
def test_decoder_matches_reference_forward_f32_kv(kind, seed):
    spec = S.tiny_olmoe_decoder() if kind == "olmoe" else S.tiny_qwen3_decoder()
    worst = run_case(spec, seed, kv_f16=False, steps=12)
    assert worst < 2e-3, worst


@gpu
def test_decoder_f16_kv_and_long_context():
    # 260 positions: the attention splits into three 128-position chunks
    worst = run_case(long_f16_spec(), 41, kv_f16=True, steps=260, check_from=250, min_gap=5e-4)
    assert worst < 1e-2, worst


@gpu
@pytest.mark.parametrize("head_size,qk_norm", [(64, None), (128, "head")])
def test_decoder_gqa8_across_chunks(head_size, qk_norm):
    # 8 q heads per kv head (config 3's grouping); 140 positions cross the
    # 128-position attention chunk boundary
    worst = run_case(gqa8_spec(head_size, qk_norm), 32, kv_f16=False, steps=140, check_from=120)
    assert worst < 2e-3, worst


@gpu
def test_decoder_qwen3_geometry_long_lm_head():
    """Config 3's attention geometry and LM head: 320 positions (three
    128-position attention chunks) teacher-forced through one layer of the
    Qwen3-shaped decoder with the f32 KV cache; logits of the last 8
    positions (the 151,936-row Q6_K LM head through gemv_kernel) against the
    reference's forward()."""
    worst = run_case(qwen3_geometry_spec(), 101, kv_f16=False, steps=320, check_from=312)
    assert worst < 2e-3, worst


@gpu
def test_decoder_qwen3_geometry_f16_cache():
    """The same geometry on the f16 KV cache (the tensor-core attention
    kernel: 8 q heads per kv head as the MMA rows, 136 positions over three
    tiles of 64): logits of the last 8 positions against the reference's
    forward() at the f16 cache's tolerance."""
    worst = run_case(qwen3_geometry_spec(), 171, kv_f16=True, steps=136, check_from=128, min_gap=5e-4)
    assert worst < 1e-2, worst


@gpu
def test_decoder_device_token_chain_matches_host_tokens():
    """gguf_decoder_step_dev fed by the previous step's argmax gives the same
    tokens and logits as gguf_decoder_step fed the same ids from the host."""
    import torch
    import vireo_b200 as V
    spec = S.tiny_olmoe_decoder()
    D = S.Decoder(spec, 33)
    runs = []
    for dev_chain in (True, False):
        G = V.Decoder(D, max_ctx=32, kv_f16=True)
        try:
            lg = torch.zeros(spec.vocab, dtype=torch.float32, device="cuda")
            nx = torch.zeros(1, dtype=torch.int32, device="cuda")
            tok = torch.tensor([5], dtype=torch.int32, device="cuda")
            seq, logs = [], []
            for pos in range(10):
                if dev_chain:
                    # the step reads its token before it writes the next one
                    G.step_dev(tok, pos, logits=lg, next=tok)
                    G.sync()
                    seq.append(int(tok.item()))
                else:
                    G.step(5 if pos == 0 else seq[-1], pos, logits=lg, next=nx)
                    G.sync()
                    seq.append(int(nx.item()))
                logs.append(lg.cpu().numpy().copy())
            runs.append((seq, np.stack(logs)))
        finally:
            G.close()
    assert runs[0][0] == runs[1][0]
    assert np.array_equal(runs[0][1], runs[1][1])


@gpu
def test_decoder_rejects_moe_of_another_dim():
    """A layer whose MoE handle was made for another hidden size is refused
    at create (the MoE block reads hb and writes x over its own dim)."""
    import vireo_b200 as V
    spec = S.tiny_olmoe_decoder(n_layers=1)
    D = S.Decoder(spec, 35)
    other = S.MoeLayer(S.MoeLayerSpec(1024, 256, 16, 4, 0, S.GGML_Q4_K, S.GGML_Q4_K, S.GGML_Q6_K), 35)
    D.layers = [D.layers[0]]
    D.layers[0].moe = other
    with pytest.raises(V.VireoError) as ei:
        V.Decoder(D, max_ctx=4)
    assert ei.value.status == -1


@gpu
def test_decoder_rejects_bad_arguments():
    import vireo_b200 as V
    spec = S.tiny_olmoe_decoder(n_layers=1)
    G = V.Decoder(S.Decoder(spec, 34), max_ctx=4)
    try:
        L = V.lib()
        assert L.gguf_decoder_step(G.h, spec.vocab, 0, None, None, None) == -1  # token out of range
        assert L.gguf_decoder_step(G.h, 0, 4, None, None, None) == -1  # position beyond max_ctx
        G.sync()
    finally:
        G.close()
