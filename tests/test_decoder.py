"""Whole decode steps on the device (gguf_decoder_*, through the C-ABI)
against the reference's own forward() (src/gguf_run.c:216-252, compiled from
the reference sources into oracle/_ref with its dense KV store and its
ExpertStore), teacher-forced on the same seeded token ids.

Tolerance on the logits: max |got - ref| / max |ref| <= 2e-3 with an f32 KV
cache (the reference's), 1e-2 with the f16 cache.  The greedy token must
agree wherever the reference's top-2 logit gap exceeds twice the largest
logit difference.
"""
import numpy as np
import pytest

from oracle import oracle as O
from vireo_b200 import synth as S

pytestmark = pytest.mark.gpu


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def tokens(seed, n, vocab):
    return (S.u64(seed, 77, n) % np.uint64(vocab)).astype(np.int64)


def run_case(spec, seed, kv_f16, steps, check_from=0):
    import torch
    import vireo_b200 as V
    if not O.ref_available():
        pytest.skip("reference library not built")
    D = S.Decoder(spec, seed)
    R = O.RefDecoder(D)
    G = V.Decoder(D, max_ctx=steps + 8, kv_f16=kv_f16)
    try:
        lg = torch.zeros(spec.vocab, dtype=torch.float32, device="cuda")
        nx = torch.zeros(1, dtype=torch.int32, device="cuda")
        worst = 0.0
        for pos, tok in enumerate(tokens(seed, steps, spec.vocab)):
            want = pos >= check_from
            G.step(int(tok), pos, logits=lg if want else None, next=nx if want else None)
            rl, rx, ra = R.step(int(tok), pos, want)
            if not want:
                continue
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
        R.close()


@pytest.mark.parametrize("kind", ["olmoe", "qwen3"])
def test_decoder_matches_reference_forward_f32_kv(kind):
    spec = S.tiny_olmoe_decoder() if kind == "olmoe" else S.tiny_qwen3_decoder()
    worst = run_case(spec, 31, kv_f16=False, steps=12)
    assert worst < 2e-3, worst


def test_decoder_f16_kv_and_long_context():
    # 300 positions: the attention splits into two 256-position chunks
    spec = S.tiny_qwen3_decoder()
    worst = run_case(spec, 32, kv_f16=True, steps=300, check_from=290)
    assert worst < 1e-2, worst


def test_decoder_gqa8_head64_no_qk_norm_across_chunks():
    # 8 q heads per kv head (config 3's grouping), 64-wide heads, no QK norm;
    # 140 positions cross the 128-position attention chunk boundary
    spec = S.DecoderSpec(2, 512, 8, 1, 64, 640, S.MoeLayerSpec(512, 256, 16, 4, 1, S.GGML_Q4_K, S.GGML_Q4_K,
                                                               S.GGML_Q6_K), qk_norm=None)
    worst = run_case(spec, 35, kv_f16=False, steps=140, check_from=120)
    assert worst < 2e-3, worst


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
