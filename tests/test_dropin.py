"""The drop-in boundary with a real model file.

A generated decoder is written as a GGUF file (vireo_b200.gguf_file) and
opened by the reference's own loader (gguf_open, src/gguf.c:79-131, and the
runner's tensor lookup, src/gguf_run.c:276-331) in two builds of the
reference's runner (oracle/dropin.py):

* as it ships (gguf_compute.c, expert_store.c);
* with gguf_compute.c and expert_store.c dropped, libvireo_b200.so linked in
  their place and the MoE hook at the top of moe_ffn, so that every layer's
  MoE block runs as one gguf_moe_ffn_host call and every other mat-vec of
  forward() (attention, LM head) goes through the library's gguf_matmul.

CPU: the writer round-trips, and the shipped reference on the file gives
exactly the logits of the reference built from the same arrays in memory
(the file holds the model the other tests use).  GPU: teacher-forced
forward() of the linked build against the shipped one, logits within 2e-3
at every step; the hook ran for every layer of every step.
"""
import os
import tempfile

import numpy as np
import pytest

from oracle import oracle as O
from vireo_b200 import gguf_file as GF
from vireo_b200 import synth as S

CASES = [("qwen3moe", S.tiny_qwen3_decoder, 32), ("olmoe", S.tiny_olmoe_decoder, 31)]
STEPS = 12


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def tokens(seed, n, vocab):
    return (S.u64(seed, 77, n) % np.uint64(vocab)).astype(np.int64)


def need_dropin():
    from oracle import dropin
    if not (os.path.exists(dropin.REF_SO) and os.path.exists(dropin.B200_SO)):
        pytest.skip("drop-in checkers not built")


@pytest.fixture
def model_file():
    d = tempfile.mkdtemp(prefix="vireo_gguf_")
    made = []

    def make(arch, spec_fn, seed):
        dec = S.Decoder(spec_fn(), seed)
        path = os.path.join(d, f"{arch}_{seed}.gguf")
        GF.write_decoder(path, dec, arch)
        made.append(path)
        return dec, path

    yield make
    for p in made:
        os.remove(p)
    os.rmdir(d)


def test_gguf_writer_round_trip(model_file):
    dec, path = model_file("qwen3moe", S.tiny_qwen3_decoder, 32)
    md, tensors = GF.read(path)
    s = dec.spec
    assert md["general.architecture"] == "qwen3moe"
    assert md["qwen3moe.block_count"] == s.n_layers and md["qwen3moe.expert_count"] == s.moe.n_experts
    assert md["qwen3moe.attention.key_length"] == s.head_size
    want = GF.decoder_tensors(dec)
    assert len(tensors) == len(want)
    for name, dims, gtype, data in want:
        got_dims, got_type, got = tensors[name]
        assert got_dims == dims and got_type == gtype, name
        assert got == bytes(np.ascontiguousarray(data).view(np.uint8).reshape(-1)), name


@pytest.mark.parametrize("arch,spec_fn,seed", CASES)
def test_reference_on_the_file_equals_reference_in_memory(model_file, arch, spec_fn, seed):
    need_dropin()
    dec, path = model_file(arch, spec_fn, seed)
    F = O.DropInDecoder(path, b200=False)
    R = O.RefDecoder(dec)
    try:
        for pos, tok in enumerate(tokens(seed, STEPS, dec.spec.vocab)):
            lf, _, af = F.step(int(tok), pos)
            lr, _, ar = R.step(int(tok), pos)
            assert np.array_equal(lf, lr), pos
            assert af == ar
    finally:
        F.close()
        R.close()


@pytest.mark.gpu
@pytest.mark.parametrize("arch,spec_fn,seed", CASES)
def test_linked_runner_matches_the_reference(model_file, arch, spec_fn, seed):
    """The runner with libvireo_b200.so in place of gguf_compute.c and
    expert_store.c (and the moe_ffn hook) against the runner as it ships,
    teacher-forced on the same file.  The seeds keep the reference's router
    away from near-ties (test_decoder checks their margins)."""
    import torch
    assert torch.cuda.is_available()
    import vireo_b200  # noqa: F401  (the library the linked runner uses, loaded first)
    need_dropin()
    dec, path = model_file(arch, spec_fn, seed)
    Ref = O.DropInDecoder(path, b200=False)
    Dev = O.DropInDecoder(path, b200=True)
    calls0 = Dev.hook_calls()  # the counter lives in the library, across cases
    try:
        worst = 0.0
        for pos, tok in enumerate(tokens(seed, STEPS, dec.spec.vocab)):
            lr, _, ar = Ref.step(int(tok), pos)
            ld, _, ad = Dev.step(int(tok), pos)
            e = rel_err(ld, lr)
            worst = max(worst, e)
            top = np.sort(lr)[::-1]
            if top[0] - top[1] > 2 * np.abs(ld - lr).max():
                assert ad == ar, (pos, ad, ar)
        assert worst < 2e-3, worst
        assert Dev.hook_calls() - calls0 == STEPS * dec.spec.n_layers
    finally:
        Dev.close()
        Ref.close()
