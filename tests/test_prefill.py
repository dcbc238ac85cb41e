"""Batched (prefill) MoE FFN (gguf_moe_prefill, tcgen05 grouped GEMMs) against
the CPU restatement of the reference's moe_ffn, token by token, on the same
bf16-rounded inputs, with and without a router bias (the imbalanced-routing
configuration adds one to the logits).

Tolerances: expert ids bit-exact on tokens whose fp64 probabilities have a
gap >= 1e-4 among the top n_used + 1; gate weights rel <= 1e-5; outputs
max |got - ref| / max |ref| <= 2e-3 per token (f16 operands, fp32
accumulation: about 2e-4 in practice).
"""
import numpy as np
import pytest

from oracle import oracle as O
from vireo_b200 import synth as S

pytestmark = pytest.mark.gpu

TOL = 2e-3


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def bf16_round(a):
    """fp32 values rounded to bf16 (round to nearest even), as fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


def margin_tokens(L, n, seed, bias, margin=1e-4):
    """n bf16-exact hidden vectors whose fp64 routing probabilities (router
    logits + bias) are separated by >= margin among the top n_used + 1."""
    s = L.spec
    R = np.frombuffer(L.router.tobytes(), dtype=np.float32).reshape(s.n_experts, s.dim).astype(np.float64)
    b = np.zeros(s.n_experts) if bias is None else bias.astype(np.float64)
    out, i = [], 0
    while len(out) < n:
        x = bf16_round(S.normal(seed, 100 + i, s.dim).astype(np.float32))
        i += 1
        l = R @ x.astype(np.float64) + b
        p = np.exp(l - l.max())
        p /= p.sum()
        top = np.sort(p)[::-1][:s.n_used + 1]
        if np.all(-np.diff(top) >= margin):
            out.append(x)
    return np.stack(out)


def run_prefill(V, L, toks, x0, bias):
    import torch
    s = L.spec
    m = V.MoeLayer(L)
    try:
        T = toks.shape[0]
        hb = torch.from_numpy(toks).cuda().to(torch.bfloat16)
        xd = torch.from_numpy(x0.copy()).cuda()
        ids = torch.full((T, s.n_used), -7, dtype=torch.int32, device="cuda")
        wts = torch.zeros((T, s.n_used), dtype=torch.float32, device="cuda")
        bd = torch.from_numpy(bias).cuda() if bias is not None else None
        V.check(V.lib().gguf_moe_prefill(m.h, hb.data_ptr(), xd.data_ptr(), T, bd.data_ptr() if bd is not None else None,
                                         ids.data_ptr(), wts.data_ptr(), None), "gguf_moe_prefill")
        m.sync()
        return xd.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
    finally:
        m.close()


CASES = [
    # dim, fe, ne, k, renorm, T, bias sigma, seed
    (512, 256, 16, 4, 1, 300, 0.5, 3),
    (1024, 512, 64, 8, 0, 200, 0.0, 4),
    (2048, 768, 128, 8, 1, 256, 0.5, 5),  # the Qwen3-30B-A3B layer shape
]


@pytest.mark.parametrize("case", CASES)
def test_prefill_matches_oracle(case):
    import torch
    assert torch.cuda.is_available()
    import vireo_b200 as V
    dim, fe, ne, k, renorm, T, bsig, seed = case
    spec = S.MoeLayerSpec(dim, fe, ne, k, renorm, S.GGML_Q4_K, S.GGML_Q4_K, S.GGML_Q6_K)
    L = S.MoeLayer(spec, seed)
    bias = (S.normal(seed, 7, ne) * bsig).astype(np.float32) if bsig > 0 else None
    toks = margin_tokens(L, T, seed, bias)
    x0 = (S.normal(seed, 8, toks.size) * 0.5).astype(np.float32).reshape(toks.shape)
    x, ids, wts = run_prefill(V, L, toks, x0, bias)
    rx, rids, rwts = O.PortMoe(L)(toks, x0, bias)
    assert np.array_equal(ids, rids), np.argwhere(ids != rids)[:5]
    assert rel_err(wts, rwts) < 1e-5, rel_err(wts, rwts)
    worst = max(rel_err(x[i] - x0[i], rx[i] - x0[i]) for i in range(T))
    assert worst < TOL, worst


def test_prefill_deterministic_and_unsupported():
    import torch
    import vireo_b200 as V
    spec = S.MoeLayerSpec(512, 256, 16, 4, 1, S.GGML_Q4_K, S.GGML_Q4_K, S.GGML_Q6_K)
    L = S.MoeLayer(spec, 11)
    toks = margin_tokens(L, 130, 11, None)
    x0 = np.zeros_like(toks)
    a = run_prefill(V, L, toks, x0, None)
    b = run_prefill(V, L, toks, x0, None)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    # a Q8_0 layer is not on the batched path: refused with a status
    spec8 = S.MoeLayerSpec(512, 256, 16, 4, 1, S.GGML_Q8_0, S.GGML_Q8_0, S.GGML_Q8_0)
    m = V.MoeLayer(S.MoeLayer(spec8, 12))
    try:
        hb = torch.zeros((4, 512), dtype=torch.bfloat16, device="cuda")
        xd = torch.zeros((4, 512), dtype=torch.float32, device="cuda")
        assert V.lib().gguf_moe_prefill(m.h, hb.data_ptr(), xd.data_ptr(), 4, None, None, None, None) == -3
    finally:
        m.close()


@pytest.mark.parametrize("ne,k", [(16, 4), (64, 8), (128, 8)])
def test_prefill_router_exact_ties(ne, k):
    """Experts 2j and 2j + 1 share one router row, so every routing
    probability is tied with its partner's bit for bit, and the selection
    must take the lower id first and keep it when a larger probability is
    inserted ahead of the pair (the reference's strict '>' scan from id 0,
    gguf_run.c:190-191).  Router entries are multiples of 1/64 and the hidden
    values small integers, so every logit is exact in bf16 operands with any
    summation order and distinct logits differ by at least 1/64: ids
    bit-exact against the oracle on every token, over several row tiles."""
    import torch
    assert torch.cuda.is_available()
    import vireo_b200 as V
    spec = S.MoeLayerSpec(512, 256, ne, k, 1, S.GGML_Q4_K, S.GGML_Q4_K, S.GGML_Q6_K)
    L = S.MoeLayer(spec, 93)
    R = L.router.view(np.float32).reshape(ne, spec.dim)
    R[:] = ((S.u64(93, 1, ne * spec.dim) % np.uint64(17)).astype(np.float32) - 8.0).reshape(R.shape) / 64.0
    R[1::2] = R[0::2]
    T = 300
    toks = ((S.u64(93, 2, T * spec.dim) % np.uint64(5)).astype(np.float32) - 2.0).reshape(T, spec.dim)
    x0 = (S.normal(93, 3, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    x, ids, wts = run_prefill(V, L, toks, x0, None)
    rx, rids, rwts = O.PortMoe(L)(toks, x0, None)
    assert (rids[:, 0] % 2 == 0).all()
    assert np.array_equal(ids, rids), np.argwhere(ids != rids)[:5]
    assert rel_err(wts, rwts) < 1e-5, rel_err(wts, rwts)
    worst = max(rel_err(x[i] - x0[i], rx[i] - x0[i]) for i in range(T))
    assert worst < TOL, worst
