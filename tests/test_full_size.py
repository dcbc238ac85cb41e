"""Parity at the sizes the benchmark runs, through the C-ABI library.

* Config 1 in full: the benchmark's 1000 seeded tokens through the
  OLMoE-shaped Q8_0 layer (gguf_moe_ffn), every token against the CPU
  restatement of the reference's moe_ffn (src/gguf_run.c:185-214).
* Config 4 in full: 8192 bf16 tokens with the benchmark's per-expert router
  bias N(0, 0.5) through the Qwen3-shaped layer (gguf_moe_prefill).  Expert
  ids are checked on every (token, slot) pair whose fp64 probability is
  separated by >= 1e-4 from its neighbours in rank order; outputs on a
  seeded sample of margin tokens spread over the experts, including every
  token of a slice of the most loaded expert's range.
* Activations with outlier channels: one 32-value group holding a value
  100x or 1000x the rest of the vector, through the mat-vec and the MoE
  layer, including the case where the outlier's weight column is zero (the
  output then does not scale with the outlier, so the precision of the
  group's other values decides the error).

Tolerances as in test_gpu_parity: ids bit-exact, gate weights rel <= 1e-5,
layer outputs max |got - ref| / max |ref| <= 2e-3 per token, mat-vec outputs
<= 1e-4.
"""
import numpy as np
import pytest

from oracle import oracle as O
from vireo_b200 import synth as S

pytestmark = pytest.mark.gpu

TOL = 2e-3
MM_TOL = 1e-4
MARGIN = 1e-4


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def bf16_round(a):
    """fp32 values rounded to bf16 (round to nearest even), as fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


@pytest.fixture(scope="module")
def V():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import vireo_b200
    return vireo_b200


def test_cfg1_all_1000_tokens(V):
    """The benchmark's workload (bench.py cfg1_moe_decode: layer seed 1234,
    1000 margin-filtered tokens) through the device entry, every token."""
    import torch
    L = S.MoeLayer(S.olmoe_q8_layer(), 1234)
    toks, _ = S.routed_tokens(L, 1000, 1234)
    n = toks.shape[0]
    x0 = (S.normal(1234, 9, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    rx, rids, rwts = O.PortMoe(L)(toks, x0)
    m = V.MoeLayer(L)
    try:
        hb, x = torch.from_numpy(toks).cuda(), torch.from_numpy(x0.copy()).cuda()
        ids = torch.zeros((n, L.spec.n_used), dtype=torch.int32, device="cuda")
        wts = torch.zeros((n, L.spec.n_used), dtype=torch.float32, device="cuda")
        m.ffn(hb, x, ids, wts)
        m.sync()
        got, gi, gw = x.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
    finally:
        m.close()
    assert np.array_equal(gi, rids), np.argwhere(gi != rids)[:5]
    assert rel_err(gw, rwts) < 1e-5
    errs = np.array([rel_err(got[i] - x0[i], rx[i] - x0[i]) for i in range(n)])
    assert errs.max() < TOL, (int(errs.argmax()), float(errs.max()))


def rank_margins(L, toks, bias):
    """Per (token, slot): the smaller fp64 probability gap to the slot's
    neighbours in rank order (slot n_used - 1 against rank n_used too)."""
    s = L.spec
    R = L.router_f64()
    lg = toks.astype(np.float64) @ R.T + bias.astype(np.float64)[None, :]
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    top = -np.sort(-p, axis=1)[:, :s.n_used + 1]
    gaps = top[:, :-1] - top[:, 1:]  # gap between rank r and r + 1
    left = np.concatenate([np.full((toks.shape[0], 1), np.inf), gaps[:, :-1]], axis=1)
    return np.minimum(left, gaps)


def test_cfg4_prefill_full_8192_tokens(V):
    """The benchmark's prefill workload (bench.py qwen3_prefill: layer seed
    1234, x ~ N(0,1) from stream 41 rounded to bf16, bias 0.5 N(0,1) from
    stream 42) through gguf_moe_prefill at its full 8192 tokens: the
    65,536 (token, slot) rows cross every per-expert range, tile table and
    row index of the dispatch."""
    import torch
    s = S.qwen3_layer()
    L = S.MoeLayer(s, 1234)
    T, d = 8192, s.dim
    toks = bf16_round(S.normal(1234, 41, T * d).astype(np.float32)).reshape(T, d)
    bias = (S.normal(1234, 42, s.n_experts) * 0.5).astype(np.float32)
    x0 = (S.normal(1234, 43, T * d) * 0.5).astype(np.float32).reshape(T, d)
    m = V.MoeLayer(L)
    try:
        hb = torch.from_numpy(toks).cuda().to(torch.bfloat16)
        xd = torch.from_numpy(x0.copy()).cuda()
        ids = torch.full((T, s.n_used), -7, dtype=torch.int32, device="cuda")
        wts = torch.zeros((T, s.n_used), dtype=torch.float32, device="cuda")
        bd = torch.from_numpy(bias).cuda()
        V.check(V.lib().gguf_moe_prefill(m.h, hb.data_ptr(), xd.data_ptr(), T, bd.data_ptr(), ids.data_ptr(),
                                         wts.data_ptr(), None), "gguf_moe_prefill")
        m.sync()
        got, gi, gw = xd.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
    finally:
        m.close()
    P = O.PortMoe(L)
    rids, rwts = P.route(toks, bias)
    mg = rank_margins(L, toks, bias)
    ok = mg >= MARGIN
    assert ok.mean() > 0.5, ok.mean()
    bad = ok & (gi != rids)
    assert not bad.any(), np.argwhere(bad)[:5]
    # gate weights of tokens whose whole selection is margin-qualified
    full = ok.all(1)
    assert rel_err(gw[full], rwts[full]) < 1e-5
    # outputs: every margin token of a slice of the heaviest expert's range,
    # plus a seeded sample over all experts
    load = np.bincount(rids.ravel(), minlength=s.n_experts)
    heavy = int(load.argmax())
    cand = np.flatnonzero(full)
    in_heavy = cand[(rids[cand] == heavy).any(1)]
    rng = np.random.default_rng(4)
    pick = set(in_heavy[:192].tolist())
    pick |= set(rng.choice(cand, size=min(448, cand.size), replace=False).tolist())
    for e in range(s.n_experts):  # at least one token per loaded expert
        hit = cand[(rids[cand] == e).any(1)]
        if hit.size:
            pick.add(int(hit[0]))
    pick = np.array(sorted(pick))
    assert pick.size >= 512
    rx, pids, _ = P(toks[pick], x0[pick], bias)
    assert np.array_equal(pids, rids[pick])
    errs = np.array([rel_err(got[i] - x0[i], rx[j] - x0[i]) for j, i in enumerate(pick)])
    assert errs.max() < TOL, (int(pick[errs.argmax()]), float(errs.max()))


def outlier_vector(seed, n, factor, j):
    x = S.normal(seed, 4, n).astype(np.float32)
    x[j] = np.float32(factor * np.abs(x).max())
    return x


@pytest.mark.parametrize("factor", [100.0, 1000.0])
@pytest.mark.parametrize("zero_col", [False, True])
@pytest.mark.parametrize("t,n,d", [(S.GGML_Q8_0, 2048, 1024), (S.GGML_Q4_K, 2048, 768),
                                   (S.GGML_Q6_K, 768, 2048)])
def test_matvec_outlier_channel(V, t, n, d, factor, zero_col):
    """One value factor x the vector's largest other magnitude, in one
    group.  zero_col: the outlier's own contribution (its weight column
    times the outlier, computed exactly on the CPU) is taken out of both the
    device result and the reference, which is the product with that weight
    column zeroed (a column cannot be zeroed inside a K-quant block)."""
    import torch
    j = 37
    w = S.tensor(t, 21, 5 + t, d, n)
    x = outlier_vector(22, n, factor, j)
    ref = O.matmul(t, w, x, n, d).astype(np.float64)
    col = np.zeros(d)
    if zero_col:
        xo = np.zeros_like(x)
        xo[j] = x[j]
        col = O.matmul(t, w, xo, n, d).astype(np.float64)
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    yd = torch.full((d,), float("nan"), dtype=torch.float32, device="cuda")
    V.gguf_matmul_dev(t, wd, xd, n, d, yd)
    V.sync()
    got = yd.cpu().numpy().astype(np.float64)
    e = rel_err(got - col, ref - col)
    print(f"type {t} n {n} d {d} factor {factor} zero_col {zero_col}: rel err {e:.2e}")
    assert e < MM_TOL, e


@pytest.mark.parametrize("factor", [100.0, 1000.0])
@pytest.mark.parametrize("name", ["cfg1", "qwen3"])
def test_moe_layer_outlier_channel(V, name, factor):
    """Tokens whose normalised hidden vector has one outlier channel through
    the decode layer.  The router's weights on that channel are zeroed (an
    outlier of this size would otherwise make the softmax one-hot and leave
    no routing margin), so the routing is decided by the other channels and
    the outlier tests the expert mat-vecs: routing bit-exact, outputs
    against the oracle."""
    import torch
    spec = S.olmoe_q8_layer() if name == "cfg1" else S.qwen3_layer()
    L = S.MoeLayer(spec, 1234)
    jj = 3 * 64 + 13
    R = L.router.view(np.float32).reshape(spec.n_experts, spec.dim)
    R[:, jj] = 0.0
    toks, _ = S.routed_tokens(L, 8, 61)
    hbv = toks.copy()
    for i in range(hbv.shape[0]):
        hbv[i, jj] = np.float32(factor * np.abs(hbv[i]).max())
    x0 = (S.normal(62, 3, hbv.size) * 0.3).astype(np.float32).reshape(hbv.shape)
    rx, rids, rwts = O.PortMoe(L)(hbv, x0)
    m = V.MoeLayer(L)
    try:
        hb, x = torch.from_numpy(hbv).cuda(), torch.from_numpy(x0.copy()).cuda()
        ids = torch.zeros((8, spec.n_used), dtype=torch.int32, device="cuda")
        m.ffn(hb, x, ids)
        m.sync()
        got, gi = x.cpu().numpy(), ids.cpu().numpy()
    finally:
        m.close()
    assert np.array_equal(gi, rids)
    errs = [rel_err(got[i] - x0[i], rx[i] - x0[i]) for i in range(8)]
    print(f"{name} factor {factor}: worst rel err {max(errs):.2e}")
    assert max(errs) < TOL, errs
