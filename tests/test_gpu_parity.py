"""Parity of the CUDA path (through the C-ABI library) with the reference.

Expected values come from the compiled reference (golden fixtures) and from
the bit-exact CPU restatement (oracle/), run on the same seeded inputs.

Tolerances (the north star's bar):
* dequantisation and expert ids: bit-exact;
* MoE-layer outputs: max |got - ref| / max |ref| <= 2e-3 per output vector;
* mat-vec outputs: the same measure <= MM_TOL = 1e-4.  The kernels multiply
  the exact quantised weights by activations carried as two int8 digits per
  value under one fp32 scale per 32 values (|error| <= max|x| / 64516 of the
  group), with exact integer accumulation and fp32 block sums: about 2e-5 on
  random inputs.
"""
import numpy as np
import pytest

from oracle import oracle as O
from vireo_b200 import synth as S

pytestmark = pytest.mark.gpu

TOL = 2e-3
MM_TOL = 1e-4
TYPES = [S.GGML_F32, S.GGML_F16, S.GGML_Q8_0, S.GGML_Q5_0, S.GGML_Q4_K, S.GGML_Q6_K]


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def same_or_both_nan(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


@pytest.fixture(scope="module")
def V():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import vireo_b200
    return vireo_b200


@pytest.mark.parametrize("t", TYPES)
def test_dequant_row_bit_exact(V, golden, t):
    src, ref = golden[f"deq_{t}_src"], golden[f"deq_{t}_out"]
    got = V.gguf_dequant_row(t, src, ref.size)
    assert same_or_both_nan(got, ref)


@pytest.mark.parametrize("t", TYPES)
def test_dequant_row_device_pointers(V, golden, t):
    import torch
    src, ref = golden[f"deq_{t}_src"], golden[f"deq_{t}_out"]
    s = torch.from_numpy(src).cuda()
    out = torch.zeros(ref.size, dtype=torch.float32, device="cuda")
    V.gguf_dequant_row(t, s, ref.size, out)
    assert same_or_both_nan(out.cpu().numpy(), ref)


@pytest.mark.parametrize("t", TYPES)
def test_matmul_golden(V, golden, t):
    for k in [k for k in golden.files if k.startswith(f"mm_{t}_") and k.endswith("_w")]:
        _, _, n, d, _ = k.split("_")
        n, d = int(n), int(d)
        w, x, y = golden[k], golden[k[:-1] + "x"], golden[k[:-1] + "y"]
        got = V.gguf_matmul(t, w, x, n, d)
        assert rel_err(got, y) < MM_TOL, (k, rel_err(got, y))


SHAPES = [(S.GGML_Q8_0, 2048, 1024), (S.GGML_Q8_0, 1024, 2048), (S.GGML_Q4_K, 2048, 768),
          (S.GGML_Q4_K, 2048, 1024), (S.GGML_Q6_K, 768, 2048), (S.GGML_Q6_K, 1024, 2048),
          (S.GGML_Q6_K, 2048, 4096), (S.GGML_Q4_K, 4096, 256), (S.GGML_Q8_0, 256, 16),
          (S.GGML_Q8_0, 96, 40), (S.GGML_Q4_K, 512, 24), (S.GGML_F32, 2048, 128),
          (S.GGML_Q5_0, 2048, 1024), (S.GGML_Q5_0, 768, 2048), (S.GGML_Q5_0, 256, 16), (S.GGML_Q5_0, 96, 40)]


@pytest.mark.parametrize("t,n,d", SHAPES)
def test_matmul_shapes_device(V, t, n, d):
    import torch
    w = S.tensor(t, 21, 5 + t, d, n)
    x = (S.normal(21, 6, n) * 1.7).astype(np.float32)
    ref = O.matmul(t, w, x, n, d)
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    yd = torch.full((d,), float("nan"), dtype=torch.float32, device="cuda")
    V.gguf_matmul_dev(t, wd, xd, n, d, yd)
    V.sync()
    got = yd.cpu().numpy()
    assert rel_err(got, ref) < MM_TOL, rel_err(got, ref)
    # host-pointer entry gives the same numbers
    assert np.array_equal(V.gguf_matmul(t, w, x, n, d), got)


def test_matmul_registered_weights(V):
    t, n, d = S.GGML_Q4_K, 2048, 256
    w = S.tensor(t, 3, 3, d, n)
    x = S.normal(3, 4, n).astype(np.float32)
    ref = O.matmul(t, w, x, n, d)
    lib = V.lib()
    V.check(lib.gguf_weights_register(w.ctypes.data, w.nbytes), "register")
    try:
        got = V.gguf_matmul(t, w[S.row_bytes(t, n) * 16:], x, n, d - 16)
        assert rel_err(got, ref[16:]) < MM_TOL
    finally:
        V.check(lib.gguf_weights_unregister(w.ctypes.data), "unregister")


MOE = ["tiny_q8", "tiny_k", "cfg1_olmoe_q8", "olmoe_q4km", "qwen3"]


def golden_layer(golden, name):
    sp = golden[f"moe_{name}_spec"]
    spec = S.MoeLayerSpec(int(sp[0]), int(sp[1]), int(sp[2]), int(sp[3]), int(sp[4]),
                          int(sp[6]), int(sp[7]), int(sp[8]), router_type=int(sp[5]))
    return S.MoeLayer(spec, int(sp[9]))


def check_moe(x0, x, ids, wts, rx, rids, rwts):
    assert np.array_equal(ids, rids), (ids, rids)
    assert rel_err(wts, rwts) < 1e-5
    for i in range(x.shape[0]):
        e = rel_err(x[i] - x0[i], rx[i] - x0[i])
        assert e < TOL, (i, e)


@pytest.mark.parametrize("name", MOE)
def test_moe_golden_host_api(V, golden, name):
    L = golden_layer(golden, name)
    m = V.MoeLayer(L)
    x0 = golden[f"moe_{name}_x0"]
    x, ids, wts = m.ffn_host(golden[f"moe_{name}_hb"], x0)
    check_moe(x0, x, ids, wts, golden[f"moe_{name}_x"], golden[f"moe_{name}_ids"], golden[f"moe_{name}_wts"])
    m.close()


@pytest.mark.parametrize("name", ["cfg1_olmoe_q8", "qwen3", "olmoe_q4km"])
def test_moe_many_tokens_device_api(V, golden, name):
    import torch
    L = golden_layer(golden, name)
    toks, _ = S.routed_tokens(L, 48, 77)
    x0 = (S.normal(77, 9, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    rx, rids, rwts = O.PortMoe(L)(toks, x0)
    m = V.MoeLayer(L)
    hb, x = torch.from_numpy(toks).cuda(), torch.from_numpy(x0.copy()).cuda()
    ids = torch.zeros((48, L.spec.n_used), dtype=torch.int32, device="cuda")
    wts = torch.zeros((48, L.spec.n_used), dtype=torch.float32, device="cuda")
    m.ffn(hb, x, ids, wts)
    m.sync()
    check_moe(x0, x.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy(), rx, rids, rwts)
    # deterministic: a second run gives identical bits
    x2 = torch.from_numpy(x0.copy()).cuda()
    m.ffn(hb, x2)
    m.sync()
    assert torch.equal(x, x2)
    m.close()


@pytest.mark.parametrize("gt,dt,dim,fe,ne,k", [(S.GGML_Q5_0, S.GGML_Q6_K, 512, 256, 16, 4),
                                               (S.GGML_Q4_K, S.GGML_Q5_0, 2048, 768, 32, 8),
                                               (S.GGML_Q5_0, S.GGML_Q5_0, 1024, 512, 16, 4)])
def test_moe_q5_0_experts(V, gt, dt, dim, fe, ne, k):
    """Q5_0 expert matrices (gguf_compute.c:68-82) on the decode path: a
    layer with Q5_0 gate/up, one with Q5_0 down, one with both, against the
    CPU oracle."""
    import torch
    spec = S.MoeLayerSpec(dim, fe, ne, k, 1, gt, gt, dt)
    L = S.MoeLayer(spec, 71)
    toks, _ = S.routed_tokens(L, 24, 71)
    x0 = (S.normal(71, 9, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    rx, rids, rwts = O.PortMoe(L)(toks, x0)
    m = V.MoeLayer(L)
    try:
        hb, x = torch.from_numpy(toks).cuda(), torch.from_numpy(x0.copy()).cuda()
        ids = torch.zeros((toks.shape[0], k), dtype=torch.int32, device="cuda")
        wts = torch.zeros((toks.shape[0], k), dtype=torch.float32, device="cuda")
        m.ffn(hb, x, ids, wts)
        m.sync()
        check_moe(x0, x.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy(), rx, rids, rwts)
    finally:
        m.close()


@pytest.mark.parametrize("name", ["cfg1_olmoe_q8", "qwen3"])
def test_moe_router_exact_ties(V, golden, name):
    """Experts 2j and 2j + 1 share one router row, so every probability is
    tied with its partner's bit for bit, and the selection must take the
    lower id first (the reference's strict '>' scan from id 0,
    gguf_run.c:190-191).  Router entries are multiples of 1/64 and the
    hidden values small integers, so every logit is exact in any summation
    order and distinct logits differ by at least 1/64: ids bit-exact against
    the oracle on every token."""
    import torch
    L = golden_layer(golden, name)
    s = L.spec
    R = L.router.view(np.float32).reshape(s.n_experts, s.dim)
    R[:] = ((S.u64(91, 1, s.n_experts * s.dim) % np.uint64(17)).astype(np.float32) - 8.0).reshape(R.shape) / 64.0
    R[1::2] = R[0::2]
    n = 12
    toks = ((S.u64(91, 2, n * s.dim) % np.uint64(5)).astype(np.float32) - 2.0).reshape(n, s.dim)
    x0 = (S.normal(91, 3, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    rx, rids, rwts = O.PortMoe(L)(toks, x0)
    assert (rids[:, 0] % 2 == 0).all()  # the lower id of the top pair first
    m = V.MoeLayer(L)
    try:
        hb, x = torch.from_numpy(toks).cuda(), torch.from_numpy(x0.copy()).cuda()
        ids = torch.zeros((n, s.n_used), dtype=torch.int32, device="cuda")
        wts = torch.zeros((n, s.n_used), dtype=torch.float32, device="cuda")
        m.ffn(hb, x, ids, wts)
        m.sync()
        check_moe(x0, x.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy(), rx, rids, rwts)
    finally:
        m.close()


@pytest.mark.parametrize("gated", [True, False])
@pytest.mark.parametrize("gt,dt,ffn", [(S.GGML_Q4_K, S.GGML_Q6_K, 2048), (S.GGML_Q8_0, S.GGML_Q8_0, 768)])
def test_shared_expert_after_routed_block(V, gated, gt, dt, ffn):
    """A shared-expert layer (Qwen2-MoE with the sigmoid gate, DeepSeek
    without): gguf_moe_ffn then gguf_moe_shexp_ffn on one stream give
    x += MoE(hb), then x += s * down(silu(gate hb) * (up hb)), s =
    sigmoid(gate_inp . hb) or 1; against the CPU restatement of the
    reference's moe_ffn followed by the same expert arithmetic
    (gguf_run.c:202-208) on the shared tensors, each mat-vec by the restated
    gguf_matmul.  The shared expert's width differs from the routed
    experts'."""
    import ctypes as C
    import torch
    spec = S.MoeLayerSpec(1024, 512, 16, 4, 1, S.GGML_Q4_K, S.GGML_Q4_K, S.GGML_Q6_K)
    L = S.MoeLayer(spec, 81)
    sh = S.SharedExpert(spec.dim, ffn, gt, gt, dt, 81, gated=gated)
    toks, _ = S.routed_tokens(L, 12, 81)
    n = toks.shape[0]
    x0 = (S.normal(81, 9, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    rx, rids, _ = O.PortMoe(L)(toks, x0)
    ref = rx.astype(np.float64).copy()
    for i in range(n):
        g = O.matmul(gt, sh.gate, toks[i], spec.dim, ffn)
        u = O.matmul(gt, sh.up, toks[i], spec.dim, ffn)
        h = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
        y = O.matmul(dt, sh.down, h, ffn, spec.dim).astype(np.float64)
        sc = 1.0 / (1.0 + np.exp(-float(np.dot(sh.gate_inp.astype(np.float64), toks[i])))) if gated else 1.0
        ref[i] += sc * y
    m = V.MoeLayer(L)
    e = V.SharedExpert(sh)
    try:
        st = torch.cuda.Stream()
        sp = C.c_void_p(st.cuda_stream)
        hb, x = torch.from_numpy(toks).cuda(), torch.from_numpy(x0.copy()).cuda()
        ids = torch.zeros((n, spec.n_used), dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        m.ffn(hb, x, ids, stream=sp)
        e.ffn(hb, x, stream=sp)
        m.sync(sp)
        e.sync(sp)
        got, gi = x.cpu().numpy(), ids.cpu().numpy()
    finally:
        e.close()
        m.close()
    assert np.array_equal(gi, rids)
    errs = [rel_err(got[i] - x0[i], ref[i] - x0[i]) for i in range(n)]
    assert max(errs) < TOL, errs


def test_moe_unsupported_layer_is_rejected(V):
    spec = S.MoeLayerSpec(512, 256, 8, 2, 0, S.GGML_F16, S.GGML_F16, S.GGML_Q8_0)
    L = S.MoeLayer(spec, 1)
    with pytest.raises(V.VireoError) as ei:
        V.MoeLayer(L)
    assert ei.value.status == -3


def expert_out(L, e, x):
    """One expert's FFN output on the CPU oracle: down(silu(gate x) * up x)
    (gguf_run.c:202-208), each mat-vec by the restated gguf_matmul."""
    s = L.spec
    sl = lambda a, n: a.view(np.uint8).ravel()[e * (a.nbytes // s.n_experts):(e + 1) * (a.nbytes // s.n_experts)]
    g = O.matmul(s.gate_type, sl(L.gate, 0), x, s.dim, s.ffn_exp)
    u = O.matmul(s.up_type, sl(L.up, 0), x, s.dim, s.ffn_exp)
    h = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
    return O.matmul(s.down_type, sl(L.down, 0), h, s.ffn_exp, s.dim)


def expert_ptrs(L, m, ids):
    """Device addresses [n][k][3] of the selected experts' slices (experts outermost)."""
    s = L.spec
    gs, us, ds = m.gate.numel() // s.n_experts, m.up.numel() // s.n_experts, m.down.numel() // s.n_experts
    out = np.zeros(ids.shape + (3,), dtype=np.uint64)
    for idx, e in np.ndenumerate(ids):
        if e >= 0:
            out[idx] = (m.gate.data_ptr() + int(e) * gs, m.up.data_ptr() + int(e) * us, m.down.data_ptr() + int(e) * ds)
    return out


@pytest.mark.parametrize("name", ["cfg1_olmoe_q8", "qwen3"])
def test_moe_routed_matches_router(V, golden, name):
    """The routing-override entry (gguf_moe_ffn_routed) given the router's own
    selection reproduces the router path bit for bit; a different selection
    matches the CPU oracle run with that selection."""
    import torch
    L = golden_layer(golden, name)
    n = 6
    toks, _ = S.routed_tokens(L, n, 91)
    x0 = (S.normal(91, 3, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    m = V.MoeLayer(L)
    k = L.spec.n_used
    hb, xa = torch.from_numpy(toks).cuda(), torch.from_numpy(x0.copy()).cuda()
    ids = torch.zeros((n, k), dtype=torch.int32, device="cuda")
    wts = torch.zeros((n, k), dtype=torch.float32, device="cuda")
    m.ffn(hb, xa, ids, wts)
    m.sync()
    hid, hwt = ids.cpu().numpy(), wts.cpu().numpy()
    ptrs = expert_ptrs(L, m, hid)
    xb = torch.from_numpy(x0.copy()).cuda()
    V.check(V.lib().gguf_moe_ffn_routed(m.h, hb.data_ptr(), xb.data_ptr(), n, hid.ctypes.data, hwt.ctypes.data,
                                        ptrs.ctypes.data, None), "gguf_moe_ffn_routed")
    m.sync()
    assert torch.equal(xa, xb)
    # an arbitrary route (reversed expert order, one unused slot) against the oracle's experts
    rid = hid[:, ::-1].copy()
    rid[:, -1] = -1
    rwt = np.linspace(0.05, 0.3, k, dtype=np.float32)[None, :].repeat(n, 0)
    xc = torch.from_numpy(x0.copy()).cuda()
    rptrs = expert_ptrs(L, m, rid)  # named: the library reads it during the call
    V.check(V.lib().gguf_moe_ffn_routed(m.h, hb.data_ptr(), xc.data_ptr(), n, rid.ctypes.data, rwt.ctypes.data,
                                        rptrs.ctypes.data, None), "gguf_moe_ffn_routed")
    m.sync()
    got = xc.cpu().numpy()
    for i in range(n):
        ref = x0[i].astype(np.float64).copy()
        for t in range(k):
            if rid[i, t] >= 0:
                ref += float(rwt[i, t]) * expert_out(L, int(rid[i, t]), toks[i]).astype(np.float64)
        e = rel_err(got[i] - x0[i], ref - x0[i])
        assert e < TOL, (i, e)
    m.close()


def test_moe_store_backed_matches_routed(V, golden):
    """gguf_moe_ffn_store: experts leased from an ExpertStore over a host image
    of the layer (budget of 12 experts for 8 per token, so lookups miss and
    evict) give the same bits as the routed entry with the layer's own device
    tensors, and the budget holds once each token's leases have ended."""
    import ctypes as C
    import torch
    L = golden_layer(golden, "qwen3")
    s = L.spec
    n = 5
    toks, _ = S.routed_tokens(L, n, 17)
    x0 = (S.normal(17, 2, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    m = V.MoeLayer(L)
    lib = V.lib()
    image = np.concatenate([L.gate.view(np.uint8).ravel(), L.up.view(np.uint8).ravel(), L.down.view(np.uint8).ravel()])
    G, U = L.gate.nbytes, L.up.nbytes
    gs, us, ds = G // s.n_experts, U // s.n_experts, L.down.nbytes // s.n_experts
    store = lib.expert_store_create_host(image.ctypes.data, image.nbytes, 12 * (gs + us + ds), 1, s.n_experts)
    assert store
    try:
        for e in range(s.n_experts):
            sl = V.ExpertSlices(e * gs, G + e * us, G + U + e * ds, gs, us, ds)
            lib.expert_store_register(store, 0, e, C.byref(sl))
        rng = np.random.default_rng(5)
        rid = np.stack([rng.choice(s.n_experts, s.n_used, replace=False) for _ in range(n)]).astype(np.int32)
        rwt = rng.uniform(0.05, 0.3, (n, s.n_used)).astype(np.float32)
        hb = torch.from_numpy(toks).cuda()
        xa, xb = torch.from_numpy(x0.copy()).cuda(), torch.from_numpy(x0.copy()).cuda()
        stream = torch.cuda.current_stream().cuda_stream
        for i in range(n):
            V.check(lib.gguf_moe_ffn_store(m.h, store, 0, hb[i].data_ptr(), xa[i].data_ptr(),
                                           rid[i].ctypes.data, rwt[i].ctypes.data, C.c_void_p(stream)),
                    "gguf_moe_ffn_store")
            torch.cuda.synchronize()  # this token's leases end before the next lookups
        rptrs = expert_ptrs(L, m, rid)  # named: the library reads it during the call
        V.check(lib.gguf_moe_ffn_routed(m.h, hb.data_ptr(), xb.data_ptr(), n, rid.ctypes.data, rwt.ctypes.data,
                                        rptrs.ctypes.data, C.c_void_p(stream)), "routed")
        torch.cuda.synchronize()
        assert torch.equal(xa, xb)
        st = V.ExpertStats()
        lib.expert_store_stats(store, C.byref(st))
        assert st.requests == n * s.n_used and st.misses > 12 and st.resident_bytes <= st.capacity_bytes
    finally:
        lib.expert_store_destroy(store)
        m.close()
