"""gguf_moe_ffn_noalloc: the MoE decode kernel with its scratch in a fixed
device array (no device allocation), checked against gguf_moe_ffn on the
same layer and tokens, on two calls in a row.

Collected last on purpose: it must pass after the other GPU tests (device
already set up, other handles created and destroyed) as well as alone in a
fresh process (the call then does the per-device set-up itself).
"""
import ctypes as C

import numpy as np
import pytest

from vireo_b200 import synth as S

pytestmark = pytest.mark.gpu

TOL = 2e-3  # max |got - ref| / max |ref| per output vector


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("formats", [(S.GGML_Q4_K, S.GGML_Q6_K, 1), (S.GGML_Q8_0, S.GGML_Q8_0, 0)])
def test_noalloc_matches_handle_path(formats):
    import torch
    import vireo_b200 as V
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    gu, dn, renorm = formats
    spec = S.MoeLayerSpec(1024, 512, 16, 4, renorm, gu, gu, dn)
    layer = S.MoeLayer(spec, 4242)
    n = 3
    toks, _ = S.routed_tokens(layer, n, 4242)
    x0 = (S.normal(4242, 5, toks.size) * 0.3).astype(np.float32).reshape(toks.shape)
    m = V.MoeLayer(layer)
    try:
        hb = torch.from_numpy(toks).cuda()
        xa = torch.from_numpy(x0.copy()).cuda()
        ids_a = torch.zeros((n, spec.n_used), dtype=torch.int32, device="cuda")
        wts_a = torch.zeros((n, spec.n_used), dtype=torch.float32, device="cuda")
        m.ffn(hb, xa, ids_a, wts_a)
        m.sync()
        ref_x, ref_ids, ref_wts = xa.cpu().numpy(), ids_a.cpu().numpy(), wts_a.cpu().numpy()
        lib = V.lib()
        for call in range(2):
            xb = torch.from_numpy(x0.copy()).cuda()
            ids_b = torch.full((n, spec.n_used), -7, dtype=torch.int32, device="cuda")
            wts_b = torch.zeros((n, spec.n_used), dtype=torch.float32, device="cuda")
            st = lib.gguf_moe_ffn_noalloc(C.byref(m.desc), hb.data_ptr(), xb.data_ptr(), n, ids_b.data_ptr(),
                                          wts_b.data_ptr(), None)
            assert st == 0, (call, st)
            torch.cuda.synchronize()
            assert np.array_equal(ids_b.cpu().numpy(), ref_ids), call
            assert rel_err(wts_b.cpu().numpy(), ref_wts) < 1e-6, call
            got = xb.cpu().numpy()
            for i in range(n):
                e = rel_err(got[i] - x0[i], ref_x[i] - x0[i])
                assert e < TOL, (call, i, e)
    finally:
        m.close()
