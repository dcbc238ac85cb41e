"""The CPU restatement (oracle/vireo_oracle.c) against the reference's own
outputs (tests/golden/reference_vectors.npz, made by gen_golden.py from the
compiled reference).  Everything here is bit-exact: same rounding steps,
same FMA placement, same reduction trees."""
import hashlib

import numpy as np
import pytest

from oracle import oracle as O
from vireo_b200 import synth as S

TYPES = [S.GGML_F32, S.GGML_F16, S.GGML_Q8_0, S.GGML_Q5_0, S.GGML_Q4_K, S.GGML_Q6_K]


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def same_or_both_nan(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return np.array_equal(bits(a)[~nan], bits(b)[~nan]) and np.array_equal(np.isnan(a), np.isnan(b))


def test_f16_all_values(golden):
    P = O.port()
    got = np.array([np.float32(P.orc_f16_to_f32(h)).view(np.uint32) for h in range(65536)], dtype=np.uint32)
    assert np.array_equal(got, golden["f16_bits"])


@pytest.mark.parametrize("t", TYPES)
def test_dequant_row(golden, t):
    src = golden[f"deq_{t}_src"]
    ref = golden[f"deq_{t}_out"]
    got = O.dequant_row(t, src, ref.size)
    assert same_or_both_nan(got, ref)


@pytest.mark.parametrize("t", TYPES)
def test_matmul(golden, t):
    keys = [k for k in golden.files if k.startswith(f"mm_{t}_") and k.endswith("_w")]
    assert keys
    for k in keys:
        _, _, n, d, _ = k.split("_")
        n, d = int(n), int(d)
        w, x, y = golden[k], golden[k[:-1] + "x"], golden[k[:-1] + "y"]
        assert np.array_equal(bits(O.matmul(t, w, x, n, d)), bits(y)), k


MOE = ["tiny_q8", "tiny_k", "cfg1_olmoe_q8", "olmoe_q4km", "qwen3"]


def layer_from(golden, name):
    sp = golden[f"moe_{name}_spec"]
    spec = S.MoeLayerSpec(*[int(v) for v in sp[:9]][:5], int(sp[6]), int(sp[7]), int(sp[8]),
                          router_type=int(sp[5]))
    return S.MoeLayer(spec, int(sp[9]))


@pytest.mark.parametrize("name", MOE)
def test_moe_ffn(golden, name):
    L = layer_from(golden, name)
    h = hashlib.sha256()
    for a in (L.router, L.gate, L.up, L.down):
        h.update(np.ascontiguousarray(a).view(np.uint8).tobytes())
    assert h.digest() == golden[f"moe_{name}_sha"].tobytes(), "synthetic generator drifted"
    x, ids, wts = O.PortMoe(L)(golden[f"moe_{name}_hb"], golden[f"moe_{name}_x0"])
    assert np.array_equal(ids, golden[f"moe_{name}_ids"])
    assert np.array_equal(bits(wts), bits(golden[f"moe_{name}_wts"]))
    assert np.array_equal(bits(x), bits(golden[f"moe_{name}_x"]))


def test_routed_tokens_margin():
    """Generated tokens keep every top-(k+1) logit gap >= 1e-4 (fp64)."""
    L = S.MoeLayer(S.MoeLayerSpec(512, 256, 16, 4, 1, S.GGML_Q4_K, S.GGML_Q4_K, S.GGML_Q6_K), 5)
    toks, _ = S.routed_tokens(L, 32, 5)
    lg = toks.astype(np.float64) @ L.router_f64().T
    top = -np.sort(-lg, axis=1)[:, :5]
    assert (np.diff(-top, axis=1) >= 1e-4).all()
