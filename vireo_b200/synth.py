"""Seeded synthetic GGUF weights and activations for the MoE FFN path.

No real checkpoints or datasets exist on the build or GPU machines, so every
weight and token vector is drawn from a counter-based generator: value i of
stream s under seed k is ``mix64(key(k, s) + (i + 1) * PHI)`` where ``mix64``
is the splitmix64 finaliser.  Being counter-based, any slice can be produced
independently (and later on the device with the same arithmetic), and the
bytes do not depend on the numpy version.

Block layouts follow the GGUF formats the reference reads
(vireo src/gguf_compute.c:38-42 block structs, src/gguf.c:27-38 sizes):
Q8_0 34 B / 32 values, Q4_K 144 B / 256, Q6_K 210 B / 256, Q5_0 22 B / 32.
"""
from __future__ import annotations

import numpy as np

PHI = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_SK = np.uint64(0xD1B54A32D192ED03)

GGML_F32, GGML_F16, GGML_Q5_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 6, 8, 12, 14
BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q5_0: (32, 22), GGML_Q8_0: (32, 34),
         GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210)}
TYPE_NAME = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q5_0: "Q5_0", GGML_Q8_0: "Q8_0",
             GGML_Q4_K: "Q4_K", GGML_Q6_K: "Q6_K"}

_CHUNK = 1 << 18


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _key(seed: int, stream: int) -> np.uint64:
    with np.errstate(over="ignore"):
        a = np.array([seed & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64)
        b = np.array([stream & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64)
        return _mix64(a ^ (b * _SK) ^ PHI)[0]


def u64(seed: int, stream: int, n: int, start: int = 0, out: np.ndarray | None = None) -> np.ndarray:
    """n raw 64-bit values of stream ``stream`` starting at counter ``start``."""
    out = np.empty(n, dtype=np.uint64) if out is None else out
    k = _key(seed, stream)
    m = min(n, _CHUNK)
    z = np.empty(m, dtype=np.uint64)
    t = np.empty(m, dtype=np.uint64)
    s30, s27, s31 = np.uint64(30), np.uint64(27), np.uint64(31)
    with np.errstate(over="ignore"):
        for c0 in range(0, n, _CHUNK):
            c1 = min(n, c0 + _CHUNK)
            w = c1 - c0
            zz, tt = z[:w], t[:w]
            zz[:] = np.arange(start + c0 + 1, start + c1 + 1, dtype=np.uint64)
            np.multiply(zz, PHI, out=zz)
            np.add(zz, k, out=zz)
            # splitmix64 finaliser, in place
            np.right_shift(zz, s30, out=tt); np.bitwise_xor(zz, tt, out=zz); np.multiply(zz, _M1, out=zz)
            np.right_shift(zz, s27, out=tt); np.bitwise_xor(zz, tt, out=zz); np.multiply(zz, _M2, out=zz)
            np.right_shift(zz, s31, out=tt); np.bitwise_xor(zz, tt, out=out[c0:c1])
    return out


def uniform(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    """float64 uniform on [0, 1) from the top 53 bits."""
    return (u64(seed, stream, n, start) >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)


def normal(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    """float64 standard normals by Box-Muller on consecutive uniform pairs."""
    u = uniform(seed, stream, 2 * n, 2 * start)
    u1 = 1.0 - u[0::2]
    u2 = u[1::2]
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def raw_bytes(seed: int, stream: int, nbytes: int) -> np.ndarray:
    n64 = (nbytes + 7) // 8
    return u64(seed, stream, n64).view(np.uint8)[:nbytes]


def f16_bits(v: np.ndarray) -> np.ndarray:
    return np.asarray(v, dtype=np.float64).astype(np.float16).view(np.uint16)


def row_bytes(ggml_type: int, n: int) -> int:
    be, bb = BLOCK[ggml_type]
    assert n % be == 0, (ggml_type, n)
    return n // be * bb


# ---------------------------------------------------------------------------
# block generators: (rows x n) matrices returned as flat uint8 arrays
# ---------------------------------------------------------------------------

def q8_0(seed: int, stream: int, rows: int, n: int, dscale: float = 0.02 / 127) -> np.ndarray:
    """Q8_0: fp16 d = U(0.5,1.5)*dscale, int8 quants uniform on [-127, 127]."""
    nb = rows * n // 32
    blk = np.empty((nb, 34), dtype=np.uint8)
    d = f16_bits((0.5 + uniform(seed, stream * 4 + 0, nb)) * dscale)
    blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    # a random byte b maps to floor(255 * b / 256) - 127, on [-127, 127]
    raw = raw_bytes(seed, stream * 4 + 1, nb * 32).reshape(nb, 32)
    lut = ((np.arange(256, dtype=np.int32) * 255) >> 8) - 127
    lut = lut.astype(np.int8).view(np.uint8)
    for b0 in range(0, nb, 1 << 16):
        b1 = min(nb, b0 + (1 << 16))
        blk[b0:b1, 2:34] = lut[raw[b0:b1]]
    return blk.reshape(-1)


def q4_k(seed: int, stream: int, rows: int, n: int, dscale: float = 9e-5,
         mscale: float = 6.5e-4) -> np.ndarray:
    """Q4_K: fp16 d = U(0.5,1.5)*dscale, dmin = U(0.5,1.5)*mscale, uniform
    random 6-bit scales/mins (all 96 packed bits random) and nibbles."""
    nb = rows * n // 256
    blk = np.empty((nb, 144), dtype=np.uint8)
    blk[:, 0:2] = f16_bits((0.5 + uniform(seed, stream * 4 + 0, nb)) * dscale).view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = f16_bits((0.5 + uniform(seed, stream * 4 + 1, nb)) * mscale).view(np.uint8).reshape(nb, 2)
    rest = raw_bytes(seed, stream * 4 + 2, nb * 140).reshape(nb, 140)
    blk[:, 4:144] = rest
    return blk.reshape(-1)


def q6_k(seed: int, stream: int, rows: int, n: int, dscale: float = 2.5e-5) -> np.ndarray:
    """Q6_K: random 6-bit quants (ql/qh bits), int8 scales uniform on
    [-128, 127], fp16 d = U(0.5,1.5)*dscale."""
    nb = rows * n // 256
    blk = np.empty((nb, 210), dtype=np.uint8)
    blk[:, 0:208] = raw_bytes(seed, stream * 4 + 0, nb * 208).reshape(nb, 208)
    blk[:, 208:210] = f16_bits((0.5 + uniform(seed, stream * 4 + 1, nb)) * dscale).view(np.uint8).reshape(nb, 2)
    return blk.reshape(-1)


def q5_0(seed: int, stream: int, rows: int, n: int, dscale: float = 1e-3) -> np.ndarray:
    nb = rows * n // 32
    blk = np.empty((nb, 22), dtype=np.uint8)
    blk[:, 0:2] = f16_bits((0.5 + uniform(seed, stream * 4 + 0, nb)) * dscale).view(np.uint8).reshape(nb, 2)
    blk[:, 2:22] = raw_bytes(seed, stream * 4 + 1, nb * 20).reshape(nb, 20)
    return blk.reshape(-1)


def f32(seed: int, stream: int, rows: int, n: int, std: float = 0.02) -> np.ndarray:
    return (normal(seed, stream, rows * n) * std).astype(np.float32).view(np.uint8)


def f16(seed: int, stream: int, rows: int, n: int, std: float = 0.02) -> np.ndarray:
    return f16_bits(normal(seed, stream, rows * n) * std).view(np.uint8)


def tensor(ggml_type: int, seed: int, stream: int, rows: int, n: int, **kw) -> np.ndarray:
    fn = {GGML_Q8_0: q8_0, GGML_Q4_K: q4_k, GGML_Q6_K: q6_k, GGML_Q5_0: q5_0,
          GGML_F32: f32, GGML_F16: f16}[ggml_type]
    return fn(seed, stream, rows, n, **kw)


# ---------------------------------------------------------------------------
# MoE layers and routed tokens
# ---------------------------------------------------------------------------

class MoeLayerSpec:
    """Shapes and formats of one MoE FFN layer (reference fields, gguf_run.c:
    dim, ffn_exp, n_experts, n_used, topk_renorm; tensor types per
    ffn_gate_exps / ffn_up_exps / ffn_down_exps)."""

    def __init__(self, dim, ffn_exp, n_experts, n_used, topk_renorm,
                 gate_type, up_type, down_type, router_type=GGML_F32, router_std=0.02):
        self.dim, self.ffn_exp, self.n_experts, self.n_used = dim, ffn_exp, n_experts, n_used
        self.topk_renorm = int(topk_renorm)
        self.gate_type, self.up_type, self.down_type = gate_type, up_type, down_type
        self.router_type, self.router_std = router_type, router_std

    @property
    def gate_slice(self):
        return self.ffn_exp * row_bytes(self.gate_type, self.dim)

    @property
    def up_slice(self):
        return self.ffn_exp * row_bytes(self.up_type, self.dim)

    @property
    def down_slice(self):
        return self.dim * row_bytes(self.down_type, self.ffn_exp)

    @property
    def expert_bytes(self):
        return self.gate_slice + self.up_slice + self.down_slice

    @property
    def router_bytes(self):
        return self.n_experts * row_bytes(self.router_type, self.dim)

    def bytes_per_token(self):
        """Algorithmic HBM bytes for one decode token: the router matrix, the
        n_used experts' three matrices, and the fp32 input/residual/output
        vectors (hidden in, residual in, residual out, plus 16 B ids/weights
        rounding is ignored)."""
        return self.router_bytes + self.n_used * self.expert_bytes + 2 * 4 * self.dim

    def flops_per_token(self):
        fe, d = self.ffn_exp, self.dim
        return 2 * self.n_experts * d + self.n_used * (3 * 2 * d * fe)


class MoeLayer:
    """A generated layer: router (fp32 or other type), and the three 3-D expert
    tensors as raw GGUF bytes with experts outermost (as in GGUF files)."""

    def __init__(self, spec: MoeLayerSpec, seed: int, layer: int = 0, expert_scales=None):
        self.spec, self.seed, self.layer = spec, seed, layer
        s = spec
        base = 1000 * (layer + 1)
        self.router = tensor(s.router_type, seed, base + 1, s.n_experts, s.dim,
                             **({"std": s.router_std} if s.router_type in (GGML_F32, GGML_F16) else {}))
        kw = expert_scales or {}
        self.gate = tensor(s.gate_type, seed, base + 2, s.n_experts * s.ffn_exp, s.dim, **kw.get("gate", {}))
        self.up = tensor(s.up_type, seed, base + 3, s.n_experts * s.ffn_exp, s.dim, **kw.get("up", {}))
        self.down = tensor(s.down_type, seed, base + 4, s.n_experts * s.dim, s.ffn_exp, **kw.get("down", {}))

    def router_f64(self) -> np.ndarray:
        s = self.spec
        if s.router_type == GGML_F32:
            return self.router.view(np.float32).astype(np.float64).reshape(s.n_experts, s.dim)
        if s.router_type == GGML_F16:
            return self.router.view(np.float16).astype(np.float64).reshape(s.n_experts, s.dim)
        raise ValueError("router type must be F32 or F16 for margin filtering")


class SharedExpert:
    """A generated shared expert (the Qwen2-MoE / DeepSeek always-on expert
    FFN): gate and up [ffn][dim], down [dim][ffn] as raw GGUF bytes, and,
    with ``gated``, an fp32 gate vector [dim] (Qwen2-MoE's
    ffn_gate_inp_shexp)."""

    def __init__(self, dim, ffn, gate_type, up_type, down_type, seed, gated=True, layer: int = 0):
        self.dim, self.ffn = dim, ffn
        self.gate_type, self.up_type, self.down_type = gate_type, up_type, down_type
        base = 1000 * (layer + 1) + 500
        self.gate = tensor(gate_type, seed, base + 2, ffn, dim)
        self.up = tensor(up_type, seed, base + 3, ffn, dim)
        self.down = tensor(down_type, seed, base + 4, dim, ffn)
        self.gate_inp = (normal(seed, base + 5, dim) * 0.05).astype(np.float32) if gated else None


def routed_tokens(layer: MoeLayer, n_tok: int, seed: int, stream: int = 7,
                  margin: float = 1e-4, bias=None, dtype=np.float32):
    """n_tok token vectors x ~ N(0,1) whose fp64 router logits (plus an
    optional per-expert bias) have every gap among the top n_used+1 order
    statistics at least ``margin``; candidates failing that are skipped.
    Returns (tokens [n_tok, dim], candidate indices used)."""
    s = layer.spec
    R = layer.router_f64()
    k1 = min(s.n_used + 1, s.n_experts)
    out = np.empty((n_tok, s.dim), dtype=dtype)
    used = []
    c = 0
    batch = max(64, n_tok)
    while len(used) < n_tok:
        cand = normal(seed, stream, batch * s.dim, start=c * s.dim).reshape(batch, s.dim)
        cand = cand.astype(dtype)
        logits = cand.astype(np.float64) @ R.T
        if bias is not None:
            logits = logits + np.asarray(bias, dtype=np.float64)[None, :]
        top = -np.sort(-logits, axis=1)[:, :k1]
        gaps = top[:, :-1] - top[:, 1:]
        ok = np.all(gaps >= margin, axis=1)
        for i in np.nonzero(ok)[0]:
            if len(used) == n_tok:
                break
            out[len(used)] = cand[i]
            used.append(c + i)
        c += batch
    return out, np.array(used, dtype=np.int64)


# the five reference configurations' MoE layer shapes
def olmoe_q8_layer() -> MoeLayerSpec:
    """Config 1: OLMoE-1B-7B-shaped layer, Q8_0 experts, no renorm."""
    return MoeLayerSpec(2048, 1024, 64, 8, 0, GGML_Q8_0, GGML_Q8_0, GGML_Q8_0)


def olmoe_q4km_layer() -> MoeLayerSpec:
    """Config 2's MoE layer: Q4_K gate/up, Q6_K down, 64 experts top-8."""
    return MoeLayerSpec(2048, 1024, 64, 8, 0, GGML_Q4_K, GGML_Q4_K, GGML_Q6_K)


def qwen3_layer() -> MoeLayerSpec:
    """Configs 3-5: Qwen3-30B-A3B-shaped layer, 128 experts top-8 renorm."""
    return MoeLayerSpec(2048, 768, 128, 8, 1, GGML_Q4_K, GGML_Q4_K, GGML_Q6_K)


# ---------------------------------------------------------------------------
# whole decoders (configs 2 and 3): attention + MoE layers
# ---------------------------------------------------------------------------

class DecoderSpec:
    """Shapes and formats of a MoE decoder (the Model fields of the reference
    runner, gguf_run.c:146-155).  qk_norm: "full" (one RMSNorm over all heads,
    OLMoE), "head" (per-head, Qwen3) or None."""

    def __init__(self, n_layers, dim, n_heads, n_kv_heads, head_size, vocab, moe: MoeLayerSpec,
                 qk_norm="full", attn_type=GGML_Q4_K, embd_type=GGML_Q4_K, lm_type=GGML_Q6_K,
                 eps=1e-5, rope_base=10000.0):
        self.n_layers, self.dim, self.n_heads, self.n_kv_heads = n_layers, dim, n_heads, n_kv_heads
        self.head_size, self.vocab, self.moe, self.qk_norm = head_size, vocab, moe, qk_norm
        self.attn_type, self.embd_type, self.lm_type = attn_type, embd_type, lm_type
        self.eps, self.rope_base = float(eps), float(rope_base)
        assert moe.dim == dim

    @property
    def q_dim(self):
        return self.n_heads * self.head_size

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.head_size

    def attn_bytes(self):
        """Weight bytes of one layer's attention block (q, k, v, o matrices
        and the F32 norm vectors)."""
        rb = row_bytes
        b = self.q_dim * rb(self.attn_type, self.dim) + 2 * self.kv_dim * rb(self.attn_type, self.dim)
        b += self.dim * rb(self.attn_type, self.q_dim) + 2 * 4 * self.dim
        if self.qk_norm == "full":
            b += 4 * (self.q_dim + self.kv_dim)
        elif self.qk_norm == "head":
            b += 8 * self.head_size
        return b

    def weight_bytes_per_token(self):
        """Algorithmic weight bytes of one decode step with logits: every
        layer's attention and router rows and its n_used experts, the final
        norm, the LM head, and one embedding row."""
        m = self.moe
        per_layer = self.attn_bytes() + m.router_bytes + m.n_used * m.expert_bytes
        return self.n_layers * per_layer + self.vocab * row_bytes(self.lm_type, self.dim) + 4 * self.dim \
            + row_bytes(self.embd_type, self.dim)

    def kv_bytes_per_position(self, elem_bytes=2):
        """KV cache bytes read per cached position per decode step."""
        return self.n_layers * 2 * self.kv_dim * elem_bytes


class DecoderLayer:
    def __init__(self, spec: DecoderSpec, seed: int, layer: int):
        s = spec
        base = 100000 + 100 * layer
        self.attn_norm = (1.0 + 0.1 * normal(seed, base + 1, s.dim)).astype(np.float32)
        self.ffn_norm = (1.0 + 0.1 * normal(seed, base + 2, s.dim)).astype(np.float32)
        self.wq = tensor(s.attn_type, seed, base + 3, s.q_dim, s.dim)
        self.wk = tensor(s.attn_type, seed, base + 4, s.kv_dim, s.dim)
        self.wv = tensor(s.attn_type, seed, base + 5, s.kv_dim, s.dim)
        self.wo = tensor(s.attn_type, seed, base + 6, s.dim, s.q_dim)
        if s.qk_norm == "full":
            self.q_norm = (1.0 + 0.1 * normal(seed, base + 7, s.q_dim)).astype(np.float32)
            self.k_norm = (1.0 + 0.1 * normal(seed, base + 8, s.kv_dim)).astype(np.float32)
        elif s.qk_norm == "head":
            self.q_norm = (1.0 + 0.1 * normal(seed, base + 7, s.head_size)).astype(np.float32)
            self.k_norm = (1.0 + 0.1 * normal(seed, base + 8, s.head_size)).astype(np.float32)
        else:
            self.q_norm = self.k_norm = None
        self.moe = MoeLayer(s.moe, seed, layer=layer)


class Decoder:
    """A generated decoder: embedding, layers, final norm, LM head."""

    def __init__(self, spec: DecoderSpec, seed: int, n_distinct_layers: int | None = None):
        """n_distinct_layers: generate only that many layers and repeat them
        (large configurations, where the device copies still get distinct
        addresses per layer)."""
        s = spec
        self.spec, self.seed = s, seed
        self.tok_embd = tensor(s.embd_type, seed, 90001, s.vocab, s.dim)
        self.out_norm = (1.0 + 0.1 * normal(seed, 90002, s.dim)).astype(np.float32)
        self.lm_head = tensor(s.lm_type, seed, 90003, s.vocab, s.dim)
        nd = s.n_layers if n_distinct_layers is None else max(1, min(n_distinct_layers, s.n_layers))
        made = [DecoderLayer(s, seed, l) for l in range(nd)]
        self.layers = [made[l % nd] for l in range(s.n_layers)]


def tiny_olmoe_decoder(n_layers=2) -> DecoderSpec:
    return DecoderSpec(n_layers, 512, 4, 4, 128, 512,
                       MoeLayerSpec(512, 256, 16, 4, 0, GGML_Q4_K, GGML_Q4_K, GGML_Q6_K), qk_norm="full")


def tiny_qwen3_decoder(n_layers=2) -> DecoderSpec:
    return DecoderSpec(n_layers, 512, 8, 2, 128, 768,
                       MoeLayerSpec(512, 256, 32, 8, 1, GGML_Q4_K, GGML_Q4_K, GGML_Q6_K), qk_norm="head",
                       eps=1e-6, rope_base=1000000.0)


def olmoe_decoder() -> DecoderSpec:
    """Config 2: OLMoE-1B-7B-shaped, 16 layers, 16 heads x 128, full-width QK
    norm, vocab 50304, 64 experts top-8 (no renorm), Q4_K attention and
    gate/up, Q6_K down and LM head."""
    return DecoderSpec(16, 2048, 16, 16, 128, 50304, olmoe_q4km_layer(), qk_norm="full")


def qwen3_decoder() -> DecoderSpec:
    """Config 3: Qwen3-30B-A3B-shaped, 48 layers, 32 q / 4 kv heads x 128,
    per-head QK norm, vocab 151936, 128 experts top-8 renormalised."""
    return DecoderSpec(48, 2048, 32, 4, 128, 151936, qwen3_layer(), qk_norm="head", eps=1e-6,
                       rope_base=1000000.0)
