"""ctypes access to the parity checkers (test infrastructure only).

* ``port()``  — oracle/_build/liboracle.so, the CPU restatement in
  vireo_oracle.c (each function there cites the reference file:line).
* ``ref()``   — oracle/_ref/libvireo_ref.so, the reference's own sources
  compiled from the reference tree plus ref_harness.c (absent if the
  reference was never available to build it).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may use this
module; the product library never loads either file.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libvireo_ref.so")
REF_SO_V4 = os.path.join(HERE, "_ref", "libvireo_ref_v4.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


def build(ref: bool = True) -> None:
    """Compile the checkers; the reference libraries too when ref is set and
    the environment variable VIREO_REF_SRC names the reference source tree
    (otherwise the prebuilt ones are kept)."""
    targets = ["port"] + (["ref", "ref_store_test"] if ref else [])
    extra = [f"REF={os.environ['VIREO_REF_SRC']}"] if ref and os.environ.get("VIREO_REF_SRC") else []
    subprocess.run(["make", "-s", "-C", HERE] + extra + targets, check=True,
                   env={**os.environ, "OCC": os.environ.get("ORACLE_CC", "gcc")})


def build_dropin() -> bool:
    """The drop-in checkers (oracle/dropin.py) when VIREO_REF_SRC names the
    reference source tree; False when it does not (prebuilt ones are kept)."""
    src = os.environ.get("VIREO_REF_SRC")
    if not src or not os.path.isdir(os.path.join(src, "src")):
        return False
    from oracle import dropin
    dropin.build(src, os.environ.get("ORACLE_CC", "gcc"))
    return True


def host_has_avx512() -> bool:
    """The x86-64-v4 feature set (AVX-512 F, BW, CD, DQ, VL) on this host."""
    try:
        with open("/proc/cpuinfo") as f:
            flags = next((l.split(":", 1)[1].split() for l in f if l.startswith("flags")), [])
    except OSError:
        return False
    return all(x in flags for x in ("avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"))


def ref_build() -> str:
    """Which reference library ref() loads on this host: "x86-64-v4" or "x86-64-v3"."""
    return "x86-64-v4" if host_has_avx512() and os.path.exists(REF_SO_V4) else "x86-64-v3"


class OrcMoeLayer(C.Structure):
    _fields_ = [("dim", C.c_int), ("ffn_exp", C.c_int), ("n_experts", C.c_int),
                ("n_used", C.c_int), ("topk_renorm", C.c_int),
                ("router_type", C.c_uint32), ("gate_type", C.c_uint32),
                ("up_type", C.c_uint32), ("down_type", C.c_uint32),
                ("router", C.c_void_p), ("gate", C.c_void_p), ("up", C.c_void_p),
                ("down", C.c_void_p),
                ("gate_nbytes", C.c_uint64), ("up_nbytes", C.c_uint64),
                ("down_nbytes", C.c_uint64)]


class ExpertStats(C.Structure):
    """Mirror of ExpertStats (reference src/expert_store.h:22-25)."""
    _fields_ = [(n, C.c_uint64) for n in ("requests", "hits", "misses", "bytes_read",
                                          "resident_bytes", "capacity_bytes",
                                          "experts_resident")]


_port = None
_ref = None


def port():
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build(ref=False)
        lib = C.CDLL(PORT_SO)
        lib.orc_f16_to_f32.argtypes = [C.c_uint16]
        lib.orc_f16_to_f32.restype = C.c_float
        lib.orc_dequant_row.argtypes = [C.c_uint32, _u8p, _f32p, C.c_int]
        lib.orc_dequant_row.restype = C.c_int
        lib.orc_matmul.argtypes = [_f32p, _f32p, C.c_uint32, _u8p, C.c_int, C.c_int]
        lib.orc_matmul.restype = C.c_int
        lib.orc_moe_ffn.argtypes = [C.POINTER(OrcMoeLayer), _f32p, _f32p, _i32p, _f32p, C.c_void_p]
        lib.orc_moe_ffn.restype = C.c_int
        lib.orc_moe_ffn_batch.argtypes = [C.POINTER(OrcMoeLayer), C.c_int, _f32p, _f32p, _i32p, _f32p]
        lib.orc_moe_ffn_batch.restype = C.c_int
        lib.orc_moe_ffn_batch_bias.argtypes = [C.POINTER(OrcMoeLayer), C.c_int, _f32p, _f32p, _i32p, _f32p,
                                               C.c_void_p]
        lib.orc_moe_ffn_batch_bias.restype = C.c_int
        lib.orc_route_batch_bias.argtypes = [C.POINTER(OrcMoeLayer), C.c_int, _f32p, _i32p, _f32p, C.c_void_p]
        lib.orc_route_batch_bias.restype = C.c_int
        lib.orc_expert_ffn.argtypes = [C.POINTER(OrcMoeLayer), C.c_int, _f32p, _f32p]
        lib.orc_expert_ffn.restype = C.c_int
        lib.orc_set_threads.argtypes = [C.c_int]
        lib.orc_max_threads.restype = C.c_int
        _port = lib
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO + " (reference library not built)")
        lib = C.CDLL(REF_SO_V4 if ref_build() == "x86-64-v4" else REF_SO)
        lib.gguf_f16_to_f32.argtypes = [C.c_uint16]
        lib.gguf_f16_to_f32.restype = C.c_float
        lib.gguf_dequant_row.argtypes = [C.c_uint32, _u8p, _f32p, C.c_int]
        lib.gguf_dequant_row.restype = None
        lib.ref_matmul.argtypes = [_f32p, _f32p, C.c_uint32, _u8p, C.c_int, C.c_int]
        lib.ref_matmul.restype = None
        lib.ref_moe_create.argtypes = [C.c_int] * 5 + [C.c_uint32, C.c_void_p, C.c_uint64] * 4 + [C.c_uint64]
        lib.ref_moe_create.restype = C.c_void_p
        lib.ref_moe_ffn.argtypes = [C.c_void_p, _f32p, _f32p, _i32p, _f32p]
        lib.ref_moe_ffn.restype = C.c_int
        lib.ref_moe_ffn_batch.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p, _i32p, _f32p]
        lib.ref_moe_ffn_batch.restype = C.c_int
        lib.ref_moe_stats.argtypes = [C.c_void_p, C.POINTER(ExpertStats)]
        lib.ref_moe_destroy.argtypes = [C.c_void_p]
        lib.ref_set_threads.argtypes = [C.c_int]
        lib.ref_max_threads.restype = C.c_int
        lib.ref_decoder_create.argtypes = [C.c_int] * 6 + [C.c_float, C.c_float] + [C.c_int] * 4 + [C.c_void_p] * 4
        lib.ref_decoder_create.restype = C.c_void_p
        lib.ref_decoder_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        lib.ref_decoder_forward.restype = C.c_int
        lib.ref_decoder_destroy.argtypes = [C.c_void_p]
        lib.ref_decoder_destroy.restype = None
        lib.ref_decoder_fill_kv.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
        lib.ref_decoder_fill_kv.restype = None
        lib.ref_decoder_last_gap.argtypes = []
        lib.ref_decoder_last_gap.restype = C.c_double
        # the reference's own ExpertStore (src/expert_store.c, compiled into the same library)
        lib.expert_store_create.argtypes = [C.c_int, C.c_uint64, C.c_int, C.c_int]
        lib.expert_store_create.restype = C.c_void_p
        lib.expert_store_register.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        lib.expert_store_register.restype = None
        lib.expert_store_lookup.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        lib.expert_store_lookup.restype = C.c_int
        lib.expert_store_release.argtypes = [C.c_void_p, C.c_void_p]
        lib.expert_store_release.restype = None
        lib.expert_store_stats.argtypes = [C.c_void_p, C.POINTER(ExpertStats)]
        lib.expert_store_stats.restype = None
        lib.expert_store_destroy.argtypes = [C.c_void_p]
        lib.expert_store_destroy.restype = None
        _ref = lib
    return _ref


# ---------------------------------------------------------------------------
# convenience wrappers over numpy arrays
# ---------------------------------------------------------------------------

def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint8).reshape(-1)


def dequant_row(ggml_type: int, src, n: int, lib=None) -> np.ndarray:
    lib = lib or port()
    out = np.zeros(n, dtype=np.float32)
    if lib is _ref:
        lib.gguf_dequant_row(ggml_type, _u8(src), out, n)
    else:
        lib.orc_dequant_row(ggml_type, _u8(src), out, n)
    return out


def matmul(ggml_type: int, w, x, n: int, d: int, lib=None) -> np.ndarray:
    lib = lib or port()
    y = np.zeros(d, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if lib is _ref:
        lib.ref_matmul(y, x, ggml_type, _u8(w), n, d)
    else:
        lib.orc_matmul(y, x, ggml_type, _u8(w), n, d)
    return y


class PortMoe:
    """The restated moe_ffn over a synth.MoeLayer (arrays kept alive here)."""

    def __init__(self, layer):
        s = layer.spec
        self.layer = layer
        self._keep = [_u8(layer.router), _u8(layer.gate), _u8(layer.up), _u8(layer.down)]
        self.desc = OrcMoeLayer(s.dim, s.ffn_exp, s.n_experts, s.n_used, s.topk_renorm,
                                s.router_type, s.gate_type, s.up_type, s.down_type,
                                self._keep[0].ctypes.data, self._keep[1].ctypes.data,
                                self._keep[2].ctypes.data, self._keep[3].ctypes.data,
                                self._keep[1].nbytes, self._keep[2].nbytes, self._keep[3].nbytes)

    def __call__(self, hb, x=None, bias=None):
        """Returns (x_out, ids, wts) for a batch of independent tokens; bias
        (optional, [n_experts]) is added to the router logits before the
        softmax (the restated function with bias=None is the reference's)."""
        s = self.layer.spec
        hb = np.ascontiguousarray(hb, dtype=np.float32).reshape(-1, s.dim)
        n = hb.shape[0]
        x = np.zeros_like(hb) if x is None else np.array(x, dtype=np.float32).reshape(n, s.dim)
        k = min(s.n_used, 64)
        ids = np.zeros((n, k), dtype=np.int32)
        wts = np.zeros((n, k), dtype=np.float32)
        if bias is None:
            port().orc_moe_ffn_batch(C.byref(self.desc), n, hb.reshape(-1), x.reshape(-1),
                                     ids.reshape(-1), wts.reshape(-1))
        else:
            b = np.ascontiguousarray(bias, dtype=np.float32)
            port().orc_moe_ffn_batch_bias(C.byref(self.desc), n, hb.reshape(-1), x.reshape(-1),
                                          ids.reshape(-1), wts.reshape(-1), b.ctypes.data)
        return x, ids, wts


    def route(self, hb, bias=None):
        """The routing alone (router, optional bias, softmax, top-k, renorm):
        (ids, wts) for a batch of tokens, as __call__ returns them."""
        s = self.layer.spec
        hb = np.ascontiguousarray(hb, dtype=np.float32).reshape(-1, s.dim)
        n = hb.shape[0]
        k = min(s.n_used, 64)
        ids = np.zeros((n, k), dtype=np.int32)
        wts = np.zeros((n, k), dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        port().orc_route_batch_bias(C.byref(self.desc), n, hb.reshape(-1), ids.reshape(-1), wts.reshape(-1),
                                    None if b is None else b.ctypes.data)
        return ids, wts

    def expert(self, e: int, hb) -> np.ndarray:
        """One expert's FFN output (before the gate weight) for one token:
        the body of the reference's per-expert loop, gguf_run.c:202-208."""
        s = self.layer.spec
        hb = np.ascontiguousarray(hb, dtype=np.float32).reshape(s.dim)
        out = np.zeros(s.dim, dtype=np.float32)
        if port().orc_expert_ffn(C.byref(self.desc), int(e), hb, out):
            raise ValueError(f"bad expert id {e}")
        return out


class RefTensorIn(C.Structure):
    _fields_ = [("type", C.c_uint32), ("data", C.c_void_p), ("nbytes", C.c_uint64), ("dim0", C.c_uint64)]


class RefDecoder:
    """The reference's own forward() (gguf_run.c:216-252, through
    ref_harness.c) over a synth.Decoder: its dense KV store and its
    ExpertStore, one decode step per call."""

    def __init__(self, dec):
        s = dec.spec
        m = s.moe
        self.dec = dec
        keep = []

        def t(ggml_type, arr, dim0):
            if arr is None:
                return RefTensorIn(0, None, 0, 0)
            a = _u8(arr)
            keep.append(a)
            return RefTensorIn(ggml_type, a.ctypes.data, a.nbytes, dim0)

        F32 = 0
        tok = t(s.embd_type, dec.tok_embd, s.dim)
        on = t(F32, dec.out_norm, s.dim)
        lm = t(s.lm_type, dec.lm_head, s.dim)
        rows = []
        for ly in dec.layers:
            qn = s.head_size if s.qk_norm == "head" else s.q_dim
            kn = s.head_size if s.qk_norm == "head" else s.kv_dim
            rows += [t(F32, ly.attn_norm, s.dim), t(s.attn_type, ly.wq, s.dim), t(s.attn_type, ly.wk, s.dim),
                     t(s.attn_type, ly.wv, s.dim), t(s.attn_type, ly.wo, s.q_dim), t(F32, ly.ffn_norm, s.dim),
                     t(F32, ly.q_norm, qn), t(F32, ly.k_norm, kn), t(m.router_type, ly.moe.router, s.dim),
                     t(m.gate_type, ly.moe.gate, s.dim), t(m.up_type, ly.moe.up, s.dim),
                     t(m.down_type, ly.moe.down, m.ffn_exp)]
        arr = (RefTensorIn * len(rows))(*rows)
        self._keep = (keep, tok, on, lm, arr)
        self.h = ref().ref_decoder_create(s.n_layers, s.dim, s.n_heads, s.n_kv_heads, s.head_size, s.vocab, s.eps,
                                          s.rope_base, m.n_experts, m.n_used, m.ffn_exp, m.topk_renorm,
                                          C.byref(tok), C.byref(on), C.byref(lm), arr)
        if not self.h:
            raise RuntimeError("ref_decoder_create failed")

    def step(self, token: int, pos: int, want_logits: bool = True):
        """(logits or None, residual x, argmax or -1)"""
        s = self.dec.spec
        lg = np.zeros(s.vocab, dtype=np.float32)
        x = np.zeros(s.dim, dtype=np.float32)
        a = ref().ref_decoder_forward(self.h, int(token), int(pos), int(want_logits), lg.ctypes.data,
                                      x.ctypes.data)
        return (lg if want_logits else None), x, a

    def fill_kv(self, n_pos: int, seed: int = 1) -> None:
        """Seeded K/V for positions [0, n_pos) of every layer and kv head,
        through the reference's own kv_append (timing at long context)."""
        ref().ref_decoder_fill_kv(self.h, int(n_pos), int(seed))

    def last_gap(self) -> float:
        """Smallest log-probability gap among the top n_used + 1 router
        choices over every layer of the last step (a near-tie when ~0)."""
        return float(ref().ref_decoder_last_gap())

    def close(self):
        if getattr(self, "h", None):
            ref().ref_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefMoe:
    """The reference's own moe_ffn (through ref_harness.c) over a synth.MoeLayer."""

    def __init__(self, layer, cap_bytes: int = 0):
        s = layer.spec
        self.layer = layer
        self._keep = [_u8(layer.router), _u8(layer.gate), _u8(layer.up), _u8(layer.down)]
        r = self._keep
        self.h = ref().ref_moe_create(s.dim, s.ffn_exp, s.n_experts, s.n_used, s.topk_renorm,
                                      s.router_type, r[0].ctypes.data, r[0].nbytes,
                                      s.gate_type, r[1].ctypes.data, r[1].nbytes,
                                      s.up_type, r[2].ctypes.data, r[2].nbytes,
                                      s.down_type, r[3].ctypes.data, r[3].nbytes, cap_bytes)
        if not self.h:
            raise RuntimeError("ref_moe_create failed")

    def __call__(self, hb, x=None):
        s = self.layer.spec
        hb = np.ascontiguousarray(hb, dtype=np.float32).reshape(-1, s.dim)
        n = hb.shape[0]
        x = np.zeros_like(hb) if x is None else np.array(x, dtype=np.float32).reshape(n, s.dim)
        k = min(s.n_used, 64)
        ids = np.zeros((n, k), dtype=np.int32)
        wts = np.zeros((n, k), dtype=np.float32)
        ref().ref_moe_ffn_batch(self.h, n, hb.reshape(-1), x.reshape(-1), ids.reshape(-1), wts.reshape(-1))
        return x, ids, wts

    def stats(self) -> ExpertStats:
        st = ExpertStats()
        ref().ref_moe_stats(self.h, C.byref(st))
        return st

    def close(self):
        if self.h:
            ref().ref_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DropInDecoder:
    """The reference's decoder opened from a GGUF file by its own loader
    (oracle/dropin_harness.c): b200=False is the reference as it ships;
    b200=True is the same runner with gguf_compute.c and expert_store.c
    replaced by libvireo_b200.so and every MoE block run by gguf_moe_ffn_host
    from the hook at the top of moe_ffn."""

    def __init__(self, path: str, b200: bool):
        from oracle import dropin
        so = dropin.B200_SO if b200 else dropin.REF_SO
        if not os.path.exists(so):
            raise FileNotFoundError(so + " (drop-in checker not built)")
        lib = C.CDLL(so)
        lib.dropin_open.argtypes = [C.c_char_p]
        lib.dropin_open.restype = C.c_void_p
        lib.dropin_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        lib.dropin_forward.restype = C.c_int
        lib.dropin_close.argtypes = [C.c_void_p]
        lib.dropin_close.restype = None
        lib.dropin_vocab.argtypes = [C.c_void_p]
        lib.dropin_vocab.restype = C.c_int
        lib.dropin_dim.argtypes = [C.c_void_p]
        lib.dropin_dim.restype = C.c_int
        lib.dropin_hook_calls.argtypes = []
        lib.dropin_hook_calls.restype = C.c_long
        self.lib = lib
        self.h = lib.dropin_open(path.encode())
        if not self.h:
            raise RuntimeError(f"dropin_open failed on {path}")
        self.vocab = lib.dropin_vocab(self.h)
        self.dim = lib.dropin_dim(self.h)

    def step(self, token: int, pos: int, want_logits: bool = True):
        """(logits or None, residual x after the step, argmax or -1)."""
        lg = np.zeros(self.vocab, dtype=np.float32)
        x = np.zeros(self.dim, dtype=np.float32)
        a = self.lib.dropin_forward(self.h, int(token), int(pos), int(want_logits), lg.ctypes.data, x.ctypes.data)
        return (lg if want_logits else None), x, a

    def hook_calls(self) -> int:
        return int(self.lib.dropin_hook_calls())

    def close(self):
        if self.h:
            self.lib.dropin_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
