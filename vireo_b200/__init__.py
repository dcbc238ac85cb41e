"""vireo-b200: vireo's MoE FFN hot path, B200-native (sm_100a).

The product is the C-ABI shared library ``libvireo_b200.so`` built from
``csrc/`` (headers in ``include/``).  This package loads it with ctypes and
mirrors the reference interface for Python callers:

* ``gguf_matmul`` / ``gguf_dequant_row`` / ``gguf_f16_to_f32`` — the three
  functions of the reference's gguf_compute.h (vireo src/gguf_compute.h:8-10);
* ``MoeLayer`` — the MoE FFN block (reference moe_ffn, src/gguf_run.c:185-214)
  behind ``gguf_moe_*``.

There is no fallback: if the library is missing or no CUDA device is
present, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvireo_b200.so")

VIREO_OK = 0
STATUS = {0: "ok", -1: "invalid argument", -2: "CUDA runtime error", -3: "unsupported tensor type or shape",
          -4: "device wait timed out", -5: "out of memory", -6: "I/O error", -7: "no CUDA device"}


class VireoError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        super().__init__(f"{what}: {STATUS.get(status, status)} ({status})")
        self.status = status


def build(jobs: int = 8) -> str:
    """Compile libvireo_b200.so for sm_100a (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", "-C", HERE, f"-j{jobs}"], check=True)
    return LIB_PATH


class GgufTensor(C.Structure):
    """gguf_tensor (reference src/gguf.h:36-45), ABI-identical."""
    _fields_ = [("name_ptr", C.c_char_p), ("name_len", C.c_uint64), ("n_dims", C.c_uint32),
                ("dims", C.c_uint64 * 4), ("ggml_type", C.c_uint32), ("offset", C.c_uint64),
                ("data", C.c_void_p), ("n_elems", C.c_uint64), ("nbytes", C.c_uint64)]


class GgufMoeDesc(C.Structure):
    _fields_ = [("dim", C.c_int), ("ffn_exp", C.c_int), ("n_experts", C.c_int), ("n_used", C.c_int),
                ("topk_renorm", C.c_int), ("router_type", C.c_uint32), ("gate_type", C.c_uint32),
                ("up_type", C.c_uint32), ("down_type", C.c_uint32), ("router", C.c_void_p),
                ("gate_exps", C.c_void_p), ("up_exps", C.c_void_p), ("down_exps", C.c_void_p),
                ("gate_nbytes", C.c_uint64), ("up_nbytes", C.c_uint64), ("down_nbytes", C.c_uint64)]


class GgufMoeShexpDesc(C.Structure):
    _fields_ = [("dim", C.c_int), ("ffn", C.c_int), ("gate_type", C.c_uint32), ("up_type", C.c_uint32),
                ("down_type", C.c_uint32), ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
                ("gate_inp", C.c_void_p)]


class ExpertStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("requests", "hits", "misses", "bytes_read", "resident_bytes",
                                          "capacity_bytes", "experts_resident")]


class ExpertSlices(C.Structure):
    _fields_ = [("gate_off", C.c_uint64), ("up_off", C.c_uint64), ("down_off", C.c_uint64),
                ("gate_bytes", C.c_uint32), ("up_bytes", C.c_uint32), ("down_bytes", C.c_uint32)]


class ExpertView(C.Structure):
    _fields_ = [("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p), ("slot", C.c_void_p)]


class ExpertStatsExt(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("h2d_bytes", "copies", "evictions", "over_budget_loads")]


_lib = None


def lib():
    """The loaded C-ABI library (raises if it was never built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: run vireo_b200.build() (no CPU fallback exists)")
        L = C.CDLL(LIB_PATH)
        L.gguf_f16_to_f32.argtypes = [C.c_uint16]
        L.gguf_f16_to_f32.restype = C.c_float
        L.gguf_dequant_row.argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_int]
        L.gguf_dequant_row.restype = None
        L.gguf_matmul.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(GgufTensor), C.c_int, C.c_int]
        L.gguf_matmul.restype = None
        L.vireo_last_error.restype = C.c_int
        L.vireo_status_string.argtypes = [C.c_int]
        L.vireo_status_string.restype = C.c_char_p
        L.vireo_device_init.argtypes = [C.c_int]
        L.gguf_matmul_dev.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(GgufTensor), C.c_int, C.c_int, C.c_void_p]
        L.gguf_dequant_row_dev.argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.gguf_weights_register.argtypes = [C.c_void_p, C.c_uint64]
        L.gguf_weights_unregister.argtypes = [C.c_void_p]
        L.vireo_sync.argtypes = [C.c_void_p]
        L.gguf_moe_create.argtypes = [C.POINTER(GgufMoeDesc), C.POINTER(C.c_void_p)]
        L.gguf_moe_ffn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.gguf_moe_ffn_host.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.gguf_moe_sync.argtypes = [C.c_void_p, C.c_void_p]
        L.gguf_moe_set_expert_ptrs.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        L.gguf_moe_destroy.argtypes = [C.c_void_p]
        L.gguf_moe_shexp_create.argtypes = [C.POINTER(GgufMoeShexpDesc), C.POINTER(C.c_void_p)]
        L.gguf_moe_shexp_ffn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.gguf_moe_shexp_sync.argtypes = [C.c_void_p, C.c_void_p]
        L.gguf_moe_shexp_destroy.argtypes = [C.c_void_p]
        L.gguf_moe_ffn_noalloc.argtypes = [C.POINTER(GgufMoeDesc), C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                           C.c_void_p, C.c_void_p]
        L.gguf_moe_destroy.restype = None
        L.gguf_moe_ffn_routed.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_void_p]
        L.gguf_moe_ffn_store.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p]
        L.gguf_moe_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_void_p]
        # expert parallelism (include/gguf_moe.h)
        L.gguf_moe_ep_unique_id.argtypes = [C.c_void_p]
        L.gguf_moe_ep_place.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.gguf_moe_ep_rows.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.gguf_moe_ep_create.argtypes = [C.POINTER(GgufMoeDesc), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                         C.POINTER(C.c_void_p)]
        L.gguf_moe_prefill_ep.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_void_p]
        L.gguf_moe_ep_sync.argtypes = [C.c_void_p, C.c_void_p]
        L.gguf_moe_ep_layer.argtypes = [C.c_void_p]
        L.gguf_moe_ep_layer.restype = C.c_void_p
        L.gguf_moe_ep_destroy.argtypes = [C.c_void_p]
        L.gguf_moe_ep_destroy.restype = None
        # ExpertStore (include/expert_store.h)
        L.expert_store_create.argtypes = [C.c_int, C.c_uint64, C.c_int, C.c_int]
        L.expert_store_create.restype = C.c_void_p
        L.expert_store_create_host.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_int, C.c_int]
        L.expert_store_create_host.restype = C.c_void_p
        L.expert_store_register.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(ExpertSlices)]
        L.expert_store_register.restype = None
        L.expert_store_lookup.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(ExpertView)]
        L.expert_store_lookup_async.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(ExpertView), C.c_void_p]
        L.expert_store_release.argtypes = [C.c_void_p, C.POINTER(ExpertView)]
        L.expert_store_release.restype = None
        L.expert_store_release_after.argtypes = [C.c_void_p, C.POINTER(ExpertView), C.c_void_p]
        L.expert_store_stats.argtypes = [C.c_void_p, C.POINTER(ExpertStats)]
        L.expert_store_stats.restype = None
        L.expert_store_stats_ext.argtypes = [C.c_void_p, C.POINTER(ExpertStatsExt)]
        L.expert_store_stats_ext.restype = None
        L.expert_store_destroy.argtypes = [C.c_void_p]
        L.expert_store_destroy.restype = None
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != VIREO_OK:
        raise VireoError(status, what)


def _ptr(a) -> int:
    """Address of a numpy array or torch tensor."""
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


# ---------------------------------------------------------------------------
# gguf_compute.h mirror
# ---------------------------------------------------------------------------

def gguf_f16_to_f32(h: int) -> float:
    return lib().gguf_f16_to_f32(h)


def gguf_dequant_row(ggml_type: int, src, n: int, out=None):
    """Reference gguf_dequant_row; src/out numpy (host) or torch CUDA tensors."""
    if out is None:
        out = np.zeros(n, dtype=np.float32)
    lib().gguf_dequant_row(ggml_type, _ptr(src), _ptr(out), n)
    check(lib().vireo_last_error(), "gguf_dequant_row")
    return out


def make_tensor(ggml_type: int, data) -> GgufTensor:
    t = GgufTensor()
    t.ggml_type = ggml_type
    t.data = _ptr(data)
    return t


def gguf_matmul(ggml_type: int, w, x, n: int, d: int, y=None):
    """Reference gguf_matmul: y[d] = W[d x n] . x[n] (host or device buffers)."""
    if y is None:
        y = np.zeros(d, dtype=np.float32)
    t = make_tensor(ggml_type, w)
    lib().gguf_matmul(_ptr(y), _ptr(x), C.byref(t), n, d)
    check(lib().vireo_last_error(), "gguf_matmul")
    return y


def gguf_matmul_dev(ggml_type: int, w, x, n: int, d: int, y, stream=None) -> None:
    t = make_tensor(ggml_type, w)
    check(lib().gguf_matmul_dev(_ptr(y), _ptr(x), C.byref(t), n, d, stream), "gguf_matmul_dev")


def sync(stream=None) -> None:
    check(lib().vireo_sync(stream), "vireo_sync")


# ---------------------------------------------------------------------------
# MoE block (gguf_moe.h)
# ---------------------------------------------------------------------------

class MoeLayer:
    """One MoE FFN layer resident in HBM, evaluated by gguf_moe_ffn.

    ``layer`` is a ``vireo_b200.synth.MoeLayer`` or any object with ``spec``
    (dim, ffn_exp, n_experts, n_used, topk_renorm, *_type) and raw GGUF byte
    arrays ``router``, ``gate``, ``up``, ``down`` (experts outermost).
    Device memory is held in torch tensors (plumbing only)."""

    def __init__(self, layer, device: int = 0):
        import torch
        s = layer.spec
        self.spec = s
        self.device = torch.device("cuda", device)
        up = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).to(self.device)
        self.router, self.gate, self.up, self.down = up(layer.router), up(layer.gate), up(layer.up), up(layer.down)
        self.desc = GgufMoeDesc(s.dim, s.ffn_exp, s.n_experts, s.n_used, s.topk_renorm, s.router_type,
                                s.gate_type, s.up_type, s.down_type, self.router.data_ptr(),
                                self.gate.data_ptr(), self.up.data_ptr(), self.down.data_ptr(),
                                self.gate.numel(), self.up.numel(), self.down.numel())
        h = C.c_void_p()
        check(lib().gguf_moe_create(C.byref(self.desc), C.byref(h)), "gguf_moe_create")
        self.h = h

    def ffn(self, hb, x, ids=None, wts=None, stream=None) -> None:
        """Device tensors: hb/x [n_tok, dim] fp32 (x updated), ids/wts [n_tok, n_used]."""
        n = hb.shape[0] if hb.dim() > 1 else 1
        check(lib().gguf_moe_ffn(self.h, hb.data_ptr(), x.data_ptr(), n,
                                 ids.data_ptr() if ids is not None else None,
                                 wts.data_ptr() if wts is not None else None, stream), "gguf_moe_ffn")

    def sync(self, stream=None) -> None:
        check(lib().gguf_moe_sync(self.h, stream), "gguf_moe_sync")

    def ffn_host(self, hb: np.ndarray, x: np.ndarray | None = None):
        """Host buffers through gguf_moe_ffn_host; returns (x_out, ids, wts)."""
        s = self.spec
        hb = np.ascontiguousarray(hb, dtype=np.float32).reshape(-1, s.dim)
        n = hb.shape[0]
        x = np.zeros_like(hb) if x is None else np.array(x, dtype=np.float32).reshape(n, s.dim)
        ids = np.zeros((n, s.n_used), dtype=np.int32)
        wts = np.zeros((n, s.n_used), dtype=np.float32)
        check(lib().gguf_moe_ffn_host(self.h, hb.ctypes.data, x.ctypes.data, n, ids.ctypes.data, wts.ctypes.data),
              "gguf_moe_ffn_host")
        return x, ids, wts

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().gguf_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ep_place(expected_load, world: int) -> np.ndarray:
    """gguf_moe_ep_place: expert -> rank by expected load (host only)."""
    load = np.ascontiguousarray(expected_load, dtype=np.float64)
    owner = np.zeros(load.size, dtype=np.int32)
    check(lib().gguf_moe_ep_place(load.ctypes.data, load.size, world, owner.ctypes.data), "gguf_moe_ep_place")
    return owner


def ep_rows(counts, owner, rank: int):
    """gguf_moe_ep_rows (host only): (dst_off [n_experts], rows_here) for
    `rank` given the [world][n_experts] pair counts and the placement."""
    c = np.ascontiguousarray(counts, dtype=np.int32)
    o = np.ascontiguousarray(owner, dtype=np.int32)
    world, ne = c.shape
    off = np.zeros(ne, dtype=np.int32)
    here = C.c_int32()
    check(lib().gguf_moe_ep_rows(c.ctypes.data, o.ctypes.data, ne, world, rank, off.ctypes.data, C.byref(here)),
          "gguf_moe_ep_rows")
    return off, int(here.value)


def ep_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().gguf_moe_ep_unique_id(buf), "gguf_moe_ep_unique_id")
    return buf.raw


class SharedExpert:
    """A shared expert (gguf_moe_shexp_*): ``sh`` is a
    ``vireo_b200.synth.SharedExpert`` (dim, ffn, *_type, raw GGUF ``gate``,
    ``up``, ``down`` and an optional fp32 ``gate_inp``)."""

    def __init__(self, sh, device: int = 0):
        import torch
        dev = torch.device("cuda", device)
        up = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).to(dev)
        self._keep = [up(sh.gate), up(sh.up), up(sh.down)]
        gi = None
        if sh.gate_inp is not None:
            gi = torch.from_numpy(np.ascontiguousarray(sh.gate_inp, dtype=np.float32)).to(dev)
            self._keep.append(gi)
        g, u, dn = self._keep[:3]
        self.desc = GgufMoeShexpDesc(sh.dim, sh.ffn, sh.gate_type, sh.up_type, sh.down_type, g.data_ptr(),
                                     u.data_ptr(), dn.data_ptr(), gi.data_ptr() if gi is not None else None)
        h = C.c_void_p()
        check(lib().gguf_moe_shexp_create(C.byref(self.desc), C.byref(h)), "gguf_moe_shexp_create")
        self.h = h

    def ffn(self, hb, x, stream=None) -> None:
        n = hb.shape[0] if hb.dim() > 1 else 1
        check(lib().gguf_moe_shexp_ffn(self.h, hb.data_ptr(), x.data_ptr(), n, stream), "gguf_moe_shexp_ffn")

    def sync(self, stream=None) -> None:
        check(lib().gguf_moe_shexp_sync(self.h, stream), "gguf_moe_shexp_sync")

    def close(self) -> None:
        if self.h:
            lib().gguf_moe_shexp_destroy(self.h)
            self.h = None


class MoeLayerEP:
    """One rank's share of an expert-parallel MoE layer (gguf_moe_ep_*).
    Every rank constructs it with the same owner table and unique id."""

    def __init__(self, layer, owner, rank: int, world: int, uid: bytes, max_tokens: int, device: int = 0):
        import torch
        s = layer.spec
        self.spec = s
        dev = torch.device("cuda", device)
        up = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).to(dev)
        self._keep = [up(layer.router), up(layer.gate), up(layer.up), up(layer.down)]
        r, g, u, dn = self._keep
        self.desc = GgufMoeDesc(s.dim, s.ffn_exp, s.n_experts, s.n_used, s.topk_renorm, s.router_type,
                                s.gate_type, s.up_type, s.down_type, r.data_ptr(), g.data_ptr(), u.data_ptr(),
                                dn.data_ptr(), g.numel(), u.numel(), dn.numel())
        self.owner = np.ascontiguousarray(owner, dtype=np.int32)
        buf = C.create_string_buffer(uid, 128)
        h = C.c_void_p()
        check(lib().gguf_moe_ep_create(C.byref(self.desc), self.owner.ctypes.data, rank, world, max_tokens, buf,
                                       C.byref(h)), "gguf_moe_ep_create")
        self.h = h

    def prefill(self, hb_bf16, x, bias=None, ids=None, wts=None, stream=None) -> None:
        n = hb_bf16.shape[0]
        check(lib().gguf_moe_prefill_ep(self.h, hb_bf16.data_ptr(), x.data_ptr(), n,
                                        bias.data_ptr() if bias is not None else None,
                                        ids.data_ptr() if ids is not None else None,
                                        wts.data_ptr() if wts is not None else None, stream), "gguf_moe_prefill_ep")

    def sync(self, stream=None) -> None:
        check(lib().gguf_moe_ep_sync(self.h, stream), "gguf_moe_ep_sync")

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().gguf_moe_ep_destroy(self.h)
            self.h = None


class GgufDecoderDesc(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("dim", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_size", C.c_int), ("vocab", C.c_int), ("eps", C.c_float), ("rope_base", C.c_float),
                ("max_ctx", C.c_int), ("kv_f16", C.c_int), ("tok_embd_type", C.c_uint32), ("tok_embd", C.c_void_p),
                ("out_norm", C.c_void_p), ("lm_head_type", C.c_uint32), ("lm_head", C.c_void_p)]


class GgufDecoderLayer(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p), ("wq_type", C.c_uint32),
                ("wk_type", C.c_uint32), ("wv_type", C.c_uint32), ("wo_type", C.c_uint32), ("wq", C.c_void_p),
                ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p), ("bq", C.c_void_p), ("bk", C.c_void_p),
                ("bv", C.c_void_p), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("q_norm_len", C.c_int),
                ("k_norm_len", C.c_int), ("moe", C.c_void_p)]


def _decoder_api(L):
    if getattr(L, "_decoder_api", False):
        return
    L.gguf_decoder_create.argtypes = [C.POINTER(GgufDecoderDesc), C.c_void_p, C.POINTER(C.c_void_p)]
    L.gguf_decoder_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    L.gguf_decoder_step_dev.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    L.gguf_decoder_hidden.argtypes = [C.c_void_p]
    L.gguf_decoder_hidden.restype = C.c_void_p
    L.gguf_decoder_sync.argtypes = [C.c_void_p, C.c_void_p]
    L.gguf_decoder_destroy.argtypes = [C.c_void_p]
    L.gguf_decoder_destroy.restype = None
    L._decoder_api = True


class Decoder:
    """A whole MoE decoder on the device (gguf_decoder_*): the reference's
    forward() (src/gguf_run.c:216-252) one step per call.  ``dec`` is a
    ``vireo_b200.synth.Decoder`` (or any object with the same fields).  Each
    layer gets its own device copy of its tensors, also when the generated
    layers repeat, so no step reads another layer's bytes out of L2."""

    def __init__(self, dec, max_ctx: int, kv_f16: bool = True, device: int = 0):
        import torch
        L = lib()
        _decoder_api(L)
        s = dec.spec
        self.spec = s
        dev = torch.device("cuda", device)
        self.device = dev
        uploaded = {}

        def up(a):
            """a device copy per call (distinct addresses), uploaded once per host array"""
            if a is None:
                return None
            key = id(a)
            if key not in uploaded:
                uploaded[key] = torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).to(dev)
                return uploaded[key]
            return uploaded[key].clone()

        self._keep = []
        keep = self._keep.append
        ptr = lambda t: t.data_ptr() if t is not None else None
        tok, on, lm = up(dec.tok_embd), up(dec.out_norm), up(dec.lm_head)
        keep(tok), keep(on), keep(lm)
        self.desc = GgufDecoderDesc(s.n_layers, s.dim, s.n_heads, s.n_kv_heads, s.head_size, s.vocab, s.eps,
                                    s.rope_base, max_ctx, int(kv_f16), s.embd_type, ptr(tok), ptr(on), s.lm_type,
                                    ptr(lm))
        self.moe = []
        rows = []
        for ly in dec.layers:
            t = [up(a) for a in (ly.attn_norm, ly.ffn_norm, ly.wq, ly.wk, ly.wv, ly.wo, ly.q_norm, ly.k_norm)]
            for x in t:
                keep(x)
            m = _DeviceMoe(ly.moe, up)
            self.moe.append(m)
            qn = s.head_size if s.qk_norm == "head" else s.q_dim
            kn = s.head_size if s.qk_norm == "head" else s.kv_dim
            rows.append(GgufDecoderLayer(ptr(t[0]), ptr(t[1]), s.attn_type, s.attn_type, s.attn_type, s.attn_type,
                                         ptr(t[2]), ptr(t[3]), ptr(t[4]), ptr(t[5]), None, None, None, ptr(t[6]),
                                         ptr(t[7]), qn if t[6] is not None else 0, kn if t[7] is not None else 0,
                                         m.h))
        self.layers = (GgufDecoderLayer * len(rows))(*rows)
        h = C.c_void_p()
        check(L.gguf_decoder_create(C.byref(self.desc), self.layers, C.byref(h)), "gguf_decoder_create")
        self.h = h

    def step(self, token: int, pos: int, logits=None, next=None, stream=None) -> None:
        """Device tensors logits [vocab] fp32 / next [1] int32, or None."""
        check(lib().gguf_decoder_step(self.h, int(token), int(pos), logits.data_ptr() if logits is not None else None,
                                      next.data_ptr() if next is not None else None, stream), "gguf_decoder_step")

    def step_dev(self, token, pos: int, logits=None, next=None, stream=None) -> None:
        """token: device int32 tensor [1] (e.g. the previous step's next)."""
        check(lib().gguf_decoder_step_dev(self.h, token.data_ptr(), int(pos),
                                          logits.data_ptr() if logits is not None else None,
                                          next.data_ptr() if next is not None else None, stream),
              "gguf_decoder_step_dev")

    def sync(self, stream=None) -> None:
        check(lib().gguf_decoder_sync(self.h, stream), "gguf_decoder_sync")

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().gguf_decoder_destroy(self.h)
            self.h = None
        for m in getattr(self, "moe", []):
            m.close()
        self.moe = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _DeviceMoe:
    """A gguf_moe handle over device copies made by `up` (Decoder's uploader)."""

    def __init__(self, layer, up):
        s = layer.spec
        self.spec = s
        self.router, self.gate, self.up, self.down = up(layer.router), up(layer.gate), up(layer.up), up(layer.down)
        self.desc = GgufMoeDesc(s.dim, s.ffn_exp, s.n_experts, s.n_used, s.topk_renorm, s.router_type,
                                s.gate_type, s.up_type, s.down_type, self.router.data_ptr(),
                                self.gate.data_ptr(), self.up.data_ptr(), self.down.data_ptr(),
                                self.gate.numel(), self.up.numel(), self.down.numel())
        h = C.c_void_p()
        check(lib().gguf_moe_create(C.byref(self.desc), C.byref(h)), "gguf_moe_create")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().gguf_moe_destroy(self.h)
            self.h = None
