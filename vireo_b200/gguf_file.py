"""GGUF v3 model files for generated (random-init) decoders.

The reference reads models only from GGUF files: gguf_open (src/gguf.c:79-131)
maps the file, parses the metadata and the tensor table, and the runner's
loader (src/gguf_run.c:276-315) takes the shapes from the "<arch>.*" keys and
the tensors by their llama.cpp names.  ``write_decoder`` writes a
``synth.Decoder`` in that layout, so the reference's own loader can open it;
``read`` parses a file back (header, metadata, tensor table and data) for
checks.

Layout (little-endian): "GGUF", version u32 = 3, tensor count u64, metadata
count u64; each metadata entry = key (u64 length + bytes), value type u32,
value; each tensor entry = name, n_dims u32, dims u64 x n_dims (dims[0] the
row length), ggml type u32, offset u64 from the data section; the data
section starts at the next multiple of general.alignment (32) and every
tensor's offset is a multiple of it.
"""
from __future__ import annotations

import struct

import numpy as np

from . import synth as S

# metadata value types (wire enum, src/gguf.h)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
ALIGN = 32
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
           I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        atype, items = v
        body = b"".join(_str(x) if atype == STRING else struct.pack(_SCALAR[atype], x) for x in items)
        return struct.pack("<IQ", atype, len(items)) + body
    return struct.pack(_SCALAR[vtype], v)


def write(path: str, metadata, tensors) -> None:
    """metadata: [(key, type, value)]; tensors: [(name, dims, ggml_type,
    bytes-like)] in file order."""
    out = bytearray(b"GGUF")
    out += struct.pack("<IQQ", 3, len(tensors), len(metadata))
    for key, vtype, v in metadata:
        out += _str(key) + struct.pack("<I", vtype) + _value(vtype, v)
    offsets, off = [], 0
    for _, _, _, data in tensors:
        offsets.append(off)
        off += (np.ascontiguousarray(data).nbytes + ALIGN - 1) // ALIGN * ALIGN
    for (name, dims, gtype, _), o in zip(tensors, offsets):
        out += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", x) for x in dims)
        out += struct.pack("<IQ", gtype, o)
    out += b"\0" * ((-len(out)) % ALIGN)
    for (_, _, _, data), o in zip(tensors, offsets):
        b = bytes(np.ascontiguousarray(data).view(np.uint8).reshape(-1))
        out += b + b"\0" * ((-len(b)) % ALIGN)
    with open(path, "wb") as f:
        f.write(out)


def decoder_tensors(dec: S.Decoder):
    """The tensors of a generated decoder under the runner's names
    (src/gguf_run.c:297-315), dims as GGUF stores them (row length first)."""
    s, m = dec.spec, dec.spec.moe
    t = [("token_embd.weight", [s.dim, s.vocab], s.embd_type, dec.tok_embd),
         ("output_norm.weight", [s.dim], S.GGML_F32, dec.out_norm),
         ("output.weight", [s.dim, s.vocab], s.lm_type, dec.lm_head)]
    for l, ly in enumerate(dec.layers):
        b = f"blk.{l}."
        t += [(b + "attn_norm.weight", [s.dim], S.GGML_F32, ly.attn_norm),
              (b + "attn_q.weight", [s.dim, s.q_dim], s.attn_type, ly.wq),
              (b + "attn_k.weight", [s.dim, s.kv_dim], s.attn_type, ly.wk),
              (b + "attn_v.weight", [s.dim, s.kv_dim], s.attn_type, ly.wv),
              (b + "attn_output.weight", [s.q_dim, s.dim], s.attn_type, ly.wo),
              (b + "ffn_norm.weight", [s.dim], S.GGML_F32, ly.ffn_norm)]
        if ly.q_norm is not None:
            t += [(b + "attn_q_norm.weight", [ly.q_norm.size], S.GGML_F32, ly.q_norm),
                  (b + "attn_k_norm.weight", [ly.k_norm.size], S.GGML_F32, ly.k_norm)]
        e = ly.moe
        t += [(b + "ffn_gate_inp.weight", [s.dim, m.n_experts], m.router_type, e.router),
              (b + "ffn_gate_exps.weight", [s.dim, m.ffn_exp, m.n_experts], m.gate_type, e.gate),
              (b + "ffn_up_exps.weight", [s.dim, m.ffn_exp, m.n_experts], m.up_type, e.up),
              (b + "ffn_down_exps.weight", [m.ffn_exp, s.dim, m.n_experts], m.down_type, e.down)]
    return t


def write_decoder(path: str, dec: S.Decoder, arch: str) -> None:
    """A generated decoder as a GGUF file the reference runner loads: arch
    "qwen3moe" (per-head QK norm, renormalised top-k) or "olmoe" (full-width
    QK norm, raw top-k probabilities); the per-arch keys are the ones its
    loader reads (src/gguf_run.c:276-293)."""
    s, m = dec.spec, dec.spec.moe
    a = arch
    md = [("general.architecture", STRING, a),
          ("general.alignment", U32, ALIGN),
          (f"{a}.block_count", U32, s.n_layers),
          (f"{a}.embedding_length", U32, s.dim),
          (f"{a}.feed_forward_length", U32, m.ffn_exp),
          (f"{a}.attention.head_count", U32, s.n_heads),
          (f"{a}.attention.head_count_kv", U32, s.n_kv_heads),
          (f"{a}.attention.layer_norm_rms_epsilon", F32, s.eps),
          (f"{a}.rope.freq_base", F32, s.rope_base),
          (f"{a}.attention.key_length", U32, s.head_size),
          (f"{a}.expert_count", U32, m.n_experts),
          (f"{a}.expert_used_count", U32, m.n_used),
          (f"{a}.expert_feed_forward_length", U32, m.ffn_exp),
          (f"{a}.expert_weights_norm", U32, int(m.topk_renorm))]
    write(path, md, decoder_tensors(dec))


def _rd(buf, off, fmt):
    v = struct.unpack_from(fmt, buf, off)
    return (v[0] if len(v) == 1 else v), off + struct.calcsize(fmt)


def _rd_str(buf, off):
    n, off = _rd(buf, off, "<Q")
    return bytes(buf[off:off + n]).decode(), off + n


def read(path: str):
    """(metadata {key: value}, tensors {name: (dims, ggml_type, bytes)})."""
    buf = memoryview(open(path, "rb").read())
    assert bytes(buf[:4]) == b"GGUF"
    (ver, nt, nkv), off = _rd(buf, 4, "<IQQ")
    assert ver in (2, 3)
    md = {}
    for _ in range(nkv):
        key, off = _rd_str(buf, off)
        vtype, off = _rd(buf, off, "<I")
        if vtype == STRING:
            val, off = _rd_str(buf, off)
        elif vtype == ARRAY:
            (atype, n), off = _rd(buf, off, "<IQ")
            val = []
            for _ in range(n):
                if atype == STRING:
                    x, off = _rd_str(buf, off)
                else:
                    x, off = _rd(buf, off, _SCALAR[atype])
                val.append(x)
        else:
            val, off = _rd(buf, off, _SCALAR[vtype])
        md[key] = val
    align = md.get("general.alignment", ALIGN)
    infos = []
    for _ in range(nt):
        name, off = _rd_str(buf, off)
        nd, off = _rd(buf, off, "<I")
        dims = []
        for _ in range(nd):
            x, off = _rd(buf, off, "<Q")
            dims.append(x)
        (gtype, toff), off = _rd(buf, off, "<IQ")
        infos.append((name, dims, gtype, toff))
    data0 = off + (-off) % align
    tensors = {}
    for name, dims, gtype, toff in infos:
        n = int(np.prod(dims))
        nbytes = S.row_bytes(gtype, dims[0]) * (n // dims[0])
        tensors[name] = (dims, gtype, bytes(buf[data0 + toff:data0 + toff + nbytes]))
    return md, tensors
