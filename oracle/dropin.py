"""Builds the drop-in checkers (test infrastructure, never product code).

    python -m oracle.dropin <reference source tree>

_ref/dropin_ref.so    dropin_harness.c over the reference's unmodified
                      sources: src/gguf_run.c (included), gguf.c,
                      gguf_compute.c, expert_store.c and the KV store files.
_ref/dropin_b200.so   the same with gguf_compute.c and expert_store.c left
                      out and libvireo_b200.so linked in their place, and the
                      MoE hook placed at the top of moe_ffn
                      (src/gguf_run.c:185) in a temporary copy of gguf_run.c
                      made for the compile and deleted after it.

Both are compiled with the reference's flags (its Makefile: -O3
-funroll-loops -fopenmp -std=c11) for x86-64-v3; only the libraries land in
oracle/_ref, nothing of the reference's source.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")
REF_SO = os.path.join(OUT, "dropin_ref.so")
B200_SO = os.path.join(OUT, "dropin_b200.so")

# the first line of moe_ffn in the reference (src/gguf_run.c:185) and the
# hook the integration notes add at its top
MOE_FFN_LINE = "static void moe_ffn(Model*m,int layer,float*hb){"
HOOK_DECL = "static int vireo_moe_hook(Model*m,int layer,float*hb);\n"
HOOK_CALL = "\n    if(vireo_moe_hook(m,layer,hb)) return;  /* the whole block on the GPU */"
OPT = ["-O3", "-march=x86-64-v3", "-funroll-loops", "-fopenmp", "-std=c11", "-fPIC", "-w"]


def kv_sources(src):
    return [os.path.join(src, f) for f in ("kvstore_dense.c", "kvstore_ooc.c", "select/select_all.c",
                                           "select/select_recent.c", "select/select_topk.c")]


def build(ref: str, cc: str = "gcc") -> None:
    src = os.path.join(ref, "src")
    if not os.path.isfile(os.path.join(src, "gguf_run.c")):
        raise FileNotFoundError(src)
    os.makedirs(OUT, exist_ok=True)
    harness = os.path.join(HERE, "dropin_harness.c")
    kv = kv_sources(src)
    subprocess.run([cc] + OPT + ["-I", src, "-shared", "-Wl,-Bsymbolic", harness,
                                 os.path.join(src, "gguf.c"), os.path.join(src, "gguf_compute.c"),
                                 os.path.join(src, "expert_store.c")] + kv + ["-lm", "-o", REF_SO], check=True)
    text = open(os.path.join(src, "gguf_run.c")).read()
    if text.count(MOE_FFN_LINE) != 1:
        raise RuntimeError("moe_ffn's first line not found once in gguf_run.c")
    tmp = tempfile.mkdtemp(prefix="vireo_dropin_")
    try:
        with open(os.path.join(tmp, "gguf_run.c"), "w") as f:
            f.write(text.replace(MOE_FFN_LINE, HOOK_DECL + MOE_FFN_LINE + HOOK_CALL))
        lib = os.path.join(ROOT, "vireo_b200")
        subprocess.run([cc] + OPT + ["-DVIREO_DROPIN", "-I", tmp, "-I", src, "-I", os.path.join(ROOT, "include"),
                                     "-shared", "-Wl,-Bsymbolic", harness, os.path.join(src, "gguf.c")] + kv +
                       ["-L", lib, "-lvireo_b200", "-Wl,-rpath,$ORIGIN/../../vireo_b200", "-lm", "-o", B200_SO],
                       check=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    build(sys.argv[1])
