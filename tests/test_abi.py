"""The C-ABI boundary without a GPU: the library builds, loads, and exports
every function declared in include/*.h; calls fail loudly (no CPU fallback)
when no device is present."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = {}
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not fn.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", fn)).read()
        src = re.sub(r"/\*.*?\*/", " ", src, flags=re.S)
        src = re.sub(r"//[^\n]*", " ", src)
        src = "\n".join(l for l in src.splitlines()
                        if not l.strip().startswith("#") and 'extern "C"' not in l and l.strip() != "}")
        for stmt in src.split(";"):
            s = " ".join(stmt.split())
            if "(" not in s or "typedef" in s or "{" in s.split("(")[0]:
                continue
            m = re.search(r"([A-Za-z_]\w*)\s*\($", s.split("(")[0] + "(")
            if m:
                names[m.group(1)] = fn
    return names


def test_headers_declare_reference_interface():
    names = declared_functions()
    for ref in ["gguf_f16_to_f32", "gguf_dequant_row", "gguf_matmul", "expert_store_create",
                "expert_store_register", "expert_store_lookup", "expert_store_release",
                "expert_store_stats", "expert_store_destroy"]:
        if ref.startswith("expert_store") and not os.path.exists(os.path.join(ROOT, "include", "expert_store.h")):
            continue
        assert ref in names, ref


def test_library_exports_every_declared_symbol():
    import vireo_b200
    if not os.path.exists(vireo_b200.LIB_PATH):
        vireo_b200.build()
    lib = C.CDLL(vireo_b200.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_f16_host_function_matches_reference_vectors(golden):
    import numpy as np
    import vireo_b200
    L = vireo_b200.lib()
    got = np.array([np.float32(L.gguf_f16_to_f32(h)).view(np.uint32) for h in range(65536)], dtype=np.uint32)
    assert np.array_equal(got, golden["f16_bits"])


def test_no_device_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    import numpy as np
    import vireo_b200
    with pytest.raises(vireo_b200.VireoError):
        vireo_b200.gguf_matmul(8, np.zeros(34 * 8 * 16, np.uint8), np.zeros(256, np.float32), 256, 16)
