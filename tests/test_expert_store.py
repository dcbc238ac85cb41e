"""ExpertStore on the GPU (include/expert_store.h) against the reference's
behaviour (vireo src/expert_store.c) and its own unit test.

* The reference's test program (tests/test_expert_store.c), compiled unchanged
  against this library by oracle/Makefile (oracle/_ref/test_expert_store_b200),
  must print PASS.
* The same properties restated here through the C-ABI: every expert's bytes
  come back exactly, the device budget holds although every expert is touched,
  a leased expert survives a flood of other lookups, eviction is LRU by last
  use, an unregistered expert gives -1 and a zeroed view.
* The device-only store over a host image (create_host), async lookups and
  deferred releases.
"""
import ctypes as C
import os
import subprocess
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_TEST = os.path.join(ROOT, "oracle", "_ref", "test_expert_store_b200")

NL, NE = 4, 16
SIZES = (3072, 3072, 2048)  # gate, up, down bytes per expert


def pattern(layer, expert, sl, n):
    """Deterministic bytes of one slice (splitmix-style hash of its position)."""
    i = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):  # arithmetic mod 2^64 on purpose
        z = i + np.uint64(0x9E3779B97F4A7C15) * np.uint64(1 + layer * 64 + expert * 4 + sl)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return ((z ^ (z >> np.uint64(31))) & np.uint64(0xFF)).astype(np.uint8)


def expert_file():
    """Backing bytes and slice locations: experts back to back (gate, up, down)."""
    blobs, locs, off = [], {}, 0
    for l in range(NL):
        for e in range(NE):
            offs = []
            for sl, n in enumerate(SIZES):
                blobs.append(pattern(l, e, sl, n))
                offs.append(off)
                off += n
            locs[(l, e)] = offs
    return np.concatenate(blobs), locs


@pytest.fixture(scope="module")
def V():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import vireo_b200
    return vireo_b200


def register_all(V, s, locs):
    L = V.lib()
    for (l, e), offs in locs.items():
        sl = V.ExpertSlices(offs[0], offs[1], offs[2], *SIZES)
        L.expert_store_register(s, l, e, C.byref(sl))


def stats(V, s):
    st = V.ExpertStats()
    V.lib().expert_store_stats(s, C.byref(st))
    return st


def test_reference_unit_test_passes():
    if not os.path.exists(REF_TEST):
        pytest.skip("oracle/_ref/test_expert_store_b200 was not built (reference tree absent at build time)")
    r = subprocess.run([REF_TEST], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout + r.stderr


def test_fd_store_bytes_budget_lease_lru(V):
    L = V.lib()
    data, locs = expert_file()
    ebytes = sum(SIZES)
    with tempfile.TemporaryFile() as f:
        f.write(data.tobytes())
        f.flush()
        s = L.expert_store_create(f.fileno(), ebytes * 10, NL, NE)
        assert s
        try:
            register_all(V, s, locs)
            # every expert's bytes, read through the (host-readable) view
            for (l, e) in locs:
                v = V.ExpertView()
                assert L.expert_store_lookup(s, l, e, C.byref(v)) == 0
                for ptr, sl in ((v.gate, 0), (v.up, 1), (v.down, 2)):
                    got = np.frombuffer(C.string_at(ptr, SIZES[sl]), dtype=np.uint8)
                    assert np.array_equal(got, pattern(l, e, sl, SIZES[sl])), (l, e, sl)
                L.expert_store_release(s, C.byref(v))
                assert v.gate is None and v.slot is None  # release zeroes the view
            st = stats(V, s)
            assert st.resident_bytes <= st.capacity_bytes == ebytes * 10
            assert st.misses == 64 and st.requests == 64 and st.experts_resident == 10
            assert st.bytes_read == 64 * ebytes
            # LRU: the 10 resident experts are the last 10 touched (layer 3, experts 6..15)
            before = stats(V, s).hits
            v = V.ExpertView()
            for e in range(6, 16):
                assert L.expert_store_lookup(s, 3, e, C.byref(v)) == 0
                L.expert_store_release(s, C.byref(v))
            assert stats(V, s).hits == before + 10
            # lease pin: (0, 0) leased, then a flood of other lookups
            pinned = V.ExpertView()
            assert L.expert_store_lookup(s, 0, 0, C.byref(pinned)) == 0
            for l in range(NL):
                for e in range(1, NE):
                    assert L.expert_store_lookup(s, l, e, C.byref(v)) == 0
                    L.expert_store_release(s, C.byref(v))
            got = np.frombuffer(C.string_at(pinned.gate, SIZES[0]), dtype=np.uint8)
            assert np.array_equal(got, pattern(0, 0, 0, SIZES[0]))
            assert stats(V, s).resident_bytes <= ebytes * 10
            L.expert_store_release(s, C.byref(pinned))
            # unregistered expert: -1 and a zeroed view
            s2 = L.expert_store_create(f.fileno(), 0, 1, 2)
            try:
                v.gate = 1234
                assert L.expert_store_lookup(s2, 0, 1, C.byref(v)) == -1
                assert v.gate is None and v.slot is None
            finally:
                L.expert_store_destroy(s2)
        finally:
            L.expert_store_destroy(s)


def test_all_leased_goes_over_budget(V):
    L = V.lib()
    data, locs = expert_file()
    ebytes = sum(SIZES)
    with tempfile.TemporaryFile() as f:
        f.write(data.tobytes())
        f.flush()
        s = L.expert_store_create(f.fileno(), ebytes * 2, 1, NE)
        try:
            for e in range(NE):
                offs = locs[(0, e)]
                L.expert_store_register(s, 0, e, C.byref(V.ExpertSlices(offs[0], offs[1], offs[2], *SIZES)))
            views = [V.ExpertView() for _ in range(3)]
            for e, v in enumerate(views):
                assert L.expert_store_lookup(s, 0, e, C.byref(v)) == 0
            st = stats(V, s)
            assert st.experts_resident == 3 and st.resident_bytes == 3 * ebytes  # over budget, all leased
            for e, v in enumerate(views):
                got = np.frombuffer(C.string_at(v.down, SIZES[2]), dtype=np.uint8)
                assert np.array_equal(got, pattern(0, e, 2, SIZES[2]))
                L.expert_store_release(s, C.byref(v))
            v = views[0]
            assert L.expert_store_lookup(s, 0, 5, C.byref(v)) == 0  # evicts back under budget
            L.expert_store_release(s, C.byref(v))
            assert stats(V, s).resident_bytes <= 2 * ebytes
        finally:
            L.expert_store_destroy(s)


def cudart():
    import glob
    import site
    for d in site.getsitepackages():
        for p in glob.glob(os.path.join(d, "nvidia", "cuda_runtime", "lib", "libcudart.so*")):
            return C.CDLL(p)
    return C.CDLL("libcudart.so")


def test_host_image_store_async_and_deferred_release(V):
    import torch
    L = V.lib()
    rt = cudart()
    rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    data, locs = expert_file()
    ebytes = sum(SIZES)
    s = L.expert_store_create_host(data.ctypes.data, data.nbytes, ebytes * 4, NL, NE)
    assert s
    stream = torch.cuda.Stream()
    try:
        register_all(V, s, locs)
        views = []
        for e in range(4):  # fills the budget, no eviction
            v = V.ExpertView()
            assert L.expert_store_lookup_async(s, 1, e, C.byref(v), C.c_void_p(stream.cuda_stream)) == 0
            views.append((e, v))
        stream.synchronize()
        for e, v in views:
            host = np.empty(SIZES[1], dtype=np.uint8)
            assert rt.cudaMemcpy(host.ctypes.data, v.up, SIZES[1], 2) == 0  # device -> host
            assert np.array_equal(host, pattern(1, e, 1, SIZES[1]))
        # deferred release: leases end with the stream's work; all four stay pinned until then
        blocker = torch.empty(1 << 24, device="cuda")
        with torch.cuda.stream(stream):
            for _ in range(20):
                blocker.mul_(1.0001)  # queued work the releases wait for
        for e, v in views:
            assert L.expert_store_release_after(s, C.byref(v), C.c_void_p(stream.cuda_stream)) == 0
        stream.synchronize()
        v = V.ExpertView()
        assert L.expert_store_lookup(s, 2, 0, C.byref(v)) == 0  # needs one eviction: leases have ended
        L.expert_store_release(s, C.byref(v))
        ext = V.ExpertStatsExt()
        L.expert_store_stats_ext(s, C.byref(ext))
        assert ext.copies == 5 and ext.h2d_bytes == 5 * ebytes and ext.evictions == 1
        assert ext.over_budget_loads == 0
    finally:
        L.expert_store_destroy(s)


STATS_FIELDS = ("requests", "hits", "misses", "bytes_read", "resident_bytes", "capacity_bytes", "experts_resident")


def stats_tuple(st):
    return tuple(int(getattr(st, f)) for f in STATS_FIELDS)


def test_store_stats_match_reference_golden(V, golden):
    """The reference's capped pager on the tiny Q8_0 layer (cap = 3 experts,
    6 tokens of 2 experts, tests/golden/gen_golden.py): the same lookups and
    releases, in moe_ffn's order (lookup, compute, release per selected expert,
    gguf_run.c:199-210), give the reference's counters exactly."""
    from vireo_b200 import synth as S
    sp = golden["moe_tiny_q8_spec"]
    spec = S.MoeLayerSpec(int(sp[0]), int(sp[1]), int(sp[2]), int(sp[3]), int(sp[4]), int(sp[6]), int(sp[7]),
                          int(sp[8]), router_type=int(sp[5]))
    ids = golden["moe_tiny_q8_ids"]
    L = V.lib()
    gs, us, ds = spec.gate_slice, spec.up_slice, spec.down_slice
    G, U = gs * spec.n_experts, us * spec.n_experts
    with tempfile.TemporaryFile() as f:
        f.write(b"\0" * (G + U + ds * spec.n_experts))
        f.flush()
        s = L.expert_store_create(f.fileno(), 3 * spec.expert_bytes, 1, spec.n_experts)
        try:
            for e in range(spec.n_experts):
                L.expert_store_register(s, 0, e, C.byref(V.ExpertSlices(e * gs, G + e * us, G + U + e * ds,
                                                                         gs, us, ds)))
            v = V.ExpertView()
            for row in ids:
                for e in row:
                    assert L.expert_store_lookup(s, 0, int(e), C.byref(v)) == 0
                    L.expert_store_release(s, C.byref(v))
            got = stats_tuple(stats(V, s))
        finally:
            L.expert_store_destroy(s)
    assert got == tuple(int(v) for v in golden["es_tiny_q8_stats"]), got


@pytest.mark.parametrize("uniform", [True, False])
def test_store_policy_matches_reference_step_by_step(V, uniform):
    """The device store and the reference's own store (src/expert_store.c,
    compiled into oracle/_ref) driven by the same seeded sequence of lookups,
    held leases and releases over slices whose sizes are not multiples of 256
    bytes (equal for every expert, or different per expert): identical
    counters after every step, and the bytes behind every view intact."""
    from oracle import oracle as O
    if not O.ref_available():
        pytest.skip("reference library not built")
    R = O.ref()
    L = V.lib()
    nl, ne = 2, 8
    sizes = {}
    blobs, off = [], 0
    for l in range(nl):
        for e in range(ne):
            sz = (1000, 1000, 700) if uniform else (1000 + 40 * e, 1000 + 24 * l, 700 + 56 * e)
            offs = []
            for k, n in enumerate(sz):
                blobs.append(pattern(l, e, k, n))
                offs.append(off)
                off += n
            sizes[(l, e)] = (offs, sz)
    data = np.concatenate(blobs)
    cap = int(3.5 * data.nbytes / (nl * ne))
    rng = np.random.default_rng(31 if uniform else 32)
    with tempfile.TemporaryFile() as f:
        f.write(data.tobytes())
        f.flush()
        ours = L.expert_store_create(f.fileno(), cap, nl, ne)
        ref = R.expert_store_create(f.fileno(), cap, nl, ne)
        assert ours and ref
        held = []
        try:
            for (l, e), (offs, sz) in sizes.items():
                loc = V.ExpertSlices(offs[0], offs[1], offs[2], *sz)
                L.expert_store_register(ours, l, e, C.byref(loc))
                R.expert_store_register(ref, l, e, C.byref(loc))
            for step in range(300):
                op = rng.random()
                if op < 0.25 and held:
                    vo, vr = held.pop(int(rng.integers(len(held))))
                    L.expert_store_release(ours, C.byref(vo))
                    R.expert_store_release(ref, C.byref(vr))
                else:
                    l, e = int(rng.integers(nl)), int(rng.integers(ne))
                    vo, vr = V.ExpertView(), V.ExpertView()
                    assert L.expert_store_lookup(ours, l, e, C.byref(vo)) == 0
                    assert R.expert_store_lookup(ref, l, e, C.byref(vr)) == 0
                    offs, sz = sizes[(l, e)]
                    for ptr, k in ((vo.gate, 0), (vo.up, 1), (vo.down, 2)):
                        got = np.frombuffer(C.string_at(ptr, sz[k]), dtype=np.uint8)
                        assert np.array_equal(got, pattern(l, e, k, sz[k])), (step, l, e, k)
                    if op < 0.45 and len(held) < 3:
                        held.append((vo, vr))
                    else:
                        L.expert_store_release(ours, C.byref(vo))
                        R.expert_store_release(ref, C.byref(vr))
                so, sr = V.ExpertStats(), O.ExpertStats()
                L.expert_store_stats(ours, C.byref(so))
                R.expert_store_stats(ref, C.byref(sr))
                assert stats_tuple(so) == stats_tuple(sr), (step, stats_tuple(so), stats_tuple(sr))
        finally:
            for vo, vr in held:
                L.expert_store_release(ours, C.byref(vo))
                R.expert_store_release(ref, C.byref(vr))
            L.expert_store_destroy(ours)
            R.expert_store_destroy(ref)


def test_async_hit_waits_for_a_copy_started_by_another_stream(V):
    """A miss looked up for stream A and then a hit on the same expert for
    stream B (before A's copy is known complete): B's kernel sees the
    expert's bytes, because every async lookup orders its stream after the
    expert's copy.  The NULL stream stands for the legacy default stream."""
    import torch
    L = V.lib()
    rt = cudart()
    rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    data, locs = expert_file()
    s = L.expert_store_create_host(data.ctypes.data, data.nbytes, 0, NL, NE)
    assert s
    a, b = torch.cuda.Stream(), torch.cuda.Stream()
    try:
        register_all(V, s, locs)
        for e in range(NE):
            va, vb = V.ExpertView(), V.ExpertView()
            assert L.expert_store_lookup_async(s, 2, e, C.byref(va), C.c_void_p(a.cuda_stream)) == 0
            assert L.expert_store_lookup_async(s, 2, e, C.byref(vb), C.c_void_p(b.cuda_stream)) == 0
            assert vb.down == va.down
            out = torch.empty(SIZES[2], dtype=torch.uint8, device="cuda")
            # a device -> device copy on stream b reads the view in b's stream order
            rt.cudaMemcpyAsync.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p]
            assert rt.cudaMemcpyAsync(out.data_ptr(), vb.down, SIZES[2], 3, C.c_void_p(b.cuda_stream)) == 0
            b.synchronize()
            assert np.array_equal(out.cpu().numpy(), pattern(2, e, 2, SIZES[2])), e
            vn = V.ExpertView()
            assert L.expert_store_lookup_async(s, 2, e, C.byref(vn), None) == 0  # legacy stream: a hit
            for v, st in ((va, a), (vb, b)):
                assert L.expert_store_release_after(s, C.byref(v), C.c_void_p(st.cuda_stream)) == 0
            L.expert_store_release(s, C.byref(vn))
        torch.cuda.synchronize()
    finally:
        L.expert_store_destroy(s)
