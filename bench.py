"""Benchmark of the MoE FFN hot path (vireo moe_ffn) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (synthetic, seeded):
  cfg1_moe_decode   config 1: OLMoE-1B-7B-shaped MoE layer, Q8_0 experts,
                    64 experts top-8, batch-1 decode (default)
  qwen3_moe_decode  the MoE layer of config 3: Qwen3-30B-A3B-shaped, Q4_K
                    gate/up, Q6_K down, 128 experts top-8 renormalised

A step is T decode tokens, each one batch-1 pass of a token through an MoE
layer (router -> top-k -> gate/up/SwiGLU -> down -> combine).  Tokens rotate
over NL device copies of the layer so the same weights are not re-read out
of L2 between tokens (reuse distance NL x bytes/token > 126 MB L2).

Decode does not shard (batch 1): with --gpus N every rank runs its own
replica ("replicas only", weak scaling); value = all ranks' tokens / max
rank time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from vireo_b200 import synth as S  # noqa: E402

WORKLOADS = {
    "cfg1_moe_decode": dict(spec=S.olmoe_q8_layer, seed=1234, config=1,
                            desc="OLMoE-1B-7B-shaped MoE layer, Q8_0, 64 experts top-8, batch-1 decode"),
    "qwen3_moe_decode": dict(spec=S.qwen3_layer, seed=1234, config=3,
                             desc="Qwen3-30B-A3B-shaped MoE layer, Q4_K gate/up + Q6_K down, 128 experts "
                                  "top-8 renorm, batch-1 decode"),
    "qwen3_prefill": dict(spec=S.qwen3_layer, seed=1234, config=4,
                          desc="Qwen3-30B-A3B-shaped MoE layer, 8192 bf16 tokens, router logits + per-expert bias "
                               "N(0,0.5), Q4_K gate/up + Q6_K down, 128 experts top-8 renorm, batched prefill"),
    "olmoe_decoder": dict(spec=S.olmoe_decoder, seed=1234, config=2, prompt=4096, gen=256,
                          desc="OLMoE-1B-7B-shaped decoder (16 layers, 16 heads x 128, vocab 50304, 64 experts "
                               "top-8, Q4_K attention and gate/up, Q6_K down and LM head), 4096-token seeded "
                               "prompt then greedy batch-1 decode"),
    "qwen3_decoder": dict(spec=S.qwen3_decoder, seed=1234, config=3, prompt=8192, gen=256,
                          desc="Qwen3-30B-A3B-shaped decoder (48 layers, 32 q / 4 kv heads x 128, vocab 151936, "
                               "128 experts top-8 renorm, Q4_K attention and gate/up, Q6_K down and LM head), "
                               "8192-token context then greedy batch-1 decode"),
    "qwen3_cached_decode": dict(spec=S.qwen3_layer, seed=1234, config=5,
                                desc="Qwen3-30B-A3B-shaped 48-layer MoE stack, experts in pinned host memory "
                                     "behind a 4 GiB device ExpertStore, Zipf(1.1) routing, batch-1 decode"),
}
PREFILL_TOKENS = 8192
PREFILL_FLOPS = 622_770_257_920  # 8192 x (8 x 3 x 2 x 2048 x 768 + 2 x 128 x 2048)
CACHED_LAYERS = 48
CACHE_BYTES = 4 << 30
ZIPF_S = 1.1
L2_BYTES = 126 * 1024 * 1024


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_launch(workload):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary, if one exists for this workload."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(workload)
    except Exception:
        return None


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.index, self.proc, self.path = index, None, f"/tmp/vireo_clocks_{os.getpid()}.csv"

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()
            self.f.close()

    def summary(self):
        try:
            rows = [l.split(",") for l in open(self.path).read().strip().splitlines()]
        except Exception:
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_rate(layer, toks, seconds, threads, warm=4):
    """The reference's own moe_ffn (compiled from its sources, oracle/_ref)
    on this host: tokens/s over a bounded sample of about ``seconds``."""
    from oracle import oracle as O
    O.build(ref=False)
    kind = "reference" if O.ref_available() else "port"
    impl = O.RefMoe(layer) if kind == "reference" else O.PortMoe(layer)
    if kind == "reference":
        O.ref().ref_set_threads(threads)
    else:
        O.port().orc_set_threads(threads)
    impl(toks[:warm])  # first touches load every expert the sample needs
    n, t0 = 0, time.perf_counter()
    while True:
        i = n % len(toks)
        impl(toks[i:i + 1])
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 8:
            break
    if kind == "reference":
        impl.close()
    return n / el, n, el, kind


def ref_build_name(kind):
    """Compiler target of the reference library that produced a CPU rate."""
    if kind != "reference":
        return "port"
    from oracle import oracle as O
    return O.ref_build()


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, spec_w):
    """--impl reference: the reference's own moe_ffn (compiled from its
    sources, oracle/_ref) on the host cores, over the same layer and the same
    tokens as our arm, T tokens per step.  Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    spec = spec_w["spec"]()
    layer = S.MoeLayer(spec, spec_w["seed"])
    T = args.tokens
    toks, _ = S.routed_tokens(layer, min(T, 1000), spec_w["seed"])
    nt = toks.shape[0]
    th = host_threads()
    from oracle import oracle as O
    O.build(ref=False)
    kind = "reference" if O.ref_available() else "port"
    impl = O.RefMoe(layer) if kind == "reference" else O.PortMoe(layer)
    (O.ref().ref_set_threads if kind == "reference" else O.port().orc_set_threads)(th)

    def step():
        done = 0
        while done < T:
            n = min(nt, T - done)
            impl(toks[:n])
            done += n

    impl(toks[:8])
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    tps = args.steps * T / el
    per_tok = spec.bytes_per_token()
    line = {"metric": "moe_decode_tok_per_s", "value": tps, "unit": "tok/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF blocks, random-init weights)",
            "config": {"workload": args.workload, "desc": spec_w["desc"], "baseline_config": spec_w["config"],
                       "tokens_per_step": T, "batch": 1, "parallelism": "host cores",
                       "l2": "host caches (the reference's CPU path)", "bytes_per_token": per_tok},
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": th, "kind": kind,
                             "build": O.ref_build() if kind == "reference" else "port",
                             "sample": f"{args.steps} steps x {T} tokens, OMP threads={th}"},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if kind == "reference":
        impl.close()
    print(json.dumps(line), flush=True)


SUB_RECORDS = {
    # name: (workload, steps, warmup, CPU-baseline seconds)
    "cfg4_prefill": ("qwen3_prefill", 10, 3, 8.0),
    "cfg3_decoder": ("qwen3_decoder", 64, 3, 8.0),
    "cfg5_cached": ("qwen3_cached_decode", 3, 2, 6.0),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="cfg1_moe_decode", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=1000, help="decode tokens per step")
    ap.add_argument("--copies", type=int, default=8, help="layer copies rotated per token")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true",
                    help="cfg1_moe_decode: skip the config 3/4/5 sub-records")
    ap.add_argument("--sub", default=None,
                    help="cfg1_moe_decode: comma-separated sub-records to run (default: all of "
                         + ", ".join(SUB_RECORDS) + ")")
    ap.add_argument("--prompt", type=int, default=None, help="decoder workloads: prompt tokens (default: the config's)")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder workloads: layer count (default: the config's; fewer layers only for profiling "
                         "runs, the line then names the count)")
    ap.add_argument("--timeline", default=None,
                    help="prefill only: after the timed steps, record 3 more steps under the CUDA activity "
                         "profiler and write each rank's kernel timeline to TIMELINE.rank<r>.txt (not timed)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, wl)
    runner = {"qwen3_cached_decode": run_cached, "qwen3_prefill": run_prefill, "olmoe_decoder": run_decoder,
              "qwen3_decoder": run_decoder}.get(args.workload, run_cfg1)
    try:
        line = runner(args, wl)
        if runner is run_cfg1 and not args.no_sub:
            want = list(SUB_RECORDS) if args.sub is None else [x for x in args.sub.split(",") if x]
            world = int(os.environ.get("WORLD_SIZE", "1"))
            for name in want:
                wname, steps, warm, cpu_s = SUB_RECORDS[name]
                if name == "cfg5_cached" and world > 1:
                    # every rank would pin its own 18.8 GB host image; decode
                    # runs replicas only, so the 1-GPU record stands for it
                    if line is not None:
                        line[name] = {"skipped": "one GPU only (replicas; the N=1 record stands)"}
                    continue
                sub = argparse.Namespace(**vars(args))
                sub.workload, sub.steps, sub.warmup, sub.cpu_seconds = wname, steps, warm, cpu_s
                sub.prompt, sub.timeline = None, None
                sub.no_cpu_baseline = args.no_cpu_baseline or cpu_s <= 0
                rec = SUB_RUNNERS[wname](sub, WORKLOADS[wname])
                if line is not None:
                    line[name] = rec
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        dist_stop()


_DIST = {"started": False}


def dist_start():
    """(world, rank, local rank) of this process; the first call sets the
    CUDA device and, under torchrun, starts the NCCL process group (short
    timeout: ranks that wait for one another end with an error)."""
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not _DIST["started"]:
        torch.cuda.set_device(local)
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", local))
        _DIST["started"] = True
    return world, rank, local


def dist_stop():
    if _DIST["started"] and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()
    _DIST["started"] = False


def run_cfg1(args, wl):
    """Config 1 (and the Qwen3 layer in decode): T batch-1 decode tokens per
    step through gguf_moe_ffn, one launch per token, rotating over layer
    copies."""
    import torch
    import vireo_b200 as V

    world, rank, local = dist_start()
    V.check(V.lib().vireo_device_init(local), "vireo_device_init")

    spec = wl["spec"]()
    layer = S.MoeLayer(spec, wl["seed"])
    T = args.tokens
    toks, _ = S.routed_tokens(layer, min(T, 1000), wl["seed"])
    NL = max(1, args.copies)
    per_tok = spec.bytes_per_token()

    layers = [V.MoeLayer(layer, local)]
    for _ in range(NL - 1):  # identical bytes at different addresses: no L2 reuse across tokens
        layers.append(V.MoeLayer(layer, local))
    dev = torch.device("cuda", local)
    hb = torch.from_numpy(toks).to(dev)
    nt = hb.shape[0]
    x = torch.zeros_like(hb)
    stream = torch.cuda.Stream(dev)
    sp = stream.cuda_stream

    ffn = V.lib().gguf_moe_ffn
    d_bytes = 4 * spec.dim
    calls = [(layers[i % NL].h, hb.data_ptr() + (i % nt) * d_bytes, x.data_ptr() + (i % nt) * d_bytes, 1,
              None, None, sp) for i in range(T)]

    def step():
        for a in calls:
            if ffn(*a):
                raise RuntimeError("gguf_moe_ffn failed")

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    for m in layers[:1]:
        m.sync(sp)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize(dev)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    st = layers[0].sync(sp)
    t_sec = ms / 1e3
    if world > 1:
        tt = torch.tensor([t_sec], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_sec = float(tt.item())
    tokens_all = args.steps * T * world
    value = tokens_all / t_sec
    launches = args.steps * T

    # end to end through the host C-ABI call (pinned host buffers, copies in
    # the timed region), per-token round trips as a decode loop makes them
    e2e = None
    n_e2e = min(200, T)
    hb_h = torch.from_numpy(toks[:n_e2e].copy()).pin_memory()
    x_h = torch.zeros_like(hb_h).pin_memory()
    ids_h = torch.zeros((n_e2e, spec.n_used), dtype=torch.int32).pin_memory()
    w_h = torch.zeros((n_e2e, spec.n_used), dtype=torch.float32).pin_memory()
    L = V.lib()

    fh = L.gguf_moe_ffn_host
    hcalls = [(layers[i % NL].h, hb_h[i].data_ptr(), x_h[i].data_ptr(), 1, ids_h[i].data_ptr(),
               w_h[i].data_ptr()) for i in range(n_e2e)]

    def e2e_step():
        for a in hcalls:
            if fh(*a):
                raise RuntimeError("gguf_moe_ffn_host failed")

    for _ in range(2):
        e2e_step()
    t0 = time.perf_counter()
    e2e_iters = max(3, args.steps // 4)
    for _ in range(e2e_iters):
        e2e_step()
    el = time.perf_counter() - t0
    e2e_tps = e2e_iters * n_e2e / el
    if world > 1:
        tt = torch.tensor([el], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        e2e_tps = e2e_iters * n_e2e * world / float(tt.item())
    # the step's tokens through the host API in one call per layer copy (the
    # step's T tokens split over the NL copies, tokens of a call one after
    # another on the device): one round trip per call instead of per token
    per_call = max(1, T // NL)
    hb_s = torch.from_numpy(np.ascontiguousarray(np.resize(toks, (NL * per_call, spec.dim)))).pin_memory()
    x_s = torch.zeros_like(hb_s).pin_memory()
    ids_s = torch.zeros((NL * per_call, spec.n_used), dtype=torch.int32).pin_memory()
    w_s = torch.zeros((NL * per_call, spec.n_used), dtype=torch.float32).pin_memory()
    d = spec.dim
    bcalls = [(layers[j].h, hb_s.data_ptr() + j * per_call * 4 * d, x_s.data_ptr() + j * per_call * 4 * d, per_call,
               ids_s.data_ptr() + j * per_call * 4 * spec.n_used, w_s.data_ptr() + j * per_call * 4 * spec.n_used)
              for j in range(NL)]

    def e2e_batched_step():
        for a in bcalls:
            if fh(*a):
                raise RuntimeError("gguf_moe_ffn_host failed")

    e2e_batched_step()
    t0 = time.perf_counter()
    for _ in range(e2e_iters):
        e2e_batched_step()
    elb = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([elb], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        elb = float(tt.item())
    e2e_b = e2e_iters * NL * per_call * world / elb
    # the same grouping on device pointers (tokens of one copy back to back):
    # shows whether consecutive tokens on one copy gain from L2
    gcalls = [(layers[(i // per_call) % NL].h, hb.data_ptr() + (i % nt) * d * 4, x.data_ptr() + (i % nt) * d * 4, 1,
               None, None, sp) for i in range(NL * per_call)]
    torch.cuda.synchronize(dev)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(max(1, args.steps // 4)):
        for a in gcalls:
            if ffn(*a):
                raise RuntimeError("gguf_moe_ffn failed")
    g1.record(stream)
    torch.cuda.synchronize(dev)
    grouped_tps = max(1, args.steps // 4) * NL * per_call / (g0.elapsed_time(g1) / 1e3)
    e2e = {"value": e2e_b, "unit": "tok/s", "h2d_bytes_per_step": T * 2 * 4 * d,
           "d2h_bytes_per_step": T * (4 * d + 8 * spec.n_used),
           "note": f"gguf_moe_ffn_host, pinned host buffers: the step's {T} tokens in {NL} calls of {per_call} "
                   f"tokens (one per layer copy), x / ids / wts returned and the status checked per call",
           "per_token_calls": {"value": e2e_tps, "unit": "tok/s",
                               "note": "one gguf_moe_ffn_host call per token (a synchronous decode hook)"},
           "device_rate_same_grouping": {"value": grouped_tps, "unit": "tok/s",
                                         "note": "gguf_moe_ffn on device pointers with the tokens grouped by layer "
                                                 "copy as in the host calls (L2 reuse check against value)"}}

    peak, peak_kind = peaks()
    per_launch_s = t_sec / launches if world == 1 else ms / 1e3 / launches
    achieved = per_tok / per_launch_s / 1e9
    tr = traffic_per_launch(args.workload)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": tr, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": per_tok,
                "kernel": "moe_decode_kernel (one launch per token)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        th = host_threads()
        rate, n, el, kind = cpu_reference_rate(layer, toks, args.cpu_seconds, th)
        cpu = {"value": rate, "unit": "tok/s", "cores": th, "kind": kind, "build": ref_build_name(kind),
               "sample": f"{n} tokens of the same workload in {el:.1f} s, OMP threads={th}"}

    if rank == 0:
        line = {"metric": "moe_decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_sec / args.steps * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded GGUF blocks, random-init weights)",
                "config": {"workload": args.workload, "desc": wl["desc"], "baseline_config": wl["config"],
                           "tokens_per_step": T, "batch": 1, "parallelism": f"replicas x{world}",
                           "l2": f"{NL} layer copies rotated per token (reuse distance "
                                 f"{NL * per_tok / 2**20:.0f} MiB > 126 MiB L2)",
                           "bytes_per_token": per_tok},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clk.summary(), "hbm_gbs": achieved}
    for m in layers:
        m.close()
    return line if rank == 0 else None


def run_prefill(args, wl):
    """Config 4: one MoE layer over 8192 tokens at once.  One GPU:
    gguf_moe_prefill (router GEMM + top-k, expert dispatch, Q4_K gate/up and
    Q6_K down grouped GEMMs on the tcgen05 tensor cores, combine).  N GPUs:
    gguf_moe_prefill_ep, expert parallel: each rank routes 8192/N of the
    tokens, experts are placed on ranks by expected load (the router bias),
    and the kernels store the rows into their experts' ranks and the outputs
    back over NVLink peer memory.
    A step is the whole 8192-token batch (strong scaling)."""
    import ctypes as C
    import torch
    import vireo_b200 as V

    world, rank, local = dist_start()
    L = V.lib()
    V.check(L.vireo_device_init(local), "vireo_device_init")
    spec = wl["spec"]()
    layer = S.MoeLayer(spec, wl["seed"])
    T, d = PREFILL_TOKENS, spec.dim
    if T % world:
        raise SystemExit(f"{T} tokens do not split over {world} ranks")
    Tl = T // world
    dev = torch.device("cuda", local)
    x_all = torch.from_numpy(S.normal(wl["seed"], 41, T * d).astype(np.float32).reshape(T, d)).to(torch.bfloat16)
    x_bf = x_all[rank * Tl:(rank + 1) * Tl].contiguous()
    bias_np = (S.normal(wl["seed"], 42, spec.n_experts) * 0.5).astype(np.float32)
    bias = torch.from_numpy(bias_np).to(dev)
    hb = x_bf.to(dev)
    x = torch.zeros((Tl, d), dtype=torch.float32, device=dev)
    ids = torch.empty((Tl, spec.n_used), dtype=torch.int32, device=dev)
    wts = torch.empty((Tl, spec.n_used), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    if world > 1:
        owner = V.ep_place(np.exp(bias_np.astype(np.float64)), world)
        uid = [V.ep_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(uid, src=0)
        ep = V.MoeLayerEP(layer, owner, rank, world, uid[0], Tl, local)
        # prep, router, count, exchange, dispatch, barrier, scan, expand,
        # gate/up, down, barrier, combine
        fn, handle, sync, launches = L.gguf_moe_prefill_ep, ep.h, L.gguf_moe_ep_sync, 12
        what = "gguf_moe_prefill_ep"
    else:
        m = V.MoeLayer(layer, local)
        # prep, router, scan, place, gate/up, down, combine
        fn, handle, sync, launches = L.gguf_moe_prefill, m.h, L.gguf_moe_sync, 7
        what = "gguf_moe_prefill"

    def step(hb_p, x_p):
        V.check(fn(handle, hb_p, x_p, Tl, bias.data_ptr(), ids.data_ptr(), wts.data_ptr(), sp), what)

    for _ in range(args.warmup):
        step(hb.data_ptr(), x.data_ptr())
    V.check(sync(handle, sp), "sync")
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(args.steps):
            step(hb.data_ptr(), x.data_ptr())
        e1.record(stream)
        torch.cuda.synchronize(dev)
    V.check(sync(handle, sp), "sync")
    t_sec = e0.elapsed_time(e1) / 1e3
    if world > 1:
        tt = torch.tensor([t_sec], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_sec = float(tt.item())
    value = args.steps * T / t_sec

    if args.timeline:
        write_timeline(args.timeline, rank, lambda: step(hb.data_ptr(), x.data_ptr()), 3)
    shares = None
    try:
        shares = kernel_shares(lambda: step(hb.data_ptr(), x.data_ptr()), 2)
    except Exception as ex:  # the profiler is a diagnostic; the timed numbers stand without it
        shares = [{"error": str(ex)[:120]}]

    # end to end: hidden states and residual from pinned host memory, residual back
    hb_h = x_bf.pin_memory()
    x_h = torch.zeros((Tl, d), dtype=torch.float32).pin_memory()
    n_e2e = max(3, args.steps // 4)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        with torch.cuda.stream(stream):
            hb.copy_(hb_h, non_blocking=True)
            x.copy_(x_h, non_blocking=True)
        step(hb.data_ptr(), x.data_ptr())
        with torch.cuda.stream(stream):
            x_h.copy_(x, non_blocking=True)
        stream.synchronize()
    el = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([el], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        el = float(tt.item())
    e2e_tps = n_e2e * T / el

    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        peak, peak_kind = float(pk["bf16_tflops_sustained"]), "measured (bf16 sustained)"
    except Exception:
        peak, peak_kind = 1400.0, "fallback (sustained)"
    achieved = PREFILL_FLOPS * args.steps / t_sec / 1e12 / world  # per GPU, against one GPU's peak
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        th = host_threads()
        toks, _ = S.routed_tokens(layer, 64, wl["seed"])
        rate, n, el, kind = cpu_reference_rate(layer, toks, args.cpu_seconds, th)
        cpu = {"value": rate, "unit": "tok/s", "cores": th, "kind": kind, "build": ref_build_name(kind),
               "sample": f"{n} tokens through the reference's moe_ffn (one token at a time, its only "
                         f"path) in {el:.1f} s, OMP threads={th}, no router bias"}
    if rank == 0:
        line = {"metric": "moe_prefill_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_sec / args.steps * 1e3,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded GGUF blocks, random-init weights, N(0,1) bf16 tokens)",
                "config": {"workload": args.workload, "desc": wl["desc"], "baseline_config": wl["config"],
                           "tokens_per_step": T, "tokens_per_rank": Tl,
                           "parallelism": f"ep{world}" if world > 1 else "single GPU",
                           "l2": "391 MB of expert weights + 34 MB of tokens per step, above the 126 MB L2"},
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                             "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                             "algorithmic_flops_per_step": PREFILL_FLOPS,
                             "kernel": "whole step per GPU (router, dispatch, gate/up, down, combine"
                                       + (", peer-memory dispatch and return)" if world > 1 else ")")},
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_tps, "unit": "tok/s", "h2d_bytes_per_step": T * d * (2 + 4),
                        "d2h_bytes_per_step": T * d * 4,
                        "note": "bf16 tokens + fp32 residual in from pinned host, residual out (all ranks)"},
                "gpu_launches": launches * args.steps, "clocks": clk.summary(),
                "kernel_shares": shares}
    if world > 1:
        ep.close()
    else:
        m.close()
    return line if rank == 0 else None


def cpu_decoder_rate(dec, seconds, threads, ctx=0):
    """The reference's own forward() (oracle/_ref, its dense KV store and
    ExpertStore) over 1- and 2-layer slices of the same decoder, with every
    layer's KV store holding ctx positions (seeded through the reference's
    kv_append) so that each timed step attends over ctx + 1 positions;
    seconds per token for the full layer count by a linear fit (a + b L: the
    LM head and embedding plus L layers)."""
    from oracle import oracle as O
    if not O.ref_available():
        return None
    O.ref().ref_set_threads(threads)
    per = {}
    for nl in (1, 2):
        sub = S.Decoder.__new__(S.Decoder)
        sub.spec = S.DecoderSpec(nl, dec.spec.dim, dec.spec.n_heads, dec.spec.n_kv_heads, dec.spec.head_size,
                                 dec.spec.vocab, dec.spec.moe, dec.spec.qk_norm, dec.spec.attn_type,
                                 dec.spec.embd_type, dec.spec.lm_type, dec.spec.eps, dec.spec.rope_base)
        sub.seed, sub.tok_embd, sub.out_norm, sub.lm_head = dec.seed, dec.tok_embd, dec.out_norm, dec.lm_head
        sub.layers = dec.layers[:nl]
        R = O.RefDecoder(sub)
        try:
            if ctx:
                R.fill_kv(ctx, 5)
            R.step(1, ctx, True)
            n, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < seconds / 2 and n < 64:
                R.step((7 * n + 3) % dec.spec.vocab, ctx + n + 1, True)
                n += 1
            per[nl] = (time.perf_counter() - t0) / n
        finally:
            R.close()
    b = per[2] - per[1]
    a = per[1] - b
    full = a + b * dec.spec.n_layers
    return full, per


def run_decoder(args, wl):
    """Configs 2 and 3: whole decode steps (gguf_decoder_step_dev: every
    layer's attention and MoE block, the final norm, the LM head and the
    greedy argmax on the device; each step's token is the previous step's
    argmax, read on the device).  The prompt is fed first (seeded ids, no LM
    head, as the reference's prompt steps); a step of the timed region is
    one generated token."""
    import torch
    import vireo_b200 as V

    world, rank, local = dist_start()
    L = V.lib()
    V.check(L.vireo_device_init(local), "vireo_device_init")
    spec = wl["spec"]()
    if args.layers:
        spec = S.DecoderSpec(args.layers, spec.dim, spec.n_heads, spec.n_kv_heads, spec.head_size, spec.vocab, spec.moe,
                             spec.qk_norm, spec.attn_type, spec.embd_type, spec.lm_type, spec.eps, spec.rope_base)
    P, gen = (wl["prompt"] if args.prompt is None else args.prompt), max(args.steps, 1)
    dec = S.Decoder(spec, wl["seed"], n_distinct_layers=1)
    dev = torch.device("cuda", local)
    G = V.Decoder(dec, max_ctx=P + gen + args.warmup + 40, kv_f16=True, device=local)
    stream = torch.cuda.Stream(dev)
    sp = stream.cuda_stream
    prompt = (S.u64(wl["seed"], 55, P) % np.uint64(spec.vocab)).astype(np.int64)
    tok = torch.zeros(1, dtype=torch.int32, device=dev)
    t0 = time.perf_counter()
    for pos in range(P):
        G.step(int(prompt[pos]), pos, stream=sp)
    G.sync(sp)
    prompt_s = time.perf_counter() - t0
    pos = P
    with torch.cuda.stream(stream):
        tok.fill_(int(prompt[-1]))
    for _ in range(args.warmup):
        G.step_dev(tok, pos, next=tok, stream=sp)
        pos += 1
    G.sync(sp)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx0 = pos
    with Clocks(local) as clk:
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(gen):
            G.step_dev(tok, pos, next=tok, stream=sp)
            pos += 1
        e1.record(stream)
        torch.cuda.synchronize(dev)
    G.sync(sp)
    t_sec = e0.elapsed_time(e1) / 1e3
    if world > 1:
        tt = torch.tensor([t_sec], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_sec = float(tt.item())
    value = gen * world / t_sec
    # end to end: the host API with a host token per step and the next token
    # read back to the host every step
    n_e2e = min(gen, 32)
    nxt = torch.zeros(1, dtype=torch.int32, device=dev)
    host_tok = int(tok.item())
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        G.step(host_tok, pos, next=nxt, stream=sp)
        pos += 1
        stream.synchronize()
        host_tok = int(nxt.item())
    e2e_tps = n_e2e * world / (time.perf_counter() - t0)
    G.sync(sp)
    if args.timeline:
        # two more greedy steps at the full context under the CUDA activity
        # profiler (untimed)
        tl_pos = [pos]

        def tl_step():
            with torch.cuda.stream(stream):
                G.step_dev(tok, tl_pos[0], next=tok, stream=sp)
            tl_pos[0] += 1

        write_timeline(args.timeline, rank, tl_step, 2)
        pos = tl_pos[0]
        G.sync(sp)

    avg_ctx = ctx0 + gen / 2
    wbytes = spec.weight_bytes_per_token()
    kvb = spec.kv_bytes_per_position(2) * avg_ctx
    per_tok = wbytes + kvb
    peak, peak_kind = peaks()
    achieved = per_tok * gen / t_sec / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        th = host_threads()
        r = cpu_decoder_rate(dec, args.cpu_seconds, th, ctx=ctx0)
        if r:
            from oracle import oracle as O
            full, per = r
            cpu = {"value": 1.0 / full, "unit": "tok/s", "cores": th, "kind": "reference",
                   "build": O.ref_build(),
                   "sample": f"the reference's forward() on 1- and 2-layer slices of this decoder, each step "
                             f"attending over {ctx0}+ cached positions (its dense KV store filled through "
                             f"kv_append) ({per[1] * 1e3:.1f} / {per[2] * 1e3:.1f} ms per token), linear in the "
                             f"layer count to {spec.n_layers} layers; OMP threads={th}"}
    if rank == 0:
        line = {"metric": "decoder_decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world,
                "steps": gen, "warmup": args.warmup, "ms_per_step": t_sec / gen * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded GGUF blocks, random-init weights, seeded prompt ids, greedy decode)",
                "config": {"workload": args.workload, "desc": wl["desc"], "baseline_config": wl["config"],
                           "layers": spec.n_layers, "prompt_tokens": P, "context_at_timed_start": ctx0,
                           "kv_cache": "f16", "batch": 1, "parallelism": f"replicas x{world}",
                           "prompt_seconds": prompt_s,
                           "l2": "every layer's weights at distinct addresses; 2 GB of weights per token"},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                             "algorithmic_bytes_per_step": per_tok,
                             "weight_bytes_per_token": wbytes, "kv_bytes_per_token": kvb,
                             "kernel": "whole decode step (all layers, LM head, argmax)"},
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4,
                        "note": "gguf_decoder_step with a host token id per step, next token read back"},
                "gpu_launches": gen * (4 * spec.n_layers + 3), "clocks": clk.summary()}
    G.close()
    return line if rank == 0 else None


def kernel_shares(step, n, top=5):
    """Per-kernel share of GPU time over n untimed steps, from the CUDA
    activity profiler (CUPTI via torch.profiler): [{name, us_per_step,
    share}] of the top kernels by total duration, for naming the limiter.
    Under torchrun the ranks meet at a barrier once every profiler is up, so
    that no rank's kernels wait on a peer still starting its profiler."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            torch.distributed.barrier()
            torch.cuda.synchronize()
        for _ in range(n):
            step()
        torch.cuda.synchronize()
    tot = {}
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            nm = e.name.split("(")[0][:80]
            tot[nm] = tot.get(nm, 0.0) + e.device_time_total
    allt = sum(tot.values()) or 1.0
    rows = sorted(tot.items(), key=lambda kv: -kv[1])[:top]
    return [{"name": k, "us_per_step": v / n, "share": v / allt} for k, v in rows]


def write_timeline(path, rank, step, n):
    """Kernel timeline of n steps from the CUDA activity profiler (CUPTI via
    torch.profiler): start offset, duration and name of every kernel, memcpy
    and memset on this rank's GPU, one line each, to path.rank<r>.txt."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            step()
        torch.cuda.synchronize()
    raw = f"{path}.rank{rank}.json"
    prof.export_chrome_trace(raw)
    with open(raw) as f:
        ev = [e for e in json.load(f)["traceEvents"] if e.get("cat") in ("kernel", "gpu_memcpy", "gpu_memset")]
    os.remove(raw)
    ev.sort(key=lambda e: e["ts"])
    t0 = ev[0]["ts"] if ev else 0
    with open(f"{path}.rank{rank}.txt", "w") as f:
        f.write("# start_us duration_us kernel\n")
        for e in ev:
            f.write(f"{e['ts'] - t0:10.1f} {e['dur']:9.1f}  {e['name'][:100]}\n")


def zipf_routes(n_tok, n_layers, ne, k, seed):
    """Per (token, layer): k distinct experts drawn from Zipf(ZIPF_S) over a
    seeded random permutation of the layer's experts; weights = the drawn
    experts' Zipf probabilities, renormalised (the routing override of the
    cached configuration)."""
    rng = np.random.default_rng(seed)
    p = np.arange(1, ne + 1, dtype=np.float64) ** -ZIPF_S
    p /= p.sum()
    perms = np.stack([rng.permutation(ne) for _ in range(n_layers)])
    ids = np.empty((n_tok, n_layers, k), dtype=np.int32)
    wts = np.empty((n_tok, n_layers, k), dtype=np.float32)
    for t in range(n_tok):
        for l in range(n_layers):
            r = rng.choice(ne, k, replace=False, p=p)
            ids[t, l] = perms[l][r]
            wts[t, l] = (p[r] / p[r].sum()).astype(np.float32)
    return ids, wts


def cpu_cached_rate(layer, seconds, threads):
    """The reference's moe_ffn with its own ExpertStore capped at the same
    share of the budget per layer (4 GiB / 48 layers), on tokens routed by
    its own router (it has no routing override): layer-tokens per second,
    divided by 48 for tokens through the whole stack."""
    from oracle import oracle as O
    if not O.ref_available():
        return None
    O.ref().ref_set_threads(threads)
    cap = CACHE_BYTES // CACHED_LAYERS
    toks, _ = S.routed_tokens(layer, 256, 99)
    R = O.RefMoe(layer, cap)
    try:
        R(toks[:8])
        n, t0 = 0, time.perf_counter()
        while True:
            R(toks[n % 256:n % 256 + 1])
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds and n >= 8:
                break
        st = R.stats()
    finally:
        R.close()
    rate = n / el
    return {"value": rate / CACHED_LAYERS, "unit": "tok/s", "cores": threads, "kind": "reference",
            "build": O.ref_build(),
            "sample": f"{n} tokens through one Qwen3-shaped layer's moe_ffn with the reference ExpertStore "
                      f"capped at {cap >> 20} MiB (4 GiB / {CACHED_LAYERS} layers; misses pread from its "
                      f"backing file) in {el:.1f} s = {rate:.1f} layer-tokens/s, / {CACHED_LAYERS} layers; "
                      f"its own routing (hit rate {st.hits / max(st.requests, 1):.2f}); OMP threads={threads}"}


def run_cached(args, wl):
    """Config 5: the 48-layer MoE stack with every expert in pinned host
    memory and a 4 GiB device ExpertStore; each layer is one
    gguf_moe_ffn_store call (async lookups, misses copied host -> device on
    the store's copy stream, routed kernel, leases released after it)."""
    import ctypes as C
    import torch
    import vireo_b200 as V

    world, rank, local = dist_start()
    L = V.lib()
    V.check(L.vireo_device_init(local), "vireo_device_init")
    spec = wl["spec"]()
    layer = S.MoeLayer(spec, wl["seed"])
    NLY, NE, k, d = CACHED_LAYERS, spec.n_experts, spec.n_used, spec.dim
    gs, us, ds = layer.gate.nbytes // NE, layer.up.nbytes // NE, layer.down.nbytes // NE
    one = np.concatenate([layer.gate.view(np.uint8).ravel(), layer.up.view(np.uint8).ravel(),
                          layer.down.view(np.uint8).ravel()])
    per = one.nbytes
    # every layer's experts in pinned host memory (18.8 GB); if the host
    # cannot pin that much, all layers alias one layer's bytes (same sizes,
    # same copies, distinct device frames)
    aliased = False
    try:
        image = torch.empty(NLY * per, dtype=torch.uint8, pin_memory=True)
        src = torch.from_numpy(one)
        for l in range(NLY):
            image[l * per:(l + 1) * per].copy_(src)
    except Exception:
        aliased = True
        image = torch.from_numpy(one).pin_memory()
    base = lambda l: 0 if aliased else l * per

    def make_store(cap):
        st = L.expert_store_create_host(image.data_ptr(), image.numel(), cap, NLY, NE)
        assert st, "expert_store_create_host failed"
        for l in range(NLY):
            for e in range(NE):
                sl = V.ExpertSlices(base(l) + e * gs, base(l) + layer.gate.nbytes + e * us,
                                    base(l) + layer.gate.nbytes + layer.up.nbytes + e * ds, gs, us, ds)
                L.expert_store_register(st, l, e, C.byref(sl))
        return st

    m = V.MoeLayer(layer, local)  # the handle (shape, scratch); experts come from the store
    T = max(1, min(args.tokens, 64))
    n_tok = (args.warmup + args.steps) * T
    ids, wts = zipf_routes(n_tok, NLY, NE, k, wl["seed"] + 7)
    hbs, _ = S.routed_tokens(layer, NLY, wl["seed"])
    dev = torch.device("cuda", local)
    hb = torch.from_numpy(hbs).to(dev)
    x = torch.zeros(d, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    fn = L.gguf_moe_ffn_store
    calls = [[(m.h, None, l, hb[l].data_ptr(), x.data_ptr(), ids[t, l].ctypes.data, wts[t, l].ctypes.data, sp)
              for l in range(NLY)] for t in range(n_tok)]

    def run_tokens(store, t0, t1):
        for t in range(t0, t1):
            for a in calls[t]:
                if fn(a[0], store, *a[2:]):
                    raise RuntimeError("gguf_moe_ffn_store failed")

    def timed(store):
        run_tokens(store, 0, args.warmup * T)
        stream.synchronize()
        s0, x0 = V.ExpertStats(), V.ExpertStatsExt()
        L.expert_store_stats(store, C.byref(s0))
        L.expert_store_stats_ext(store, C.byref(x0))
        if world > 1:
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        run_tokens(store, args.warmup * T, n_tok)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        s1, x1 = V.ExpertStats(), V.ExpertStatsExt()
        L.expert_store_stats(store, C.byref(s1))
        L.expert_store_stats_ext(store, C.byref(x1))
        return e0.elapsed_time(e1) / 1e3, s1.requests - s0.requests, s1.hits - s0.hits, x1.h2d_bytes - x0.h2d_bytes

    cached = make_store(CACHE_BYTES)
    with Clocks(local) as clk:
        t_sec, req, hits, h2d = timed(cached)
    # the same tokens with every expert resident (unbounded store, warmed by
    # touching every expert): the copy time the cached run exposes is the gap
    full = make_store(0)
    for l in range(NLY):
        vv = V.ExpertView()
        for e in range(NE):
            if L.expert_store_lookup(full, l, e, C.byref(vv)) == 0:
                L.expert_store_release(full, C.byref(vv))
    t_hit, _, _, _ = timed(full)
    L.expert_store_destroy(full)
    if world > 1:
        tt = torch.tensor([t_sec, t_hit], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_sec, t_hit = float(tt[0]), float(tt[1])
    ntimed = args.steps * T
    value = ntimed * world / t_sec

    # end to end: per token, this token's hidden vectors and residual copied in
    # from pinned host memory and the residual read back
    hb_h = torch.from_numpy(hbs).pin_memory()
    x_h = torch.zeros(d, dtype=torch.float32).pin_memory()
    n_e2e = min(T, 16)
    t0 = time.perf_counter()
    for t in range(n_e2e):
        with torch.cuda.stream(stream):
            hb.copy_(hb_h, non_blocking=True)
            x.copy_(x_h, non_blocking=True)
        run_tokens(cached, t, t + 1)
        with torch.cuda.stream(stream):
            x_h.copy_(x, non_blocking=True)
        stream.synchronize()
    e2e_tps = n_e2e / (time.perf_counter() - t0)
    L.expert_store_destroy(cached)

    layer_bytes = k * (gs + us + ds) + 2 * 4 * d  # routed launch: no router rows
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_cached_rate(layer, args.cpu_seconds, host_threads())
    peak, peak_kind = peaks()
    achieved = layer_bytes * NLY * ntimed / t_hit / 1e9
    if rank == 0:
        line = {"metric": "moe_decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_sec / args.steps * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded GGUF blocks, random-init weights, Zipf routing)",
                "config": {"workload": args.workload, "desc": wl["desc"], "baseline_config": wl["config"],
                           "layers": NLY, "tokens_per_step": T, "batch": 1, "parallelism": f"replicas x{world}",
                           "cache_bytes": CACHE_BYTES, "host_image_bytes": image.numel(),
                           "host_image": "one layer aliased by all 48" if aliased else "all 48 layers",
                           "l2": "48 layers x 8 experts x 3.06 MB per token, far above the 126 MB L2"},
                "cache": {"hit_rate": hits / max(req, 1), "requests": req,
                          "h2d_bytes_per_token": h2d / ntimed,
                          "exposed_copy_ms_per_token": max(0.0, (t_sec - t_hit) / ntimed * 1e3),
                          "all_hit_tok_per_s": ntimed * world / t_hit},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                             "algorithmic_bytes_per_launch": layer_bytes,
                             "kernel": "moe_routed_kernel (one launch per layer), all-hit run"},
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_tps * world, "unit": "tok/s", "h2d_bytes_per_step": T * (hbs.nbytes + 4 * d),
                        "d2h_bytes_per_step": T * 4 * d,
                        "note": "per token: hidden vectors + residual in from pinned host, residual out"},
                "gpu_launches": ntimed * NLY, "clocks": clk.summary()}
    m.close()
    return line if rank == 0 else None


SUB_RUNNERS = {"qwen3_prefill": run_prefill, "qwen3_decoder": run_decoder, "olmoe_decoder": run_decoder,
               "qwen3_cached_decode": run_cached}

if __name__ == "__main__":
    main()
