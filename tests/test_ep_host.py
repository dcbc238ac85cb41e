"""Expert parallelism on the host, no GPU: the library's placement and
all-to-all offset functions (gguf_moe_ep_place, gguf_moe_ep_offsets), and
the expert-parallel dataflow of gguf_moe_prefill_ep run end to end as two
gloo ranks on CPU with the CPU oracle as the expert math.

The dataflow test follows the device path step by step: each rank routes its
own tokens, sends every (token, slot) row to the rank that owns the slot's
expert (counts all-gathered, offsets from gguf_moe_ep_offsets), the owner
computes w * expert(x), the rows come back, and each token is combined in
rank order.  The result must equal the single-process restatement of the
reference's moe_ffn bit for bit (same float32 operations in the same order).
"""
import datetime
import os
import socket

import numpy as np
import pytest

from vireo_b200 import synth as S


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spec():
    return S.MoeLayerSpec(512, 256, 16, 4, 1, S.GGML_Q4_K, S.GGML_Q4_K, S.GGML_Q6_K)


def test_place_balances_load_and_counts():
    import vireo_b200 as V
    rng = np.random.default_rng(3)
    for ne, world in [(16, 2), (128, 8), (128, 4), (10, 3), (7, 7)]:
        load = rng.exponential(size=ne)
        owner = V.ep_place(load, world)
        held = np.bincount(owner, minlength=world)
        assert held.min() >= ne // world and held.max() <= -(-ne // world), held
        per = np.bincount(owner, weights=load, minlength=world)
        # greedy placement stays within one expert of a perfect split
        assert per.max() - per.min() <= load.max() + 1e-12, (per, load.max())
        assert np.array_equal(owner, V.ep_place(load, world))  # deterministic
    with pytest.raises(V.VireoError):
        V.ep_place(np.ones(4), 0)


def test_offsets_match_a_prefix_sum():
    import vireo_b200 as V
    rng = np.random.default_rng(5)
    for world in (1, 2, 5, 8):
        cnt = rng.integers(0, 50, size=(world, world)).astype(np.int32)
        for r in range(world):
            so, ro, rc, tot = V.ep_offsets(cnt, r)
            assert np.array_equal(so, np.concatenate([[0], np.cumsum(cnt[r])[:-1]]))
            assert np.array_equal(rc, cnt[:, r])
            assert np.array_equal(ro, np.concatenate([[0], np.cumsum(cnt[:, r])[:-1]]))
            assert tot == cnt[:, r].sum()
    with pytest.raises(V.VireoError):
        V.ep_offsets(-np.ones((2, 2), dtype=np.int32), 0)


def _ep_rank(rank, world, port, seed, n_tok, out_dir):
    """One gloo rank of the expert-parallel dataflow (module level: spawned)."""
    import torch
    import torch.distributed as dist

    import vireo_b200 as V
    from oracle import oracle as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        spec = _spec()
        L = S.MoeLayer(spec, seed)
        P = O.PortMoe(L)
        d, k, ne = spec.dim, spec.n_used, spec.n_experts
        toks, _ = S.routed_tokens(L, n_tok, seed)
        x0 = (S.normal(seed, 9, toks.size) * 0.5).astype(np.float32).reshape(toks.shape)
        lo, hi = n_tok * rank // world, n_tok * (rank + 1) // world
        mine, xm = toks[lo:hi], x0[lo:hi]
        T = mine.shape[0]
        # every rank places the experts the same way (a fixed synthetic load)
        owner = V.ep_place(np.arange(ne, 0, -1, dtype=np.float64) ** 1.5, world)
        # route the local tokens
        _, ids, wts = P(mine)
        dest = owner[ids.reshape(-1)]
        sendcnt = np.bincount(dest, minlength=world).astype(np.int32)
        allc = [torch.zeros(world, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(allc, torch.from_numpy(sendcnt))
        counts = torch.stack(allc).numpy()
        so, ro, rc, R = V.ep_offsets(counts, rank)
        # dispatch rows: [hidden | expert | weight], grouped by destination in pair order
        send = np.zeros((int(sendcnt.sum()), d + 2), dtype=np.float32)
        pos = np.zeros(T * k, dtype=np.int64)
        fill = so.astype(np.int64).copy()
        for p in range(T * k):
            q = dest[p]
            pos[p] = fill[q]
            fill[q] += 1
            send[pos[p], :d] = mine[p // k]
            send[pos[p], d] = ids.reshape(-1)[p]
            send[pos[p], d + 1] = wts.reshape(-1)[p]
        recv = torch.zeros((R, d + 2), dtype=torch.float32)
        dist.all_to_all_single(recv, torch.from_numpy(send), [int(c) for c in rc], [int(c) for c in sendcnt])
        recv = recv.numpy()
        # the experts held here: y = w * expert(x)
        ysend = np.zeros((R, d), dtype=np.float32)
        for i in range(R):
            e = int(recv[i, d])
            assert owner[e] == rank, (e, owner[e], rank)
            ysend[i] = np.float32(recv[i, d + 1]) * P.expert(e, recv[i, :d])
        yret = torch.zeros((send.shape[0], d), dtype=torch.float32)
        dist.all_to_all_single(yret, torch.from_numpy(ysend), [int(c) for c in sendcnt], [int(c) for c in rc])
        yret = yret.numpy()
        # combine in rank order, then the residual add
        x = xm.copy()
        for t in range(T):
            acc = np.zeros(d, dtype=np.float32)
            for i in range(k):
                acc = acc + yret[pos[t * k + i]]
            x[t] = x[t] + acc
        ref, _, _ = P(mine, xm)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.stack([x, ref]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_ep_dataflow_two_gloo_ranks_bit_exact(tmp_path, world):
    import torch.multiprocessing as mp
    mp.start_processes(_ep_rank, args=(world, _free_port(), 21, 30, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        x, ref = np.load(tmp_path / f"rank{r}.npy")
        assert x.shape[0] > 0
        assert np.array_equal(x.view(np.uint32), ref.view(np.uint32)), (r, np.abs(x - ref).max())
