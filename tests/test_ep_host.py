"""Expert parallelism on the host, no GPU: the library's placement and
row-layout functions (gguf_moe_ep_place, gguf_moe_ep_rows), and the
expert-parallel dataflow of gguf_moe_prefill_ep run end to end as two gloo
ranks on CPU with the CPU oracle as the expert math.

The dataflow test follows the device path step by step: each rank routes its
own tokens and counts pairs per expert, the counts are all-gathered, a
token's hidden row goes once to each other rank holding one of its experts
(its receive buffer) and each (token, slot) pair's metadata to the row
gguf_moe_ep_rows assigns it in its expert's range on the owning rank (gloo
stands in for the peer stores), the owner fills each row from its own tokens
or its receive buffer, finds each row's expert from the layout alone and
computes w * expert(x),
the rows return to (source rank, pair), and each token is combined in rank
order.  The result must equal the single-process restatement of the
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


def test_rows_layout_matches_the_owner_scan():
    """dst_off from gguf_moe_ep_rows against the owner's layout written out
    directly: experts in index order, each range padded to 128 rows, sources
    in rank order inside a range."""
    import vireo_b200 as V
    rng = np.random.default_rng(5)
    for world, ne in [(1, 8), (2, 16), (3, 10), (8, 128)]:
        cnt = rng.integers(0, 300, size=(world, ne)).astype(np.int32)
        cnt[:, rng.integers(0, ne)] = 0  # an expert nobody routes to
        owner = V.ep_place(rng.exponential(size=ne), world)
        base = {}
        for q in range(world):
            b = 0
            for e in range(ne):
                if owner[e] == q:
                    base[e] = b
                    b += -(-int(cnt[:, e].sum()) // 128) * 128
        for r in range(world):
            off, here = V.ep_rows(cnt, owner, r)
            for e in range(ne):
                assert off[e] == base[e] + cnt[:r, e].sum(), (world, r, e)
            assert here == sum(int(cnt[:, e].sum()) for e in range(ne) if owner[e] == r)
    with pytest.raises(V.VireoError):
        V.ep_rows(-np.ones((2, 4), dtype=np.int32), np.zeros(4, dtype=np.int32), 0)


def off_rows(counts, owner, rank, e, row):
    """True when `row` lies in expert e's range on its owner `rank` (the
    layout gguf_moe_ep_rows describes)."""
    b = 0
    for e2 in range(counts.shape[1]):
        if owner[e2] != rank:
            continue
        n = int(counts[:, e2].sum())
        if e2 == e:
            return b <= row < b + n
        b += -(-n // 128) * 128
    return False


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
        # route the local tokens; per expert, the local count and each pair's index
        _, ids, wts = P(mine)
        flat = ids.reshape(-1)
        pos = np.zeros(T * k, dtype=np.int64)
        cnt = np.zeros(ne, dtype=np.int32)
        for p in range(T * k):
            pos[p] = cnt[flat[p]]
            cnt[flat[p]] += 1
        allc = [torch.zeros(ne, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(allc, torch.from_numpy(cnt))
        counts = torch.stack(allc).numpy()
        off, here = V.ep_rows(counts, owner, rank)
        # dispatch (the peer stores of the device path, carried here by gloo):
        # a token's hidden row goes ONCE to each other rank holding one of its
        # experts, into that rank's receive buffer at slot rank * max_tok + t;
        # each pair's metadata (its row off[e] + pos on the owner, weight,
        # pair, expert, receive slot or -1 when this rank placed the row
        # itself) goes to the pair's owner
        max_tok = n_tok
        dest = owner[flat]
        tok_dest = sorted({(int(q), p // k) for p, q in enumerate(dest) if q != rank})
        # tokens with several experts on one peer send their row once: fewer
        # rows than remote pairs
        assert len(tok_dest) < int((dest != rank).sum())
        tsend = np.zeros((len(tok_dest), d + 1), dtype=np.float32)  # [hidden | receive slot]
        for j, (q, t) in enumerate(tok_dest):
            tsend[j, :d] = mine[t]
            tsend[j, d] = rank * max_tok + t
        tsendcnt = np.bincount(np.array([q for q, _ in tok_dest], dtype=np.int64), minlength=world)
        tall = [torch.zeros(world, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(tall, torch.from_numpy(tsendcnt.astype(np.int64)))
        trecvcnt = np.array([int(tall[q][rank]) for q in range(world)])
        trecv = torch.zeros((int(trecvcnt.sum()), d + 1), dtype=torch.float32)
        dist.all_to_all_single(trecv, torch.from_numpy(tsend), [int(c) for c in trecvcnt], [int(c) for c in tsendcnt])
        xr = {}
        for row in trecv.numpy():
            slot = int(row[d])
            assert slot not in xr  # one row per (source rank, token)
            xr[slot] = row[:d]
        sendcnt = np.bincount(dest, minlength=world)
        recvcnt = np.array([counts[q][owner == rank].sum() for q in range(world)])
        order = np.argsort(dest, kind="stable")
        send = np.zeros((T * k, 5), dtype=np.float32)  # [dest row | weight | pair | expert | receive slot]
        for j, p in enumerate(order):
            send[j, 0] = off[flat[p]] + pos[p]
            send[j, 1] = wts.reshape(-1)[p]
            send[j, 2] = p
            send[j, 3] = flat[p]
            send[j, 4] = -1 if dest[p] == rank else rank * max_tok + p // k
        meta = torch.zeros((int(recvcnt.sum()), 5), dtype=torch.float32)
        dist.all_to_all_single(meta, torch.from_numpy(send), [int(c) for c in recvcnt], [int(c) for c in sendcnt])
        meta = meta.numpy()
        # the owner's operand rows: rows placed by this rank come from its own
        # tokens, the others from the receive buffer (prefill_expand)
        recv = np.zeros((len(meta), d + 4), dtype=np.float32)  # [hidden | dest row | weight | pair | expert]
        recv[:, d:] = meta[:, :4]
        src = np.repeat(np.arange(world), recvcnt)
        for i in range(len(meta)):
            slot = int(meta[i, 4])
            assert (slot < 0) == (src[i] == rank)  # only the owner's own pairs skip the receive buffer
            recv[i, :d] = mine[int(meta[i, 2]) // k] if slot < 0 else xr[slot]
        rows = np.full((max(int(recv[:, d].max()) + 1 if len(recv) else 0, 1),), -1, dtype=np.int64)
        for i in range(len(recv)):
            assert rows[int(recv[i, d])] == -1  # no two pairs share a row
            rows[int(recv[i, d])] = i
        assert here == len(recv)
        # the experts held here: y = w * expert(x), returned to (source rank, pair)
        yback = np.zeros((len(recv), d), dtype=np.float32)
        for i in range(len(recv)):
            r0 = int(recv[i, d])
            held = [e2 for e2 in range(ne) if owner[e2] == rank and off_rows(counts, owner, rank, e2, r0)]
            assert held == [int(recv[i, d + 3])], (held, recv[i, d + 3])  # the layout alone names the expert
            yback[i] = np.float32(recv[i, d + 1]) * P.expert(held[0], recv[i, :d])
        ret = np.concatenate([yback, recv[:, d + 2:d + 3]], axis=1)
        got = torch.zeros((T * k, d + 1), dtype=torch.float32)
        dist.all_to_all_single(got, torch.from_numpy(ret), [int(c) for c in sendcnt], [int(c) for c in recvcnt])
        got = got.numpy()
        yret = np.zeros((T * k, d), dtype=np.float32)
        for j in range(T * k):
            yret[int(got[j, d])] = got[j, :d]
        # combine in rank order, then the residual add
        x = xm.copy()
        for t in range(T):
            acc = np.zeros(d, dtype=np.float32)
            for i in range(k):
                acc = acc + yret[t * k + i]
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
