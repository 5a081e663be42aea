"""Host logic of the data-parallel + expert-parallel MoE path, on the CPU.

The CUDA kernels (moe_ep.cu) place each routed pair in its expert owner's
receive buffer by a plan computed from every rank's per-expert counts; the
plan is restated in catnn_b200.dist. These tests check that restatement:
(1) for 1..8 ranks the rows an owner receives are, expert by expert, the
pairs the one-GPU permutation would give that expert, in the same order,
padded to the alignment, within the allocated capacity; (2) two gloo ranks
that route, dispatch, run the experts and combine through this plan produce
exactly the oracle's one-process MoE output (moe.rs:186-219 restated)."""
import os
import socket

import numpy as np
import pytest

from catnn_b200 import dist as D
from oracle import oracle as O


def _route_all(T, h, E, k, seed):
    r = np.random.default_rng(seed)
    x = r.standard_normal((T, h)).astype(np.float32)
    gate = r.standard_normal((h, E)).astype(np.float32)
    idx, w, _ = O.route(x, gate, k)
    return x, gate, idx, w


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("align", [1, 128])
def test_plan_reproduces_one_gpu_expert_order(world, align):
    B, S, h, E, k = 8, 16, 8, 8, 2
    Tg = B * S
    _, _, idx, _ = _route_all(Tg, h, E, k, 11 + world)
    El = E // world
    Tl = Tg // world
    shards = [idx[r * Tl:(r + 1) * Tl] for r in range(world)]
    counts_all = np.stack([np.bincount(s.reshape(-1), minlength=E) for s in shards])
    recv = [dict() for _ in range(world)]
    for s in range(world):
        assert D.shard(s, world, B, S) == (s * Tl, Tl)
        dest = D.ep_dest_rows(shards[s], counts_all, s, align)
        for i, e in enumerate(shards[s].reshape(-1)):
            o = D.expert_owner(int(e), E, world)
            assert dest[i] not in recv[o], "two pairs share a row"
            recv[o][int(dest[i])] = (s * Tl * k + i, int(e))
    cap = Tg * min(k, El) + El * (align - 1)
    flat = idx.reshape(-1)
    for o in range(world):
        off, tot, _ = D.ep_plan(counts_all, o, align)
        assert off[El] <= cap
        rows = recv[o]
        for j in range(El):
            e = o * El + j
            want = np.nonzero(flat == e)[0]  # one-GPU order: pairs of e in pair order
            got = [rows[r][0] for r in range(off[j], off[j] + tot[j])]
            assert np.array_equal(got, want), (o, e)
            assert all(rows[r][1] == e for r in range(off[j], off[j] + tot[j]))
            pad = off[j + 1] - off[j] - tot[j]
            assert 0 <= pad < align and (off[j + 1] - off[j]) % align == 0
            assert not any(r in rows for r in range(off[j] + tot[j], off[j + 1]))
        assert len(rows) == int(tot.sum())


def test_plan_capacity_worst_case():
    """Every token routes to rank 0's experts: the receive buffer is exactly full."""
    world, E, k, align, Tg = 4, 8, 2, 128, 256
    El = E // world
    counts_all = np.zeros((world, E), np.int64)
    counts_all[:, 0] = Tg // world
    counts_all[:, 1] = Tg // world
    off, tot, _ = D.ep_plan(counts_all, 0, align)
    assert list(tot) == [Tg, Tg] and off[El] == 2 * (-(-Tg // align) * align)
    assert off[El] <= Tg * min(k, El) + El * (align - 1)
    for o in range(1, world):
        off_o, tot_o, _ = D.ep_plan(counts_all, o, align)
        assert off_o[El] == 0 and tot_o.sum() == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, S, h, F, E, k, align = 4, 8, 16, 24, 4, 2, 4
        Tg = B * S
        r = np.random.default_rng(5)
        x = r.standard_normal((Tg, h)).astype(np.float32)
        gate = r.standard_normal((h, E)).astype(np.float32)
        w1 = (r.standard_normal((E, h, F)) * 0.3).astype(np.float32)
        w3 = (r.standard_normal((E, h, F)) * 0.3).astype(np.float32)
        w2 = (r.standard_normal((E, F, h)) * 0.3).astype(np.float32)
        off0, Tl = D.shard(rank, world, B, S)
        El = E // world
        xs = x[off0:off0 + Tl]
        idx, w, _ = O.route(xs, gate, k)  # row-local: the same as routing the global batch
        # counts of every rank
        cnt = torch.as_tensor(np.bincount(idx.reshape(-1), minlength=E), dtype=torch.int64)
        allc = [torch.empty_like(cnt) for _ in range(world)]
        dist.all_gather(allc, cnt)
        counts_all = torch.stack(allc).numpy()
        dest = D.ep_dest_rows(idx, counts_all, rank, align)
        # dispatch: (row, global pair id, x row) to each owner
        owner = idx.reshape(-1) // El
        send = [[] for _ in range(world)]
        for i in range(Tl * k):
            send[owner[i]].append(np.concatenate([[dest[i], rank * Tl * k + i], xs[i // k]]))
        rec = _exchange(send, h + 2, world)
        plan_off, plan_tot, _ = D.ep_plan(counts_all, rank, align)
        xp = np.zeros((plan_off[El], h), np.float32)
        tag = -np.ones(plan_off[El], np.int64)
        for row in rec:
            xp[int(row[0])] = row[2:]
            tag[int(row[0])] = int(row[1])
        # the experts on their received rows (padding rows are zero rows)
        yp = np.zeros_like(xp)
        for j in range(El):
            e = rank * El + j
            a, b = plan_off[j], plan_off[j + 1]
            if b > a:
                yp[a:b] = O.swiglu(xp[a:b], w1[e], w3[e], w2[e])
        # combine: each received row goes back to its pair's rank
        back = [[] for _ in range(world)]
        for row in range(plan_off[El]):
            if tag[row] >= 0:
                s = int(tag[row]) // (Tl * k)
                back[s].append(np.concatenate([[int(tag[row]) - s * Tl * k], yp[row]]))
        got = _exchange(back, h + 1, world)
        ye = np.zeros((Tl * k, h), np.float32)
        for row in got:
            ye[int(row[0])] = row[1:]
        y = np.zeros((Tl, h), np.float32)
        for t in range(Tl):
            for j in range(k):
                y[t] += w[t, j] * ye[t * k + j]
        np.save(os.path.join(outdir, f"y{rank}.npy"), y)
        # the NCCL group id travels over the same host group
        obj = [D.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        np.save(os.path.join(outdir, f"id{rank}.npy"), np.frombuffer(obj[0], np.uint8))
    finally:
        dist.destroy_process_group()


def _exchange(send, width, world):
    """Uneven all-to-all of float64 rows over gloo."""
    import torch
    import torch.distributed as dist
    sizes = torch.tensor([len(s) for s in send], dtype=torch.int64)
    rsizes = torch.empty_like(sizes)
    dist.all_to_all_single(rsizes, sizes)
    flat = [np.asarray(s, np.float64).reshape(-1, width) for s in send]
    buf = torch.as_tensor(np.concatenate(flat) if sum(map(len, flat)) else np.zeros((0, width)))
    out = torch.empty(int(rsizes.sum()), width, dtype=torch.float64)
    dist.all_to_all_single(out, buf, output_split_sizes=rsizes.tolist(), input_split_sizes=sizes.tolist())
    return out.numpy()


def test_two_gloo_ranks_match_one_process_moe(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    B, S, h, F, E, k = 4, 8, 16, 24, 4, 2
    r = np.random.default_rng(5)
    x = r.standard_normal((B * S, h)).astype(np.float32)
    gate = r.standard_normal((h, E)).astype(np.float32)
    w1 = (r.standard_normal((E, h, F)) * 0.3).astype(np.float32)
    w3 = (r.standard_normal((E, h, F)) * 0.3).astype(np.float32)
    w2 = (r.standard_normal((E, F, h)) * 0.3).astype(np.float32)
    ref = O.moe(x, gate, w1, w3, w2, k)
    got = np.concatenate([np.load(tmp_path / f"y{q}.npy") for q in range(world)])
    assert np.array_equal(got, ref), np.abs(got - ref).max()
    ids = [np.load(tmp_path / f"id{q}.npy") for q in range(world)]
    assert ids[0].size == D.COMM_ID_BYTES and np.array_equal(ids[0], ids[1])
