"""Expert parallelism: the dispatch plan, the pair metadata, the return
order and the two all-to-all exchanges, on CPU with 2 gloo ranks.  The expert
arithmetic and the final sum are stand-ins passed to ep_forward (the CUDA
experts are tested on GPUs); what is checked here is that every (token, slot)
reaches the rank that owns its expert and comes back to exactly its place, so
the layer equals the same functions applied on one process — bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from titan_b200.expert_parallel import (_membership, balanced_placement, pairs_from_meta,
                                        plan_dispatch, return_addresses, return_slots,
                                        slot_experts)

H, E, K = 64, 8, 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _routing(T, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32) \
        if T else torch.zeros(0, K, dtype=torch.int32)
    sc = torch.rand(T, K, generator=g).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    return x, idx, sc


def _expert_mats():
    g = torch.Generator().manual_seed(1234)
    return torch.randn(E, H, H, generator=g) * 0.1


def _expert_out(mats, e, x):
    """Stand-in for expert e on one row: bf16(x @ M_e)."""
    return (x.float() @ mats[e]).to(torch.bfloat16)


def _combine(ys, inv, sc):
    """Stand-in for the block's weighted sum: fp32 in slot order, bf16 once."""
    T = sc.shape[0]
    out = torch.zeros(T, H)
    for t in range(T):
        for j in range(K):
            out[t] += sc[t, j].float() * ys[int(inv[t * K + j])].float()
    return out.to(torch.bfloat16)


def test_plan_dispatch_dedupes_per_destination():
    x, idx, sc = _routing(9, seed=3)
    world, epr = 4, E // 4
    plan = plan_dispatch(idx, epr, world)
    dest = idx.long() // epr
    want = [(t, d) for d in range(world) for t in range(9) if (dest[t] == d).any()]
    got = list(zip(plan.send_token.tolist(),
                   np.repeat(np.arange(world), plan.send_counts.tolist()).tolist()))
    assert got == want
    for r, (t, d) in enumerate(want):
        for j in range(K):
            e = int(idx[t, j])
            assert int(plan.local_ids[r, j]) == (e - d * epr if e // epr == d else -1)


def test_pairs_and_return_slots():
    ids = torch.tensor([[1, -1, 0], [-1, 2, -1], [2, 3, -1]], dtype=torch.int32)
    pr, pe = pairs_from_meta(ids)
    assert pr.tolist() == [0, 0, 1, 2, 2]
    assert pe.tolist() == [1, 0, 2, 2, 3]
    x, idx, sc = _routing(6, seed=5)
    plan = plan_dispatch(idx, E // 2, 2)
    inv = return_slots(plan, 6, K)
    assert sorted(inv.tolist()) == list(range(6 * K))   # every slot exactly once


@pytest.mark.parametrize("world", [2, 4])
def test_peer_exchange_host_plan(world):
    """The host side of the peer-memory transport: destination rows (pos,
    counts) as peer_forward computes them, the metadata rows a dispatch
    writes (simulated here), and the owner's slot list and return addresses
    read back from a buffer whose unwritten rows hold stale ids.  Every
    (source, token, slot) must be served once, by the owner of its expert,
    and be returned to ret row token*k + slot of its source."""
    epr, cap = E // world, 9
    tokens = [9, 0, 4, 7][:world]
    g = torch.Generator().manual_seed(77)
    meta = [torch.randint(-1, epr, (world, cap, K + 1), generator=g, dtype=torch.int32)
            for _ in range(world)]                  # stale rows from an earlier layer
    rows_in = [torch.zeros(world, dtype=torch.int32) for _ in range(world)]
    idxs = []
    for s in range(world):
        _, idx, _ = _routing(tokens[s], seed=40 + s)
        idxs.append(idx)
        dest, member = _membership(idx, epr, world)
        pos = (torch.cumsum(member.to(torch.int32), 0, dtype=torch.int32) - 1).t().contiguous()
        counts = member.sum(0, dtype=torch.int32)
        for t in range(tokens[s]):
            for d in range(world):
                if not member[t, d]:
                    continue
                r = int(pos[d, t])
                assert 0 <= r < int(counts[d])
                for j in range(K):
                    e = int(idx[t, j])
                    meta[d][s, r, j] = e - d * epr if e // epr == d else -1
                meta[d][s, r, K] = t
        for d in range(world):
            rows_in[d][s] = counts[d]
    served = {}
    H_, ret_off = 32, 4096
    peers = torch.tensor([(s + 1) << 40 for s in range(world)], dtype=torch.int64)
    for d in range(world):
        se = slot_experts(meta[d], rows_in[d], epr)
        addr = return_addresses(meta[d], se, peers, ret_off, H_)
        assert bool((addr[se < 0] == 0).all())
        assert se.dtype == torch.int32 and se.shape == (world * cap * K,)
        for f in torch.nonzero(se >= 0).flatten().tolist():
            s, i, slot = f // (cap * K), (f // K) % cap, f % K
            t = int(meta[d][s, i, K])
            assert int(idxs[s][t, slot]) == d * epr + int(se[f])
            off = int(addr[f]) - int(peers[s]) - ret_off
            assert off % (2 * H_) == 0 and off // (2 * H_) == t * K + slot
            key = (s, t * K + slot)
            assert key not in served
            served[key] = d
    assert sorted(served) == [(s, i) for s in range(world) for i in range(tokens[s] * K)]


def test_balanced_placement():
    world, E = 4, 16
    load = [100, 90, 1, 1, 80, 2, 3, 70, 1, 1, 60, 5, 1, 50, 1, 4]
    perm = balanced_placement(load, world)
    assert sorted(perm) == list(range(E))
    per_rank = [sum(load[e] for e in perm[r * 4:(r + 1) * 4]) for r in range(world)]
    contiguous = [sum(load[r * 4:(r + 1) * 4]) for r in range(world)]
    assert max(per_rank) - min(per_rank) <= max(load)
    assert max(per_rank) < max(contiguous)
    with pytest.raises(ValueError):
        balanced_placement(load[:15], world)


def _worker(rank, world, port, tokens, q, placed=False):
    import torch.distributed as dist
    from titan_b200.expert_parallel import ep_forward
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        epr = E // world
        mats = _expert_mats()
        x, idx, sc = _routing(tokens[rank], seed=100 + rank)

        # with a placement, rank r holds experts perm[r*epr:(r+1)*epr] and the
        # ids travel as places (as ExpertParallelMoE maps them)
        perm = balanced_placement(list(range(E, 0, -1)), world) if placed else list(range(E))
        place = torch.empty(E, dtype=torch.int32)
        place[torch.tensor(perm)] = torch.arange(E, dtype=torch.int32)

        def expert_fn(rows, pair_row, pair_exp):
            out = torch.empty(pair_row.numel(), H, dtype=torch.bfloat16)
            for p in range(pair_row.numel()):
                e = perm[rank * epr + int(pair_exp[p])]
                out[p] = _expert_out(mats, e, rows[int(pair_row[p]):int(pair_row[p]) + 1])[0]
            return out

        for _ in range(2):                       # two layers in a row on one group
            y = ep_forward(x, place[idx.long()], epr, expert_fn,
                           lambda ys, inv: _combine(ys, inv, sc))
        T = x.shape[0]
        ys_full = torch.empty(T * K, H, dtype=torch.bfloat16)
        for t in range(T):
            for j in range(K):
                ys_full[t * K + j] = _expert_out(mats, int(idx[t, j]), x[t:t + 1])[0]
        ref = _combine(ys_full, torch.arange(T * K), sc)
        q.put((rank, bool(torch.equal(y, ref)), tuple(y.shape)))
    except Exception as exc:                     # report instead of hanging the peer
        q.put((rank, repr(exc), None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,placed", [((7, 5), False), ((6, 0), False), ((7, 5), True)],
                         ids=["both", "one_rank_empty", "placed"])
def test_ep_forward_two_gloo_ranks(tokens, placed):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tokens, q, placed))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, shape in sorted(results):
        assert ok is True, f"rank {rank}: {ok}"
        assert shape == (tokens[rank], H)


def _skipping_worker(rank, world, port, q):
    """Rank 1 leaves before the layer's exchange (its post never comes); rank
    0 must get an error from its exchange within the process group's short
    timeout, not hang and not return a result."""
    import datetime
    import time

    import torch.distributed as dist
    from titan_b200.expert_parallel import ep_forward
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    try:
        epr = E // world
        mats = _expert_mats()
        x, idx, sc = _routing(6, seed=300 + rank)
        if rank == 1:
            time.sleep(8)                          # never joins the exchange
            q.put((rank, "skipped"))
            return

        def expert_fn(rows, pair_row, pair_exp):
            out = torch.empty(pair_row.numel(), H, dtype=torch.bfloat16)
            for p in range(pair_row.numel()):
                out[p] = _expert_out(mats, rank * epr + int(pair_exp[p]),
                                     rows[int(pair_row[p]):int(pair_row[p]) + 1])[0]
            return out

        t0 = time.monotonic()
        try:
            ep_forward(x, idx, epr, expert_fn, lambda ys, inv: _combine(ys, inv, sc))
            q.put((rank, "returned a result"))
        except Exception as exc:                   # the expected outcome
            q.put((rank, f"raised after {time.monotonic() - t0:.1f}s: {type(exc).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_ep_forward_peer_that_never_posts_raises():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_skipping_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1] == "skipped"
    assert results[0].startswith("raised"), results[0]
