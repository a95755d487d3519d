"""Expert parallelism on GPUs: the token-local part (router, top-k, shared
expert: tmoe_moe_local), the routed experts of a rank on received rows
(tmoe_moe_experts, or tmoe_moe_experts_slots storing into the sources'
buffers), both transports (NCCL exchanges; peer-memory dispatch, slot list,
flags and bounded waits) and the block's weighted sum (tmoe_moe_combine),
through ExpertParallelMoE, with and without an expert placement.  The layer
must equal the single-GPU block bit for bit on the int8 path, with and
without a shared expert, and stay within the north-star tolerance of the
oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from gpu_util import bf, load_block, nbf
from helpers import assert_bf16_close, f32, rel_rms

pytestmark = pytest.mark.gpu

SHAPE = dict(H=1024, E=32, k=8, I=256, Is=512)
SHAPE0 = dict(SHAPE, Is=0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _opts(min_tokens):
    from titan_b200 import _lib
    o = _lib.Options()
    o.min_tokens, o.int8_prefill, o.down_int8, o.wsum_mode, o.gemm_kernel = min_tokens, 1, 1, 0, 0
    return o


def _compare(oracle, L, x, y_ep):
    ry, _, _, ops = oracle.moe_prefill(L, x, int8_mode=3, parts=True)
    assert_bf16_close(y_ep, ry, what="EP vs oracle block", operands=ops, operand_ulps=4)
    assert rel_rms(f32(y_ep), f32(ry)) < 0.01


def _blocks(oracle, device, shape, seed):
    from titan_b200 import SparseMoeBlock
    L = oracle.make_layer(seed=seed, **shape)
    blk = SparseMoeBlock(shape["H"], shape["E"], shape["k"], shape["I"], shape["Is"], device=device,
                         init=False)
    load_block(blk, L)
    return L, blk


def test_ep_single_rank_matches_block(cuda, oracle):
    import torch.distributed as dist
    from titan_b200.expert_parallel import ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1)
    try:
        L0, blk0 = _blocks(oracle, cuda, SHAPE0, 33)
        ep0 = ExpertParallelMoE(blk0)
        L, blk = _blocks(oracle, cuda, SHAPE, 31)
        ep = ExpertParallelMoE(blk)
        for T in (150, 7):
            x = oracle.make_x(T, SHAPE["H"], seed=T)
            y0 = ep0(bf(x), options=_opts(1))
            assert torch.equal(y0.view(torch.int16), blk0(bf(x), options=_opts(1)).view(torch.int16))
            y = ep(bf(x), options=_opts(1))
            assert torch.equal(y.view(torch.int16), blk(bf(x), options=_opts(1)).view(torch.int16))
            torch.cuda.synchronize()
            _compare(oracle, L, x, nbf(y))
    finally:
        dist.destroy_process_group()


def test_ep_peer_single_rank_matches_block(cuda, oracle):
    """The peer-memory transport on one rank: the dispatch and return
    kernels write through the rank's own buffer and the flags; two layers
    share one exchange and run in turn, with calls of different sizes and an
    empty call; every output bit-identical to the single-GPU block."""
    import torch.distributed as dist
    from titan_b200.expert_parallel import ExpertParallelMoE, PeerExchange
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1)
    try:
        ex = PeerExchange(160, SHAPE["H"], SHAPE["k"])
        L0, blk0 = _blocks(oracle, cuda, SHAPE0, 33)
        L, blk = _blocks(oracle, cuda, SHAPE, 31)
        eps = (ExpertParallelMoE(blk0, exchange=ex), ExpertParallelMoE(blk, exchange=ex))
        for T in (150, 7, 160, 1, 150):
            x = oracle.make_x(T, SHAPE["H"], seed=T)
            for ep, b in zip(eps, (blk0, blk)):
                y = ep(bf(x), options=_opts(1))
                yb = b(bf(x), options=_opts(1))
                assert torch.equal(y.view(torch.int16), yb.view(torch.int16)), T
        y = eps[1](bf(oracle.make_x(0, SHAPE["H"], seed=1)), options=_opts(1))
        assert y.shape == (0, SHAPE["H"])
        # a placement permutes the experts (here reversed) without changing a bit
        placed = ExpertParallelMoE(blk, exchange=ex, placement=list(range(SHAPE["E"]))[::-1])
        for T in (150, 3):
            x = oracle.make_x(T, SHAPE["H"], seed=40 + T)
            y = placed(bf(x), options=_opts(1))
            assert torch.equal(y.view(torch.int16), blk(bf(x), options=_opts(1)).view(torch.int16))
        x = oracle.make_x(150, SHAPE["H"], seed=5)
        y = ExpertParallelMoE(blk, exchange=ex)(bf(x), options=_opts(1))
        torch.cuda.synchronize()
        _compare(oracle, L, x, nbf(y))
        ex.check()
        ex.close()
    finally:
        dist.destroy_process_group()


def test_ep_slots_kernel_matches_tensor_statement(cuda):
    """tmoe_ep_slots against its tensor statement (slot_experts,
    return_addresses) on a 3-source buffer holding random metadata: rows past
    each source's count, negative ids and ids of other ranks must come out as
    -1 with a NULL address, and a source whose wait gave up (-1) as no rows."""
    import ctypes as C
    from titan_b200 import _lib
    from titan_b200.expert_parallel import _view, return_addresses, slot_experts
    lib = _lib.load()
    W, cap, k, H, epr = 3, 37, 5, 256, 6
    offs = (C.c_size_t * 4)()
    nb = lib.tmoe_ep_buffer_bytes(W, cap, H, k, cap, offs)
    ptr = C.c_void_p()
    _lib.check(lib.tmoe_ep_alloc(nb, C.byref(ptr)))
    try:
        meta = _view(ptr.value + offs[1], (W, cap, k + 1), torch.int32, cuda)
        g = torch.Generator(device=cuda).manual_seed(3)
        meta[..., :k] = torch.randint(-2, epr + 3, (W, cap, k), generator=g, device=cuda,
                                      dtype=torch.int32)
        meta[..., k] = torch.randint(0, cap, (W, cap), generator=g, device=cuda, dtype=torch.int32)
        peers = torch.tensor([ptr.value + (s << 30) for s in range(W)], dtype=torch.int64,
                             device=cuda)
        for rows in ([cap, 0, 11], [5, -1, cap]):
            rows_in = torch.tensor(rows, dtype=torch.int32, device=cuda)
            se = torch.full((W * cap * k,), 99, dtype=torch.int32, device=cuda)
            yr = torch.full((W * cap * k,), 99, dtype=torch.int64, device=cuda)
            _lib.check(lib.tmoe_ep_slots(ptr, offs, rows_in.data_ptr(), W, cap, k, epr, H,
                                         peers.data_ptr(), se.data_ptr(), yr.data_ptr(), None))
            want = slot_experts(meta, rows_in, epr)
            assert torch.equal(se, want)
            assert torch.equal(yr, return_addresses(meta, want, peers, int(offs[2]), H))
            assert int((want >= 0).sum()) > 0
    finally:
        torch.cuda.synchronize()
        _lib.check(lib.tmoe_ep_free(ptr))


def _timeout_child(q):
    import ctypes as C
    try:
        from titan_b200 import _lib
        lib = _lib.load()
        torch.cuda.set_device(0)
        world, offs = 2, (C.c_size_t * 4)()
        nb = lib.tmoe_ep_buffer_bytes(world, 8, 1024, 8, 8, offs)
        ptr = C.c_void_p()
        _lib.check(lib.tmoe_ep_alloc(nb, C.byref(ptr)))
        counts = torch.full((world,), 7, dtype=torch.int32, device="cuda")
        # epoch 5: nothing ever posts it, so both waits must give up
        _lib.check(lib.tmoe_ep_wait(ptr, offs, 0, world, 5, counts.data_ptr(), None))
        torch.cuda.synchronize()
        got = counts.tolist()
        # an owner whose dispatch wait gave up passes count -1 on with its
        # return post; the source's wait reads it and the guard NaN-fills y
        peers = torch.tensor([ptr.value], dtype=torch.int64, device="cuda")
        rows_in = torch.tensor([-1], dtype=torch.int32, device="cuda")
        _lib.check(lib.tmoe_ep_post_return(rows_in.data_ptr(), 1, 0, peers.data_ptr(), offs, 6,
                                           None))
        ret = torch.full((1,), 7, dtype=torch.int32, device="cuda")
        _lib.check(lib.tmoe_ep_wait(ptr, offs, 1, 1, 6, ret.data_ptr(), None))
        y = torch.ones(4, 1024, dtype=torch.bfloat16, device="cuda")
        _lib.check(lib.tmoe_ep_guard(ret.data_ptr(), 1, y.data_ptr(), y.numel(), None))
        ok = torch.zeros(1, dtype=torch.int32, device="cuda")
        y2 = torch.ones(4, 1024, dtype=torch.bfloat16, device="cuda")
        _lib.check(lib.tmoe_ep_guard(ok.data_ptr(), 1, y2.data_ptr(), y2.numel(), None))
        torch.cuda.synchronize()
        got = (got, ret.tolist(), bool(torch.isnan(y).all()), bool((y2 == 1).all()))
        status = int(lib.tmoe_device_status())
        _lib.check(lib.tmoe_ep_free(ptr))
        q.put((got, status, None))
    except Exception as exc:
        q.put((None, None, repr(exc)))


def test_ep_wait_gives_up_and_reports(cuda):
    """A flag that nothing sets: the wait kernel gives up after its bounded
    time, writes count -1, the context stays usable, and tmoe_device_status
    reports TMOE_ERR_TIMEOUT (5).  A failed dispatch wait is carried into the
    return (tmoe_ep_post_return posts -1) and the source's guard turns the
    layer output into NaN.  In a child process: the error is sticky
    for the life of the library."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_timeout_child, args=(q,))
    p.start()
    got, status, err = q.get(timeout=300)
    p.join(timeout=60)
    assert err is None, err
    counts, ret, y_nan, y_kept = got
    assert counts == [-1, -1]
    assert ret == [-1], "a poisoned return post must read as count -1"
    assert y_nan, "the guard must NaN-fill the output of a failed layer"
    assert y_kept, "the guard must leave a valid layer's output alone"
    assert status == 5


def _worker(rank, world, port, layer_arrays, T, q):
    import torch.distributed as dist
    sys_path = os.path.dirname(os.path.abspath(__file__))
    import sys
    sys.path.insert(0, sys_path)
    sys.path.insert(0, os.path.dirname(sys_path))
    from gpu_util import bf, load_block, nbf
    from oracle import oracle
    from titan_b200 import SparseMoeBlock
    from titan_b200.expert_parallel import ExpertParallelMoE, PeerExchange
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        dev = torch.device("cuda", rank)
        x = oracle.make_x(T, SHAPE["H"], seed=500 + rank)
        out = {}
        ex = PeerExchange(128, SHAPE["H"], SHAPE["k"]) if layer_arrays == "peer" else None
        refs = []
        for shape, seed, tag in ((SHAPE0, 33, "plain"), (SHAPE, 31, "shared")):
            L = oracle.make_layer(seed=seed, **shape)
            blk = SparseMoeBlock(shape["H"], shape["E"], shape["k"], shape["I"], shape["Is"],
                                 device=dev, init=False)
            load_block(blk, L)
            yb = nbf(blk(bf(x, dev=dev), options=_opts(1)))
            ry, _, _, ops = oracle.moe_prefill(L, x, int8_mode=3, parts=True)
            refs.append((tag, blk, yb, ry, ops))
        # the oracle's CPU time differs between ranks: line the ranks up
        # before the first exchange so no device wait runs long
        dist.barrier()
        for tag, blk, yb, ry, ops in refs:
            if ex is None:
                ep = ExpertParallelMoE(blk)
                y = nbf(ep(bf(x, dev=dev), options=_opts(1)))
                out[tag] = (y, yb, ry, ops)
                continue
            ep = ExpertParallelMoE(blk, exchange=ex)
            for i in range(3):                         # the exchange reused call after call
                y = nbf(ep(bf(x, dev=dev), options=_opts(1)))
                out[f"{tag}_{i}"] = (y, yb, ry, ops)
            # experts interleaved over the ranks by a placement
            E = shape["E"]
            ep = ExpertParallelMoE(blk, exchange=ex,
                                   placement=[e for r in range(world) for e in range(r, E, world)])
            out[f"{tag}_placed"] = (nbf(ep(bf(x, dev=dev), options=_opts(1))), yb, ry, ops)
        if ex is not None:
            from titan_b200 import _lib
            out["status"] = int(_lib.load().tmoe_device_status())
            ex.close()
        q.put((rank, out, None, None))
    except Exception as exc:
        q.put((rank, repr(exc), None, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_nccl(oracle):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, None, (120, 40)[r], q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, out, _, _ in sorted(res, key=lambda r: r[0]):
        assert not isinstance(out, str), f"rank {rank}: {out}"
        y, yb, _, _ = out["plain"]
        assert np.array_equal(y, yb), f"rank {rank}: EP differs from the single-GPU block"
        y, yb, ry, ops = out["shared"]
        assert np.array_equal(y, yb), f"rank {rank}: EP with a shared expert differs from the block"
        assert_bf16_close(y, ry, what=f"EP rank {rank}", operands=ops, operand_ulps=4)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_peer_memory(oracle):
    """The peer-memory transport over two GPUs (CUDA IPC mappings, NVLink
    stores, epoch flags): bit-identical to the single-GPU block on each
    rank's tokens, calls in a row, ranks with unequal tokens."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, "peer", (120, 40)[r], q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, out, _, _ in sorted(res, key=lambda r: r[0]):
        assert not isinstance(out, str), f"rank {rank}: {out}"
        assert out.pop("status") == 0, f"rank {rank}: a device wait timed out"
        for tag, (y, yb, ry, ops) in out.items():
            assert np.array_equal(y, yb), f"rank {rank} {tag}: peer EP differs from the block"
            assert_bf16_close(y, ry, what=f"peer EP rank {rank} {tag}", operands=ops,
                              operand_ulps=4)
