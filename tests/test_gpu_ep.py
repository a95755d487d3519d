"""Expert parallelism on GPUs: the token-local part (router, top-k, shared
expert: tmoe_moe_local), the routed experts of a rank on received rows
(tmoe_moe_experts), the NCCL exchanges and the block's weighted sum
(tmoe_moe_combine), through ExpertParallelMoE.  The layer must equal the
single-GPU block bit for bit on the int8 path, with and without a shared
expert, and stay within the north-star tolerance of the oracle."""
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


def _worker(rank, world, port, layer_arrays, T, q):
    import torch.distributed as dist
    sys_path = os.path.dirname(os.path.abspath(__file__))
    import sys
    sys.path.insert(0, sys_path)
    sys.path.insert(0, os.path.dirname(sys_path))
    from gpu_util import bf, load_block, nbf
    from oracle import oracle
    from titan_b200 import SparseMoeBlock
    from titan_b200.expert_parallel import ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        dev = torch.device("cuda", rank)
        x = oracle.make_x(T, SHAPE["H"], seed=500 + rank)
        out = {}
        for shape, seed, tag in ((SHAPE0, 33, "plain"), (SHAPE, 31, "shared")):
            L = oracle.make_layer(seed=seed, **shape)
            blk = SparseMoeBlock(shape["H"], shape["E"], shape["k"], shape["I"], shape["Is"],
                                 device=dev, init=False)
            load_block(blk, L)
            ep = ExpertParallelMoE(blk)
            y = nbf(ep(bf(x, dev=dev), options=_opts(1)))
            yb = nbf(blk(bf(x, dev=dev), options=_opts(1)))
            ry, _, _, ops = oracle.moe_prefill(L, x, int8_mode=3, parts=True)
            out[tag] = (y, yb, ry, ops)
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
