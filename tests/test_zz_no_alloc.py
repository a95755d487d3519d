"""tmoe_gather_qmm_int8_static (the entry point that allocates nothing) against
tmoe_gather_qmm_int8 (caller-supplied workspace), both called through the C
ABI on the same inputs, twice in a row.  The file name sorts last so the test
also runs after every other GPU test of the session."""
import ctypes as C

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close

pytestmark = pytest.mark.gpu


def _inputs(R, E, N, K, seed, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(R, K, generator=g) * 1.5).to(torch.bfloat16).to(dev)
    w = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, N, K // 8), generator=g, dtype=torch.int64)
    w = w.to(torch.int32).to(dev)
    s = (torch.rand(E, N, K // 64, generator=g) * 0.01 + 1e-3).to(torch.bfloat16).to(dev)
    b = (-8 * s.float() + torch.randn(E, N, K // 64, generator=g).to(dev) * 1e-3).to(torch.bfloat16)
    ids = torch.sort(torch.randint(0, E, (R,), generator=g, dtype=torch.int32)).values.to(dev)
    return x, w, s, b, ids


def _bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("R,E,N,K", [(1000, 64, 512, 1024),     # single-CTA routing plan
                                     (3000, 32, 256, 2048)])    # multi-CTA routing plan
def test_static_scratch_gather_matches_workspace_gather(cuda, R, E, N, K):
    from titan_b200 import _lib, ops
    lib = _lib.load()
    x, w, s, b, ids = _inputs(R, E, N, K, seed=R, dev=cuda)
    st, bt = ops.prepare_tables(s, b)
    need = lib.tmoe_gather_qmm_int8_workspace_size(R, E, N, K)
    assert need <= lib.tmoe_static_scratch_bytes()
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    ref = torch.empty(R, N, dtype=torch.bfloat16, device=cuda)
    _lib.check(lib.tmoe_gather_qmm_int8(x.data_ptr(), w.data_ptr(), st.data_ptr(), bt.data_ptr(),
                                        ids.data_ptr(), R, E, N, K, ws.data_ptr(), need,
                                        ref.data_ptr(), stream), "tmoe_gather_qmm_int8")
    refb = _bits(ref)
    for call in range(2):
        y = torch.full((R, N), float("nan"), dtype=torch.bfloat16, device=cuda)
        _lib.check(lib.tmoe_gather_qmm_int8_static(x.data_ptr(), w.data_ptr(), st.data_ptr(),
                                                   bt.data_ptr(), ids.data_ptr(), R, E, N, K,
                                                   y.data_ptr(), stream),
                   "tmoe_gather_qmm_int8_static")
        torch.cuda.synchronize(cuda)
        got = _bits(y)
        assert np.isfinite((got.astype(np.uint32) << 16).view(np.float32)).all()
        # same kernels on the same inputs: identical, which is inside the
        # parity bar of the int8 gather (1 bf16 ULP of the reference order)
        assert_bf16_close(got, refb, ulps=1, rel=0, what=f"static scratch, call {call}")
        assert np.array_equal(got, refb), f"call {call}"


def test_static_scratch_rejects_oversized_calls(cuda):
    from titan_b200 import _lib
    lib = _lib.load()
    R, E, N, K = 20000, 64, 512, 2048
    assert lib.tmoe_gather_qmm_int8_workspace_size(R, E, N, K) > lib.tmoe_static_scratch_bytes()
    rc = lib.tmoe_gather_qmm_int8_static(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16),
                                         C.c_void_p(16), C.c_void_p(16), R, E, N, K,
                                         C.c_void_p(16), None)
    assert rc == 6
    assert "static scratch" in _lib.last_error()
