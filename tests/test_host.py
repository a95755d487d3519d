"""Host-side logic, no GPU: the C ABI loads and exports every declared
symbol, argument validation returns typed errors before any launch, the
workspace queries are consistent, and the overlay installs / uninstalls the
way engine/patches/moe-int8/patch.py:140-168 does."""
import ctypes as C
import os
import re
import weakref

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "titan_moe.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tmoe_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(built_lib):
    lib = C.CDLL(built_lib.LIB_PATH)
    names = _declared_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding types every declared entry point
    assert set(names) == set(built_lib.EXPORTED)


def test_abi_version(built_lib):
    assert built_lib.load().tmoe_abi_version() == built_lib.ABI_VERSION


def test_invalid_arguments_are_reported_before_launch(built_lib):
    lib = built_lib.load()
    rc = lib.tmoe_route_sort(None, 10, 8, None, 0, None, None, None, None, None, None, 0, None)
    assert rc == 1 and "bad arguments" in built_lib.last_error()
    fake = C.c_void_p(16)
    # N not a multiple of 128 -> unsupported, no device access
    rc = lib.tmoe_gather_qmm_int8(fake, fake, fake, fake, fake, 4, 2, 100, 256, fake, 1 << 30,
                                  fake, None)
    assert rc == 2 and "N % 128" in built_lib.last_error()
    # workspace too small -> workspace error
    rc = lib.tmoe_gather_qmm_int8(fake, fake, fake, fake, fake, 4, 2, 128, 256, fake, 1, fake, None)
    assert rc == 6
    with pytest.raises(built_lib.WorkspaceError):
        built_lib.check(rc, "x")
    # router limits
    rc = lib.tmoe_router_topk(fake, fake, 1, 100, 8, 2, fake, fake, fake, None, None)
    assert rc == 2


def test_workspace_queries_are_host_only_and_monotone(built_lib):
    lib = built_lib.load()
    a = lib.tmoe_gather_qmm_int8_workspace_size(1000, 64, 1024, 2048)
    b = lib.tmoe_gather_qmm_int8_workspace_size(4000, 64, 1024, 2048)
    assert 0 < a < b
    L = built_lib.Layer()
    L.hidden, L.num_experts, L.top_k, L.moe_inter, L.shared_inter = 2048, 512, 10, 512, 512
    o = built_lib.Options()
    o.min_tokens, o.down_int8, o.int8_prefill = 512, 1, 1
    dec = lib.tmoe_moe_workspace_size(C.byref(L), 8, C.byref(o))
    pre = lib.tmoe_moe_workspace_size(C.byref(L), 4096, C.byref(o))
    assert 0 < dec < pre
    assert lib.tmoe_route_workspace_size(100, 512) == 0       # one-CTA plan
    assert lib.tmoe_route_workspace_size(100000, 512) > 0


def test_forward_rejects_missing_tables_for_int8(built_lib):
    lib = built_lib.load()
    L = built_lib.Layer()
    L.hidden, L.num_experts, L.top_k, L.moe_inter = 2048, 64, 4, 512
    for n in ("router_w", "gate_up_w", "gate_up_s", "gate_up_b", "down_w", "down_s", "down_b"):
        setattr(L, n, 256)
    o = built_lib.Options()
    o.min_tokens, o.int8_prefill, o.down_int8 = 16, 1, 1
    rc = lib.tmoe_moe_forward(C.byref(L), 256, 64, C.byref(o), 256, 1 << 40, 256, None, None, None)
    assert rc == 1 and "prepared tables" in built_lib.last_error()


def test_ops_refuse_cpu_tensors():
    from titan_b200 import InvalidArgument, ops
    x = torch.zeros(4, 1, 256, dtype=torch.bfloat16)
    w = torch.zeros(2, 128, 32, dtype=torch.int32)
    s = torch.zeros(2, 128, 4, dtype=torch.bfloat16)
    with pytest.raises(InvalidArgument):
        ops.gather_qmm(x, w, s, s, rhs_indices=torch.zeros(4, dtype=torch.int32))
    with pytest.raises(NotImplementedError):
        ops.gather_qmm(x, w, s, s, rhs_indices=torch.zeros(4, dtype=torch.int32), bits=8)


def test_supported_int8_predicate():
    from titan_b200 import ops
    x = torch.zeros(4096, 1, 2048, dtype=torch.bfloat16)
    w = torch.zeros(64, 1024, 256, dtype=torch.int32)
    s = torch.zeros(64, 1024, 32, dtype=torch.bfloat16)
    idx = torch.zeros(4096, dtype=torch.int32)
    assert ops.supported_int8(x, w, s, s, idx)
    assert not ops.supported_int8(x.float(), w, s, s, idx)
    assert not ops.supported_int8(x, w, s, s, idx, group_size=128)
    assert not ops.supported_int8(x, w, s[:, :100], s, idx)


def test_patch_install_is_idempotent_and_reversible():
    from titan_b200 import ops, patch
    from titan_b200.switch_layers import SwitchGLU
    orig_op, orig_fwd = ops.gather_qmm, SwitchGLU.forward
    try:
        assert patch.install(enabled=True, min_tokens=256) is True
        assert patch.install() is False               # marker makes it idempotent
        assert ops.gather_qmm is not orig_op and getattr(ops.gather_qmm, "_titan_moe_int8")
        assert SwitchGLU.forward is not orig_fwd
        o = patch.block_options()
        assert (o.int8_prefill, o.down_int8, o.min_tokens) == (1, 1, 256)
    finally:
        patch.uninstall()
    assert ops.gather_qmm is orig_op and SwitchGLU.forward is orig_fwd
    o = patch.block_options()
    assert o.int8_prefill == 0 and o.down_int8 == 0


def test_should_route_predicate_follows_reference(monkeypatch):
    """patch.py:78-102: sorted only, token floor, skip_down rule."""
    from titan_b200 import patch
    x = torch.zeros(8192, 1, 2048, dtype=torch.bfloat16)
    w = torch.zeros(64, 1024, 256, dtype=torch.int32)
    s = torch.zeros(64, 1024, 32, dtype=torch.bfloat16)
    idx = torch.zeros(8192, dtype=torch.int32)
    kw = dict(rhs_indices=idx, sorted_indices=True)
    try:
        patch.install(enabled=True, min_tokens=512, min_rows=4096)
        assert patch._should_route(x, w, (s, s), kw)
        assert not patch._should_route(x, w, (s, s), dict(kw, sorted_indices=False))
        patch._ctx["tokens"] = 100                    # a 100-token chunk is below the floor
        assert not patch._should_route(x, w, (s, s), kw)
        patch._ctx["tokens"] = None
        assert not patch._should_route(x[:1000], w, (s, s), dict(kw, rhs_indices=idx[:1000]))
        patch.install(enabled=True, skip_down=True)
        xd = torch.zeros(8192, 1, 512, dtype=torch.bfloat16)
        assert not patch._should_route(xd, w[:, :, :64], (s[:, :, :8], s[:, :, :8]), kw)
        patch.install(enabled=False)
        assert not patch._should_route(x, w, (s, s), kw)
    finally:
        patch._ctx["tokens"] = None
        patch.uninstall()


def test_env_configuration(monkeypatch):
    from titan_b200 import patch
    monkeypatch.setenv("OMLX_MOE_INT8_PREFILL", "1")
    monkeypatch.setenv("OMLX_MOE_INT8_MIN_TOKENS", "1024")
    monkeypatch.setenv("OMLX_MOE_INT8_SKIP_DOWN", "1")
    try:
        patch.install(enabled=None)
        o = patch.block_options()
        assert (o.int8_prefill, o.min_tokens, o.down_int8) == (1, 1024, 0)
    finally:
        patch.uninstall()


def test_table_cache_never_serves_another_tensors_tables(monkeypatch):
    """The per-weight table cache is keyed by id(); an id reused by a new
    tensor (after the old one was freed) must not return the old tables."""
    from titan_b200 import ops
    built = []
    monkeypatch.setattr(ops, "build_tables", lambda w, s, b: built.append(w) or ops.Int8Tables(s, b, s[..., 0].float()))
    ops.clear_tables()
    try:
        w1 = torch.zeros(2, 128, 8, dtype=torch.int32)
        s1 = torch.zeros(2, 128, 1, dtype=torch.bfloat16)
        b1 = torch.zeros_like(s1)
        t1 = ops.cached_tables(w1, s1, b1)
        assert ops.cached_tables(w1, s1, b1) is t1 and len(built) == 1
        s1.add_(1)                                   # in-place update of the scales
        assert ops.cached_tables(w1, s1, b1) is not t1 and len(built) == 2
        # forge the id collision: a stale entry under the new tensor's key
        w2 = torch.zeros(2, 128, 8, dtype=torch.int32)
        s2 = torch.zeros(2, 128, 1, dtype=torch.bfloat16)
        b2 = torch.zeros_like(s2)
        key = (id(w2), tuple(w2.shape), s2.data_ptr())
        ops._TABLES[key] = ((s2._version, b2._version), t1, weakref.ref(w1), weakref.ref(s1))
        t2 = ops.cached_tables(w2, s2, b2)
        assert t2 is not t1 and built[-1] is w2
    finally:
        ops.clear_tables()
