"""Checkpoint loader: the plan over a synthetic MLX-layout checkpoint (CPU),
and a loaded block against the oracle (GPU).  The reference's plan test
(tests/model/test_loader_plan.py) asserts every checkpoint tensor is covered
exactly once; the same property is checked here for the MoE block's plan."""
import json
import os

import numpy as np
import pytest

from titan_b200 import _lib
from titan_b200 import loader as LD

H, E, K, I, IS = 128, 8, 2, 64, 128


def _checkpoint(tmp, oracle, layers=2, quant=None, drop_up=False):
    rng = np.random.default_rng(3)
    tensors, dtypes, keep = {}, {}, {}

    def put(name, arr, dt):
        tensors[name] = arr
        dtypes[name] = dt

    put("language_model.model.embed_tokens.weight",
        oracle.f32_to_bf16(rng.standard_normal((32, H), dtype=np.float32)), "BF16")
    for l in range(layers):
        L = oracle.make_layer(H=H, E=E, k=K, I=I, Is=IS, seed=10 + l)
        keep[l] = L
        p = f"language_model.model.layers.{l}."
        put(p + "self_attn.q_proj.weight",
            oracle.f32_to_bf16(rng.standard_normal((H, H), dtype=np.float32)), "BF16")
        put(p + "mlp.gate.weight", L.wr, "BF16")
        for q, a in (("weight", (L.gu_w, "U32")), ("scales", (L.gu_s, "BF16")),
                     ("biases", (L.gu_b, "BF16"))):
            arr, dt = a
            put(p + f"mlp.switch_mlp.gate_proj.{q}", arr[:, :I], dt)
            if not drop_up:
                put(p + f"mlp.switch_mlp.up_proj.{q}", arr[:, I:], dt)
        for q, a in (("weight", (L.dn_w, "U32")), ("scales", (L.dn_s, "BF16")),
                     ("biases", (L.dn_b, "BF16"))):
            put(p + f"mlp.switch_mlp.down_proj.{q}", a[0], a[1])
        for q, a in (("weight", (L.sgu_w[0], "U32")), ("scales", (L.sgu_s[0], "BF16")),
                     ("biases", (L.sgu_b[0], "BF16"))):
            put(p + f"mlp.shared_expert.gate_proj.{q}", a[0][:IS], a[1])
            put(p + f"mlp.shared_expert.up_proj.{q}", a[0][IS:], a[1])
        for q, a in (("weight", (L.sdn_w[0], "U32")), ("scales", (L.sdn_s[0], "BF16")),
                     ("biases", (L.sdn_b[0], "BF16"))):
            put(p + f"mlp.shared_expert.down_proj.{q}", a[0], a[1])
        put(p + "mlp.shared_expert_gate.weight", L.wg[None], "BF16")
    names = sorted(tensors)
    half = len(names) // 2
    for i, part in enumerate((names[:half], names[half:])):       # two shards
        LD.write_safetensors(os.path.join(tmp, f"model-{i:05d}.safetensors"),
                             {n: tensors[n] for n in part}, {n: dtypes[n] for n in part})
    cfg = {"text_config": {"num_experts_per_tok": K},
           "quantization": quant or {"group_size": 64, "bits": 4}}
    json.dump(cfg, open(os.path.join(tmp, "config.json"), "w"))
    return tensors, keep


def test_plan_covers_every_tensor_once_and_fuses_gate_rows_first(tmp_path, oracle):
    tensors, keep = _checkpoint(str(tmp_path), oracle)
    plan = LD.build_plan(str(tmp_path), layer=1)
    seen = [s for e in plan.entries for s in e.sources]
    assert sorted(seen) == sorted(tensors)              # every tensor exactly once
    assert plan.prefix == "language_model.model.layers.1.mlp."
    fused = {e.target: e for e in plan.entries if e.action == LD.FUSE}
    assert set(fused) == {f"{o}.gate_up_proj.{q}" for o in ("switch_mlp", "shared_expert")
                          for q in ("weight", "scales", "biases")}
    assert fused["switch_mlp.gate_up_proj.weight"].shape == (E, 2 * I, H // 8)
    assert fused["shared_expert.gate_up_proj.scales"].shape == (2 * IS, H // 64)
    drops = [e for e in plan.entries if e.action == LD.DROP]
    assert any("layers.0" in e.sources[0] for e in drops)
    arrs = LD.plan_arrays(plan, LD.checkpoint_tensors(str(tmp_path)))
    L = keep[1]
    assert np.array_equal(arrs["switch_mlp.gate_up_proj.weight"], L.gu_w)   # gate rows first
    assert np.array_equal(arrs["switch_mlp.gate_up_proj.biases"], L.gu_b)
    assert np.array_equal(arrs["shared_expert.gate_up_proj.weight"], L.sgu_w[0])
    assert np.array_equal(arrs["switch_mlp.down_proj.scales"], L.dn_s)
    assert np.array_equal(arrs["gate_weight"], L.wr)
    assert len(plan.quant) == 6 and all(
        q == {"group_size": 64, "bits": 4, "mode": "affine"} for q in plan.quant.values())


def test_plan_refuses_other_quantisation_and_missing_halves(tmp_path, oracle):
    d1 = tmp_path / "a"
    d1.mkdir()
    _checkpoint(str(d1), oracle, layers=1, quant={
        "group_size": 64, "bits": 4,
        "language_model.model.layers.0.mlp.switch_mlp.down_proj": {"group_size": 32, "bits": 8}})
    with pytest.raises(_lib.Unsupported):
        LD.build_plan(str(d1), layer=0)
    d2 = tmp_path / "b"
    d2.mkdir()
    _checkpoint(str(d2), oracle, layers=1, drop_up=True)
    with pytest.raises(_lib.InvalidArgument):
        LD.build_plan(str(d2), layer=0)
    with pytest.raises(_lib.InvalidArgument):
        LD.build_plan(str(d2), layer=5)


@pytest.mark.gpu
def test_loaded_block_matches_oracle(tmp_path, cuda, oracle):
    from gpu_util import bf, nbf
    from helpers import assert_bf16_close
    _, keep = _checkpoint(str(tmp_path), oracle)
    blk = LD.load_moe_block(str(tmp_path), 1, device=cuda)
    L = keep[1]
    x = oracle.make_x(96, H, seed=4)
    o = _lib.Options()
    o.min_tokens, o.int8_prefill, o.down_int8, o.wsum_mode = 1, 1, 1, 0
    y, idx, sc = blk(bf(x), options=o, return_routing=True)
    ry, ridx, rsc, ops = oracle.moe_prefill(L, x, int8_mode=3, parts=True)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert_bf16_close(nbf(y), ry, what="loaded block", operands=ops, operand_ulps=4)
