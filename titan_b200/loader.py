"""Checkpoint loading for the MoE block: safetensors headers, a plan, a load.

Mirrors the reference loader's split (titan/adapters/mlx/loader.py:1-31,
162-283): ``build_plan`` reads only the safetensors headers and
``config.json`` and decides, for every tensor, exactly one of LOAD (into a
block parameter), FUSE (the routed or shared expert's gate and up
projections, concatenated on the output axis with the gate rows first, the
layout of loader.py:440-470 and switch_layers.py:229-232) or DROP (with the
reason: not on the MoE block's path).  ``load_moe_block`` executes the plan
for one decoder layer from memory-mapped shards.  Affine quantisation groups
run along the input axis, so every output row carries its own scale and bias
and the concatenation is exact.

Per-tensor quantisation overrides (``config.json`` "quantization" entries
keyed by module path, moe-int8/REPORT.md:40-55) are honoured; the kernels
take 4-bit affine groups of 64 only, so any other spec raises Unsupported.

The safetensors format is read directly: an 8-byte little-endian header
length, a JSON header of name -> {dtype, shape, data_offsets}, then the raw
little-endian data.
"""
from __future__ import annotations

import json
import os
import re
import struct
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib

_DTYPES = {"BF16": (np.uint16, torch.bfloat16), "F16": (np.float16, torch.float16),
           "F32": (np.float32, torch.float32), "U32": (np.uint32, torch.int32),
           "I32": (np.int32, torch.int32), "U8": (np.uint8, torch.uint8)}

LOAD, FUSE, DROP = "load", "fuse", "drop"

# parameter suffixes of one MoE block, relative to "<layer>.mlp."
_ROUTED = re.compile(r"^switch_mlp\.(gate_proj|up_proj|down_proj)\.(weight|scales|biases)$")
_SHARED = re.compile(r"^shared_expert\.(gate_proj|up_proj|down_proj)\.(weight|scales|biases)$")
_ROUTER = "gate.weight"
_SHARED_GATE = "shared_expert_gate.weight"


@dataclass(frozen=True)
class TensorMeta:
    name: str
    dtype: str
    shape: tuple
    file: str
    offset: int          # byte offset of the data in the file
    nbytes: int


def read_header(path: str) -> dict[str, TensorMeta]:
    """The tensors of one safetensors file (header only)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        head = json.loads(f.read(n))
    base = 8 + n
    out = {}
    for name, d in head.items():
        if name == "__metadata__":
            continue
        a, b = d["data_offsets"]
        out[name] = TensorMeta(name, d["dtype"], tuple(d["shape"]), path, base + a, b - a)
    return out


def checkpoint_tensors(model_dir: str) -> dict[str, TensorMeta]:
    """Every tensor of every *.safetensors shard in model_dir."""
    out = {}
    for fn in sorted(os.listdir(model_dir)):
        if fn.endswith(".safetensors"):
            out.update(read_header(os.path.join(model_dir, fn)))
    return out


def write_safetensors(path: str, tensors: dict[str, np.ndarray], dtypes: dict[str, str]) -> None:
    """A safetensors file from numpy arrays (dtype names as in the format);
    the writer of the tests' synthetic checkpoints."""
    head, off, blobs = {}, 0, []
    for name, arr in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        head[name] = {"dtype": dtypes[name], "shape": list(arr.shape),
                      "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(head).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


@dataclass
class PlanEntry:
    action: str
    sources: tuple
    target: str | None     # block parameter path (LOAD / FUSE)
    shape: tuple
    dtype: str
    reason: str = ""


@dataclass
class LoaderPlan:
    layer: int
    prefix: str                          # "<...>.layers.N.mlp."
    entries: list = field(default_factory=list)
    quant: dict = field(default_factory=dict)

    def targets(self) -> list[str]:
        return [e.target for e in self.entries if e.target]

    def summary(self) -> str:
        c: dict[str, int] = {}
        for e in self.entries:
            c[e.action] = c.get(e.action, 0) + 1
        return ", ".join(f"{k}={v}" for k, v in sorted(c.items()))


def _layer_prefix(tensors, layer: int) -> str:
    pat = re.compile(rf"^(.*?(?:^|\.)layers\.{layer}\.mlp\.)")
    for name in sorted(tensors):
        m = pat.match(name)
        if m and name[len(m.group(1)):] in (_ROUTER,):
            return m.group(1)
    raise _lib.InvalidArgument(f"no MoE router ('layers.{layer}.mlp.gate.weight') in the checkpoint")


def _quant_spec(config: dict, module_path: str) -> dict:
    q = config.get("quantization") or config.get("quantization_config") or {}
    spec = q.get(module_path)
    if not isinstance(spec, dict):
        spec = {"group_size": q.get("group_size", 64), "bits": q.get("bits", 4),
                "mode": q.get("mode", "affine")}
    return {"group_size": spec.get("group_size", 64), "bits": spec.get("bits", 4),
            "mode": spec.get("mode", "affine")}


def build_plan(model_dir: str | None = None, layer: int = 0, *, tensors=None,
               config: dict | None = None) -> LoaderPlan:
    """Decide where every tensor goes for the MoE block of decoder `layer`.
    Reads headers only.  Every tensor of the checkpoint appears in exactly
    one entry."""
    if tensors is None:
        tensors = checkpoint_tensors(model_dir)
    if config is None:
        cfg_path = os.path.join(model_dir, "config.json") if model_dir else None
        config = json.load(open(cfg_path)) if cfg_path and os.path.exists(cfg_path) else {}
    prefix = _layer_prefix(tensors, layer)
    plan = LoaderPlan(layer, prefix)
    fuse: dict[tuple[str, str], dict[str, TensorMeta]] = {}
    for name in sorted(tensors):
        meta = tensors[name]
        if not name.startswith(prefix):
            plan.entries.append(PlanEntry(DROP, (name,), None, meta.shape, meta.dtype,
                                          "not part of this layer's MoE block"))
            continue
        rel = name[len(prefix):]
        m = _ROUTED.match(rel) or _SHARED.match(rel)
        if m and m.group(1) in ("gate_proj", "up_proj"):
            owner = "switch_mlp" if rel.startswith("switch_mlp") else "shared_expert"
            fuse.setdefault((owner, m.group(2)), {})[m.group(1)] = meta
            continue
        if m:
            owner = "switch_mlp" if rel.startswith("switch_mlp") else "shared_expert"
            plan.entries.append(PlanEntry(LOAD, (name,), f"{owner}.down_proj.{m.group(2)}",
                                          meta.shape, meta.dtype))
        elif rel == _ROUTER:
            plan.entries.append(PlanEntry(LOAD, (name,), "gate_weight", meta.shape, meta.dtype))
        elif rel == _SHARED_GATE:
            plan.entries.append(PlanEntry(LOAD, (name,), "shared_expert_gate_weight", meta.shape,
                                          meta.dtype))
        else:
            plan.entries.append(PlanEntry(DROP, (name,), None, meta.shape, meta.dtype,
                                          "not a tensor of the MoE block"))
    for (owner, suffix), parts in sorted(fuse.items()):
        missing = {"gate_proj", "up_proj"} - set(parts)
        if missing:
            raise _lib.InvalidArgument(f"{prefix}{owner}: cannot fuse, missing {sorted(missing)}")
        g, u = parts["gate_proj"], parts["up_proj"]
        ax = 1 if owner == "switch_mlp" else 0
        if g.dtype != u.dtype or g.shape[:ax] != u.shape[:ax] or g.shape[ax + 1:] != u.shape[ax + 1:]:
            raise _lib.InvalidArgument(f"{prefix}{owner}: gate/up mismatch {g.shape} {u.shape}")
        shape = g.shape[:ax] + (g.shape[ax] + u.shape[ax],) + g.shape[ax + 1:]
        plan.entries.append(PlanEntry(FUSE, (g.name, u.name), f"{owner}.gate_up_proj.{suffix}",
                                      shape, g.dtype, "[gate | up] on the output axis"))
    for owner in ("switch_mlp", "shared_expert"):
        for proj in ("gate_proj", "up_proj", "down_proj"):
            path = f"{prefix}{owner}.{proj}"
            if any(src.startswith(path + ".") for e in plan.entries for src in e.sources):
                spec = _quant_spec(config, path.rstrip("."))
                if spec != {"group_size": 64, "bits": 4, "mode": "affine"}:
                    raise _lib.Unsupported(f"{path}: quantisation {spec} (the kernels take "
                                           "affine 4-bit groups of 64)")
                plan.quant[path] = spec
    plan.entries.sort(key=lambda e: (e.action, e.target or "", e.sources[0]))
    return plan


def _read(meta: TensorMeta) -> np.ndarray:
    npdt = _DTYPES[meta.dtype][0]
    mm = np.memmap(meta.file, dtype=np.uint8, mode="r", offset=meta.offset, shape=(meta.nbytes,))
    return mm.view(npdt).reshape(meta.shape)


def _to_param(arr: np.ndarray, like: torch.Tensor) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if like.dtype == torch.bfloat16:
        t = t.view(torch.int16).view(torch.bfloat16)
    elif like.dtype == torch.int32 and t.dtype != torch.int32:
        t = t.view(torch.int32)
    return t


def plan_arrays(plan: LoaderPlan, tensors: dict[str, TensorMeta]) -> dict[str, np.ndarray]:
    """Execute a plan on the host: target -> array (memory-mapped for LOAD,
    concatenated for FUSE)."""
    out = {}
    for e in plan.entries:
        if not e.target:
            continue
        parts = [_read(tensors[s]) for s in e.sources]
        out[e.target] = parts[0] if e.action == LOAD else np.concatenate(
            parts, axis=1 if e.target.startswith("switch_mlp") else 0)
    return out


def load_moe_block(model_dir: str, layer: int, device=None, plan: LoaderPlan | None = None):
    """A titan_b200.SparseMoeBlock holding decoder `layer`'s MoE weights."""
    from .moe_block import SparseMoeBlock
    tensors = checkpoint_tensors(model_dir)
    if plan is None:
        plan = build_plan(model_dir, layer, tensors=tensors)
    by_target = {e.target: e for e in plan.entries if e.target}
    gu = by_target["switch_mlp.gate_up_proj.weight"].shape
    dn = by_target["switch_mlp.down_proj.weight"].shape
    E, H = by_target["gate_weight"].shape
    I = gu[1] // 2
    Is = by_target["shared_expert.gate_up_proj.weight"].shape[0] // 2 \
        if "shared_expert.gate_up_proj.weight" in by_target else 0
    if dn != (E, H, I // 8):
        raise _lib.InvalidArgument(f"down_proj {dn} does not match E={E} H={H} I={I}")
    k = None
    cfg_path = os.path.join(model_dir, "config.json")
    if os.path.exists(cfg_path):
        cfg = json.load(open(cfg_path))
        tc = cfg.get("text_config", cfg)
        k = tc.get("num_experts_per_tok")
    if not k:
        raise _lib.InvalidArgument("config.json gives no num_experts_per_tok")
    blk = SparseMoeBlock(H, E, k, I, Is, device=device, init=False)
    params = dict(blk.named_parameters())
    params.update(dict(blk.named_buffers()))
    with torch.no_grad():
        for target, arr in plan_arrays(plan, tensors).items():
            dst = params[target]
            dst.copy_(_to_param(arr, dst).reshape(dst.shape).to(dst.device))
    blk.prepare()
    return blk
