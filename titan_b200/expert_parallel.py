"""Expert parallelism for the quantised MoE block.

Experts are sharded over W ranks, expert e on rank e // (E / W); the router
and the shared expert stay data-parallel (each rank serves its own tokens).
A layer takes two all-to-all exchanges (the reference runs one device and has
no counterpart; the partitioning follows its block,
titan/adapters/mlx/vendor/mlx_vlm/models/qwen3_5_moe/language.py:60-91):

  dispatch  each token row goes once to every rank that owns at least one of
            its k experts (deduplicated per destination rank, not per
            expert), with the k-wide local expert ids of the slots served
            there (-1 elsewhere);
  combine   each owner returns one bf16 row per (token, slot) it served: the
            expert output itself, the same bits the single-device block
            computes for that slot.

The source then runs the block's own weighted sum (clone mode, with the
sigmoid-gated shared expert) over the k outputs of every token, so the
expert-parallel layer reproduces the single-device layer bit for bit wherever
the experts' arithmetic is fixed-order (the int8 path).

Two transports carry the exchanges:

  NCCL      ``torch.distributed`` all-to-alls (NCCL on GPUs, gloo in the CPU
            tests).  The dispatch plan is computed on the device with tensor
            ops; the host reads only the exchanged counts, which the
            variable-size all-to-all needs.
  peer      (:class:`PeerExchange`) every rank's receive buffers are mapped
            into every other rank through CUDA IPC and the library's kernels
            write into them over NVLink: tmoe_ep_dispatch stores each token
            row straight into its owners' receive rows, and the owners' down
            GEMM (tmoe_moe_experts_slots) stores every expert output row
            straight into the source's return row from its epilogue, so the
            return exchange is part of the expert kernel.  Epoch-tagged flags
            (tmoe_ep_wait) replace the collectives, and the receive buffers
            have a fixed capacity, so no count ever goes to the host.

The expert arithmetic is ``tmoe_moe_experts`` and the final sum
``tmoe_moe_combine`` from libtitan_moe.so, and the token-local part (router,
top-k, shared expert) ``tmoe_moe_local`` with the block's own kernels.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib, ops

__all__ = ["DispatchPlan", "plan_dispatch", "pairs_from_meta", "return_slots",
           "ExpertParallelMoE", "PeerExchange", "balanced_placement", "ep_forward"]


@dataclass
class DispatchPlan:
    send_token: torch.Tensor    # [S] local token of each sent row (destination-major)
    send_counts: torch.Tensor   # [W] rows per destination rank (int64)
    local_ids: torch.Tensor     # [S, k] int32 local expert id per slot, -1 if not on that rank


def _compact(flags: torch.Tensor, n: int, values: torch.Tensor) -> torch.Tensor:
    """values[flags] in order, for an n = flags.sum() the caller already knows
    (no host synchronisation): positions from a cumulative sum, the rest of
    the rows sent to a dummy slot n that is dropped."""
    pos = torch.cumsum(flags.to(torch.int64), 0) - 1
    pos = torch.where(flags, pos, torch.full_like(pos, n))
    out = values.new_empty((n + 1,) + tuple(values.shape[1:]))
    out.index_copy_(0, pos, values)
    return out[:n]


def _membership(idx: torch.Tensor, experts_per_rank: int, world: int):
    T = idx.shape[0]
    dest = idx.long() // experts_per_rank                          # [T, k]
    member = torch.zeros(T, world, dtype=torch.bool, device=idx.device)
    if T:
        member.scatter_(1, dest, True)
    return dest, member


def plan_dispatch(idx: torch.Tensor, experts_per_rank: int, world: int,
                  n_rows: int | None = None) -> DispatchPlan:
    """Deduplicated dispatch plan of one rank's tokens; idx [T, k] global
    expert ids.  Rows are ordered by destination rank, then by token.  n_rows
    (the number of rows sent, if the caller knows it) avoids a host sync."""
    T, k = idx.shape
    dest, member = _membership(idx, experts_per_rank, world)
    send_counts = member.sum(0).to(torch.int64)
    flat = member.t().reshape(-1)                                   # destination-major
    if n_rows is None:
        n_rows = int(flat.sum())
    dev = idx.device
    t_idx = _compact(flat, n_rows, torch.arange(T, device=dev).repeat(world))
    d_idx = _compact(flat, n_rows, torch.arange(world, device=dev).repeat_interleave(T))
    on_d = dest[t_idx] == d_idx[:, None]                           # [S, k]
    local = torch.where(on_d, idx[t_idx].long() - d_idx[:, None] * experts_per_rank,
                        torch.full_like(dest[t_idx], -1)).to(torch.int32)
    return DispatchPlan(t_idx, send_counts, local.contiguous())


def pairs_from_meta(local_ids: torch.Tensor, n_pairs: int | None = None):
    """Received k-wide metadata -> the (row, local expert) pairs this rank
    serves, row-major (row, then slot).  n_pairs (if known) avoids a host
    sync."""
    R, k = local_ids.shape
    flags = (local_ids >= 0).reshape(-1)
    if n_pairs is None:
        n_pairs = int(flags.sum())
    rows = torch.arange(R, device=local_ids.device).repeat_interleave(k)
    pair_row = _compact(flags, n_pairs, rows)
    pair_exp = _compact(flags, n_pairs, local_ids.reshape(-1))
    return pair_row.to(torch.int32).contiguous(), pair_exp.to(torch.int32).contiguous()


def return_slots(plan: DispatchPlan, T: int, k: int) -> torch.Tensor:
    """Where each (token, slot) lands in the combine buffer: the owners send
    their pair outputs back in the order of the sent rows (destination, then
    token) and, inside a row, of the slots; inv [T*k] int32.  Every (token,
    slot) is served on exactly one rank, so all T*k entries are written."""
    dev = plan.local_ids.device
    valid = (plan.local_ids >= 0).reshape(-1)
    pos = (torch.cumsum(valid.to(torch.int64), 0) - 1).to(torch.int32)
    tgt = (plan.send_token.long()[:, None] * k + torch.arange(k, device=dev)[None, :]).reshape(-1)
    tgt = torch.where(valid, tgt, torch.full_like(tgt, T * k))
    inv = torch.empty(T * k + 1, dtype=torch.int32, device=dev)
    inv.index_copy_(0, tgt, pos)
    return inv[:T * k]


def _exchange(t: torch.Tensor, send_counts: list[int], recv_counts: list[int], group) -> torch.Tensor:
    out = torch.empty((sum(recv_counts),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t.contiguous(), recv_counts, send_counts, group=group)
    return out


def _wire(t: torch.Tensor) -> torch.Tensor:
    """Rows travel as int32 words (every backend moves those; gloo has no
    16-bit types); a row's bytes must be a multiple of 4."""
    return t.contiguous().view(torch.int32)


def _words(x: torch.Tensor) -> int:
    """int32 words per row of x on the wire."""
    return x.shape[1] * x.element_size() // 4


def _unwire(t: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    return t.view(like.dtype)


def _mark(marks, name):
    if marks is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((name, ev))


def ep_forward(x: torch.Tensor, idx: torch.Tensor, experts_per_rank: int, expert_fn: Callable,
               combine_fn: Callable, group=None, marks: list | None = None):
    """One expert-parallel MoE layer on this rank's tokens x [T, H] with their
    expert ids idx [T, k].  expert_fn(rows, pair_row, pair_exp) -> [P, H]
    bf16 applies this rank's experts to the pairs it serves;
    combine_fn(ys, inv) -> [T, H] bf16 forms the output from every token's k
    expert outputs ys[inv[t*k + j]].  marks (GPU runs): a list that receives
    (phase, CUDA event) after each phase, for timing."""
    world = dist.get_world_size(group)
    T, k = idx.shape
    # counts first (rows and pairs per destination), the one host sync of
    # the layer (the variable-size all-to-all needs them on the host)
    dest, member = _membership(idx, experts_per_rank, world)
    pair_counts = torch.bincount(dest.reshape(-1), minlength=world)[:world]
    counts = torch.stack([member.sum(0).to(torch.int64), pair_counts.to(torch.int64)], 1)
    _mark(marks, "plan")
    recv = torch.empty_like(counts)
    dist.all_to_all_single(recv, counts, group=group)
    c = counts.cpu()
    rc = recv.cpu()
    _mark(marks, "counts")
    rows_out, rows_in = c[:, 0].tolist(), rc[:, 0].tolist()
    pairs_back, pairs_recv = c[:, 1].tolist(), rc[:, 1].tolist()
    plan = plan_dispatch(idx, experts_per_rank, world, n_rows=sum(rows_out))
    # one exchange per direction: each sent row carries its k local expert
    # ids as k extra int32 words after the row's words
    H = x.shape[1]
    payload = torch.cat([_wire(x[plan.send_token]), plan.local_ids.view(torch.int32)], 1)
    got = _exchange(payload, rows_out, rows_in, group)
    nw = _words(x)
    rows = _unwire(got[:, :nw].contiguous(), x).reshape(-1, H)
    ids = got[:, nw:].contiguous()
    _mark(marks, "dispatch")
    pair_row, pair_exp = pairs_from_meta(ids, n_pairs=sum(pairs_recv))
    y_pairs = expert_fn(rows, pair_row, pair_exp)
    _mark(marks, "experts")
    back = _unwire(_exchange(_wire(y_pairs), pairs_recv, pairs_back, group), y_pairs)
    _mark(marks, "return")
    y = combine_fn(back, return_slots(plan, T, k))
    _mark(marks, "combine")
    return y


class _DeviceArray:
    """Raw device memory seen by torch.as_tensor (CUDA array interface)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def _view(ptr: int, shape: tuple, dtype: torch.dtype, device) -> torch.Tensor:
    code = {torch.int32: "<i4", torch.int16: "<i2"}[dtype]
    return torch.as_tensor(_DeviceArray(ptr, shape, code), device=device)


class PeerExchange:
    """The expert-parallel exchange of one rank over NVLink peer memory.

    One device allocation per rank (tmoe_ep_alloc; layout in
    include/titan_moe.h) holds the rows other ranks send here, their expert
    ids and token indices, the returned expert outputs of this rank's own
    tokens, and the epoch-tagged flags.  Every rank maps every other rank's
    allocation through CUDA IPC (handles swapped with one
    ``all_gather_object``), so the library's kernels store into peers
    directly.  One exchange serves any number of layers in turn: the layers
    of a step run one after another, and each call advances the epoch.
    ``cap`` is the most tokens a rank passes to one layer call.  Creating
    and :meth:`close` are collective over ``group``."""

    def __init__(self, cap: int, hidden: int, top_k: int, group=None, device=None):
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.cap, self.hidden, self.top_k = int(cap), int(hidden), int(top_k)
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        self.offsets = (C.c_size_t * 4)()
        nbytes = lib.tmoe_ep_buffer_bytes(self.world, self.cap, self.hidden, self.top_k,
                                          self.cap, self.offsets)
        if nbytes == 0:
            raise _lib.InvalidArgument(f"bad exchange shape: cap={cap}, H={hidden}, k={top_k}")
        self.nbytes = int(nbytes)
        ptr = C.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.tmoe_ep_alloc(self.nbytes, C.byref(ptr)), "tmoe_ep_alloc")
        self.ptr = ptr.value
        handle = C.create_string_buffer(64)
        if self.world > 1:
            _lib.check(lib.tmoe_ipc_handle(self.ptr, handle), "tmoe_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        peers = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    peers.append(self.ptr)
                    continue
                p = C.c_void_p()
                _lib.check(lib.tmoe_ipc_open(C.create_string_buffer(h, 64), C.byref(p)),
                           "tmoe_ipc_open")
                self._opened.append(p.value)
                peers.append(p.value)
        self.peers = torch.tensor(peers, dtype=torch.int64, device=self.device)
        W, k = self.world, self.top_k
        self.counters = torch.zeros(W + 1, dtype=torch.int32, device=self.device)
        self.rows_in = torch.zeros(W, dtype=torch.int32, device=self.device)
        self.returned = torch.zeros(W, dtype=torch.int32, device=self.device)
        self.slot_exp = torch.empty(W * self.cap * k, dtype=torch.int32, device=self.device)
        self.y_rows = torch.empty(W * self.cap * k, dtype=torch.int64, device=self.device)
        self.epoch = 0
        o = [int(v) for v in self.offsets]
        W, k, H = self.world, self.top_k, self.hidden
        self.rows = _view(self.ptr + o[0], (W * self.cap, H), torch.int16,
                          self.device).view(torch.bfloat16)
        self.meta = _view(self.ptr + o[1], (W, self.cap, k + 1), torch.int32, self.device)
        self.ret = _view(self.ptr + o[2], (self.cap * k, H), torch.int16,
                         self.device).view(torch.bfloat16)
        self.ret_offset = o[2]
        self._ar = {}

    def arange(self, n: int) -> torch.Tensor:
        a = self._ar.get(n)
        if a is None:
            a = self._ar[n] = torch.arange(n, dtype=torch.int32, device=self.device)
        return a

    def check(self) -> None:
        """Raise DeviceTimeout if a wait of the library has given up (a rank
        did not post its flag within the bound); synchronises the host."""
        _lib.check(_lib.load().tmoe_device_status(), "peer exchange")

    def close(self) -> None:
        """Unmap the peers' buffers, wait for every rank to do the same, and
        free this rank's buffer (collective)."""
        if self.ptr is None:
            return
        torch.cuda.synchronize(self.device)
        lib = _lib.load()
        for p in self._opened:
            _lib.check(lib.tmoe_ipc_close(p), "tmoe_ipc_close")
        self._opened = []
        dist.barrier(group=self.group)
        self.rows = self.meta = self.ret = None
        _lib.check(lib.tmoe_ep_free(self.ptr), "tmoe_ep_free")
        self.ptr = None


def slot_experts(meta: torch.Tensor, rows_in: torch.Tensor, experts_per_rank: int) -> torch.Tensor:
    """The slot-form pair list of a PeerExchange's metadata meta [W, cap, k+1]:
    slot j of received row (source s, i) is served here by local expert
    meta[s, i, j] when the row was written this layer (i < rows_in[s]) and
    that id is one of this rank's experts; -1 otherwise.  int32 [W*cap*k].
    The tensor statement of tmoe_ep_slots (tests check one against the
    other)."""
    W, cap, k1 = meta.shape
    live = torch.arange(cap, dtype=torch.int32, device=meta.device)[None, :] < rows_in[:, None]
    ids = meta[..., :k1 - 1]
    ok = live[..., None] & (ids >= 0) & (ids < experts_per_rank)
    return torch.where(ok, ids, -1).reshape(-1)


def return_addresses(meta: torch.Tensor, slot_exp: torch.Tensor, peers: torch.Tensor,
                     ret_offset: int, hidden: int) -> torch.Tensor:
    """Where the output of slot j of received row (s, i) goes: the ret row
    token*k + j of source s's buffer (peers [W] int64 base addresses), token =
    meta[s, i, k]; 0 for a slot not served (slot_exp -1).  int64 [W*cap*k].
    With slot_experts, the tensor statement of tmoe_ep_slots."""
    W, cap, k1 = meta.shape
    k = k1 - 1
    tok = meta[..., k].long()
    slot = torch.arange(k, dtype=torch.int64, device=meta.device)
    addr = (peers[:, None, None] + ret_offset + (tok[..., None] * k + slot) * (2 * hidden)).reshape(-1)
    return torch.where(slot_exp >= 0, addr, 0)


def peer_forward(x: torch.Tensor, idx: torch.Tensor, ex: PeerExchange, experts_per_rank: int,
                 expert_fn: Callable, combine_fn: Callable, marks: list | None = None):
    """One expert-parallel MoE layer over peer memory (the PeerExchange
    transport), the same layer as :func:`ep_forward` without a host
    synchronisation: every count stays on the device.

    expert_fn(rows, slot_exp, y_addr) applies this rank's experts to the
    served slots of the received rows and stores slot f's output at address
    y_addr[f] (the sources' ret rows; tmoe_moe_experts_slots).  A wait that
    gives up anywhere in the layer (an owner's dispatch wait is passed on as
    a return count of -1) turns this rank's output into NaN, and
    :meth:`PeerExchange.check` (tmoe_device_status) raises DeviceTimeout;
    callers check at their step boundary."""
    W, rank, cap = ex.world, ex.rank, ex.cap
    T, k = idx.shape
    H = x.shape[1]
    if T > cap:
        raise _lib.InvalidArgument(f"{T} tokens exceed the exchange capacity {cap}")
    if k != ex.top_k or H != ex.hidden:
        raise _lib.InvalidArgument("layer shape differs from the exchange's")
    lib = _lib.load()
    stream = ops.stream_ptr(x.device)
    ex.epoch += 1
    ep = ex.epoch
    _lib.check(lib.tmoe_ep_dispatch(x.data_ptr(), idx.data_ptr(), T, k, H, experts_per_rank, W,
                                    rank, ex.peers.data_ptr(), ex.offsets, cap, ep,
                                    ex.counters.data_ptr(), stream), "tmoe_ep_dispatch")
    _lib.check(lib.tmoe_ep_wait(ex.ptr, ex.offsets, 0, W, ep, ex.rows_in.data_ptr(), stream),
               "tmoe_ep_wait")
    _mark(marks, "dispatch")
    _lib.check(lib.tmoe_ep_slots(ex.ptr, ex.offsets, ex.rows_in.data_ptr(), W, cap, k,
                                 experts_per_rank, H, ex.peers.data_ptr(), ex.slot_exp.data_ptr(),
                                 ex.y_rows.data_ptr(), stream), "tmoe_ep_slots")
    _mark(marks, "slots")
    expert_fn(ex.rows, ex.slot_exp, ex.y_rows)
    # count -1 to every source when a dispatch wait above gave up
    _lib.check(lib.tmoe_ep_post_return(ex.rows_in.data_ptr(), W, rank, ex.peers.data_ptr(),
                                       ex.offsets, ep, stream), "tmoe_ep_post_return")
    _mark(marks, "experts+return")
    _lib.check(lib.tmoe_ep_wait(ex.ptr, ex.offsets, 1, W, ep, ex.returned.data_ptr(), stream),
               "tmoe_ep_wait")
    _mark(marks, "wait")
    y = combine_fn(ex.ret[:T * k], None)      # returned rows are token-major
    # a negative return count (an owner's or this rank's wait gave up): the
    # output becomes NaN and tmoe_device_status reports the timeout
    _lib.check(lib.tmoe_ep_guard(ex.returned.data_ptr(), W, y.data_ptr(), y.numel(), stream),
               "tmoe_ep_guard")
    _mark(marks, "combine")
    return y


def balanced_placement(load, world: int) -> list[int]:
    """An expert placement for ``world`` ranks from per-expert load (token
    counts, say): longest-processing-time greedy, the most loaded expert
    first onto the rank with the least load that still has a free place, E/W
    places per rank.  Returns perm: rank r holds experts perm[r*E/W:(r+1)*E/W]
    in that order."""
    load = [float(v) for v in load]
    E = len(load)
    if E % world:
        raise _lib.InvalidArgument(f"{E} experts do not split over {world} ranks")
    epr = E // world
    order = sorted(range(E), key=lambda e: (-load[e], e))
    total = [0.0] * world
    places: list[list[int]] = [[] for _ in range(world)]
    for e in order:
        r = min((r for r in range(world) if len(places[r]) < epr), key=lambda r: (total[r], r))
        places[r].append(e)
        total[r] += load[e]
    return [e for r in range(world) for e in sorted(places[r])]


class ExpertParallelMoE(torch.nn.Module):
    """A SparseMoeBlock sharded over the ranks of ``group``: this rank holds
    E/W routed experts and a full copy of the router and the shared expert;
    the constructor slices them out of a full block.  Without a placement
    rank r holds experts [r*E/W, (r+1)*E/W); with one (a permutation of the
    experts, e.g. from balanced_placement, the same on every rank) it holds
    placement[r*E/W:(r+1)*E/W], and the router's expert ids are mapped to
    their places before the exchanges (one gather; the outputs keep every
    bit, since a slot's expert and the slot order are unchanged)."""

    def __init__(self, block, group=None, exchange: PeerExchange | None = None,
                 placement=None):
        super().__init__()
        self.group = group
        self.exchange = exchange
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        E = block.num_experts
        if E % world:
            raise _lib.InvalidArgument(f"{E} experts do not split over {world} ranks")
        self.world, self.rank, self.epr = world, rank, E // world
        self.hidden, self.top_k = block.hidden, block.top_k
        self.moe_inter = block.moe_inter
        lo, hi = rank * self.epr, (rank + 1) * self.epr
        sm = block.switch_mlp
        dev = block.gate_weight.device
        self.place = None
        if placement is not None:
            perm = torch.as_tensor(list(placement), dtype=torch.int64)
            if perm.numel() != E or not torch.equal(perm.sort().values, torch.arange(E)):
                raise _lib.InvalidArgument("placement must be a permutation of the experts")
            place = torch.empty(E, dtype=torch.int32)
            place[perm] = torch.arange(E, dtype=torch.int32)
            self.place = place.to(dev)                  # expert -> its place
            mine = perm[lo:hi].to(dev)
        else:
            mine = torch.arange(lo, hi, device=dev)
        self.gate_weight = block.gate_weight
        self.gu = tuple(t.index_select(0, mine.to(t.device)).contiguous() for t in
                        (sm.gate_up_proj.weight, sm.gate_up_proj.scales, sm.gate_up_proj.biases))
        self.dn = tuple(t.index_select(0, mine.to(t.device)).contiguous() for t in
                        (sm.down_proj.weight, sm.down_proj.scales, sm.down_proj.biases))
        self.tables = (ops.build_tables(*self.gu), ops.build_tables(*self.dn))
        self.shared_expert = block.shared_expert
        self.shared_gate = block.shared_expert_gate_weight
        self.shared_inter = block.shared_inter
        self.num_experts = E
        se = block.shared_expert
        self.shared_tables = () if se is None else (
            ops.build_tables(se.gate_up_proj.weight, se.gate_up_proj.scales, se.gate_up_proj.biases),
            ops.build_tables(se.down_proj.weight, se.down_proj.scales, se.down_proj.biases))
        self._layer = None
        self._local = None

    def _layer_struct(self) -> _lib.Layer:
        if self._layer is None:
            L = _lib.Layer()
            L.hidden, L.num_experts, L.top_k = self.hidden, self.epr, self.top_k
            L.moe_inter, L.shared_inter = self.moe_inter, 0
            L.gate_up_w, L.gate_up_s, L.gate_up_b = (t.data_ptr() for t in self.gu)
            L.down_w, L.down_s, L.down_b = (t.data_ptr() for t in self.dn)
            L.gate_up_st, L.gate_up_bt = self.tables[0].scales_t.data_ptr(), self.tables[0].biases_t.data_ptr()
            L.down_st, L.down_bt = self.tables[1].scales_t.data_ptr(), self.tables[1].biases_t.data_ptr()
            L.gate_up_rs = self.tables[0].row_scale.data_ptr()
            L.down_rs = self.tables[1].row_scale.data_ptr()
            self._layer = L
        return self._layer

    def _local_struct(self) -> _lib.Layer:
        """The token-local part of the layer: the full router and the shared
        expert (routed-expert fields left empty)."""
        if self._local is None:
            L = _lib.Layer()
            L.hidden, L.num_experts, L.top_k = self.hidden, self.num_experts, self.top_k
            L.moe_inter, L.shared_inter = self.moe_inter, self.shared_inter
            L.router_w = self.gate_weight.data_ptr()
            if self.shared_expert is not None:
                se, t = self.shared_expert, self.shared_tables
                L.shared_gate_up_w = se.gate_up_proj.weight.data_ptr()
                L.shared_gate_up_s = se.gate_up_proj.scales.data_ptr()
                L.shared_gate_up_b = se.gate_up_proj.biases.data_ptr()
                L.shared_down_w = se.down_proj.weight.data_ptr()
                L.shared_down_s = se.down_proj.scales.data_ptr()
                L.shared_down_b = se.down_proj.biases.data_ptr()
                L.shared_gate_up_st, L.shared_gate_up_bt = t[0].scales_t.data_ptr(), t[0].biases_t.data_ptr()
                L.shared_down_st, L.shared_down_bt = t[1].scales_t.data_ptr(), t[1].biases_t.data_ptr()
                L.shared_gate_up_rs = t[0].row_scale.data_ptr()
                L.shared_down_rs = t[1].row_scale.data_ptr()
                L.shared_gate_w = self.shared_gate.data_ptr()
            self._local = L
        return self._local

    def local(self, xf, options: _lib.Options | None = None):
        """Router, top-k, shared expert and its gate logit on this rank's
        tokens (tmoe_moe_local): the block's own kernels."""
        T, dev = xf.shape[0], xf.device
        idx = torch.empty(T, self.top_k, dtype=torch.int32, device=dev)
        scores = torch.empty(T, self.top_k, dtype=torch.bfloat16, device=dev)
        shared_out = gate_logit = None
        if self.shared_expert is not None:
            shared_out = torch.empty(T, self.hidden, dtype=torch.bfloat16, device=dev)
            gate_logit = torch.empty(T, dtype=torch.float32, device=dev)
        if T == 0:
            return idx, scores, shared_out, gate_logit
        L = self._local_struct()
        opt = options if options is not None else _lib.Options(512, 1, 0, 1, 0)
        lib = _lib.load()
        nb = lib.tmoe_moe_local_workspace_size(L, T, opt)
        ws = ops.workspace(nb, dev, "ep_local")
        _lib.check(lib.tmoe_moe_local(L, xf.data_ptr(), T, opt, ws.data_ptr(), ws.numel(),
                                      idx.data_ptr(), scores.data_ptr(),
                                      None if gate_logit is None else gate_logit.data_ptr(),
                                      None if shared_out is None else shared_out.data_ptr(),
                                      ops.stream_ptr(dev)),
                   "tmoe_moe_local")
        return idx, scores, shared_out, gate_logit

    def experts(self, rows, pair_row, pair_exp, options: _lib.Options | None = None):
        """This rank's routed experts on received rows (tmoe_moe_experts)."""
        R, P = rows.shape[0], pair_row.numel()
        y = torch.empty(P, self.hidden, dtype=torch.bfloat16, device=rows.device)
        if P == 0:
            return y
        L = self._layer_struct()
        opt = options if options is not None else _lib.Options(512, 1, 0, 1, 0)
        lib = _lib.load()
        nb = lib.tmoe_moe_experts_workspace_size(L, R, P, opt)
        ws = ops.workspace(nb, rows.device, "ep")
        _lib.check(lib.tmoe_moe_experts(L, rows.data_ptr(), R, pair_row.data_ptr(),
                                        pair_exp.data_ptr(), P, opt, ws.data_ptr(), ws.numel(),
                                        y.data_ptr(), ops.stream_ptr(rows.device)),
                   "tmoe_moe_experts")
        return y

    def experts_slots(self, rows, slot_exp, y_addr, options: _lib.Options | None = None):
        """This rank's routed experts on the served slots of rows (slot_exp
        [R*k], -1: not served), slot f's output row stored at address
        y_addr[f] (tmoe_moe_experts_slots)."""
        R = rows.shape[0]
        if R == 0:
            return
        L = self._layer_struct()
        opt = options if options is not None else _lib.Options(512, 1, 0, 1, 0)
        lib = _lib.load()
        nb = lib.tmoe_moe_experts_workspace_size(L, R, R * self.top_k, opt)
        ws = ops.workspace(nb, rows.device, "ep")
        _lib.check(lib.tmoe_moe_experts_slots(L, rows.data_ptr(), R, slot_exp.data_ptr(), opt,
                                              ws.data_ptr(), ws.numel(), y_addr.data_ptr(),
                                              ops.stream_ptr(rows.device)),
                   "tmoe_moe_experts_slots")

    def combine(self, ys, inv, scores, shared_out, gate_logit, mode: int = 0):
        """The block's weighted sum plus gated shared expert (tmoe_moe_combine);
        inv None: ys is already token-major."""
        T, k = scores.shape
        y = torch.empty(T, self.hidden, dtype=torch.bfloat16, device=scores.device)
        if T == 0:
            return y
        _lib.call("tmoe_moe_combine", ys.data_ptr(), None if inv is None else inv.data_ptr(),
                  scores.data_ptr(), T, k,
                  self.hidden, mode, None if shared_out is None else shared_out.data_ptr(),
                  None if gate_logit is None else gate_logit.data_ptr(), y.data_ptr(),
                  ops.stream_ptr(scores.device))
        return y

    def forward(self, x: torch.Tensor, options: _lib.Options | None = None,
                marks: list | None = None) -> torch.Tensor:
        xf = x.reshape(-1, self.hidden).contiguous()
        _mark(marks, "start")
        idx, scores, shared_out, gate_logit = self.local(xf, options)
        if self.place is not None and idx.numel():
            idx = self.place[idx.long()]
        _mark(marks, "local")
        mode = options.wsum_mode if options is not None else 0
        experts = lambda *a: self.experts(*a, options=options)  # noqa: E731
        combine = lambda ys, inv: self.combine(ys, inv, scores, shared_out, gate_logit, mode)  # noqa: E731
        if self.exchange is not None:
            y = peer_forward(xf, idx, self.exchange, self.epr,
                             lambda *a: self.experts_slots(*a, options=options), combine, marks)
        else:
            y = ep_forward(xf, idx, self.epr, experts, combine, self.group, marks)
        return y.reshape(x.shape)
