"""Multi-token and expert-parallel selected-expert MoE.

The reference runs one token at a time through
``MoeExecutor::execute_selected_moe_cuda`` (crates/objeta-cuda/src/moe.rs:
352-751) and has no expert parallelism; this module is the multi-token,
multi-GPU form of the same layer:

* ``router_topk_batched``: the reference router (deepseek_single_layer_moe.rs:
  720-740) for T tokens, one CTA per token;
* ``moe_pairs``: the layer over a list of (expert, token) pairs, each pair's
  unweighted down-projection output in its own row;
* ``moe_combine``: the weighted top-k combine per token, in slot order, with
  the reference's arithmetic (out = 0; out += w * down; moe.rs:1319-1321);
* ``DispatchPlan`` / ``ExpertParallelMoe``: experts of a layer block-
  partitioned over the ranks of a process group (expert e on rank
  e // (E / G)); every rank routes its own tokens, the routing table is
  all-gathered, token rows go to the experts' ranks with one all-to-all, the
  pair outputs come back with a second, and each token's owner combines
  them in slot order.  Every pair output is computed by the same row
  programs whichever rank runs it, so the result does not depend on the
  number of ranks.

Collectives are ``torch.distributed`` calls (NCCL on GPUs, gloo on CPU); the
compute is the CUDA library unless a test supplies another ``compute``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from .quant import _dev_ptr

c_size = ctypes.c_size_t
c_int = ctypes.c_int
c_void_p = ctypes.c_void_p

_lib.register_signatures({
    "objb_moe_pairs_scratch_bytes": (c_int, [c_void_p, c_size, c_size, ctypes.POINTER(c_size)]),
    "objb_moe_pairs_device": (c_int, [c_void_p, c_size, c_void_p, c_void_p, c_void_p, c_void_p, c_size,
                                      c_void_p, c_void_p, c_size, ctypes.c_float, c_void_p]),
    "objb_moe_pairs_tc_scratch_bytes": (c_int, [c_void_p, c_size, c_size, ctypes.POINTER(c_size)]),
    "objb_moe_pairs_tc_device": (c_int, [c_void_p, c_size, c_void_p, c_void_p, c_void_p, c_void_p, c_size,
                                         c_void_p, c_void_p, c_size, ctypes.c_float, c_void_p]),
    "objb_moe_pairs_official_tc_scratch_bytes": (c_int, [c_void_p, c_size, c_size, ctypes.POINTER(c_size)]),
    "objb_moe_pairs_official_tc_device": (c_int, [c_void_p, c_size, c_void_p, c_void_p, c_void_p, c_void_p, c_size,
                                                  c_void_p, c_void_p, c_size, ctypes.c_float, c_void_p]),
    "objb_moe_combine_device": (c_int, [c_void_p, c_size, c_void_p, c_void_p, c_size, c_size, c_size, c_void_p,
                                        c_void_p]),
    "objb_router_topk_batched_device": (c_int, [c_void_p, c_size, c_size, c_size, c_int, c_void_p, c_void_p,
                                                c_void_p]),
    "objb_ep_build_pairs_device": (c_int, [c_void_p, c_size, c_size, c_size, c_size, c_size, c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_void_p]),
    "objb_ep_partial_combine_device": (c_int, [c_void_p, c_void_p, c_void_p, c_size, c_size, c_size, c_size,
                                               c_size, c_size, c_void_p, c_void_p]),
    "objb_ep_sum_partials_device": (c_int, [c_void_p, c_size, c_size, c_size, c_void_p, c_void_p]),
    "objb_ep_packed_rows": (c_size, [c_size, c_size, c_size]),
    "objb_ep_pack_device": (c_int, [c_void_p, c_void_p, c_void_p, c_size, c_size, c_size, c_void_p, c_void_p]),
    "objb_ep_build_pairs_packed_device": (c_int, [c_void_p, c_size, c_size, c_size, c_size, c_size, c_size,
                                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "objb_ep_partial_combine_packed_device": (c_int, [c_void_p, c_void_p, c_size, c_size, c_size, c_size, c_size,
                                                      c_size, c_size, c_void_p, c_void_p]),
    "objb_deepseek_gate_device": (c_int, [c_void_p, c_void_p, c_void_p, c_size, c_void_p, c_void_p, c_size, c_size,
                                          c_size, c_size, c_int, ctypes.c_float, c_void_p, c_void_p, c_void_p]),
})

SOFTMAX, SIGMOID, SQRT_SOFTPLUS = 0, 1, 2


def deepseek_gate(d_gate_weight, d_hidden, top_k: int, score_func: int = SQRT_SOFTPLUS, route_scale: float = 1.5,
                  d_gate_bias=None, d_tid2eid=None, d_input_ids=None, stream=None):
    """The DeepSeek V4 gate (cpu_gate_ref, dsl_moe.rs:768-881) on the device
    for T tokens: d_gate_weight f32 [E, H], d_hidden f32 [T, H]; returns
    (ids int32 [T, k], weights f32 [T, k])."""
    import torch
    E, H = d_gate_weight.shape
    hid = d_hidden.reshape(-1, H)
    T = hid.shape[0]
    ids = torch.empty(T, top_k, dtype=torch.int32, device=hid.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=hid.device)
    _lib.call("objb_deepseek_gate_device", _dev_ptr(d_gate_weight),
              _dev_ptr(d_gate_bias) if d_gate_bias is not None else None,
              _dev_ptr(d_tid2eid) if d_tid2eid is not None else None,
              0 if d_tid2eid is None else d_tid2eid.numel(), _dev_ptr(hid),
              _dev_ptr(d_input_ids) if d_input_ids is not None else None, T, E, H, top_k, int(score_func),
              float(route_scale), _dev_ptr(ids), _dev_ptr(w), _lib.stream_handle(stream))
    return ids, w


def ep_build_pairs(ids_all, rank: int, num_experts: int, stream=None):
    """This rank's pairs from the routing table ids_all [G, T, k] (device
    int32), built on the device: returns (pair_expert, pair_token, pair_out,
    count) device int32 tensors; the arrays have G*T*k entries of which the
    first ``count`` are used.  pair_token indexes the all-gathered token rows
    [G*T, H]; pair_out is the routing entry's flat index (s*T + t)*k + j."""
    import torch
    G, T, K = ids_all.shape
    n = G * T * K
    buf = torch.empty(3 * n + 1, dtype=torch.int32, device=ids_all.device)
    pe, pt, po, cnt = buf[:n], buf[n:2 * n], buf[2 * n:3 * n], buf[3 * n:]
    _lib.call("objb_ep_build_pairs_device", _dev_ptr(ids_all), G, T, K, num_experts, rank, _dev_ptr(pe),
              _dev_ptr(pt), _dev_ptr(po), _dev_ptr(cnt), _lib.stream_handle(stream))
    return pe, pt, po, cnt


def ep_partial_combine(ids_all, w_all, v, rank: int, num_experts: int, out_dim: int, stream=None):
    """Per routing row (s, t): the slot-order fold of w * v over the slots
    whose expert lives on this rank -> partial [G, T, out_dim]."""
    import torch
    G, T, K = ids_all.shape
    part = torch.empty(G, T, out_dim, dtype=torch.float32, device=v.device)
    _lib.call("objb_ep_partial_combine_device", _dev_ptr(ids_all), _dev_ptr(w_all), _dev_ptr(v), G, T, K,
              num_experts, rank, out_dim, _dev_ptr(part), _lib.stream_handle(stream))
    return part


def ep_sum_partials(parts, stream=None):
    """out[t] = sum over ranks r (in rank order) of parts[r, t]."""
    import torch
    G, T, O_ = parts.shape
    out = torch.empty(T, O_, dtype=torch.float32, device=parts.device)
    _lib.call("objb_ep_sum_partials_device", _dev_ptr(parts), G, T, O_, _dev_ptr(out), _lib.stream_handle(stream))
    return out


def ep_packed_rows(tokens: int, top_k: int, hidden: int) -> int:
    """Rows of H floats in one rank's packed exchange buffer: its T token rows,
    then its ids and weights (objb_ep_packed_rows)."""
    return int(_lib.load().objb_ep_packed_rows(tokens, top_k, hidden))


def ep_pack(x, ids, w, send, stream=None):
    """Packs this rank's step (x [T, H] f32, ids [T, k] int32, w [T, k] f32)
    into send [ep_packed_rows(T, k, H), H] for the one all-gather."""
    T, H = x.shape
    K = ids.shape[1]
    _lib.call("objb_ep_pack_device", _dev_ptr(x), _dev_ptr(ids), _dev_ptr(w), T, K, H, _dev_ptr(send),
              _lib.stream_handle(stream))
    return send


def ep_build_pairs_packed(recv, world: int, tokens: int, top_k: int, rank: int, num_experts: int, stream=None):
    """ep_build_pairs reading the ids from the all-gathered packed buffers
    recv [G * rows, H]; pair_token indexes the rows of recv."""
    import torch
    n = world * tokens * top_k
    buf = torch.empty(3 * n + 1, dtype=torch.int32, device=recv.device)
    pe, pt, po, cnt = buf[:n], buf[n:2 * n], buf[2 * n:3 * n], buf[3 * n:]
    _lib.call("objb_ep_build_pairs_packed_device", _dev_ptr(recv), world, tokens, top_k, recv.shape[1], num_experts,
              rank, _dev_ptr(pe), _dev_ptr(pt), _dev_ptr(po), _dev_ptr(cnt), _lib.stream_handle(stream))
    return pe, pt, po, cnt


def ep_partial_combine_packed(recv, v, world: int, tokens: int, top_k: int, rank: int, num_experts: int,
                              out_dim: int, stream=None):
    """ep_partial_combine reading ids and weights from the packed buffers."""
    import torch
    part = torch.empty(world, tokens, out_dim, dtype=torch.float32, device=v.device)
    _lib.call("objb_ep_partial_combine_packed_device", _dev_ptr(recv), _dev_ptr(v), world, tokens, top_k,
              recv.shape[1], num_experts, rank, out_dim, _dev_ptr(part), _lib.stream_handle(stream))
    return part


def router_topk_batched(d_logits, top_k: int, renormalize: bool = False, stream=None):
    """Router of T tokens: d_logits [T, E] f32 -> (ids [T, k] int32,
    weights [T, k] f32), each row as ``router_topk`` computes it."""
    import torch
    T, E = d_logits.shape
    ids = torch.empty(T, top_k, dtype=torch.int32, device=d_logits.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=d_logits.device)
    _lib.call("objb_router_topk_batched_device", _dev_ptr(d_logits), T, E, top_k, int(bool(renormalize)),
              _dev_ptr(ids), _dev_ptr(w), _lib.stream_handle(stream))
    return ids, w


def moe_pairs(layer, pair_expert, pair_token, d_x, d_v, pair_out=None, swiglu_limit: float = 0.0, stream=None,
              d_count=None):
    """v[pair_out[p]] = down_e(SwiGLU(gate_e x_t, up_e x_t)) with
    e = pair_expert[p], t = pair_token[p] (device int32 tensors); d_x [T, H],
    d_v [V, O] f32.  ``pair_out`` None writes row p.  ``d_count``: a device
    int32 with the number of pairs to run (the arrays' length is the cap)."""
    P = pair_expert.numel()
    T = d_x.shape[0]
    _lib.call("objb_moe_pairs_device", ctypes.byref(layer._c), P, _dev_ptr(d_count) if d_count is not None else None,
              _dev_ptr(pair_expert), _dev_ptr(pair_token), _dev_ptr(pair_out) if pair_out is not None else None, T,
              _dev_ptr(d_x), _dev_ptr(d_v), d_v.shape[0], float(swiglu_limit), _lib.stream_handle(stream))
    return d_v


def moe_pairs_tc(layer, pair_expert, pair_token, d_x, d_v, pair_out=None, swiglu_limit: float = 0.0, stream=None,
                 d_count=None):
    """moe_pairs for Q4_0 layers on the tensor cores (tcgen05 kind::i8):
    runs of equal experts are taken 32 pairs at a time per 256-row weight
    tile (a CTA pair).  Same arguments; pairs must be grouped by expert."""
    P = pair_expert.numel()
    T = d_x.shape[0]
    _lib.call("objb_moe_pairs_tc_device", ctypes.byref(layer._c), P,
              _dev_ptr(d_count) if d_count is not None else None, _dev_ptr(pair_expert), _dev_ptr(pair_token),
              _dev_ptr(pair_out) if pair_out is not None else None, T, _dev_ptr(d_x), _dev_ptr(d_v), d_v.shape[0],
              float(swiglu_limit), _lib.stream_handle(stream))
    return d_v


def moe_pairs_official_tc(layer, pair_expert, pair_token, d_x, d_v, pair_out=None, swiglu_limit: float = 10.0,
                          stream=None, d_count=None):
    """The official DeepSeek routed experts (act_quant -> FP8 x FP4 gate/up ->
    SwiGLU clamping up only -> act_quant -> FP8 x FP4 down) over (expert,
    token) pairs on block-scaled tensor-core MMAs; layer: a split FP4
    ``MoeLayer`` with scale tables.  Same pair arguments as ``moe_pairs``;
    pairs grouped by expert; rows unweighted."""
    P = pair_expert.numel()
    T = d_x.shape[0]
    _lib.call("objb_moe_pairs_official_tc_device", ctypes.byref(layer._c), P,
              _dev_ptr(d_count) if d_count is not None else None, _dev_ptr(pair_expert), _dev_ptr(pair_token),
              _dev_ptr(pair_out) if pair_out is not None else None, T, _dev_ptr(d_x), _dev_ptr(d_v), d_v.shape[0],
              float(swiglu_limit), _lib.stream_handle(stream))
    return d_v


# Token slots (tokens x top_k per rank) from which ExpertParallelMoe's
# "auto" mode takes the grouped tensor-core path: below this the CUDA-core
# pair programs, which stream each pair's experts straight from HBM, are
# faster (measured on B200 at hidden 2048 / intermediate 512, top-8).
GROUPED_MIN_SLOTS = 256


def grouped_supported(layer) -> bool:
    """The grouped tensor-core pairs path takes Q4_0 layers (16-byte aligned
    experts) whose hidden and intermediate sizes are multiples of 256."""
    return (int(layer.fmt) == 0 and layer._tensors[3] is None and (layer._c.flags & 1) == 0
            and layer.hidden % 256 == 0 and layer.intermediate % 256 == 0)


def moe_pairs_scratch_bytes(layer, num_pairs: int, num_tokens: int) -> int:
    n = c_size()
    _lib.call("objb_moe_pairs_scratch_bytes", ctypes.byref(layer._c), num_pairs, num_tokens, ctypes.byref(n))
    return int(n.value)


def moe_combine(d_v, slot_row, d_w, d_out, stream=None):
    """d_out[t] = sum_j d_w[t, j] * d_v[slot_row[t, j]] in slot order."""
    T, K = slot_row.shape
    _lib.call("objb_moe_combine_device", _dev_ptr(d_v), d_v.shape[0], _dev_ptr(slot_row), _dev_ptr(d_w), T, K,
              d_v.shape[1], _dev_ptr(d_out), _lib.stream_handle(stream))
    return d_out


@dataclass
class DispatchPlan:
    """Where every (token, slot) of every rank goes, computed identically on
    all ranks from the all-gathered routing table ``ids_all`` [G, T, k].

    Buffers, all grouped by peer rank in ascending order:

    * x send: this rank's tokens that need rank r (ascending token index);
    * x recv: rank s's tokens that need this rank (ascending);
    * v send: one row per pair computed here, ordered (source rank, token,
      slot); pairs are *computed* in expert order (``pair_*`` arrays) and
      written to ``pair_out``;
    * v recv: this rank's (token, slot) outputs, ordered (owner rank, token,
      slot); ``slot_row[t, j]`` is the row holding token t's slot j.
    """
    world: int
    rank: int
    experts_per_rank: int
    send_idx: np.ndarray          # [sum send_counts] token indices
    send_counts: list
    recv_counts: list
    pair_expert: np.ndarray       # [P] local expert index
    pair_token: np.ndarray        # [P] row of the x recv buffer
    pair_out: np.ndarray          # [P] row of the v send buffer
    v_send_counts: list
    v_recv_counts: list
    slot_row: np.ndarray          # [T, k] row of the v recv buffer

    @staticmethod
    def build(ids_all: np.ndarray, rank: int, world: int, num_experts: int) -> "DispatchPlan":
        ids_all = np.asarray(ids_all, dtype=np.int64)
        G, T, K = ids_all.shape
        if G != world:
            raise ValueError(f"routing table has {G} ranks, world is {world}")
        if num_experts % world:
            raise ValueError(f"num_experts {num_experts} is not divisible by world {world}")
        if ids_all.size and (ids_all.min() < 0 or ids_all.max() >= num_experts):
            raise ValueError("expert id out of range in routing table")
        epr = num_experts // world
        owner = ids_all // epr                                   # [G, T, K]
        # needs[s, t, r]: token t of rank s has a slot on rank r
        needs = np.zeros((G, T, G), dtype=bool)
        gi, ti, _ = np.indices(owner.shape)
        needs[gi.ravel(), ti.ravel(), owner.ravel()] = True
        # x send (mine) and x recv (others' tokens that need me)
        send_lists = [np.nonzero(needs[rank, :, r])[0] for r in range(G)]
        send_idx = np.concatenate(send_lists) if send_lists else np.zeros(0, np.int64)
        send_counts = [int(len(v)) for v in send_lists]
        recv_lists = [np.nonzero(needs[s, :, rank])[0] for s in range(G)]
        recv_counts = [int(len(v)) for v in recv_lists]
        # pairs computed here, in v-send order (source rank, token, slot)
        pe, pt = [], []
        v_send_counts = []
        row0 = 0
        for s in range(G):
            pos = {int(t): row0 + i for i, t in enumerate(recv_lists[s])}
            row0 += len(recv_lists[s])
            mask = owner[s] == rank                               # [T, K]
            tt, jj = np.nonzero(mask)                             # row-major: token, then slot
            pe.append(ids_all[s, tt, jj] - rank * epr)
            pt.append(np.array([pos[int(t)] for t in tt], dtype=np.int64))
            v_send_counts.append(int(len(tt)))
        pe = np.concatenate(pe) if pe else np.zeros(0, np.int64)
        pt = np.concatenate(pt) if pt else np.zeros(0, np.int64)
        out_rows = np.arange(len(pe), dtype=np.int64)
        order = np.argsort(pe, kind="stable")                     # compute grouped by expert
        # v recv: my (token, slot) outputs grouped by owner rank
        mine = owner[rank]                                        # [T, K]
        slot_row = np.zeros((T, K), dtype=np.int64)
        v_recv_counts = []
        row = 0
        for r in range(G):
            tt, jj = np.nonzero(mine == r)
            slot_row[tt, jj] = row + np.arange(len(tt))
            row += len(tt)
            v_recv_counts.append(int(len(tt)))
        return DispatchPlan(world=G, rank=rank, experts_per_rank=epr, send_idx=send_idx.astype(np.int64),
                            send_counts=send_counts, recv_counts=recv_counts,
                            pair_expert=pe[order].astype(np.int32), pair_token=pt[order].astype(np.int32),
                            pair_out=out_rows[order].astype(np.int32), v_send_counts=v_send_counts,
                            v_recv_counts=v_recv_counts, slot_row=slot_row.astype(np.int32))

    @property
    def num_pairs(self) -> int:
        return int(self.pair_expert.size)

    def exchange_bytes(self, hidden: int, out_dim: int) -> dict:
        """Bytes this rank sends to other ranks (dispatch, combine)."""
        me = self.rank
        disp = sum(c for r, c in enumerate(self.send_counts) if r != me) * hidden * 4
        comb = sum(c for s, c in enumerate(self.v_send_counts) if s != me) * out_dim * 4
        return {"dispatch": disp, "combine": comb}


class ExpertParallelMoe:
    """One MoE layer whose experts are split over the ranks of ``group``.

    ``layer``: this rank's shard, a ``MoeLayer`` holding experts
    [rank * E / G, (rank + 1) * E / G) in local order.  ``forward(x, ids, w)``
    takes this rank's T tokens (x [T, H], ids / w [T, k] from the router) and
    returns their outputs [T, O].  T must be the same on every rank.

    ``compute(plan, x_recv, n_rows) -> v_send`` and ``combine(v_recv, plan,
    w) -> out`` default to the CUDA library; tests on CPU pass their own.
    Paths:

    * one rank (default compute): on the device, bit-identical to the
      single-token launch on the CUDA-core pair programs;
    * several ranks, ``exchange="device"`` (default compute): no host round
      trip -- all-gathers of the routing table, weights and token rows, the
      pair list built on the device, pair launches with a device-side count,
      a per-rank partial combine (slot order) and one all-to-all of the
      partials, summed on the token owner in rank order.  Deterministic, and
      within the reference tolerance of the one-rank result, but the
      association of the combine depends on the rank count;
    * ``exchange="host"`` or ``plan_on_host=True`` (and any injected compute):
      the routing table goes to the host, a ``DispatchPlan`` sends only the
      needed token rows and pair outputs, and the owner combines in slot
      order -- bit-identical for any rank count.

    ``grouped``: "auto" (default) runs the pairs on the grouped tensor-core
    path (``moe_pairs_tc``) when the layer supports it and this rank's token
    slots T * k reach ``GROUPED_MIN_SLOTS``; "on" always (the layer must
    support it), "off" never.  Its rows are within the reference tolerance of
    the CUDA-core ones and, like them, depend only on (expert, token row), so
    the choice -- made from T * k, not from the rank count -- keeps results
    independent of the number of ranks."""

    def __init__(self, layer, num_experts: int, top_k: int, rank: int = 0, world: int = 1, group=None,
                 out_dim: int | None = None, compute=None, combine=None, swiglu_limit: float = 0.0,
                 plan_on_host: bool = False, exchange: str = "device", grouped: str = "auto"):
        self.layer = layer
        self.num_experts = int(num_experts)
        self.top_k = int(top_k)
        self.rank, self.world, self.group = int(rank), int(world), group
        self.out_dim = int(out_dim if out_dim is not None else layer.out_dim)
        self.swiglu_limit = float(swiglu_limit)
        self._compute = compute or self._cuda_compute
        self._combine = combine or self._cuda_combine
        self._device_only = compute is None and combine is None and not plan_on_host
        if exchange not in ("device", "host"):
            raise ValueError(f"exchange must be 'device' or 'host', not {exchange!r}")
        self._device_exchange = self._device_only and exchange == "device"
        if grouped not in ("auto", "on", "off"):
            raise ValueError(f"grouped must be 'auto', 'on' or 'off', not {grouped!r}")
        if grouped == "on" and (layer is None or not grouped_supported(layer)):
            raise ValueError("grouped='on' needs a Q4_0 layer with hidden, intermediate multiples of 256")
        self.grouped = grouped
        self.last_plan = None
        self.phase_events = None  # a list: forward() appends (phase, CUDA event) boundaries to it
        self._pin = None     # pinned int32 staging for plan arrays (grow-only)
        self._dmeta = None   # device copy (grow-only)
        self._slot_cache = {}

    def _stage(self, arrays, dev):
        """One H2D copy of the int32 plan arrays; returns device views.  The
        staging buffer is reused: the host sync of the next step's routing
        table orders the copy before any rewrite."""
        import torch
        n = sum(int(a.size) for a in arrays)
        if self._pin is None or self._pin.numel() < n:
            cap = max(1024, 1 << (n - 1).bit_length())
            self._pin = torch.empty(cap, dtype=torch.int32, pin_memory=True)
            self._dmeta = torch.empty(cap, dtype=torch.int32, device=dev)
        host = self._pin.numpy()
        off = 0
        for a in arrays:
            host[off:off + a.size] = a.ravel()
            off += a.size
        self._dmeta[:n].copy_(self._pin[:n], non_blocking=True)
        views, off = [], 0
        for a in arrays:
            views.append(self._dmeta[off:off + a.size].view(a.shape))
            off += a.size
        return views

    def _pairs_fn(self, slots: int):
        """moe_pairs or moe_pairs_tc for a step with `slots` = T * k token slots."""
        if self.grouped == "on":
            return moe_pairs_tc
        if self.grouped == "auto" and slots >= GROUPED_MIN_SLOTS and grouped_supported(self.layer):
            return moe_pairs_tc
        return moe_pairs

    # ---- default (CUDA) compute and combine
    def _cuda_compute(self, plan: DispatchPlan, x_recv, n_rows: int):
        import torch
        dev = x_recv.device
        v = torch.empty(n_rows, self.out_dim, dtype=torch.float32, device=dev)
        if plan.num_pairs == 0:
            return v
        pe, pt, po, slot = self._stage([plan.pair_expert, plan.pair_token, plan.pair_out, plan.slot_row], dev)
        self._staged_slot = slot
        self._pairs_fn(plan.slot_row.size)(self.layer, pe, pt, x_recv, v, pair_out=po,
                                           swiglu_limit=self.swiglu_limit, stream=torch.cuda.current_stream(dev))
        return v

    def _cuda_combine(self, v_recv, plan: DispatchPlan, w):
        import torch
        T, K = plan.slot_row.shape
        out = torch.empty(T, self.out_dim, dtype=torch.float32, device=w.device)
        slot = getattr(self, "_staged_slot", None)
        if slot is None or plan.num_pairs == 0:
            (slot,) = self._stage([plan.slot_row], w.device)
        self._staged_slot = None
        return moe_combine(v_recv, slot, w.contiguous(), out, stream=torch.cuda.current_stream(w.device))

    def _forward_one_rank(self, x, ids, w):
        """World size 1: no host round trip.  Pairs are the (token, slot)
        entries grouped by expert on the device (objb_ep_build_pairs_device
        with one rank: a count per expert, a scan, a scatter, one launch;
        within an expert the order is the atomics', which changes no row, as
        a pair's row depends on its expert and token alone); pair p's output
        goes to row t * k + j, which the combine reads in slot order."""
        import torch
        T, K = ids.shape
        if T == 1:
            # one token: the fused single-token launch (the pairs' rows are
            # bit-identical to it), without the sort and the separate combine
            out = torch.empty(1, self.out_dim, dtype=torch.float32, device=x.device)
            self.layer.forward_selected(ids[0].to(torch.int32).contiguous(), w[0].contiguous(), x[0].contiguous(),
                                        d_out=out[0], swiglu_limit=self.swiglu_limit,
                                        stream=torch.cuda.current_stream(x.device))
            return out
        flat = ids.reshape(-1).to(torch.int32)
        key = (T, K, x.device)
        if key not in self._slot_cache:
            self._slot_cache[key] = torch.arange(T * K, dtype=torch.int32, device=x.device).view(T, K)
        slot = self._slot_cache[key]
        stream = torch.cuda.current_stream(x.device)
        self._mark("start", stream)
        pair_expert, pair_token, perm, cnt = ep_build_pairs(flat.view(1, T, K), 0, self.num_experts, stream=stream)
        self._mark("sort", stream)
        v = torch.empty(T * K, self.out_dim, dtype=torch.float32, device=x.device)
        self._pairs_fn(T * K)(self.layer, pair_expert, pair_token, x.contiguous(), v, pair_out=perm,
                              swiglu_limit=self.swiglu_limit, stream=stream, d_count=cnt)
        self._mark("pairs", stream)
        out = torch.empty(T, self.out_dim, dtype=torch.float32, device=x.device)
        moe_combine(v, slot, w.contiguous(), out, stream=stream)
        self._mark("combine", stream)
        return out

    def _mark(self, name, stream):
        """Records a phase boundary when the step is instrumented."""
        if self.phase_events is not None:
            import torch
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            self.phase_events.append((name, ev))

    def _forward_device_exchange(self, x, ids, w):
        """One all-gather of every rank's packed step (token rows, ids,
        weights), the pair list built from it on the device, the pairs, a
        per-rank partial combine and one all-to-all of the partials."""
        import torch
        import torch.distributed as dist
        G, (T, K) = self.world, ids.shape
        H = x.shape[1]
        dev = x.device
        stream = torch.cuda.current_stream(dev)
        rows = ep_packed_rows(T, K, H)
        send = torch.empty(rows, H, dtype=torch.float32, device=dev)
        self._mark("start", stream)
        ep_pack(x.contiguous(), ids.to(torch.int32).contiguous(), w.contiguous(), send, stream=stream)
        recv = torch.empty(G * rows, H, dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(recv, send, group=self.group)
        self._mark("pack+all_gather", stream)
        pe, pt, po, cnt = ep_build_pairs_packed(recv, G, T, K, self.rank, self.num_experts, stream=stream)
        v = torch.empty(G * T * K, self.out_dim, dtype=torch.float32, device=dev)
        self._pairs_fn(T * K)(self.layer, pe, pt, recv, v, pair_out=po, swiglu_limit=self.swiglu_limit,
                              stream=stream, d_count=cnt)
        self._mark("build_pairs+pairs", stream)
        part = ep_partial_combine_packed(recv, v, G, T, K, self.rank, self.num_experts, self.out_dim, stream=stream)
        self._mark("partial_combine", stream)
        got = torch.empty_like(part)
        dist.all_to_all_single(got, part, group=self.group)
        self._mark("all_to_all", stream)
        out = ep_sum_partials(got, stream=stream)
        self._mark("sum", stream)
        return out

    # ---- the layer
    def plan(self, ids) -> DispatchPlan:
        import torch
        import torch.distributed as dist
        ids = ids.to(torch.int32).contiguous()
        if self.world > 1:
            parts = [torch.empty_like(ids) for _ in range(self.world)]
            dist.all_gather(parts, ids, group=self.group)
            ids_all = torch.stack(parts).cpu().numpy()
        else:
            ids_all = ids.cpu().numpy()[None]
        return DispatchPlan.build(ids_all, self.rank, self.world, self.num_experts)

    def forward(self, x, ids, w):
        import torch
        import torch.distributed as dist
        if self.world == 1 and self._device_only:
            self.last_plan = None
            return self._forward_one_rank(x, ids, w)
        if self._device_exchange:
            self.last_plan = None
            return self._forward_device_exchange(x, ids, w)
        plan = self.plan(ids)
        self.last_plan = plan
        H = x.shape[1]
        if self.world > 1:
            idx = torch.from_numpy(plan.send_idx).to(x.device)
            x_send = x.index_select(0, idx)
            x_recv = torch.empty(sum(plan.recv_counts), H, dtype=x.dtype, device=x.device)
            dist.all_to_all_single(x_recv, x_send, plan.recv_counts, plan.send_counts, group=self.group)
        else:
            # one rank: every token needs rank 0 and arrives in token order
            x_recv = x
        v_send = self._compute(plan, x_recv, sum(plan.v_send_counts))
        if self.world > 1:
            v_recv = torch.empty(sum(plan.v_recv_counts), self.out_dim, dtype=v_send.dtype, device=v_send.device)
            dist.all_to_all_single(v_recv, v_send, plan.v_recv_counts, plan.v_send_counts, group=self.group)
        else:
            v_recv = v_send
        return self._combine(v_recv, plan, w)


class CachedExpertCompute:
    """Per-rank compute for ``ExpertParallelMoe`` when this rank's experts
    live in host memory and reach the GPU through a ``CudaExpertCache``
    (device LRU + admission, uploads on the cache's side stream): the pairs
    of a step go to ``MoeExecutor.execute_pairs``, which resolves each
    distinct expert once.  ``experts`` are this rank's ``ExpertWeights`` in
    local order."""

    def __init__(self, executor, cache, experts, hidden: int, intermediate: int, out_dim: int, layer_id: int = 0,
                 fmt=0):
        self.executor, self.cache = executor, cache
        self.table = executor.expert_table(experts)
        self.hidden, self.intermediate, self.out_dim = int(hidden), int(intermediate), int(out_dim)
        self.layer_id, self.fmt = int(layer_id), fmt
        self.last_telemetry = None

    def __call__(self, plan: DispatchPlan, x_recv, n_rows: int):
        import torch
        v = torch.empty(n_rows, self.out_dim, dtype=torch.float32, device=x_recv.device)
        if plan.num_pairs == 0:
            return v
        self.last_telemetry = self.executor.execute_pairs(
            self.table, plan.pair_expert, plan.pair_token, x_recv.contiguous(), v, self.hidden, self.intermediate,
            self.out_dim, self.layer_id, cache=self.cache, pair_out=plan.pair_out, fmt=self.fmt,
            stream=torch.cuda.current_stream(x_recv.device))
        return v
