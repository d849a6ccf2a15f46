"""Expert parallelism with token dispatch over ``torch.distributed`` all-to-all (NCCL).

The reference's expert-parallel layer replicates every token on every rank and adds the
ranks' partial outputs with a ``psum`` (``qwen38_tpu/experts.py:130-131``, placement
``parallel.py:64-87``); :func:`qk_b200.experts.expert_parallel` keeps that form. This
module is the dispatch form of the same layer: each rank holds its own tokens and a
contiguous range of ``experts_per_rank`` experts, sends every route's token row to the
rank that owns the expert, runs its experts on what it receives, sends the expert outputs
back, and combines them per token in ascending expert order in FP32
(``experts.py:66-76,129-131``). The result equals the single-device layer on the same
tokens. Per layer it moves ``routes * hidden * 2`` bytes each way over NVLink instead of
all-reducing ``tokens * hidden * 4`` bytes.

    fn = ExpertAllToAll(group, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K",
                        hidden=2048, intermediate=512, experts_per_rank=E // world)
    out = fn(gate, up, down, x, ids, weights)   # this rank's tokens -> bf16 [B, hidden]

``ops`` carries the four local steps; the default uses this library's kernels
(``qk_ep_plan``, ``qk_gather_rows``, ``qk_moe_forward`` with top_k 1, ``qk_ep_combine``).
"""

from dataclasses import dataclass

import torch

from . import _lib
from .quant import GGML_TYPE, normalize_qtype


@dataclass
class Plan:
    send_counts: torch.Tensor   # int32 [world]
    send_rows: torch.Tensor     # int32 [B * k]: token of each send slot (rank-major)
    send_expert: torch.Tensor   # int32 [B * k]: global expert of each send slot
    route_slot: torch.Tensor    # int32 [B, k]: send slot of route (b, j), or -1
    route_weight: torch.Tensor  # float32 [B, k]: merged route weight (0 when dropped)


class DeviceOps:
    """The local steps on the GPU through the C ABI."""

    def __init__(self, types, hidden, intermediate):
        self.types = types
        self.hidden = hidden
        self.intermediate = intermediate
        self._ws = {}

    def plan(self, ids, weights, experts_per_rank, world):
        B, k = ids.shape
        dev = ids.device
        p = Plan(torch.empty(world, dtype=torch.int32, device=dev),
                 torch.empty(max(B * k, 1), dtype=torch.int32, device=dev),
                 torch.empty(max(B * k, 1), dtype=torch.int32, device=dev),
                 torch.empty((B, k), dtype=torch.int32, device=dev),
                 torch.empty((B, k), dtype=torch.float32, device=dev))
        _lib.call("qk_ep_plan", _lib.ptr(ids), _lib.ptr(weights), B, k, experts_per_rank, world,
                  _lib.ptr(p.send_counts), _lib.ptr(p.send_rows), _lib.ptr(p.send_expert),
                  _lib.ptr(p.route_slot), _lib.ptr(p.route_weight), _lib.stream_handle(dev))
        return p

    def gather(self, x, rows):
        out = torch.empty((rows.numel(), x.shape[1]), dtype=x.dtype, device=x.device)
        if rows.numel():
            _lib.call("qk_gather_rows", _lib.ptr(x), _lib.ptr(rows), rows.numel(), x.shape[1],
                      _lib.ptr(out), _lib.stream_handle(x.device))
        return out

    def local_ffn(self, gate, up, down, x, experts, first_expert):
        """bf16(h Wd^T) of each received row for its (global) expert: qk_moe_forward with
        top_k 1 and route weight 1, whose combine returns the expert output unchanged."""
        n = x.shape[0]
        out = torch.empty((n, self.hidden), dtype=torch.bfloat16, device=x.device)
        if n == 0:
            return out
        desc = _lib.MoeDesc(*(GGML_TYPE[t] for t in self.types), self.hidden, self.intermediate,
                            gate.shape[0], first_expert, 1)
        need = int(_lib.load().qk_moe_workspace_bytes(desc, n))
        key = x.device.index
        ws = self._ws.get(key)
        if ws is None or ws.numel() < need:
            ws = self._ws[key] = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        ones = torch.ones((n, 1), dtype=torch.bfloat16, device=x.device)
        ids = experts.to(torch.int32).reshape(n, 1).contiguous()
        _lib.call("qk_moe_forward", desc, _lib.ptr(gate), _lib.ptr(up), _lib.ptr(down), _lib.ptr(x),
                  _lib.ptr(ids), _lib.ptr(ones), n, _lib.QK_OUT_BF16, _lib.ptr(out), _lib.ptr(ws),
                  ws.numel(), _lib.stream_handle(x.device))
        return out

    def combine(self, y, plan, ids, hidden):
        B, k = ids.shape
        out = torch.empty((B, hidden), dtype=torch.bfloat16, device=ids.device)
        _lib.call("qk_ep_combine", _lib.ptr(y) if y.numel() else None, _lib.ptr(plan.route_slot),
                  _lib.ptr(ids), _lib.ptr(plan.route_weight), B, k, hidden, _lib.QK_OUT_BF16,
                  _lib.ptr(out), _lib.stream_handle(ids.device))
        return out


class ExpertAllToAll:
    """Routed expert FFN with token dispatch; see the module docstring."""

    def __init__(self, group, *, gate_type, up_type, down_type, hidden, intermediate,
                 experts_per_rank, ops=None):
        self.group = group
        self.types = tuple(normalize_qtype(t) for t in (gate_type, up_type, down_type))
        self.hidden = hidden
        self.intermediate = intermediate
        self.experts_per_rank = experts_per_rank
        self.ops = ops or DeviceOps(self.types, hidden, intermediate)

    def _rank_world(self):
        if self.group is None:
            return 0, 1
        import torch.distributed as dist

        return dist.get_rank(self.group), dist.get_world_size(self.group)

    def _all_to_all(self, out, inp, out_splits, in_splits):
        if self.group is None:
            out.copy_(inp)
            return
        import torch.distributed as dist

        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def __call__(self, gate, up, down, x, ids, weights):
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise TypeError("x must be a [B, hidden] tensor")
        if ids.dim() != 2 or ids.shape[0] != x.shape[0] or weights.shape != ids.shape:
            raise ValueError("ids and weights must be [B, top_k]")
        if gate.shape[0] != self.experts_per_rank:
            raise ValueError("gate, up and down must hold this rank's experts_per_rank experts")
        rank, world = self._rank_world()
        x = x.contiguous()
        ids = ids.to(torch.int32).contiguous()
        weights = weights.contiguous()
        plan = self.ops.plan(ids, weights, self.experts_per_rank, world)
        # counts: every rank learns how many rows each peer sends it
        recv_counts = torch.empty_like(plan.send_counts)
        self._all_to_all(recv_counts, plan.send_counts, None, None)
        send_splits = [int(c) for c in plan.send_counts.cpu()]
        recv_splits = [int(c) for c in recv_counts.cpu()]
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        # dispatch: token rows and their expert ids to the owning ranks
        x_send = self.ops.gather(x, plan.send_rows[:n_send])
        x_recv = x.new_empty((n_recv, self.hidden))
        self._all_to_all(x_recv, x_send, recv_splits, send_splits)
        e_recv = plan.send_expert.new_empty(n_recv)
        self._all_to_all(e_recv, plan.send_expert[:n_send].contiguous(), recv_splits, send_splits)
        # this rank's experts on the received rows, then the outputs back to their tokens
        y_recv = self.ops.local_ffn(gate, up, down, x_recv, e_recv, rank * self.experts_per_rank)
        y_send = y_recv.new_empty((n_send, self.hidden))
        self._all_to_all(y_send, y_recv, send_splits, recv_splits)
        return self.ops.combine(y_send, plan, ids, self.hidden)


__all__ = ["ExpertAllToAll", "DeviceOps", "Plan"]
