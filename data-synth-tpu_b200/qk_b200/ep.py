"""Expert parallelism with token dispatch.

Two forms of the same layer. ``ExpertAllToAll`` (the product path) moves tokens and
partial outputs through peer memory over NVLink with no host synchronisation
(``qk_ep_p2p_*``, ``csrc/ep_p2p.cu``). ``ExpertAllToAllNccl`` (below) is the variable-size
NCCL all-to-all form, whose split sizes are read back to the host every call.

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

    fn = ExpertAllToAllNccl(group, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K",
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


class ExpertAllToAllNccl:
    """Routed expert FFN with token dispatch over NCCL all-to-all; see the module docstring.
    Each call reads the per-rank send counts back to the host (two synchronisations), so it
    cannot be captured in a CUDA graph; ``ExpertAllToAll`` has neither limitation."""

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


class ExchangeRegion:
    """This rank's exchange region of the peer-to-peer layer and the table of every rank's
    region as mapped in this process (CUDA IPC handles exchanged over ``group``).

    ``regions``/``rank`` instead of ``group``: ranks emulated in one process on one device
    (test infrastructure), every region already allocated here."""

    def __init__(self, group, *, max_tokens, hidden, top_k, device, world=None, rank=None,
                 shared=None):
        import ctypes

        self.device = torch.device(device)
        lib = _lib.load()
        if shared is not None:
            world, rank = shared["world"], rank
        elif group is None:
            world, rank = 1, 0
        else:
            import torch.distributed as dist

            world, rank = dist.get_world_size(group), dist.get_rank(group)
        self.world, self.rank = world, rank
        self.max_tokens, self.hidden, self.top_k = max_tokens, hidden, top_k
        self.bytes = int(lib.qk_ep_p2p_bytes(world, max_tokens, hidden, top_k))
        if self.bytes == 0:
            raise ValueError("bad exchange geometry")
        self._opened = []
        self._owned = None
        with torch.cuda.device(self.device):
            if shared is not None:
                self.base = shared["regions"][rank]
                bases = shared["regions"]
            else:
                ptr = ctypes.c_void_p()
                _lib.check(lib.qk_device_alloc(self.bytes, ctypes.byref(ptr)))
                self._owned = ptr.value
                self.base = ptr.value
                _lib.check(lib.qk_ep_p2p_reset(ctypes.c_void_p(self.base), _lib.stream_handle(self.device)))
                torch.cuda.synchronize(self.device)
                bases = [None] * world
                bases[rank] = self.base
                if world > 1:
                    import torch.distributed as dist

                    handle = (ctypes.c_uint8 * 64)()
                    _lib.check(lib.qk_ipc_get_handle(ctypes.c_void_p(self.base), handle))
                    handles = [None] * world
                    dist.all_gather_object(handles, bytes(handle), group=group)
                    for r in range(world):
                        if r == rank:
                            continue
                        p = ctypes.c_void_p()
                        buf = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
                        _lib.check(lib.qk_ipc_open_handle(buf, ctypes.byref(p)))
                        self._opened.append(p.value)
                        bases[r] = p.value
                    # every region is cleared before any peer may write into it
                    dist.barrier(group=group)
            self.peers = torch.tensor(bases, dtype=torch.int64, device=self.device)

    @property
    def region(self):
        import ctypes

        return ctypes.c_void_p(self.base)

    def status(self):
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().qk_ep_p2p_status(self.region, _lib.stream_handle(self.device)))

    def close(self):
        import ctypes

        lib = _lib.load()
        for p in self._opened:
            lib.qk_ipc_close_handle(ctypes.c_void_p(p))
        self._opened = []
        if self._owned is not None:
            lib.qk_device_free(ctypes.c_void_p(self._owned))
            self._owned = None


class ExpertAllToAll:
    """Routed expert FFN with token dispatch over peer memory (``csrc/ep_p2p.cu``).

    Rank r of ``group`` holds experts ``[r * experts_per_rank, (r + 1) * experts_per_rank)``
    (``parallel.py:64-87``) and its own tokens (at most ``max_tokens`` per call). A call is
    three launches' worth of stream-ordered work on every rank, none of which waits for
    the host: each token row goes once to every rank that owns one of its experts; the
    owner runs its experts and returns the token's FP32 partial sum (ascending expert
    order); the source adds the partials in ascending rank order and rounds to BF16. That
    is the reference's expert-parallel arithmetic (local sum, ``psum``, cast;
    ``experts.py:128-131``); with one rank it is bit-identical to ``expert_parallel``.

    Every rank must make the same sequence of calls. The output is a view of a buffer the
    layer owns (valid until its next call) unless ``out`` is given."""

    def __init__(self, group, *, gate_type, up_type, down_type, hidden, intermediate,
                 experts_per_rank, top_k, max_tokens, device=None, region=None):
        self.types = tuple(normalize_qtype(t) for t in (gate_type, up_type, down_type))
        self.hidden, self.intermediate = hidden, intermediate
        self.experts_per_rank, self.top_k, self.max_tokens = experts_per_rank, top_k, max_tokens
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.region = region or ExchangeRegion(group, max_tokens=max_tokens, hidden=hidden,
                                               top_k=top_k, device=self.device)
        self.world, self.rank = self.region.world, self.region.rank
        self.desc = _lib.MoeDesc(*(GGML_TYPE[t] for t in self.types), hidden, intermediate,
                                 experts_per_rank, self.rank * experts_per_rank, top_k)
        need = int(_lib.load().qk_moe_workspace_bytes(self.desc, self.world * max_tokens))
        self.workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=self.device)
        self.out = torch.empty((max_tokens, hidden), dtype=torch.bfloat16, device=self.device)

    def __call__(self, gate, up, down, x, ids, weights, out=None):
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise TypeError("x must be a [B, hidden] tensor")
        B = x.shape[0]
        if ids.shape != (B, self.top_k) or weights.shape != ids.shape:
            raise ValueError("ids and weights must be [B, top_k]")
        if B > self.max_tokens:
            raise ValueError(f"batch {B} exceeds max_tokens {self.max_tokens}")
        if gate.shape[0] != self.experts_per_rank:
            raise ValueError("gate, up and down must hold this rank's experts_per_rank experts")
        if ids.dtype != torch.int32 or weights.dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
            raise TypeError("x and weights must be bfloat16, ids int32")
        out = self.out[:B] if out is None else out
        lib = _lib.load()
        st = _lib.stream_handle(self.device)
        peers, region = _lib.ptr(self.region.peers), self.region.region
        _lib.check(lib.qk_ep_p2p_dispatch(peers, region, self.world, self.rank, self.max_tokens,
                                          self.hidden, self.top_k, self.experts_per_rank,
                                          _lib.ptr(x), _lib.ptr(ids), _lib.ptr(weights), B, st))
        _lib.check(lib.qk_ep_p2p_expert(self.desc, _lib.ptr(gate), _lib.ptr(up), _lib.ptr(down),
                                        peers, region, self.world, self.rank, self.max_tokens,
                                        _lib.ptr(self.workspace), self.workspace.numel(), st))
        _lib.check(lib.qk_ep_p2p_combine(region, self.world, self.rank, self.max_tokens,
                                         self.hidden, self.top_k, self.experts_per_rank,
                                         _lib.ptr(ids), _lib.ptr(weights), B, _lib.ptr(out), st))
        return out

    def check_status(self):
        """Raise if a bounded wait on a peer gave up (synchronises the stream)."""
        self.region.status()
        _lib.call("qk_moe_check", _lib.ptr(self.workspace), _lib.stream_handle(self.device))

    def close(self):
        self.region.close()


__all__ = ["ExpertAllToAll", "ExpertAllToAllNccl", "ExchangeRegion", "DeviceOps", "Plan"]
