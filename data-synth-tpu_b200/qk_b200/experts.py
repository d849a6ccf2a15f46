"""Routed expert FFN over packed expert weights (replaces ``qwen38_tpu/experts.py:17-140``).

``expert_parallel(group, *, gate_type, up_type, down_type, hidden, intermediate, ...)``
returns ``fn(gate, up, down, x, ids, weights) -> bf16[B, hidden]`` with the reference's
positional order (``engine.py:199-201``). ``gate``/``up``/``down`` are this rank's
device-resident tiled expert tensors from :func:`parallel.put_expert_bytes`; ``x`` is
BF16 ``[B, hidden]``, ``ids`` int32 ``[B, k]``, ``weights`` BF16 ``[B, k]``, all replicated
across ranks as in the reference's ``P()`` in_specs.

Single GPU: one ``qk_moe_forward`` call writes the BF16 output. Expert parallel over a
``torch.distributed`` group (NCCL): each rank writes the FP32 sum over its own experts,
an all-reduce adds the ranks (``experts.py:130-131``, ``psum(out, "expert")``) and
``qk_cast_f32_bf16`` casts the sum to BF16.
"""

import torch

from . import _lib
from .parallel import expert_shape
from .quant import GGML_TYPE, normalize_qtype

EXPERT_ROW_TILE = 128


class ExpertFFN:
    def __init__(self, group, gate_type, up_type, down_type, hidden, intermediate, tensor_parallel=1,
                 compute="bf16"):
        self.group = group
        self.types = tuple(normalize_qtype(t) for t in (gate_type, up_type, down_type))
        self.hidden = hidden
        self.intermediate = intermediate
        self.tensor_parallel = tensor_parallel
        self.compute = compute
        self._workspace = {}
        self.tensor_group = self.expert_group = None
        self.expert_rank = 0
        if tensor_parallel > 1 and group is not None:
            self._mesh_groups()

    def _mesh_groups(self):
        """The ("expert", "tensor") mesh of parallel.py:28-33 over `group`: rank = e * tp + t.
        The tensor group of a rank is the tp ranks holding slices of its experts; the expert
        group is the ranks holding the same slice of the other experts. Every rank builds
        every group (torch.distributed.new_group is collective)."""
        import torch.distributed as dist

        tp = self.tensor_parallel
        ranks = dist.get_process_group_ranks(self.group)
        me = dist.get_rank(self.group)
        ep = len(ranks) // tp
        self.expert_rank = me // tp
        if ep == 1:
            self.tensor_group = self.group
            return
        for e in range(ep):
            g = dist.new_group([ranks[e * tp + t] for t in range(tp)])
            if e == me // tp:
                self.tensor_group = g
        for t in range(tp):
            g = dist.new_group([ranks[e * tp + t] for e in range(ep)])
            if t == me % tp:
                self.expert_group = g

    def _rank_world(self):
        if self.group is None:
            return 0, 1
        import torch.distributed as dist

        return dist.get_rank(self.group), dist.get_world_size(self.group)

    def desc(self, num_experts, first_expert, top_k):
        return _lib.MoeDesc(
            GGML_TYPE[self.types[0]], GGML_TYPE[self.types[1]], GGML_TYPE[self.types[2]],
            self.hidden, self.intermediate // self.tensor_parallel, num_experts, first_expert, top_k,
            _lib.QK_COMPUTE_INT8_Q8 if self.compute == "int8_q8" else _lib.QK_COMPUTE_BF16,
        )

    def workspace(self, desc, batch, device):
        need = int(_lib.load().qk_moe_workspace_bytes(desc, batch))
        key = (device.index, desc.num_experts, desc.top_k, desc.compute)
        buf = self._workspace.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.empty(max(need, 1), dtype=torch.uint8, device=device)
            self._workspace[key] = buf
        return buf

    def _check(self, gate, up, down, x, ids, weights):
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != self.hidden:
            raise TypeError("x must be a BF16 [B, hidden] tensor")
        if ids.dim() != 2 or ids.shape[0] != x.shape[0] or weights.shape != ids.shape:
            raise ValueError("ids and weights must be [B, top_k]")
        count = gate.shape[0]
        if up.shape[0] != count or down.shape[0] != count:
            raise ValueError("gate, up and down must hold the same experts")

    def partial(self, gate, up, down, x, ids, weights, first_expert=None):
        """FP32 ``[B, hidden]`` sum over this rank's experts (before the all-reduce)."""
        return self._run(gate, up, down, x, ids, weights, first_expert, torch.float32)

    def _run(self, gate, up, down, x, ids, weights, first_expert, out_dtype):
        self._check(gate, up, down, x, ids, weights)
        rank, _ = self._rank_world()
        count = gate.shape[0]
        first = rank * count if first_expert is None else first_expert
        batch, top_k = ids.shape
        desc = self.desc(count, first, top_k)
        device = x.device
        ws = self.workspace(desc, batch, device)
        x = x.contiguous()
        ids = ids.to(torch.int32).contiguous()
        weights = weights.to(torch.bfloat16).contiguous()
        out = torch.empty((batch, self.hidden), dtype=out_dtype, device=device)
        with torch.cuda.device(device):
            _lib.call(
                "qk_moe_forward", desc, _lib.ptr(gate), _lib.ptr(up), _lib.ptr(down),
                _lib.ptr(x), _lib.ptr(ids), _lib.ptr(weights), batch,
                _lib.QK_OUT_BF16 if out_dtype == torch.bfloat16 else _lib.QK_OUT_F32,
                _lib.ptr(out), _lib.ptr(ws), ws.numel(), _lib.stream_handle(device),
            )
        self.last_workspace = ws
        return out

    def tensor_partial(self, gate, up, down, x, ids, weights, first_expert=0):
        """Tensor parallel, first half: this rank's slice of its experts [first_expert,
        first_expert + E_local); returns the FP32 down projection of every route ``[B * k,
        hidden]`` (before the tensor all-reduce) and the workspace the combine reads."""
        self._check(gate, up, down, x, ids, weights)
        batch, top_k = ids.shape
        desc = self.desc(gate.shape[0], first_expert, top_k)
        device = x.device
        ws = self.workspace(desc, batch, device)
        x = x.contiguous()
        ids = ids.to(torch.int32).contiguous()
        weights = weights.to(torch.bfloat16).contiguous()
        y_routes = torch.empty((batch * top_k, self.hidden), dtype=torch.float32, device=device)
        with torch.cuda.device(device):
            _lib.call("qk_moe_forward_tp_partial", desc, _lib.ptr(gate), _lib.ptr(up), _lib.ptr(down),
                      _lib.ptr(x), _lib.ptr(ids), _lib.ptr(weights), batch, _lib.ptr(y_routes), _lib.ptr(ws),
                      ws.numel(), _lib.stream_handle(device))
        self.last_workspace = ws
        return y_routes, ids, ws

    def tensor_combine(self, y_routes, ids, ws, num_experts, out_dtype=torch.bfloat16):
        """Tensor parallel, second half: BF16 of each route's summed down projection,
        route-weighted and added in ascending expert order; BF16, or the FP32 sum that an
        expert-parallel all-reduce adds (``out_dtype=torch.float32``)."""
        batch, top_k = ids.shape
        desc = self.desc(num_experts, 0, top_k)
        out = torch.empty((batch, self.hidden), dtype=out_dtype, device=ids.device)
        code = _lib.QK_OUT_BF16 if out_dtype == torch.bfloat16 else _lib.QK_OUT_F32
        with torch.cuda.device(ids.device):
            _lib.call("qk_moe_forward_tp_combine", desc, _lib.ptr(y_routes), _lib.ptr(ids), batch,
                      code, _lib.ptr(out), _lib.ptr(ws), ws.numel(), _lib.stream_handle(ids.device))
        return out

    def _cast_bf16(self, partial):
        out = torch.empty(partial.shape, dtype=torch.bfloat16, device=partial.device)
        with torch.cuda.device(partial.device):
            _lib.call("qk_cast_f32_bf16", _lib.ptr(partial), _lib.ptr(out), partial.numel(),
                      _lib.stream_handle(partial.device))
        return out

    def __call__(self, gate, up, down, x, ids, weights):
        rank, world = self._rank_world()
        if self.tensor_parallel > 1:
            import torch.distributed as dist

            count = gate.shape[0]
            y_routes, ids32, ws = self.tensor_partial(gate, up, down, x, ids, weights,
                                                      self.expert_rank * count)
            dist.all_reduce(y_routes, group=self.tensor_group)  # grouped_experts.py:113-118
            if self.expert_group is None:
                return self.tensor_combine(y_routes, ids32, ws, count)
            partial = self.tensor_combine(y_routes, ids32, ws, count, torch.float32)
            dist.all_reduce(partial, group=self.expert_group)  # experts.py:130-131
            return self._cast_bf16(partial)
        if world == 1:
            return self._run(gate, up, down, x, ids, weights, None, torch.bfloat16)
        import torch.distributed as dist

        partial = self._run(gate, up, down, x, ids, weights, None, torch.float32)
        dist.all_reduce(partial, group=self.group)
        return self._cast_bf16(partial)

    def check_status(self):
        """Raise if a bounded device wait of the last call gave up (synchronises)."""
        ws = getattr(self, "last_workspace", None)
        if ws is not None:
            with torch.cuda.device(ws.device):
                _lib.call("qk_moe_check", _lib.ptr(ws), _lib.stream_handle(ws.device))


def expert_parallel(
    group=None,
    *,
    gate_type,
    up_type,
    down_type,
    hidden,
    intermediate,
    compute="bf16",
    row_tile=EXPERT_ROW_TILE,
    group_size=1,
    tensor_parallel=1,
):
    """Return the routed FFN for this process's experts; see the module docstring.

    ``compute`` "int8_q8" only changes Q8_0 projections, as in the reference
    (qwen38_tpu/experts.py:85-99): a Q8_0 down projection becomes the W8A8 integer dot of
    qwen38_tpu/compute.py:20-34 (activations quantised per 32 values, tcgen05 kind::i8 MMAs,
    FP32 scaled sum over the groups; the call then uses 32-token chunks); the k-quant gate
    and up projections compute exactly like "bf16". ``row_tile`` and
    ``group_size`` shape the reference's XLA loops and do not change results; they are
    validated and otherwise unused (the kernels tile rows by 32 and stream experts).
    """
    if compute not in {"bf16", "int8_q8"}:
        raise ValueError("Unknown expert compute policy")
    if row_tile is not None and (type(row_tile) is not int or row_tile < 1):
        raise ValueError("Expert row tile must be a positive integer or None")
    if type(group_size) is not int or group_size < 1:
        raise ValueError("Expert group size must be a positive integer")
    if type(tensor_parallel) is not int or tensor_parallel < 1:
        raise ValueError("Tensor parallel size must divide the device count")
    if tensor_parallel > 1:
        # the ("expert", "tensor") mesh of parallel.py:28-33 over `group`: rank e * tp + t holds
        # tensor slice t of expert range e (put_expert_bytes(..., rank=e, world=ep,
        # tensor_rank=t, tensor_parallel=tp))
        if group is None:
            raise ValueError("tensor parallel experts need a process group")
        import torch.distributed as dist

        if dist.get_world_size(group) % tensor_parallel:
            raise ValueError("Tensor parallel size must divide the device count")
    types = tuple(normalize_qtype(t) for t in (gate_type, up_type, down_type))
    if (types[0] != types[1] or types[0] not in ("Q6_K", "Q4_K", "Q5_K")
            or types[2] not in ("Q6_K", "Q4_K", "Q8_0", "Q5_1")):
        raise ValueError("expert kernels take gate and up both Q6_K, Q4_K or Q5_K, down Q6_K, Q4_K, Q8_0 or Q5_1")
    # the down projection reads whole GGUF blocks of intermediate (gate/up tiles pad rows to 64)
    step = 32 if types[2] in ("Q8_0", "Q5_1") else 256
    if tensor_parallel > 1 and ((intermediate // tensor_parallel) % step or intermediate % tensor_parallel):
        raise ValueError("Tensor slices must contain whole down quantization blocks")
    if hidden % 256 or intermediate % step:
        raise ValueError(f"hidden must be a multiple of 256 and intermediate a multiple of {step}")
    return ExpertFFN(group, *types, hidden, intermediate, tensor_parallel, compute)


__all__ = ["ExpertFFN", "expert_parallel", "expert_shape", "EXPERT_ROW_TILE"]
