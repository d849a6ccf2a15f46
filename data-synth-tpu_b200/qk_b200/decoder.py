"""Synthetic MoE decoder stack: the decode step the routed FFN and the Q8 attention sit in.

The model of the stack benchmark (many layers, hidden 2048, GQA 16 query / 2 KV heads of
256 over a Q8 KV cache, 512 routed SwiGLU experts of intermediate 512 with top-10 routing
plus one always-on shared expert, all experts packed Q6_K or Q4_K). One decode step per
layer, following the reference's layer order (attention_cache.py:128-172 then
math.py:277-284 and the routed FFN, engine.py:193-204), with a plain pre-norm residual:

    h  = rms(x, attn_norm)
    q | gate, k, v = h @ [Wq; Wk; Wv]^T                       (qk_linear_bf16)
    q, k = rope(rms(q, q_norm)), rope(rms(k, k_norm))          (qk_qk_norm_rope)
    cache <- Q8(k, v) at time positions[b]                      (qk_kv_q8_append)
    o  = decode attention over the cache with the gate         (qk_kv_q8_decode_attention)
    x  = x + o @ Wo^T                     (qk_linear_bf16 + qk_residual_rms_norm)
    h2 = rms(x, ffn_norm)
    ids, w = router top-k(h2)              (qk_router_logits + qk_router_topk_logits)
    ids, w += (shared, sigmoid(h2 . w_shared_router))            (qk_append_shared_route)
    x  = x + experts(h2, ids, w)                                (qk_moe_forward, routed + shared)

Every step of a layer is one launch (the MoE call is five), the whole step is captured in a
CUDA graph, and nothing is allocated per step. Weights are synthetic: BF16 projections
N(0, 0.02), FP32 router N(0, 0.02), and expert blocks of random code bytes with one FP16
block scale chosen so the decoded values have a spread of about 0.02 (the kernels' cost does
not depend on the values). The shared expert is expert ``experts`` of the packed tensors,
routed to every row with its sigmoid gate as the route weight, so its output joins the
routed sum in FP32 before the one BF16 rounding (the reference rounds the shared and routed
parts separately and adds them in BF16).
"""

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .attention_cache import CacheConfig
from .parallel import expert_shape, put_expert_bytes
from .quant import BLOCK_LAYOUTS, GGML_TYPE, normalize_qtype


def checked_argmax(logits):
    """``run.py:46-55``: per row ``(argmax, count of non-finite logits)`` as int32 ``[B, 2]``;
    the first maximum wins and a NaN counts as the maximum (``jnp.argmax``)."""
    if logits.dim() != 2 or logits.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("logits must be a BF16 or FP32 [B, V] tensor")
    logits = logits.contiguous()
    out = torch.empty((logits.shape[0], 2), dtype=torch.int32, device=logits.device)
    code = _lib.QK_OUT_BF16 if logits.dtype == torch.bfloat16 else _lib.QK_OUT_F32
    with torch.cuda.device(logits.device):
        _lib.call("qk_checked_argmax", _lib.ptr(logits), code, logits.shape[0], logits.shape[1], _lib.ptr(out),
                  _lib.stream_handle(logits.device))
    return out


@dataclass(frozen=True)
class StackConfig:
    layers: int = 48
    hidden: int = 2048
    intermediate: int = 512
    experts: int = 512
    top_k: int = 10
    query_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 10_000_000.0
    eps: float = 1e-6
    qtype: str = "Q6_K"
    down_qtype: str | None = None  # None: the same as qtype; "Q8_0": the checkpoints' type mix
    context: int = 8192
    page: int = 256


# FP16 block-scale bytes inside one raw block and the scale giving a ~0.02 value spread:
# Q6_K d (offset 208) * int8 sub-scale * (q - 32); Q4_K d (offset 0) * 6-bit scale * q - dmin.
# Q8_0 d (offset 0) * int8 code.
_SCALE_BYTES = {"Q6_K": ((208, 2.0 ** -16),), "Q4_K": ((0, 2.0 ** -11), (2, 2.0 ** -12)),
                "Q8_0": ((0, 2.0 ** -12),)}


def synthetic_expert_bytes(qtype, count, rows, width, generator, device):
    """Raw GGUF blocks ``uint8[count, rows * blocks * block_bytes]`` of random code bytes with
    fixed FP16 block scales."""
    values, size = BLOCK_LAYOUTS[qtype]
    blocks = count * rows * (width // values)
    raw = torch.randint(0, 256, (blocks, size), dtype=torch.uint8, device=device, generator=generator)
    for offset, scale in _SCALE_BYTES[qtype]:
        bits = int(np.array([scale], np.float16).view(np.uint16)[0])
        raw[:, offset] = bits & 0xFF
        raw[:, offset + 1] = bits >> 8
    return raw.view(count, -1)


class LayerWeights:
    """One layer's weights. ``experts_here`` packed experts: all routed experts plus the
    shared one (one device), or one rank's slice of routed experts plus its own copy of the
    shared expert (expert parallel)."""

    def __init__(self, cfg, generator, device, experts_here=None, expert_generator=None):
        H, hq, kv, hd = cfg.hidden, cfg.query_heads, cfg.kv_heads, cfg.head_dim

        def normal(shape, dtype=torch.bfloat16):
            return (torch.randn(shape, device=device, generator=generator) * 0.02).to(dtype)

        self.w_qkv = normal((2 * hq * hd + 2 * kv * hd, H))
        self.w_o = normal((H, hq * hd))
        self.attn_norm = torch.ones(H, dtype=torch.bfloat16, device=device)
        self.ffn_norm = torch.ones(H, dtype=torch.bfloat16, device=device)
        self.q_norm = torch.ones(hd, dtype=torch.bfloat16, device=device)
        self.k_norm = torch.ones(hd, dtype=torch.bfloat16, device=device)
        self.router = normal((cfg.experts, H), torch.float32)
        self.shared_router = normal((H,))
        self.experts = {}
        for kind in ("gate", "up", "down"):
            qtype = normalize_qtype((cfg.down_qtype or cfg.qtype) if kind == "down" else cfg.qtype)
            rows, width = expert_shape(kind, H, cfg.intermediate)
            count = cfg.experts + 1 if experts_here is None else experts_here
            raw = synthetic_expert_bytes(qtype, count, rows, width, expert_generator or generator, device)
            self.experts[kind] = put_expert_bytes(raw, kind, qtype, H, cfg.intermediate, device=device)
            del raw

    def expert_bytes(self):
        return sum(t.numel() for t in self.experts.values()) // self.experts["gate"].shape[0]

    def dense_bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.w_qkv, self.w_o, self.router, self.shared_router))


class SyntheticDecoder:
    """All layers' weights of a :class:`StackConfig` on one device, or, with a process
    ``group`` of several ranks, one rank's part of the expert-parallel model: the dense
    weights replicated, each layer's routed experts sharded (``experts / world`` per rank,
    ``parallel.py:64-87``) plus a copy of the shared expert on every rank. Each rank then
    decodes its own sequences (attention is data parallel) and the routed FFN exchanges
    tokens through :class:`qk_b200.ep.ExpertAllToAll` (peer memory, no host synchronisation,
    graph-capturable)."""

    def __init__(self, cfg, device, seed=1, group=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        if group is None:
            self.world, self.rank = 1, 0
        else:
            import torch.distributed as dist

            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if cfg.experts % self.world:
            raise ValueError("Expert count must divide expert parallel size")
        self.per = cfg.experts // self.world
        ep = self.world > 1
        # the dense weights are the same on every rank; the expert bytes differ per rank
        g = torch.Generator(device=self.device).manual_seed(seed)
        ge = torch.Generator(device=self.device).manual_seed(seed * 1000 + 7 + self.rank)
        self.layers = [LayerWeights(cfg, g, self.device, experts_here=self.per + 1 if ep else None,
                                    expert_generator=ge if ep else None) for _ in range(cfg.layers)]
        half = cfg.rotary_dim // 2
        inv = np.power(np.float32(cfg.rope_theta), -np.arange(half, dtype=np.float32) * 2 / np.float32(cfg.rotary_dim))
        self.inv_freq = torch.from_numpy(inv.astype(np.float32)).to(self.device)
        q, qd = normalize_qtype(cfg.qtype), normalize_qtype(cfg.down_qtype or cfg.qtype)
        self.desc = _lib.MoeDesc(GGML_TYPE[q], GGML_TYPE[q], GGML_TYPE[qd], cfg.hidden, cfg.intermediate,
                                 cfg.experts + 1, 0, cfg.top_k + 1)
        self.types = (q, q, qd)

    def state(self, batch, seed=2):
        """Decode state of ``batch`` sequences on this rank (with several ranks the global
        batch is ``batch * world``; every rank must create its states in the same order)."""
        if self.world > 1:
            return DecodeState(self, batch, seed + 101 * self.rank, global_batch=batch * self.world)
        return DecodeState(self, batch, seed)


class DecodeState:
    """Per-batch state of the stack: Q8 KV caches of every layer (random codes and scales,
    every slot of the context in use), a page table of ``page``-slot pages in random order,
    and every intermediate buffer of one decode step."""

    def __init__(self, model, batch, seed, global_batch=None):
        cfg, dev = model.cfg, model.device
        self.model, self.batch = model, batch
        self.global_batch = batch if global_batch is None else global_batch
        H, hq, kv, hd, T = cfg.hidden, cfg.query_heads, cfg.kv_heads, cfg.head_dim, cfg.context
        g = torch.Generator(device=dev).manual_seed(seed)
        groups = kv * hd // 32
        self.caches = []
        for _ in range(cfg.layers):
            cache = {n: torch.randint(-127, 128, (batch, T, kv * hd), dtype=torch.int8, device=dev, generator=g)
                     for n in ("k", "v")}
            cache.update({n: (torch.rand((batch * groups, T), device=dev, generator=g) * 0.02 + 0.001)
                          .to(torch.bfloat16) for n in ("k_scale", "v_scale")})
            self.caches.append(cache)
        self.cache_config = CacheConfig(kv_heads=kv, head_dim=hd, query_heads=hq, max_context=T)
        rng = np.random.default_rng(0)
        page = cfg.page if T % cfg.page == 0 else 1  # a context that is not whole pages: no paging
        table = np.stack([rng.permutation(T // page) for _ in range(batch)]) if page > 1 else None
        slots = np.arange(T)
        order = table[:, slots // page] * page + slots % page if page > 1 else np.tile(slots, (batch, 1))
        self.indices = torch.from_numpy(np.ascontiguousarray(order.astype(np.int32))).to(dev)
        self.positions = torch.full((batch,), T - 1, dtype=torch.int32, device=dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = (torch.randn((batch, H), device=dev, generator=g)).to(torch.bfloat16)
        self.h = torch.empty((batch, H), **bf)
        self.qkv = torch.empty((batch, 2 * hq * hd + 2 * kv * hd), **bf)
        self.q = torch.empty((batch, hq, hd), **bf)
        self.gate = torch.empty((batch, hq, hd), **bf)
        self.k = torch.empty((batch, kv, hd), **bf)
        self.v = torch.empty((batch, kv, hd), **bf)
        self.o = torch.empty((batch, hq, hd), **bf)
        self.a = torch.empty((batch, H), **bf)
        self.y = torch.empty((batch, H), **bf)
        k = cfg.top_k
        self.logits = torch.empty((batch, cfg.experts), dtype=torch.float32, device=dev)
        # the attention projections: this library's tcgen05 pass up to 256 rows, a library GEMM
        # beyond (their zeroed workspaces are reused by every call)
        self.own_linear = batch <= 256
        if self.own_linear:
            from .packed import linear_workspace

            self.lin_qkv = (self.qkv.shape[1], linear_workspace(batch, H, self.qkv.shape[1], dev))
            self.lin_o = (H, linear_workspace(batch, hq * hd, H, dev))
        self.ids_all = [torch.empty((batch, k + 1), dtype=torch.int32, device=dev) for _ in range(cfg.layers)]
        self.w_all = torch.empty((batch, k + 1), **bf)
        lib = _lib.load()
        self.attn_ws_bytes = int(lib.qk_kv_q8_attention_workspace_bytes(batch, T, hq, kv, hd))
        self.attn_ws = torch.empty(max(self.attn_ws_bytes, 16), dtype=torch.uint8, device=dev)
        self.moe_ws_bytes = int(lib.qk_moe_workspace_bytes(model.desc, batch))
        self.moe_ws = torch.empty(max(self.moe_ws_bytes, 16), dtype=torch.uint8, device=dev)
        self.ep = None
        if model.world > 1:
            from .ep import ExpertAllToAll

            # every rank creates its exchange in the same order (a collective set-up)
            self.ep = ExpertAllToAll(model.group, gate_type=model.types[0], up_type=model.types[1],
                                     down_type=model.types[2], hidden=H, intermediate=cfg.intermediate,
                                     experts_per_rank=model.per + 1, top_k=k + 1, max_tokens=batch, device=dev)

    def step(self):
        """One decode step of every layer on the current stream (no allocation, capturable)."""
        cfg, m = self.model.cfg, self.model
        lib = _lib.load()
        st = _lib.stream_handle(m.device)
        P = _lib.ptr
        B, H, hq, kv, hd = self.batch, cfg.hidden, cfg.query_heads, cfg.kv_heads, cfg.head_dim
        T = cfg.context
        nl = len(m.layers)
        # the first layer's attention norm; every later one runs with the residual add before it
        _lib.check(lib.qk_rms_norm(P(self.x), P(m.layers[0].attn_norm), B, H, cfg.eps, P(self.h), st))
        for li, L in enumerate(m.layers):
            cache = self.caches[li]
            if self.own_linear:
                n, ws = self.lin_qkv
                _lib.check(lib.qk_linear_bf16(P(self.h), B, H, P(L.w_qkv), n, P(self.qkv), P(ws), ws.numel(), st))
            else:
                torch.matmul(self.h, L.w_qkv.t(), out=self.qkv)
            _lib.check(lib.qk_qk_norm_rope(P(self.qkv), P(L.q_norm), P(L.k_norm), P(m.inv_freq), P(self.positions),
                                           B, hq, kv, hd, cfg.rotary_dim, cfg.eps, P(self.q), P(self.gate), P(self.k),
                                           P(self.v), st))
            _lib.check(lib.qk_kv_q8_append(P(self.k), P(self.v), _lib.QK_OUT_BF16, P(self.positions), None,
                                           P(cache["k"]), P(cache["v"]), P(cache["k_scale"]), P(cache["v_scale"]),
                                           B, T, kv, hd, st))
            _lib.check(lib.qk_kv_q8_decode_attention(
                P(self.q), P(cache["k"]), P(cache["v"]), P(cache["k_scale"]), P(cache["v_scale"]), P(self.indices),
                None, P(self.positions), P(self.gate), B, T, T, hq, kv, hd, P(self.o),
                P(self.attn_ws) if self.attn_ws_bytes else None, self.attn_ws_bytes, st))
            if self.own_linear:
                n, ws = self.lin_o
                _lib.check(lib.qk_linear_bf16(P(self.o), B, hq * hd, P(L.w_o), n, P(self.a), P(ws), ws.numel(), st))
            else:
                torch.matmul(self.o.view(B, hq * hd), L.w_o.t(), out=self.a)
            _lib.check(lib.qk_residual_rms_norm(P(self.x), P(self.a), P(L.ffn_norm), B, H, cfg.eps, P(self.x),
                                                P(self.h), st))
            # the router's logits over ~E / 4 CTAs, then one CTA per token for the selection and
            # the shared expert's route: the ids and weights of qk_router_topk +
            # qk_append_shared_route, whose 8-CTA clusters read the whole FP32 router matrix per
            # 8 tokens
            _lib.check(lib.qk_router_logits(P(self.h), P(L.router), B, H, cfg.experts, P(self.logits), st))
            ids_all = self.ids_all[li]
            shared_id, per = (cfg.experts, 0) if self.ep is None else (m.rank * (m.per + 1) + m.per, m.per)
            _lib.check(lib.qk_router_select_shared(P(self.logits), None, B, cfg.experts, cfg.top_k, P(self.h),
                                                   P(L.shared_router), H, shared_id, per, P(ids_all),
                                                   P(self.w_all), st))
            if self.ep is None:
                _lib.check(lib.qk_moe_forward(m.desc, P(L.experts["gate"]), P(L.experts["up"]),
                                              P(L.experts["down"]), P(self.h), P(ids_all), P(self.w_all), B,
                                              _lib.QK_OUT_BF16, P(self.y), P(self.moe_ws), self.moe_ws_bytes, st))
            else:
                self.ep(L.experts["gate"], L.experts["up"], L.experts["down"], self.h, ids_all, self.w_all,
                        out=self.y)
            if li + 1 < nl:  # the residual add and the next layer's attention norm
                _lib.check(lib.qk_residual_rms_norm(P(self.x), P(self.y), P(m.layers[li + 1].attn_norm), B, H,
                                                    cfg.eps, P(self.x), P(self.h), st))
            else:
                _lib.check(lib.qk_residual_add(P(self.x), P(self.y), B * H, P(self.x), st))
        return self.x

    def launches_per_step(self):
        # per layer: norm/rope, append, attention (split + merge when split), residual + FFN
        # norm, router logits, router selection + shared route, MoE (route, dispatch, gate/up,
        # down, combine; expert parallel: dispatch, wait, route, dispatch, gate/up, down,
        # combine-and-return, final combine), residual (+ the next layer's attention norm);
        # the first layer's attention norm; the 2 projections per layer (this library's, or
        # library GEMMs above 256 rows)
        attn = 2 if self.attn_ws_bytes else 1
        moe = 5 if self.ep is None else 8
        own = 2 if self.own_linear else 0
        return self.model.cfg.layers * (6 + attn + moe + own) + 1, self.model.cfg.layers * (2 - own)

    def close(self):
        if self.ep is not None:
            self.ep.close()
            self.ep = None

    def step_bytes(self):
        """Algorithmic HBM bytes of the last step on this rank: the distinct experts each layer
        routed to (shared included; with several ranks, of this rank's tokens) times their
        packed bytes, the dense weights, and the KV cache (codes and BF16 scales of every
        attended slot)."""
        cfg = self.model.cfg
        total, distinct = 0, []
        for li, L in enumerate(self.model.layers):
            n = int(torch.unique(self.ids_all[li]).numel())
            distinct.append(n)
            total += n * L.expert_bytes() + L.dense_bytes()
        kv_slot = 2 * cfg.kv_heads * cfg.head_dim + 2 * 2 * cfg.kv_heads * cfg.head_dim // 32
        total += cfg.layers * self.batch * cfg.context * kv_slot
        return total, distinct
