"""Batched static generation over the synthetic decoder stack: a prompt prefill, then greedy
decode steps (``qwen38_tpu/run.py:194`` ``prefill`` and ``:251`` ``generate``).

A :class:`StaticGeneration` holds a batch of sequences on one rank of a
:class:`~qk_b200.decoder.SyntheticDecoder` (the whole model on one GPU, or this rank's
share of the expert-parallel model):

* **Prefill** (``engine.py:449-500`` ``forward_chunk``): the whole prompt of every sequence
  is one chunk of ``batch * prompt`` tokens. Per layer: RMSNorm, the q | gate, k, v
  projection (cuBLAS), per-head q/k RMSNorm and rotary at each token's position
  (``qk_qk_norm_rope``), the chunk's keys and values quantised into the Q8 cache
  (``qk_kv_q8_append_chunk``), causal attention of the chunk over the dequantised cache
  (``qk_kv_q8_read`` feeding PyTorch's fused attention; the cache's own keys and values, as
  ``attention_cache.py:152-170`` reads them), the sigmoid output gate, the output
  projection and the residual; then the routed FFN with the shared expert over all
  ``batch * prompt`` tokens (``qk_moe_forward``: at these sizes its prefill form, 256 tokens
  per chunk, with both MMA operands in shared memory) or, expert parallel, through
  :class:`~qk_b200.ep.ExpertAllToAll`.
* **Logits and greedy choice**: the last prompt token's hidden state, the final RMSNorm, the
  tied embedding as output head (cuBLAS) and ``checked_argmax`` (``run.py:46-55``).
* **Decode**: one CUDA-graph replay per step - the chosen tokens' embeddings, every layer's
  decode step (:meth:`DecodeState.step`, Q8 cache append at the step's position and decode
  attention over all slots up to it), logits and ``checked_argmax``; the step's position
  advances on the device, so the graph is captured once.

The embedding table is ``N(0, 0.02)`` (seed 0 + 3), prompt ids uniform over the vocabulary
(seed 0); everything else is the decoder's synthetic weights.
"""

import numpy as np
import torch

from . import _lib
from .decoder import checked_argmax


class StaticGeneration:
    def __init__(self, model, batch, prompt, new_tokens, vocab=151936, seed=0):
        cfg, dev = model.cfg, model.device
        if prompt + new_tokens > cfg.context:
            raise ValueError("prompt + new tokens exceed the model's cache context")
        self.model, self.batch, self.prompt, self.new_tokens, self.vocab = model, batch, prompt, new_tokens, vocab
        H = cfg.hidden
        g = torch.Generator(device=dev).manual_seed(seed + 3)
        self.embedding = (torch.randn((vocab, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.final_norm = torch.ones(H, dtype=torch.bfloat16, device=dev)
        rng = np.random.default_rng([seed, model.rank])
        self.prompt_ids = torch.from_numpy(rng.integers(0, vocab, (batch, prompt)).astype(np.int64)).to(dev)
        self.state = model.state(batch, seed=2)
        st = self.state
        T = cfg.context
        # real generation writes and reads the same logical slots: identity page table
        st.indices.copy_(torch.arange(T, dtype=torch.int32, device=dev).expand(batch, T))
        self.generated = torch.zeros((batch, new_tokens), dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.logits = torch.empty((batch, vocab), dtype=torch.bfloat16, device=dev)
        self.hn = torch.empty((batch, H), dtype=torch.bfloat16, device=dev)
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=dev)
        self._prefill_ep = None
        self._graph = None
        self.moe_events = None  # optional: 5 CUDA events around the last layer's prefill MoE stages

    # ---- prefill --------------------------------------------------------------------
    def prefill(self):
        """Run the prompt through every layer and choose the first new token."""
        m, cfg, st = self.model, self.model.cfg, self.state
        dev = m.device
        lib = _lib.load()
        s = _lib.stream_handle(dev)
        P = _lib.ptr
        B, W, H = self.batch, self.prompt, cfg.hidden
        hq, kv, hd, T = cfg.query_heads, cfg.kv_heads, cfg.head_dim, cfg.context
        n = B * W
        bf = dict(dtype=torch.bfloat16, device=dev)
        x = self.embedding.index_select(0, self.prompt_ids.reshape(-1))  # [B * W, H]
        h = torch.empty((n, H), **bf)
        qkv = torch.empty((n, 2 * hq * hd + 2 * kv * hd), **bf)
        q = torch.empty((n, hq, hd), **bf)
        gate = torch.empty((n, hq, hd), **bf)
        k = torch.empty((n, kv, hd), **bf)
        v = torch.empty((n, kv, hd), **bf)
        a = torch.empty((n, H), **bf)
        y = torch.empty((n, H), **bf)
        ids = torch.empty((n, cfg.top_k), dtype=torch.int32, device=dev)
        w = torch.empty((n, cfg.top_k), **bf)
        ids_all = torch.empty((n, cfg.top_k + 1), dtype=torch.int32, device=dev)
        w_all = torch.empty((n, cfg.top_k + 1), **bf)
        positions = torch.arange(W, dtype=torch.int32, device=dev).repeat(B)
        start = torch.zeros(B, dtype=torch.int32, device=dev)
        read_idx = torch.arange(W, dtype=torch.int32, device=dev).expand(B, W).contiguous()
        kd = torch.empty((B, W, kv * hd), **bf)
        vd = torch.empty((B, W, kv * hd), **bf)
        if m.world == 1:
            need = int(lib.qk_moe_workspace_bytes(m.desc, n))
            ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
        else:
            from .ep import ExpertAllToAll

            if self._prefill_ep is None:
                self._prefill_ep = ExpertAllToAll(m.group, gate_type=m.types[0], up_type=m.types[1],
                                                  down_type=m.types[2], hidden=H, intermediate=cfg.intermediate,
                                                  experts_per_rank=m.per + 1, top_k=cfg.top_k + 1, max_tokens=n,
                                                  device=dev)
        for li, L in enumerate(m.layers):
            cache = st.caches[li]
            _lib.check(lib.qk_rms_norm(P(x), P(L.attn_norm), n, H, cfg.eps, P(h), s))
            torch.matmul(h, L.w_qkv.t(), out=qkv)
            _lib.check(lib.qk_qk_norm_rope(P(qkv), P(L.q_norm), P(L.k_norm), P(m.inv_freq), P(positions), n, hq, kv,
                                           hd, cfg.rotary_dim, cfg.eps, P(q), P(gate), P(k), P(v), s))
            _lib.check(lib.qk_kv_q8_append_chunk(P(k), P(v), _lib.QK_OUT_BF16, P(start), None, P(cache["k"]),
                                                 P(cache["v"]), P(cache["k_scale"]), P(cache["v_scale"]), B, W, T, kv,
                                                 hd, s))
            # the chunk attends to the cache's own (quantised) keys and values
            _lib.check(lib.qk_kv_q8_read(P(cache["k"]), P(cache["k_scale"]), P(read_idx), B, W, T, kv, hd,
                                         _lib.QK_OUT_BF16, P(kd), s))
            _lib.check(lib.qk_kv_q8_read(P(cache["v"]), P(cache["v_scale"]), P(read_idx), B, W, T, kv, hd,
                                         _lib.QK_OUT_BF16, P(vd), s))
            qh = q.view(B, W, hq, hd).transpose(1, 2)
            # each KV head serves hq / kv query heads (GQA), expanded for the fused attention
            kh = kd.view(B, W, kv, hd).transpose(1, 2).repeat_interleave(hq // kv, dim=1)
            vh = vd.view(B, W, kv, hd).transpose(1, 2).repeat_interleave(hq // kv, dim=1)
            o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, is_causal=True)
            del kh, vh
            o = o.transpose(1, 2).reshape(n, hq, hd) * torch.sigmoid(gate)
            torch.matmul(o.reshape(n, hq * hd), L.w_o.t(), out=a)
            _lib.check(lib.qk_residual_add(P(x), P(a), n * H, P(x), s))
            _lib.check(lib.qk_rms_norm(P(x), P(L.ffn_norm), n, H, cfg.eps, P(h), s))
            _lib.check(lib.qk_router_topk(P(h), P(L.router), None, n, H, cfg.experts, cfg.top_k, P(ids), P(w), None,
                                          s))
            if m.world == 1:
                _lib.check(lib.qk_append_shared_route(P(ids), P(w), n, cfg.top_k, P(h), P(L.shared_router), H,
                                                      cfg.experts, P(ids_all), P(w_all), s))
                if li == len(m.layers) - 1 and self.moe_events is not None:
                    _lib.check(lib.qk_moe_forward_profiled(m.desc, P(L.experts["gate"]), P(L.experts["up"]),
                                                           P(L.experts["down"]), P(h), P(ids_all), P(w_all), n,
                                                           _lib.QK_OUT_BF16, P(y), P(ws), ws.numel(), s,
                                                           self.moe_events))
                else:
                    _lib.check(lib.qk_moe_forward(m.desc, P(L.experts["gate"]), P(L.experts["up"]),
                                                  P(L.experts["down"]), P(h), P(ids_all), P(w_all), n,
                                                  _lib.QK_OUT_BF16, P(y), P(ws), ws.numel(), s))
            else:
                _lib.check(lib.qk_append_shared_route_ep(P(ids), P(w), n, cfg.top_k, P(h), P(L.shared_router), H,
                                                         m.per, m.rank, P(ids_all), P(w_all), s))
                self._prefill_ep(L.experts["gate"], L.experts["up"], L.experts["down"], h, ids_all, w_all, out=y)
            _lib.check(lib.qk_residual_add(P(x), P(y), n * H, P(x), s))
            del o
        # the last prompt token of every sequence: the decode state's hidden row
        st.x.copy_(x.view(B, W, H)[:, W - 1])
        st.positions.fill_(W)
        self._choose(0)
        return self.tokens

    # ---- one greedy step ------------------------------------------------------------
    def _choose(self, column):
        """Final norm, tied-embedding logits and checked_argmax of the state's hidden rows;
        the choice goes to the generated-token column ``column`` (a Python int) and feeds
        the next step."""
        m, st = self.model, self.state
        lib = _lib.load()
        s = _lib.stream_handle(m.device)
        P = _lib.ptr
        _lib.check(lib.qk_rms_norm(P(st.x), P(self.final_norm), self.batch, m.cfg.hidden, m.cfg.eps, P(self.hn), s))
        torch.matmul(self.hn, self.embedding.t(), out=self.logits)
        choice = checked_argmax(self.logits)
        self.tokens.copy_(choice[:, 0].to(torch.int64))
        self.nonfinite.add_(choice[:, 1].sum().to(torch.int32))
        self.generated[:, column] = choice[:, 0]

    def _decode_step(self):
        st = self.state
        st.x.copy_(self.embedding.index_select(0, self.tokens))
        st.step()
        # greedy choice into column positions - prompt (device-side index)
        m = self.model
        lib = _lib.load()
        s = _lib.stream_handle(m.device)
        P = _lib.ptr
        _lib.check(lib.qk_rms_norm(P(st.x), P(self.final_norm), self.batch, m.cfg.hidden, m.cfg.eps, P(self.hn), s))
        torch.matmul(self.hn, self.embedding.t(), out=self.logits)
        choice = checked_argmax(self.logits)
        self.tokens.copy_(choice[:, 0].to(torch.int64))
        self.nonfinite.add_(choice[:, 1].sum().to(torch.int32))
        col = (st.positions[:1].to(torch.int64) - (self.prompt - 1)).clamp_(0, self.new_tokens - 1)
        self.generated.index_copy_(1, col, choice[:, :1])
        st.positions.add_(1)

    def capture(self):
        """Capture the decode step's CUDA graph (the state is left as it was)."""
        if self._graph is None:
            # capture needs a side stream; the capture's own replay state is restored after
            saved = self.state.positions.clone(), self.tokens.clone(), self.state.x.clone(), self.nonfinite.clone()
            self._decode_step()  # warm-up (also allocates whatever the first call needs)
            torch.cuda.synchronize(self.model.device)
            self._graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._graph):
                self._decode_step()
            self.state.positions.copy_(saved[0])
            self.tokens.copy_(saved[1])
            self.state.x.copy_(saved[2])
            self.nonfinite.copy_(saved[3])

    def decode(self, steps=None):
        """``steps`` (default: the remaining new tokens) greedy decode steps, each one replay
        of the captured CUDA graph."""
        steps = self.new_tokens - 1 if steps is None else steps
        self.capture()
        for _ in range(steps):
            self._graph.replay()
        return self.generated

    def close(self):
        self._graph = None
        if self._prefill_ep is not None:
            self._prefill_ep.close()
            self._prefill_ep = None
        self.state.close()


__all__ = ["StaticGeneration"]
