"""Router top-k on the GPU (router part of ``qwen38_tpu/math.py:277-281``, ``routes_and_shared``).

``routes(x, router_weight, top_k, active=None)`` returns ``(ids int32[T, k], weights bf16[T, k])``:
FP32 logits ``x @ Wr^T``, accurate softmax, top-k with ties to the lower expert index
(``lax.top_k``), renormalisation with an IEEE divide, inactive rows zeroed, BF16 cast.
"""

import torch

from . import _lib


def _check_k(top_k, experts):
    if type(top_k) is not int or not 0 < top_k <= experts or top_k > 32:
        raise ValueError("Invalid expert top-k")


def routes(x, router_weight, top_k, active=None, *, return_probs=False):
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a BF16 [T, H] tensor")
    router_weight = router_weight.to(device=x.device, dtype=torch.float32).contiguous()
    T, H = x.shape
    E = router_weight.shape[0]
    if router_weight.shape[1] != H:
        raise ValueError("router weight must be [E, hidden]")
    _check_k(top_k, E)
    x = x.contiguous()
    ids = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    weights = torch.empty((T, top_k), dtype=torch.bfloat16, device=x.device)
    probs = torch.empty((T, E), dtype=torch.float32, device=x.device) if return_probs else None
    act = None if active is None else active.to(device=x.device, dtype=torch.uint8).contiguous()
    with torch.cuda.device(x.device):
        _lib.call("qk_router_topk", _lib.ptr(x), _lib.ptr(router_weight), _lib.ptr(act), T, H, E,
                  top_k, _lib.ptr(ids), _lib.ptr(weights), _lib.ptr(probs),
                  _lib.stream_handle(x.device))
    return (ids, weights, probs) if return_probs else (ids, weights)


def router_logits(x, router_weight, out=None):
    """FP32 logits ``x @ Wr^T`` ``[T, E]`` (the linear of ``math.py:277-281``) over many CTAs,
    with the same values ``routes`` selects from; ``routes_from_logits(router_logits(x, w), k)``
    equals ``routes(x, w, k)``."""
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a BF16 [T, H] tensor")
    router_weight = router_weight.to(device=x.device, dtype=torch.float32).contiguous()
    T, H = x.shape
    E = router_weight.shape[0]
    if router_weight.shape[1] != H:
        raise ValueError("router weight must be [E, hidden]")
    x = x.contiguous()
    if out is None:
        out = torch.empty((T, E), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("qk_router_logits", _lib.ptr(x), _lib.ptr(router_weight), T, H, E, _lib.ptr(out),
                  _lib.stream_handle(x.device))
    return out


def routes_from_logits(logits, top_k, active=None, *, return_probs=False):
    """The same selection from precomputed FP32 logits ``[T, E]``."""
    logits = logits.to(torch.float32).contiguous()
    T, E = logits.shape
    _check_k(top_k, E)
    ids = torch.empty((T, top_k), dtype=torch.int32, device=logits.device)
    weights = torch.empty((T, top_k), dtype=torch.bfloat16, device=logits.device)
    probs = torch.empty((T, E), dtype=torch.float32, device=logits.device) if return_probs else None
    act = None if active is None else active.to(device=logits.device, dtype=torch.uint8).contiguous()
    with torch.cuda.device(logits.device):
        _lib.call("qk_router_topk_logits", _lib.ptr(logits), _lib.ptr(act), T, E, top_k,
                  _lib.ptr(ids), _lib.ptr(weights), _lib.ptr(probs),
                  _lib.stream_handle(logits.device))
    return (ids, weights, probs) if return_probs else (ids, weights)
