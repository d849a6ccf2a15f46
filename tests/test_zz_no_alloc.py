"""qk_kv_q8_decode_attention_noalloc: decode attention whose split scratch is a fixed array
in the library's device image. Compared with the workspace entry point on the same inputs,
two calls in a row on one stream; geometries above the fixed size are refused unrun."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 16 << 20  # QK_ATTN_STATIC_SCRATCH_BYTES
HQ, KV, HD = 16, 2, 256


def _cache(torch, device, batch, T, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    groups = KV * HD // 32
    cache = {
        "k": torch.randint(-127, 128, (batch, T, KV * HD), dtype=torch.int8, generator=g),
        "v": torch.randint(-127, 128, (batch, T, KV * HD), dtype=torch.int8, generator=g),
        "k_scale": (torch.rand((batch * groups, T), generator=g) * 0.02 + 0.001).to(torch.bfloat16),
        "v_scale": (torch.rand((batch * groups, T), generator=g) * 0.02 + 0.001).to(torch.bfloat16),
    }
    return {k: v.to(device) for k, v in cache.items()}


def _inputs(torch, device, batch, S, T, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn((batch, HQ, HD), generator=g).to(torch.bfloat16).to(device)
    gate = torch.randn((batch, HQ, HD), generator=g).to(torch.bfloat16).to(device)
    idx = torch.stack([torch.randperm(T, generator=g)[:S] for _ in range(batch)]).to(torch.int32).to(device)
    lengths = torch.randint(S // 2, S, (batch,), generator=g).to(torch.int32).to(device)
    return q, gate, idx, lengths


def _args(_lib, cache, q, gate, idx, lengths, batch, S, T, out):
    return (_lib.ptr(q), _lib.ptr(cache["k"]), _lib.ptr(cache["v"]), _lib.ptr(cache["k_scale"]),
            _lib.ptr(cache["v_scale"]), _lib.ptr(idx), None, _lib.ptr(lengths), _lib.ptr(gate),
            batch, S, T, HQ, KV, HD, _lib.ptr(out))


@pytest.mark.parametrize("batch,S", [(4, 512), (32, 1024), (1, 40), (1, 8192), (150, 512)])
def test_noalloc_matches_workspace_entry_point_twice_in_a_row(cuda_device, batch, S):
    import torch

    from qk_b200 import _lib

    lib = _lib.load()
    T = S + 64
    need = int(lib.qk_kv_q8_attention_workspace_bytes(batch, S, HQ, KV, HD))
    assert need <= STATIC_SCRATCH_BYTES
    cache = _cache(torch, cuda_device, batch, T, seed=batch * 1000 + S)
    stream = _lib.stream_handle(cuda_device)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=cuda_device)
    sets = [_inputs(torch, cuda_device, batch, S, T, seed=s) for s in (11, 12)]
    refs, outs = [], []
    for q, gate, idx, lengths in sets:
        ref = torch.empty((batch, HQ, HD), dtype=torch.bfloat16, device=cuda_device)
        _lib.check(lib.qk_kv_q8_decode_attention(*_args(_lib, cache, q, gate, idx, lengths, batch, S, T, ref),
                                                 _lib.ptr(ws) if need else None, need, stream))
        refs.append(ref)
    # two calls in a row on the same stream, sharing the static scratch
    for q, gate, idx, lengths in sets:
        out = torch.full((batch, HQ, HD), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        _lib.check(lib.qk_kv_q8_decode_attention_noalloc(
            *_args(_lib, cache, q, gate, idx, lengths, batch, S, T, out), stream))
        outs.append(out)
    torch.cuda.synchronize(cuda_device)
    for ref, out in zip(refs, outs):
        r, o = ref.float(), out.float()
        assert torch.isfinite(o).all()
        err = float((o - r).abs().max() / r.abs().max())
        assert err <= 1e-3, err
    # the two input sets differ, so a stale scratch would show up as equal outputs
    assert not torch.equal(outs[0], outs[1])


def test_workspace_is_bounded_by_the_sm_count_whatever_the_batch(cuda_device):
    """One CTA per SM, at most two partial rows per KV head each: the workspace (and so the
    fixed scratch the no-alloc entry point needs) does not grow with B or S."""
    import torch

    from qk_b200 import _lib

    lib = _lib.load()
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    bound = 2 * sms * KV * (16 + 8 * HD) * 4
    for batch, S in ((1, 40), (1, 32768), (32, 32768), (150, 512), (1024, 4096)):
        need = int(lib.qk_kv_q8_attention_workspace_bytes(batch, S, HQ, KV, HD))
        assert need <= bound, (batch, S, need, bound)
    assert bound <= STATIC_SCRATCH_BYTES


def test_noalloc_refuses_a_workspace_above_the_fixed_scratch_unrun(cuda_device):
    """The refusal path, driven through a geometry the kernel accepts but whose scratch does
    not fit: 16 KV heads of 128 need 2 * SMs * 16 * (16 + 8 * 128) * 4 bytes, 19.7 MB on a
    148-SM B200, above the 16 MiB array. The call must fail before any launch, so the
    operand pointers are never dereferenced."""
    import torch

    from qk_b200 import _lib

    lib = _lib.load()
    hq, kv, hd = 16, 16, 128
    batch, S, T = 150, 4096, 4096
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    need = int(lib.qk_kv_q8_attention_workspace_bytes(batch, S, hq, kv, hd))
    assert need > STATIC_SCRATCH_BYTES, (sms, need)
    launches = _lib.launch_count()
    dummy = ctypes.c_void_p(256)
    rc = lib.qk_kv_q8_decode_attention_noalloc(*([dummy] * 6), None, dummy, None, batch, S, T, hq,
                                               kv, hd, dummy, _lib.stream_handle(cuda_device))
    assert rc == _lib.QK_ERR_WORKSPACE
    assert "fixed" in _lib.last_error() and str(need) in _lib.last_error()
    assert _lib.launch_count() == launches
