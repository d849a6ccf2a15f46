"""Q8 KV cache codec, gathers and split-KV decode attention on the GPU against the oracle."""

import numpy as np
import pytest

from oracle import kv
from oracle.precision import bf16_round
from util import bf16_tensor, rel_err, to_f32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("width", [8, 256])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_codec_codes_and_scales_bit_exact(golden, cuda_device, width, dtype):
    import torch

    from qk_b200.attention_cache import quantize

    data = golden("q8_kv.npz")
    tag = f"w{width}_{dtype}"
    x = data[f"{tag}_x"]
    xt = bf16_tensor(x, cuda_device) if dtype == "bf16" else torch.from_numpy(x).to(cuda_device)
    codes, scale = quantize(xt, min(32, width))
    np.testing.assert_array_equal(codes.cpu().numpy(), data[f"{tag}_codes"])
    np.testing.assert_array_equal(to_f32(scale), data[f"{tag}_scale"])
    assert np.count_nonzero(data[f"{tag}_unrounded_codes"] != codes.cpu().numpy()) > 0


def test_write_then_read_matches_reference_and_leaves_inactive_rows(golden, cuda_device):
    import torch

    from qk_b200.attention_cache import CacheConfig, empty_cache, read_quantized, write_quantized

    data = golden("q8_kv.npz")
    c = CacheConfig(max_context=32)
    cache = empty_cache(2, c, cuda_device)
    src = bf16_tensor(data["read_source"], cuda_device)
    write_quantized(cache, src, src, torch.tensor([31, 8]), torch.tensor([True, False]), c)
    indices = torch.tensor([[31, 0, 31, 1], [8, 0, 8, 31]], device=cuda_device)
    for dtype in (torch.float32, torch.bfloat16):
        got = to_f32(read_quantized(cache, "k", indices, c, dtype))
        expected = np.zeros((2, 4, 2, 256), np.float32)
        expected[0, [0, 2]] = data["read_reconstructed"]
        if dtype == torch.bfloat16:  # test_qwen38_kv_gather.py:94 expected.astype(dtype)
            expected = bf16_round(expected)
        np.testing.assert_array_equal(got, expected)
    for name in ("k", "v", "k_scale", "v_scale"):
        assert (cache[name].reshape(2, -1)[1] == 0).all()


@pytest.mark.parametrize("case", ["1_16_8", "2_4_32", "8_16_64"])
def test_scale_gather_wrap_clamp_golden(golden, cuda_device, case):
    import torch

    from qk_b200.attention_cache import gather_scale_plane

    data = golden("q8_kv.npz")
    batch, groups, time = map(int, case.split("_"))
    tag = f"gather_{case}"
    plane = torch.from_numpy(data[f"{tag}_plane"].view(np.int16)).to(cuda_device).view(torch.bfloat16)
    idx = torch.from_numpy(data[f"{tag}_indices"]).to(cuda_device)
    for method in ("indexed", "rowwise"):
        got = gather_scale_plane(plane, idx, groups, method=method)
        np.testing.assert_array_equal(got.view(torch.int16).cpu().numpy().view(np.uint16),
                                      data[f"{tag}_expected"])


def test_append_random_rows_matches_oracle(cuda_device):
    import torch

    from qk_b200.attention_cache import CacheConfig, empty_cache, write_quantized

    c = CacheConfig(max_context=64)
    rng = np.random.default_rng(81)
    cache = empty_cache(4, c, cuda_device)
    ref = {n: np.zeros((4, 64, 512), np.int8) for n in ("k", "v")}
    ref.update({n: np.zeros((4 * 16, 64), np.float32) for n in ("k_scale", "v_scale")})
    for step in range(5):
        key = bf16_round(rng.normal(size=(4, 2, 256)).astype(np.float32) * 3)
        val = bf16_round(rng.normal(size=(4, 2, 256)).astype(np.float32))
        t = np.array([step, step * 3, 63, -1], np.int32)
        active = np.array([True, step % 2 == 0, True, True])
        write_quantized(cache, bf16_tensor(key, cuda_device), bf16_tensor(val, cuda_device),
                        torch.from_numpy(t), torch.from_numpy(active), c)
        kv.write_quantized(ref, key, val, np.where(t < 0, t + 64, t), active, 2, 256)
    for n in ("k", "v"):
        np.testing.assert_array_equal(cache[n].cpu().numpy(), ref[n])
    for n in ("k_scale", "v_scale"):
        np.testing.assert_array_equal(to_f32(cache[n]), ref[n])


def build_cache(rng, batch, T, device, c):
    import torch

    from qk_b200.attention_cache import empty_cache, write_quantized

    cache = empty_cache(batch, c, device)
    keys = rng.normal(size=(T, batch, c.kv_heads, c.head_dim)).astype(np.float32)
    vals = rng.normal(size=(T, batch, c.kv_heads, c.head_dim)).astype(np.float32)
    # append token by token, like decode steps (attention_cache.py:139-140)
    for t in range(T):
        write_quantized(cache, bf16_tensor(keys[t], device), bf16_tensor(vals[t], device),
                        torch.full((batch,), t, dtype=torch.int32), None, c)
    return cache


@pytest.mark.parametrize("batch,S,pages", [(1, 40, False), (3, 300, False), (2, 1024, True)])
def test_decode_attention_matches_oracle(cuda_device, batch, S, pages):
    import torch

    from qk_b200.attention_cache import CacheConfig, decode_attention

    c = CacheConfig(max_context=S, query_heads=16, kv_heads=2, head_dim=256)
    rng = np.random.default_rng(S + batch)
    cache = build_cache(rng, batch, S, cuda_device, c)
    if pages:  # 256-slot pages through a random permutation page table
        P = 256
        table = np.stack([rng.permutation(S // P) for _ in range(batch)])
        slots = np.arange(S)
        indices = (table[:, slots // P] * P + slots % P).astype(np.int32)
    else:
        indices = np.tile(np.arange(S, dtype=np.int32), (batch, 1))
    lengths = rng.integers(S // 2, S, batch).astype(np.int32)
    q = bf16_round(rng.normal(size=(batch, 16, 256)).astype(np.float32))
    gate = bf16_round(rng.normal(size=(batch, 16, 256)).astype(np.float32))
    got = to_f32(decode_attention(bf16_tensor(q, cuda_device), cache, torch.from_numpy(indices), c,
                                  lengths=torch.from_numpy(lengths), gate=bf16_tensor(gate, cuda_device)))
    codes = {n: cache[n].cpu().numpy() for n in ("k", "v")}
    planes = {n: to_f32(cache[n + "_scale"]) for n in ("k", "v")}
    keys = kv.read_quantized(codes["k"], planes["k"], indices, 2, 256)
    values = kv.read_quantized(codes["v"], planes["v"], indices, 2, 256)
    mask = np.arange(S)[None, :] <= lengths[:, None]
    expected = kv.attention(q, keys, values, mask, gate)
    mx, l2 = rel_err(got, expected)
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)


def test_decode_attention_valid_mask_and_sparse_indices(cuda_device):
    import torch

    from qk_b200.attention_cache import CacheConfig, decode_attention

    c = CacheConfig(max_context=128, query_heads=16, kv_heads=2, head_dim=256)
    rng = np.random.default_rng(5)
    cache = build_cache(rng, 2, 128, cuda_device, c)
    indices = rng.integers(0, 128, (2, 77)).astype(np.int32)
    valid = rng.random((2, 77)) < 0.6
    valid[:, 0] = True
    q = bf16_round(rng.normal(size=(2, 16, 256)).astype(np.float32))
    got = to_f32(decode_attention(bf16_tensor(q, cuda_device), cache, torch.from_numpy(indices), c,
                                  valid=torch.from_numpy(valid)))
    codes = {n: cache[n].cpu().numpy() for n in ("k", "v")}
    planes = {n: to_f32(cache[n + "_scale"]) for n in ("k", "v")}
    keys = kv.read_quantized(codes["k"], planes["k"], indices, 2, 256)
    values = kv.read_quantized(codes["v"], planes["v"], indices, 2, 256)
    expected = kv.attention(q, keys, values, valid)
    mx, l2 = rel_err(got, expected)
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)


def _random_cache(torch, device, rng, batch, T, kv_heads, hd):
    """Cache tensors filled directly (random codes, scales in [0.001, 0.021)): long contexts
    without T single-token appends."""
    groups = kv_heads * hd // 32
    codes = {n: rng.integers(-127, 128, (batch, T, kv_heads * hd)).astype(np.int8) for n in ("k", "v")}
    planes = {n: bf16_round(rng.uniform(0.001, 0.021, (batch * groups, T)).astype(np.float32))
              for n in ("k", "v")}
    cache = {n: torch.from_numpy(codes[n]).to(device) for n in ("k", "v")}
    cache.update({n + "_scale": bf16_tensor(planes[n], device) for n in ("k", "v")})
    return cache, codes, planes


@pytest.mark.parametrize("batch,S,hq,kv_heads,hd,pages", [
    (1, 8192, 16, 2, 256, True),     # two pairs, each cut across dozens of CTAs
    (3, 2000, 16, 2, 256, False),    # ragged last tile (2000 = 125 * 16), contiguous slots
    (5, 777, 16, 2, 256, True),      # ragged tile inside the CTA ranges, 16-slot pages
    (2, 300, 8, 2, 128, False),      # head_dim 128, 4 query heads per KV head
    (4, 1500, 32, 4, 128, True),     # head_dim 128, 8 query heads per KV head, 4 KV heads
])
def test_decode_attention_stream_split_matches_oracle(cuda_device, batch, S, hq, kv_heads, hd, pages):
    import torch

    from qk_b200.attention_cache import CacheConfig, decode_attention

    rng = np.random.default_rng(batch * 131 + S)
    T = S + 48
    c = CacheConfig(max_context=T, query_heads=hq, kv_heads=kv_heads, head_dim=hd)
    cache, codes, planes = _random_cache(torch, cuda_device, rng, batch, T, kv_heads, hd)
    if pages:
        P = 16
        table = np.stack([rng.permutation(T // P) for _ in range(batch)])
        slots = np.arange(S)
        indices = (table[:, slots // P] * P + slots % P).astype(np.int32)
    else:
        indices = np.tile(np.arange(S, dtype=np.int32), (batch, 1))
    lengths = rng.integers(S // 2, S, batch).astype(np.int32)
    q = bf16_round(rng.normal(size=(batch, hq, hd)).astype(np.float32))
    gate = bf16_round(rng.normal(size=(batch, hq, hd)).astype(np.float32))
    got = to_f32(decode_attention(bf16_tensor(q, cuda_device), cache, torch.from_numpy(indices), c,
                                  lengths=torch.from_numpy(lengths), gate=bf16_tensor(gate, cuda_device)))
    keys = kv.read_quantized(codes["k"], planes["k"], indices, kv_heads, hd)
    values = kv.read_quantized(codes["v"], planes["v"], indices, kv_heads, hd)
    mask = np.arange(S)[None, :] <= lengths[:, None]
    expected = kv.attention(q, keys, values, mask, gate)
    mx, l2 = rel_err(got, expected)
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)


def test_decode_attention_wrapped_and_clamped_indices(cuda_device):
    """Negative cache times wrap once, out-of-range times clamp (the scale gather rule), and
    runs that are consecutive but not 8-aligned take the per-scale path."""
    import torch

    from qk_b200.attention_cache import CacheConfig, decode_attention

    rng = np.random.default_rng(17)
    batch, S, T = 2, 700, 640
    c = CacheConfig(max_context=T, query_heads=16, kv_heads=2, head_dim=256)
    cache, codes, planes = _random_cache(torch, cuda_device, rng, batch, T, 2, 256)
    indices = np.tile((np.arange(S) + 3).astype(np.int32), (batch, 1))  # consecutive, offset 3
    indices[0, :40] = rng.integers(-2 * T, 0, 40)     # negative: wrap (then clamp to 0)
    indices[1, 100:140] = rng.integers(T, 3 * T, 40)  # past the end: clamp to T - 1
    valid = rng.random((batch, S)) < 0.8
    q = bf16_round(rng.normal(size=(batch, 16, 256)).astype(np.float32))
    got = to_f32(decode_attention(bf16_tensor(q, cuda_device), cache, torch.from_numpy(indices), c,
                                  valid=torch.from_numpy(valid)))
    keys = kv.read_quantized(codes["k"], planes["k"], indices, 2, 256)
    values = kv.read_quantized(codes["v"], planes["v"], indices, 2, 256)
    expected = kv.attention(q, keys, values, valid)
    mx, l2 = rel_err(got, expected)
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)
