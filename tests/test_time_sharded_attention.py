"""Time-sharded Q8 decode attention: the cache's time axis split over ranks
(``engine.py:350-369``), partial (output, max, sum) sets all-gathered in rank order and
merged by log-sum-exp.

CPU: the shard bookkeeping, and the 2-rank protocol on ``gloo`` with the oracle's partials.
GPU: the partial kernel + combine against the single-device kernel and the oracle, ranks
emulated on one device, and two real ranks over NCCL when two GPUs are present.
"""

import os
import socket

import numpy as np
import pytest

from oracle import kv
from oracle.precision import bf16_round
from util import bf16_tensor, rel_err, to_f32


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _random_cache_np(rng, batch, T, kv_heads, hd):
    groups = kv_heads * hd // 32
    codes = {n: rng.integers(-127, 128, (batch, T, kv_heads * hd)).astype(np.int8) for n in ("k", "v")}
    planes = {n: bf16_round(rng.uniform(0.001, 0.021, (batch * groups, T)).astype(np.float32))
              for n in ("k", "v")}
    return codes, planes


# ---- CPU: bookkeeping ------------------------------------------------------------------


def test_time_shards_partition_the_context_and_writes_land_once():
    import torch

    from qk_b200.attention_cache import local_lengths, local_write_target, time_shard

    T = 96
    lengths = torch.tensor([0, 5, 31, 32, 64, 95, 200, -3], dtype=torch.int32)
    active = torch.tensor([1, 1, 1, 1, 1, 1, 1, 0], dtype=torch.bool)
    for world in (1, 2, 3, 4):
        covered, writers = [], torch.zeros(len(lengths), dtype=torch.int32)
        for rank in range(world):
            first, size = time_shard(T, rank, world)
            covered.extend(range(first, first + size))
            t, mine = local_write_target(lengths, active, first, size, T)
            writers += mine.to(torch.int32)
            clipped = lengths.clamp(0, T - 1)
            for b in range(len(lengths)):
                if mine[b]:
                    assert first + int(t[b]) == int(clipped[b])
            # local slot s valid iff first + s <= clipped length
            local = local_lengths(clipped, first)
            for b in range(len(lengths)):
                valid = [s for s in range(size) if s <= int(local[b])]
                assert valid == [s for s in range(size) if first + s <= int(clipped[b])]
        assert covered == list(range(T))
        assert writers.tolist() == [1] * 7 + [0]  # every active row written by one rank
    with pytest.raises(ValueError, match="divide evenly"):
        time_shard(100, 0, 3)
    with pytest.raises(ValueError):
        time_shard(96, 2, 2)


def test_oracle_shard_merge_equals_the_unsharded_oracle():
    rng = np.random.default_rng(44)
    batch, T, hq, kvh, hd = 3, 96, 16, 2, 256
    codes, planes = _random_cache_np(rng, batch, T, kvh, hd)
    idx = np.tile(np.arange(T, dtype=np.int32), (batch, 1))
    keys = kv.read_quantized(codes["k"], planes["k"], idx, kvh, hd)
    values = kv.read_quantized(codes["v"], planes["v"], idx, kvh, hd)
    q = bf16_round(rng.normal(size=(batch, hq, hd)).astype(np.float32))
    gate = bf16_round(rng.normal(size=(batch, hq, hd)).astype(np.float32))
    lengths = np.array([10, 50, 95])
    mask = np.arange(T)[None, :] <= lengths[:, None]
    expected = kv.attention(q, keys, values, mask, gate)
    for world in (1, 2, 4):
        size = T // world
        parts = [kv.attention_partial(q, keys[:, r * size:(r + 1) * size], values[:, r * size:(r + 1) * size],
                                      mask[:, r * size:(r + 1) * size]) for r in range(world)]
        got = kv.combine_partials(np.concatenate(parts), batch, hq, hd, gate)
        mx, l2 = rel_err(got, expected)
        assert mx < 1e-2 and l2 < 5e-3, (world, mx, l2)


def _gloo_rank(rank, world, port, path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qk_b200.attention_cache import gather_partials, local_lengths, time_shard

        rng = np.random.default_rng(45)  # the same full cache on every rank
        batch, T, hq, kvh, hd = 2, 64, 16, 2, 256
        codes, planes = _random_cache_np(rng, batch, T, kvh, hd)
        q = bf16_round(rng.normal(size=(batch, hq, hd)).astype(np.float32))
        lengths = torch.tensor([20, 63], dtype=torch.int32)
        first, size = time_shard(T, rank, world)
        local = {n: codes[n][:, first:first + size] for n in codes}
        lplanes = {n: planes[n][:, first:first + size] for n in planes}
        idx = np.tile(np.arange(size, dtype=np.int32), (batch, 1))
        keys = kv.read_quantized(local["k"], lplanes["k"], idx, kvh, hd)
        values = kv.read_quantized(local["v"], lplanes["v"], idx, kvh, hd)
        mask = np.arange(size)[None, :] <= local_lengths(lengths, first).numpy()[:, None]
        partial = torch.from_numpy(kv.attention_partial(q, keys, values, mask))
        parts = gather_partials(partial, dist.group.WORLD, world)
        got = kv.combine_partials(parts.numpy(), batch, hq, hd)
        full_idx = np.tile(np.arange(T, dtype=np.int32), (batch, 1))
        fk = kv.read_quantized(codes["k"], planes["k"], full_idx, kvh, hd)
        fv = kv.read_quantized(codes["v"], planes["v"], full_idx, kvh, hd)
        expected = kv.attention(q, fk, fv, np.arange(T)[None, :] <= lengths.numpy()[:, None])
        np.save(f"{path}.{rank}.npy", np.stack([got, expected]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_partial_gather_on_gloo(tmp_path):
    import torch.multiprocessing as mp

    path = tmp_path / "tsa"
    mp.start_processes(_gloo_rank, args=(2, _port(), str(path)), nprocs=2, start_method="spawn")
    results = [np.load(f"{path}.{r}.npy") for r in range(2)]
    np.testing.assert_array_equal(results[0][0], results[1][0])  # every rank gets the same output
    mx, l2 = rel_err(results[0][0], results[0][1])
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)


# ---- GPU --------------------------------------------------------------------------------


def _device_cache(torch, device, codes, planes, first=0, size=None):
    size = codes["k"].shape[1] - first if size is None else size
    cache = {n: torch.from_numpy(np.ascontiguousarray(codes[n][:, first:first + size])).to(device)
             for n in ("k", "v")}
    cache.update({n + "_scale": bf16_tensor(np.ascontiguousarray(planes[n][:, first:first + size]), device)
                  for n in ("k", "v")})
    return cache


@pytest.mark.gpu
@pytest.mark.parametrize("batch,S,hq,kvh,hd,pages", [
    (3, 2000, 16, 2, 256, False),
    (1, 8192, 16, 2, 256, True),
    (4, 1500, 32, 4, 128, True),
])
def test_single_partial_set_equals_the_fused_kernel(cuda_device, batch, S, hq, kvh, hd, pages):
    """R = 1: partial + combine reproduces qk_kv_q8_decode_attention bit for bit."""
    import torch

    from qk_b200.attention_cache import (CacheConfig, combine_partials, decode_attention,
                                         decode_attention_partial)

    rng = np.random.default_rng(batch * 7 + S)
    T = S + 16
    c = CacheConfig(max_context=T, query_heads=hq, kv_heads=kvh, head_dim=hd)
    codes, planes = _random_cache_np(rng, batch, T, kvh, hd)
    cache = _device_cache(torch, cuda_device, codes, planes)
    if pages:
        table = np.stack([rng.permutation(T // 16) for _ in range(batch)])
        slots = np.arange(S)
        indices = (table[:, slots // 16] * 16 + slots % 16).astype(np.int32)
    else:
        indices = np.tile(np.arange(S, dtype=np.int32), (batch, 1))
    lengths = torch.from_numpy(rng.integers(S // 3, S, batch).astype(np.int32))
    q = bf16_tensor(rng.normal(size=(batch, hq, hd)).astype(np.float32), cuda_device)
    for gate in (None, bf16_tensor(rng.normal(size=(batch, hq, hd)).astype(np.float32), cuda_device)):
        ref = decode_attention(q, cache, torch.from_numpy(indices), c, lengths=lengths, gate=gate)
        part = decode_attention_partial(q, cache, torch.from_numpy(indices), c, lengths=lengths)
        got = combine_partials(part, batch, hq, hd, gate)
        torch.cuda.synchronize(cuda_device)
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


@pytest.mark.gpu
@pytest.mark.parametrize("world,batch,T,hq,kvh,hd", [
    (2, 3, 4096, 16, 2, 256),
    (4, 2, 2048, 16, 2, 256),
    (8, 5, 1024, 16, 2, 256),
    (2, 4, 1536, 32, 4, 128),
])
def test_emulated_time_shards_match_oracle_and_single_device(cuda_device, world, batch, T, hq, kvh, hd):
    """Ranks emulated on one device: each shard's partial set over its slice of the times,
    concatenated in rank order and combined. Rows whose length ends inside the first shard
    leave the later shards with no valid slot (max -inf, sum 0)."""
    import torch

    from qk_b200.attention_cache import (CacheConfig, combine_partials, decode_attention,
                                         decode_attention_partial, local_lengths, time_shard)

    rng = np.random.default_rng(world * 100 + T)
    c = CacheConfig(max_context=T, query_heads=hq, kv_heads=kvh, head_dim=hd)
    codes, planes = _random_cache_np(rng, batch, T, kvh, hd)
    lengths = rng.integers(0, T, batch).astype(np.int32)
    lengths[0] = 5  # inside shard 0 only
    q_np = bf16_round(rng.normal(size=(batch, hq, hd)).astype(np.float32))
    gate_np = bf16_round(rng.normal(size=(batch, hq, hd)).astype(np.float32))
    q, gate = bf16_tensor(q_np, cuda_device), bf16_tensor(gate_np, cuda_device)
    lens = torch.from_numpy(lengths).to(cuda_device)
    shard_c = CacheConfig(max_context=T // world, query_heads=hq, kv_heads=kvh, head_dim=hd)
    parts = []
    for rank in range(world):
        first, size = time_shard(T, rank, world)
        cache = _device_cache(torch, cuda_device, codes, planes, first, size)
        idx = torch.arange(size, dtype=torch.int32, device=cuda_device).expand(batch, size)
        part = decode_attention_partial(q, cache, idx, shard_c, lengths=local_lengths(lens, first))
        if rank > 0:  # row 0 has no valid slot here
            st = part[batch * hq * hd:].view(batch, hq, 2)
            assert torch.isneginf(st[0, :, 0]).all() and (st[0, :, 1] == 0).all()
        parts.append(part)
    got = combine_partials(torch.cat(parts), batch, hq, hd, gate)
    full = _device_cache(torch, cuda_device, codes, planes)
    idx = torch.arange(T, dtype=torch.int32, device=cuda_device).expand(batch, T)
    single = decode_attention(q, full, idx, c, lengths=lens, gate=gate)
    mx, l2 = rel_err(to_f32(got), to_f32(single))
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)
    full_idx = np.tile(np.arange(T, dtype=np.int32), (batch, 1))
    keys = kv.read_quantized(codes["k"], planes["k"], full_idx, kvh, hd)
    values = kv.read_quantized(codes["v"], planes["v"], full_idx, kvh, hd)
    expected = kv.attention(q_np, keys, values, np.arange(T)[None, :] <= lengths[:, None], gate_np)
    mx, l2 = rel_err(to_f32(got), expected)
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)


def _two_gpu_rank(rank, world, port, path):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from qk_b200.attention_cache import (CacheConfig, TimeShardedAttention, combine_partials,
                                             decode_attention_partial, empty_cache, local_lengths,
                                             time_shard)

        batch, T, steps = 3, 512, 40
        c = CacheConfig(max_context=T, query_heads=16, kv_heads=2, head_dim=256)
        attn = TimeShardedAttention(dist.group.WORLD)
        first, size = attn.shard(c)
        cache = empty_cache(batch, CacheConfig(max_context=size, query_heads=16, kv_heads=2, head_dim=256), dev)
        rng = np.random.default_rng(71)  # the same stream of keys on both ranks
        lengths = torch.tensor([200, 250, 300], dtype=torch.int32, device=dev)
        for _ in range(steps):  # decode steps: write at lengths[b], then advance
            key = bf16_tensor(rng.normal(size=(batch, 2, 256)).astype(np.float32), dev)
            val = bf16_tensor(rng.normal(size=(batch, 2, 256)).astype(np.float32), dev)
            attn.write(cache, key, val, lengths, None, c)
            lengths += 1
        lengths -= 1
        q = bf16_tensor(rng.normal(size=(batch, 16, 256)).astype(np.float32), dev)
        got = attn(q, cache, lengths, c)
        # this rank's own emulation of both shards from the gathered caches
        caches = [torch.empty_like(cache[n]) for n in ("k", "v", "k_scale", "v_scale") for _ in range(world)]
        full = {}
        for i, n in enumerate(("k", "v", "k_scale", "v_scale")):
            parts = caches[i * world:(i + 1) * world]
            dist.all_gather(parts, cache[n].contiguous())
            full[n] = parts
        sc = CacheConfig(max_context=size, query_heads=16, kv_heads=2, head_dim=256)
        sets = []
        for r in range(world):
            f, s = time_shard(T, r, world)
            shard = {n: full[n][r] for n in full}
            idx = torch.arange(s, dtype=torch.int32, device=dev).expand(batch, s)
            sets.append(decode_attention_partial(q, shard, idx, sc, lengths=local_lengths(lengths, f)))
        ref = combine_partials(torch.cat(sets), batch, 16, 256)
        torch.cuda.synchronize(dev)
        np.save(f"{path}.{rank}.npy", np.stack([got.view(torch.int16).cpu().numpy(),
                                                ref.view(torch.int16).cpu().numpy()]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_time_sharded_attention_on_two_gpus_nccl(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = tmp_path / "tsa2"
    mp.start_processes(_two_gpu_rank, args=(2, _port(), str(path)), nprocs=2, start_method="spawn")
    r0, r1 = (np.load(f"{path}.{r}.npy") for r in range(2))
    np.testing.assert_array_equal(r0[0], r1[0])
    np.testing.assert_array_equal(r0[0], r0[1])
