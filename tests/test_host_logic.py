"""Host-side placement and expert-parallel bookkeeping, on CPU (gloo for the 2-rank case)."""

import hashlib
import os

import numpy as np
import pytest

from oracle import gguf, moe
from oracle.precision import bf16_round


def test_split_expert_bytes_matches_reference_golden(golden):
    from make_golden import SPLIT_CASES, split_inputs

    from qk_b200.parallel import split_expert_bytes
    from qk_b200.quant import block_layout

    data = golden("split_experts.npz")
    for qtype, hidden, inter, tp in SPLIT_CASES:
        for kind in ("gate", "up", "down"):
            raw = split_inputs(qtype, kind, hidden, inter, block_layout(qtype))
            got = np.ascontiguousarray(split_expert_bytes(raw, kind, qtype, hidden, inter, tp))
            tag = f"{qtype}_{kind}_{tp}"
            assert tuple(got.shape) == tuple(data[f"{tag}_shape"])
            assert hashlib.sha256(got.tobytes()).digest() == bytes(data[f"{tag}_sha256"])


def test_split_rejects_partial_blocks():
    from qk_b200.parallel import split_expert_bytes

    with pytest.raises(ValueError, match="whole down quantization blocks"):
        split_expert_bytes(np.zeros((2, 256 * 210), np.uint8), "down", "Q6_K", 256, 512, 4)
    with pytest.raises(ValueError, match="Unknown"):
        split_expert_bytes(np.zeros((2, 10), np.uint8), "side", "Q6_K", 256, 512, 1)


def test_local_expert_ranges_partition_the_experts():
    from qk_b200.parallel import local_range

    for world in (1, 2, 4, 8):
        seen = []
        for rank in range(world):
            first, count = local_range(512, rank, world)
            seen.extend(range(first, first + count))
        assert seen == list(range(512))
    with pytest.raises(ValueError):
        local_range(10, 0, 4)


def test_qtype_normalisation_and_layouts():
    from qk_b200.quant import block_layout, normalize_qtype

    assert normalize_qtype("GGMLQuantizationType.Q6_K") == "Q6_K"
    assert normalize_qtype(14) == "Q6_K" and normalize_qtype(12) == "Q4_K"
    assert block_layout("Q8_0") == (32, 34)
    with pytest.raises(ValueError, match="unsupported"):
        normalize_qtype("Q3_K")


def _ep_rank(rank, world, port, result_path):
    import torch.distributed as dist
    import torch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qk_b200.experts import expert_parallel

        hidden, inter, count, k = 256, 256, 8, 3
        rng = np.random.default_rng(0)
        raw = {n: gguf.encode_q6_k(rng.normal(0, 0.05, (count,) + shape)).reshape(count, -1)
               for n, shape in (("gate", (inter, hidden)), ("up", (inter, hidden)), ("down", (hidden, inter)))}
        x = rng.normal(size=(9, hidden)).astype(np.float32)
        ids = np.stack([rng.permutation(count)[:k] for _ in range(9)]).astype(np.int32)
        weights = bf16_round(rng.uniform(0.1, 1, (9, k)).astype(np.float32))
        per = count // world
        first = rank * per
        # the library's rank bookkeeping on a real (gloo) process group
        fn = expert_parallel(dist.group.WORLD, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K",
                             hidden=hidden, intermediate=inter)
        assert fn._rank_world() == (rank, world)
        assert fn.desc(per, first, k).first_expert == first
        part = moe.expert_ffn(raw["gate"][first:first + per], raw["up"][first:first + per],
                              raw["down"][first:first + per], x, ids, weights, gate_type="Q6_K",
                              up_type="Q6_K", down_type="Q6_K", hidden=hidden, intermediate=inter,
                              first_expert=first, partial=True)
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        if rank == 0:
            full = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights,
                                  gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K",
                                  hidden=hidden, intermediate=inter)
            np.save(result_path, np.stack([bf16_round(t.numpy()), full]))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_partials_all_reduce_to_the_layer_gloo(tmp_path):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    result = tmp_path / "ep.npy"
    mp.start_processes(_ep_rank, args=(2, port, str(result)), nprocs=2, start_method="spawn")
    got, full = np.load(result)
    assert np.max(np.abs(got - full)) <= 1e-2 * np.max(np.abs(full))
