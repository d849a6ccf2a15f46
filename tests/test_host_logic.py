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


# ---- expert parallel with token dispatch (all-to-all), orchestration on gloo ----


class _NumpyOps:
    """The four local steps of ExpertAllToAllNccl restated with the oracle (CPU, test only)."""

    def __init__(self, qtype, hidden, intermediate):
        self.qtype, self.hidden, self.intermediate = qtype, hidden, intermediate

    def plan(self, ids, weights, experts_per_rank, world):
        import torch

        from qk_b200.ep import Plan

        ids_n = ids.numpy()
        w_n = weights.float().numpy()
        B, k = ids_n.shape
        n_exp = experts_per_rank * world
        route_weight = np.zeros((B, k), np.float32)
        for b in range(B):
            for j in range(k):
                e = ids_n[b, j]
                if e < 0 or e >= n_exp or e in ids_n[b, :j]:
                    continue
                route_weight[b, j] = bf16_round(np.float32(w_n[b, j:][ids_n[b, j:] == e].sum(dtype=np.float32)))
        live = [(b, j) for b in range(B) for j in range(k) if route_weight[b, j] != 0]
        live.sort(key=lambda bj: ids_n[bj] // experts_per_rank)  # stable: token order per rank
        counts = np.bincount([ids_n[bj] // experts_per_rank for bj in live], minlength=world)
        slot = np.full((B, k), -1, np.int32)
        rows = np.zeros(max(B * k, 1), np.int32)
        expert = np.zeros(max(B * k, 1), np.int32)
        for s, (b, j) in enumerate(live):
            slot[b, j], rows[s], expert[s] = s, b, ids_n[b, j]
        return Plan(torch.from_numpy(counts.astype(np.int64)), torch.from_numpy(rows),
                    torch.from_numpy(expert), torch.from_numpy(slot), torch.from_numpy(route_weight))

    def gather(self, x, rows):
        return x[rows.long()]

    def local_ffn(self, gate, up, down, x, experts, first_expert):
        import torch

        xs = x.float().numpy()
        out = np.zeros((xs.shape[0], self.hidden), np.float32)
        for i, e in enumerate(experts.numpy()):
            le = int(e) - first_expert
            wg = moe.expert_weights(gate[le], self.qtype, self.intermediate, self.hidden)
            wu = moe.expert_weights(up[le], self.qtype, self.intermediate, self.hidden)
            wd = moe.expert_weights(down[le], self.qtype, self.hidden, self.intermediate)
            out[i] = moe.expert_forward(xs[i:i + 1], wg, wu, wd)[0]
        return torch.from_numpy(out)

    def combine(self, y, plan, ids, hidden):
        import torch

        ys = y.float().numpy()
        slot, w, ids_n = plan.route_slot.numpy(), plan.route_weight.numpy(), ids.numpy()
        out = np.zeros((ids_n.shape[0], hidden), np.float32)
        for b in range(ids_n.shape[0]):
            for j in np.argsort(np.where(slot[b] >= 0, ids_n[b], np.iinfo(np.int32).max), kind="stable"):
                if slot[b, j] >= 0:
                    out[b] = (out[b] + (ys[slot[b, j]] * w[b, j]).astype(np.float32)).astype(np.float32)
        return torch.from_numpy(bf16_round(out))


def _a2a_rank(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qk_b200.ep import ExpertAllToAllNccl

        hidden, inter, per, k = 256, 256, 3, 3
        count = per * world
        rng = np.random.default_rng(7)  # same experts on every rank
        raw = {n: gguf.encode_q6_k(rng.normal(0, 0.05, (count,) + shape)).reshape(count, -1)
               for n, shape in (("gate", (inter, hidden)), ("up", (inter, hidden)), ("down", (hidden, inter)))}
        trng = np.random.default_rng(100 + rank)  # this rank's own tokens
        B = 5 + rank
        x = bf16_round(trng.normal(size=(B, hidden)).astype(np.float32))
        ids = trng.integers(0, count, (B, k)).astype(np.int32)
        ids[0, 1] = ids[0, 0]  # a repeated expert: one route of weight bf16(w0 + w1)
        weights = bf16_round(trng.uniform(0.1, 1, (B, k)).astype(np.float32))
        weights[1, 2] = 0.0    # a dropped route
        mine = slice(rank * per, (rank + 1) * per)
        fn = ExpertAllToAllNccl(dist.group.WORLD, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K",
                            hidden=hidden, intermediate=inter, experts_per_rank=per,
                            ops=_NumpyOps("Q6_K", hidden, inter))
        got = fn(raw["gate"][mine], raw["up"][mine], raw["down"][mine], torch.from_numpy(x),
                 torch.from_numpy(ids), torch.from_numpy(weights)).numpy()
        expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type="Q6_K",
                                  up_type="Q6_K", down_type="Q6_K", hidden=hidden, intermediate=inter)
        np.save(f"{result_path}.{rank}.npy", np.stack([got, expected]))
    finally:
        dist.destroy_process_group()


def test_expert_all_to_all_dispatch_matches_single_device_layer_gloo(tmp_path):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    result = tmp_path / "a2a"
    mp.start_processes(_a2a_rank, args=(2, port, str(result)), nprocs=2, start_method="spawn")
    for rank in range(2):
        got, expected = np.load(f"{result}.{rank}.npy")
        np.testing.assert_array_equal(got, expected)


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K"])
def test_tensor_slices_are_the_split_expert_bytes(qtype):
    """put_expert_bytes' tensor slice (NumPy or torch input) equals the reference's split."""
    import torch

    from qk_b200.parallel import split_expert_bytes, tensor_slice
    from qk_b200.quant import block_layout

    hidden, inter = 512, 1024
    rng = np.random.default_rng(9)
    size = block_layout(qtype)[1]
    for kind, rows, width in (("gate", inter, hidden), ("up", inter, hidden), ("down", hidden, inter)):
        raw = rng.integers(0, 256, (3, rows * (width // 256) * size), dtype=np.uint8)
        for tp in (1, 2, 4):
            split = split_expert_bytes(raw, kind, qtype, hidden, inter, tp)
            for r in range(tp):
                np.testing.assert_array_equal(tensor_slice(raw, kind, qtype, hidden, inter, tp, r), split[r])
                got = tensor_slice(torch.from_numpy(raw), kind, qtype, hidden, inter, tp, r)
                np.testing.assert_array_equal(got.contiguous().numpy(), split[r])
    with pytest.raises(ValueError, match="whole down"):
        tensor_slice(np.zeros((1, 512 * 2 * size), np.uint8), "down", qtype, 512, 512, 4, 0)


def test_tensor_parallel_factory_contract():
    from qk_b200.experts import expert_parallel

    with pytest.raises(ValueError, match="process group"):
        expert_parallel(None, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=2048,
                        intermediate=512, tensor_parallel=2)


def _mesh_rank(rank, world, port, path):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qk_b200.experts import expert_parallel

        fn = expert_parallel(dist.group.WORLD, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=2048,
                             intermediate=512, tensor_parallel=2)
        tg = dist.get_process_group_ranks(fn.tensor_group)
        eg = dist.get_process_group_ranks(fn.expert_group)
        np.save(f"{path}.{rank}.npy", np.array([fn.expert_rank] + tg + eg))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_expert_tensor_mesh_groups_on_gloo(tmp_path):
    """The ("expert", "tensor") mesh of parallel.py:28-33 over 4 ranks with tp = 2: rank
    e * 2 + t sums its tensor slices with rank e * 2 + (1 - t) and its expert partials with
    rank (1 - e) * 2 + t."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    path = tmp_path / "mesh"
    mp.start_processes(_mesh_rank, args=(4, port, str(path)), nprocs=4, start_method="spawn")
    for rank in range(4):
        e, t = divmod(rank, 2)
        got = np.load(f"{path}.{rank}.npy").tolist()
        assert got == [e, 2 * e, 2 * e + 1, t, 2 + t]
