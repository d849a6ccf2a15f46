"""Tensor parallel inside the experts (grouped_experts.py:113-119): each tensor rank holds
every expert's slice of the intermediate channels, the FP32 down projections of the routes
are summed over the ranks before the BF16 rounding, then route-weighted and combined.

Ranks emulated on one GPU (the FP32 sum of the partials done by hand in rank order), and two
real ranks over NCCL when two GPUs are present.
"""

import os
import socket

import numpy as np
import pytest

from oracle import gguf, moe
from oracle.precision import bf16_round
from util import bf16_tensor, rel_err, to_f32

pytestmark = pytest.mark.gpu

HIDDEN, INTER = 512, 512


def _experts(qtype, count, seed):
    rng = np.random.default_rng(seed)
    return {
        "gate": gguf.encode(rng.normal(0, 0.02, (count, INTER, HIDDEN)), qtype).reshape(count, -1),
        "up": gguf.encode(rng.normal(0, 0.02, (count, INTER, HIDDEN)), qtype).reshape(count, -1),
        "down": gguf.encode(rng.normal(0, 0.02, (count, HIDDEN, INTER)), qtype).reshape(count, -1),
    }


def _tokens(B, k, count, seed):
    rng = np.random.default_rng(seed)
    x = bf16_round(rng.normal(size=(B, HIDDEN)).astype(np.float32))
    ids = np.stack([rng.choice(count, k, replace=False) for _ in range(B)]).astype(np.int32)
    ids[0, 1] = ids[0, 0]  # a repeated expert: the two routes merge into one entry
    w = bf16_round(rng.uniform(0.05, 1.0, (B, k)).astype(np.float32))
    w[1, 0] = 0.0          # a zero weight: the route drops
    return x, ids, w


def _emulated(raw, qtype, x, ids, w, tp, device):
    import torch

    from qk_b200.experts import ExpertFFN
    from qk_b200.parallel import put_expert_bytes

    fn = ExpertFFN(None, qtype, qtype, qtype, HIDDEN, INTER, tensor_parallel=tp)
    xd, idd, wd = bf16_tensor(x, device), torch.from_numpy(ids).to(device), bf16_tensor(w, device)
    total, last = None, None
    for r in range(tp):
        t = {n: put_expert_bytes(raw[n], n, qtype, HIDDEN, INTER, device=device, tensor_rank=r, tensor_parallel=tp)
             for n in raw}
        y_routes, ids32, ws = fn.tensor_partial(t["gate"], t["up"], t["down"], xd, idd, wd)
        total = y_routes.clone() if total is None else total + y_routes
        last = (ids32, ws, t["gate"].shape[0])
    ids32, ws, count = last
    return fn.tensor_combine(total, ids32, ws, count)


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K"])
def test_two_tensor_slices_match_the_whole_experts(cuda_device, qtype):
    import torch

    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes

    count, B, k = 6, 37, 4
    raw = _experts(qtype, count, 51)
    x, ids, w = _tokens(B, k, count, 52)
    got = _emulated(raw, qtype, x, ids, w, 2, cuda_device)
    whole = {n: put_expert_bytes(raw[n], n, qtype, HIDDEN, INTER, device=cuda_device) for n in raw}
    single = expert_parallel(gate_type=qtype, up_type=qtype, down_type=qtype, hidden=HIDDEN, intermediate=INTER)(
        whole["gate"], whole["up"], whole["down"], bf16_tensor(x, cuda_device), torch.from_numpy(ids).to(cuda_device),
        bf16_tensor(w, cuda_device))
    mx, l2 = rel_err(to_f32(got), to_f32(single))
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, w, gate_type=qtype, up_type=qtype,
                              down_type=qtype, hidden=HIDDEN, intermediate=INTER)
    mx, l2 = rel_err(to_f32(got), expected)
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)
    assert np.isfinite(to_f32(got)).all()


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K"])
def test_expert_by_tensor_mesh_emulated(cuda_device, qtype):
    """The ("expert", "tensor") mesh (parallel.py:28-33) with 2 expert ranks x 2 tensor
    ranks emulated on one GPU: each expert rank's tensor slices are summed in FP32 before
    the BF16 rounding (grouped_experts.py:113-119), the expert ranks' FP32 partials are then
    added (experts.py:130-131) and rounded."""
    import torch

    from qk_b200.experts import ExpertFFN, expert_parallel
    from qk_b200.parallel import put_expert_bytes

    ep, tp, per, B, k = 2, 2, 4, 29, 3
    count = ep * per
    raw = _experts(qtype, count, 71)
    x, ids, w = _tokens(B, k, count, 72)
    xd, idd, wd = bf16_tensor(x, cuda_device), torch.from_numpy(ids).to(cuda_device), bf16_tensor(w, cuda_device)
    fn = ExpertFFN(None, qtype, qtype, qtype, HIDDEN, INTER, tensor_parallel=tp)
    total = None
    for e in range(ep):
        y_sum, last = None, None
        for t in range(tp):
            mine = {n: put_expert_bytes(raw[n], n, qtype, HIDDEN, INTER, rank=e, world=ep, device=cuda_device,
                                        tensor_rank=t, tensor_parallel=tp) for n in raw}
            y_routes, ids32, ws = fn.tensor_partial(mine["gate"], mine["up"], mine["down"], xd, idd, wd, e * per)
            y_sum = y_routes.clone() if y_sum is None else y_sum + y_routes
            last = (ids32, ws)
        part = fn.tensor_combine(y_sum, last[0], last[1], per, torch.float32)
        total = part if total is None else total + part
    got = to_f32(total.to(torch.bfloat16))
    whole = {n: put_expert_bytes(raw[n], n, qtype, HIDDEN, INTER, device=cuda_device) for n in raw}
    single = expert_parallel(gate_type=qtype, up_type=qtype, down_type=qtype, hidden=HIDDEN, intermediate=INTER)(
        whole["gate"], whole["up"], whole["down"], xd, idd, wd)
    mx, l2 = rel_err(got, to_f32(single))
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, w, gate_type=qtype, up_type=qtype,
                              down_type=qtype, hidden=HIDDEN, intermediate=INTER)
    mx, l2 = rel_err(got, expected)
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


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
        from qk_b200.experts import expert_parallel
        from qk_b200.parallel import put_expert_bytes

        raw = _experts("Q6_K", 6, 61)
        x, ids, w = _tokens(21, 4, 6, 62)  # the same tokens on both ranks (replicated)
        mine = {n: put_expert_bytes(raw[n], n, "Q6_K", HIDDEN, INTER, device=dev, tensor_rank=rank,
                                    tensor_parallel=world) for n in raw}
        fn = expert_parallel(dist.group.WORLD, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K",
                             hidden=HIDDEN, intermediate=INTER, tensor_parallel=world)
        got = fn(mine["gate"], mine["up"], mine["down"], bf16_tensor(x, dev), torch.from_numpy(ids).to(dev),
                 bf16_tensor(w, dev))
        ref = _emulated(raw, "Q6_K", x, ids, w, world, dev)
        torch.cuda.synchronize(dev)
        np.save(f"{path}.{rank}.npy", np.stack([got.view(torch.int16).cpu().numpy(),
                                                ref.view(torch.int16).cpu().numpy()]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_experts_on_two_gpus_nccl(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = tmp_path / "tp2"
    mp.start_processes(_two_gpu_rank, args=(2, _port(), str(path)), nprocs=2, start_method="spawn")
    r0, r1 = (np.load(f"{path}.{r}.npy") for r in range(2))
    np.testing.assert_array_equal(r0[0], r1[0])
    np.testing.assert_array_equal(r0[0], r0[1])  # a + b is the same sum in either order
