"""Expert parallelism with token dispatch (qk_ep_plan / qk_gather_rows / qk_ep_combine and
ExpertAllToAllNccl) on the GPU: bit-identical to the single-device routed FFN."""

import os

import numpy as np
import pytest

from oracle import gguf
from oracle.precision import bf16_round
from util import bf16_tensor

pytestmark = pytest.mark.gpu

HIDDEN, INTER = 512, 256


def _experts(count, seed):
    rng = np.random.default_rng(seed)
    return {n: gguf.encode_q6_k(rng.normal(0, 0.03, (count,) + shape)).reshape(count, -1)
            for n, shape in (("gate", (INTER, HIDDEN)), ("up", (INTER, HIDDEN)), ("down", (HIDDEN, INTER)))}


def _tokens(B, k, count, seed):
    rng = np.random.default_rng(seed)
    x = bf16_round(rng.normal(size=(B, HIDDEN)).astype(np.float32))
    ids = rng.integers(0, count, (B, k)).astype(np.int32)
    ids[0, 1] = ids[0, 0]          # repeated expert
    w = bf16_round(rng.uniform(0.05, 1, (B, k)).astype(np.float32))
    w[1, 0] = 0.0                  # dropped route
    return x, ids, w


def test_plan_counts_slots_and_merged_weights(cuda_device):
    import torch

    from qk_b200.ep import DeviceOps

    _, ids, w = _tokens(40, 4, 24, 3)
    ops = DeviceOps(("Q6_K",) * 3, HIDDEN, INTER)
    plan = ops.plan(torch.from_numpy(ids).to(cuda_device), bf16_tensor(w, cuda_device), 6, 4)
    counts = plan.send_counts.cpu().numpy()
    slot = plan.route_slot.cpu().numpy()
    rw = plan.route_weight.cpu().numpy()
    rows = plan.send_rows.cpu().numpy()
    expert = plan.send_expert.cpu().numpy()
    live = slot >= 0
    assert counts.sum() == live.sum()
    # merged weights: first slot of an expert carries bf16(sum), repeats and zeros drop
    for b in range(ids.shape[0]):
        for j in range(ids.shape[1]):
            e = ids[b, j]
            if e in ids[b, :j]:
                assert slot[b, j] == -1
            else:
                want = bf16_round(np.float32(w[b, j:][ids[b, j:] == e].sum(dtype=np.float32)))
                assert rw[b, j] == want and (slot[b, j] >= 0) == (want != 0)
    # slots: rank-major, each live route has its own slot holding its token and expert
    starts = np.concatenate([[0], np.cumsum(counts)])
    for b, j in zip(*np.nonzero(live)):
        s = slot[b, j]
        assert rows[s] == b and expert[s] == ids[b, j]
        r = ids[b, j] // 6
        assert starts[r] <= s < starts[r + 1]
    assert len(set(slot[live].tolist())) == live.sum()


def test_all_to_all_layer_on_one_device_equals_routed_ffn(cuda_device):
    import torch

    from qk_b200.ep import ExpertAllToAllNccl
    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes

    count, k = 12, 4
    raw = _experts(count, 11)
    x, ids, w = _tokens(33, k, count, 12)
    t = {n: put_expert_bytes(raw[n], n, "Q6_K", HIDDEN, INTER, device=cuda_device) for n in raw}
    args = (t["gate"], t["up"], t["down"], bf16_tensor(x, cuda_device), torch.from_numpy(ids).to(cuda_device),
            bf16_tensor(w, cuda_device))
    ref = expert_parallel(gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=HIDDEN, intermediate=INTER)(*args)
    fn = ExpertAllToAllNccl(None, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=HIDDEN,
                        intermediate=INTER, experts_per_rank=count)
    got = fn(*args)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def _two_gpu_rank(rank, world, port, path):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from qk_b200.ep import ExpertAllToAllNccl
        from qk_b200.experts import expert_parallel
        from qk_b200.parallel import put_expert_bytes

        per, k = 6, 4
        count = per * world
        raw = _experts(count, 21)
        x, ids, w = _tokens(17 + 5 * rank, k, count, 30 + rank)
        mine = {n: put_expert_bytes(raw[n], n, "Q6_K", HIDDEN, INTER, rank=rank, world=world, device=dev) for n in raw}
        fn = ExpertAllToAllNccl(dist.group.WORLD, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K",
                            hidden=HIDDEN, intermediate=INTER, experts_per_rank=per)
        xd, idd, wd = bf16_tensor(x, dev), torch.from_numpy(ids).to(dev), bf16_tensor(w, dev)
        got = fn(mine["gate"], mine["up"], mine["down"], xd, idd, wd)
        every = {n: put_expert_bytes(raw[n], n, "Q6_K", HIDDEN, INTER, device=dev) for n in raw}
        ref = expert_parallel(gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=HIDDEN,
                              intermediate=INTER)(every["gate"], every["up"], every["down"], xd, idd, wd)
        torch.cuda.synchronize(dev)
        np.save(f"{path}.{rank}.npy", np.stack([got.view(torch.int16).cpu().numpy(),
                                                ref.view(torch.int16).cpu().numpy()]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_all_to_all_layer_on_two_gpus_nccl(tmp_path):
    import socket

    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = tmp_path / "ep2"
    mp.start_processes(_two_gpu_rank, args=(2, port, str(path)), nprocs=2, start_method="spawn")
    for rank in range(2):
        got, ref = np.load(f"{path}.{rank}.npy")
        np.testing.assert_array_equal(got, ref)
