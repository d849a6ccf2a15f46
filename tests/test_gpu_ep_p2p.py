"""The peer-to-peer expert-parallel layer (qk_ep_p2p_*, qk_b200.ep.ExpertAllToAll).

* One rank: bit-identical to the single-device routed FFN (expert_parallel), over several
  calls in a row (the exchange's epochs advance) with varying batch sizes, an empty batch
  included.
* W ranks emulated on one device (every region allocated in this process, the peer table
  pointing at all of them; each rank's launches run in stream order, so every wait finds its
  flag already raised): each token's output equals the reference's expert-parallel
  arithmetic - every rank's FP32 partial over its experts (qk_moe_forward with QK_OUT_F32,
  the all-reduce form's local sum) added in ascending rank order, then one BF16 rounding
  (experts.py:128-131) - bit for bit, and agrees with the oracle within the layer tolerance.
* Two GPUs: the same on two processes over NVLink (skipped with fewer GPUs).
"""

import os

import numpy as np
import pytest

from oracle import gguf, moe
from oracle.precision import bf16_round
from util import bf16_tensor, rel_err, to_f32

pytestmark = pytest.mark.gpu

HIDDEN, INTER = 512, 256


def _experts(count, seed):
    rng = np.random.default_rng(seed)
    return {n: gguf.encode_q6_k(rng.normal(0, 0.03, (count,) + shape)).reshape(count, -1)
            for n, shape in (("gate", (INTER, HIDDEN)), ("up", (INTER, HIDDEN)), ("down", (HIDDEN, INTER)))}


def _tokens(B, k, count, seed):
    rng = np.random.default_rng(seed)
    x = bf16_round(rng.normal(size=(B, HIDDEN)).astype(np.float32))
    ids = np.stack([rng.choice(count, k, replace=False) for _ in range(B)]).astype(np.int32) if B else \
        np.zeros((0, k), np.int32)
    w = bf16_round(rng.uniform(0.05, 1, (B, k)).astype(np.float32))
    if B > 3:
        ids[0, 1] = ids[0, 0]      # repeated expert: merged
        w[1, :] = 0.0              # a finished row: exactly zero
        w[2, 0] = 0.0              # one dropped route
    return x, ids, w


def _partial_sum_reference(dev, raw_dev, per, world, x, ids, w, types=("Q6_K",) * 3):
    """The expert-parallel arithmetic from the single-device kernels: each rank's FP32
    partial (QK_OUT_F32 over its expert range), added in rank order, one BF16 rounding."""
    import torch

    from qk_b200 import _lib
    from qk_b200.quant import GGML_TYPE

    B, k = ids.shape
    total = np.zeros((B, HIDDEN), np.float32)
    xd, idd, wd = bf16_tensor(x, dev), torch.from_numpy(ids).to(dev), bf16_tensor(w, dev)
    for r in range(world):
        desc = _lib.MoeDesc(*(GGML_TYPE[t] for t in types), HIDDEN, INTER, per, r * per, k)
        ws = torch.empty(int(_lib.load().qk_moe_workspace_bytes(desc, B)), dtype=torch.uint8, device=dev)
        part = torch.empty((B, HIDDEN), dtype=torch.float32, device=dev)
        sl = slice(r * per, (r + 1) * per)
        _lib.call("qk_moe_forward", desc, _lib.ptr(raw_dev["gate"][sl]), _lib.ptr(raw_dev["up"][sl]),
                  _lib.ptr(raw_dev["down"][sl]), _lib.ptr(xd), _lib.ptr(idd), _lib.ptr(wd), B, _lib.QK_OUT_F32,
                  _lib.ptr(part), _lib.ptr(ws), ws.numel(), _lib.stream_handle(dev))
        total = (total + part.cpu().numpy()).astype(np.float32)
    return bf16_round(total)


def test_one_rank_is_bit_identical_to_the_routed_ffn_over_consecutive_calls(cuda_device):
    import torch

    from qk_b200.ep import ExpertAllToAll
    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes

    count, k, max_tokens = 12, 4, 40
    raw = _experts(count, 11)
    t = {n: put_expert_bytes(raw[n], n, "Q6_K", HIDDEN, INTER, device=cuda_device) for n in raw}
    ref_fn = expert_parallel(gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=HIDDEN, intermediate=INTER)
    fn = ExpertAllToAll(None, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=HIDDEN,
                        intermediate=INTER, experts_per_rank=count, top_k=k, max_tokens=max_tokens,
                        device=cuda_device)
    try:
        for step, B in enumerate((33, 40, 0, 7, 33)):
            x, ids, w = _tokens(B, k, count, 12 + step)
            args = (t["gate"], t["up"], t["down"], bf16_tensor(x, cuda_device),
                    torch.from_numpy(ids).to(cuda_device), bf16_tensor(w, cuda_device))
            got = fn(*args).clone()
            if B == 0:
                assert got.shape == (0, HIDDEN)
                continue
            ref = ref_fn(*args)
            torch.cuda.synchronize(cuda_device)
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), step
            assert torch.all(got[1] == 0)
        fn.check_status()
    finally:
        fn.close()


@pytest.mark.parametrize("world,per,k", [(2, 6, 4), (4, 3, 4), (4, 16, 10)])
def test_emulated_ranks_match_the_expert_parallel_arithmetic(cuda_device, world, per, k):
    import torch

    from qk_b200 import _lib
    from qk_b200.ep import ExchangeRegion, ExpertAllToAll
    from qk_b200.parallel import put_expert_bytes

    count, max_tokens = per * world, 24
    raw = _experts(count, 40 + world)
    every = {n: put_expert_bytes(raw[n], n, "Q6_K", HIDDEN, INTER, device=cuda_device) for n in raw}
    lib = _lib.load()
    nbytes = int(lib.qk_ep_p2p_bytes(world, max_tokens, HIDDEN, k))
    buffers = [torch.empty(nbytes, dtype=torch.uint8, device=cuda_device) for _ in range(world)]
    for buf in buffers:
        _lib.call("qk_ep_p2p_reset", _lib.ptr(buf), _lib.stream_handle(cuda_device))
    shared = {"world": world, "regions": [buf.data_ptr() for buf in buffers]}
    layers = []
    for r in range(world):
        region = ExchangeRegion(None, max_tokens=max_tokens, hidden=HIDDEN, top_k=k, device=cuda_device,
                                rank=r, shared=shared)
        layers.append(ExpertAllToAll(None, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=HIDDEN,
                                     intermediate=INTER, experts_per_rank=per, top_k=k, max_tokens=max_tokens,
                                     device=cuda_device, region=region))
    lib = _lib.load()
    st = _lib.stream_handle(cuda_device)
    for step in range(2):
        batches = [max_tokens - 3 * r - step for r in range(world)]
        inputs = [_tokens(B, k, count, 100 * step + r) for r, B in enumerate(batches)]
        dev_in = [(bf16_tensor(x, cuda_device), torch.from_numpy(ids).to(cuda_device), bf16_tensor(w, cuda_device))
                  for x, ids, w in inputs]
        outs = [torch.empty((B, HIDDEN), dtype=torch.bfloat16, device=cuda_device) for B in batches]
        # the three phases of every rank in turn: each wait finds its flags raised
        for r, fn in enumerate(layers):
            xd, idd, wd = dev_in[r]
            _lib.check(lib.qk_ep_p2p_dispatch(_lib.ptr(fn.region.peers), fn.region.region, world, r, max_tokens,
                                              HIDDEN, k, per, _lib.ptr(xd), _lib.ptr(idd), _lib.ptr(wd),
                                              batches[r], st))
        for r, fn in enumerate(layers):
            sl = slice(r * per, (r + 1) * per)
            _lib.check(lib.qk_ep_p2p_expert(fn.desc, _lib.ptr(every["gate"][sl]), _lib.ptr(every["up"][sl]),
                                            _lib.ptr(every["down"][sl]), _lib.ptr(fn.region.peers),
                                            fn.region.region, world, r, max_tokens, _lib.ptr(fn.workspace),
                                            fn.workspace.numel(), st))
        for r, fn in enumerate(layers):
            _, idd, wd = dev_in[r]
            _lib.check(lib.qk_ep_p2p_combine(fn.region.region, world, r, max_tokens, HIDDEN, k, per, _lib.ptr(idd),
                                             _lib.ptr(wd), batches[r], _lib.ptr(outs[r]), st))
        torch.cuda.synchronize(cuda_device)
        for r, fn in enumerate(layers):
            fn.region.status()
            x, ids, w = inputs[r]
            want = _partial_sum_reference(cuda_device, every, per, world, x, ids, w)
            got = to_f32(outs[r])
            np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
            expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, w, gate_type="Q6_K",
                                      up_type="Q6_K", down_type="Q6_K", hidden=HIDDEN, intermediate=INTER)
            mx, l2 = rel_err(got, expected)
            assert mx < 1e-2 and l2 < 2e-3, (r, mx, l2)
            np.testing.assert_array_equal(got[1], 0)


def _two_gpu_rank(rank, world, port, path):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    fn = None
    try:
        from qk_b200.ep import ExpertAllToAll
        from qk_b200.parallel import put_expert_bytes

        per, k, max_tokens = 6, 4, 32
        count = per * world
        raw = _experts(count, 21)
        mine = {n: put_expert_bytes(raw[n], n, "Q6_K", HIDDEN, INTER, rank=rank, world=world, device=dev)
                for n in raw}
        every = {n: put_expert_bytes(raw[n], n, "Q6_K", HIDDEN, INTER, device=dev) for n in raw}
        fn = ExpertAllToAll(dist.group.WORLD, gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=HIDDEN,
                            intermediate=INTER, experts_per_rank=per, top_k=k, max_tokens=max_tokens, device=dev)
        results = []
        for step in range(3):
            x, ids, w = _tokens(17 + 5 * rank + step, k, count, 30 + 10 * step + rank)
            got = fn(mine["gate"], mine["up"], mine["down"], bf16_tensor(x, dev), torch.from_numpy(ids).to(dev),
                     bf16_tensor(w, dev)).clone()
            torch.cuda.synchronize(dev)
            want = _partial_sum_reference(dev, every, per, world, x, ids, w)
            results.append(np.array_equal(to_f32(got).view(np.uint32), want.view(np.uint32)))
        fn.check_status()
        np.save(f"{path}.{rank}.npy", np.array(results))
        dist.barrier()
    finally:
        if fn is not None:
            torch.cuda.synchronize(dev)
            dist.barrier()
            fn.close()
        dist.destroy_process_group()


def test_peer_to_peer_layer_on_two_gpus(tmp_path):
    import socket

    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = tmp_path / "p2p"
    mp.start_processes(_two_gpu_rank, args=(2, port, str(path)), nprocs=2, start_method="spawn")
    for rank in range(2):
        assert np.load(f"{path}.{rank}.npy").all(), rank
