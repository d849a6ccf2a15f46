"""Decoder-layer glue kernels and one layer of the synthetic decoder stack against the oracle.

The stack's step is checked stage by stage: each stage's GPU output is compared with the
oracle applied to the GPU's own input of that stage, so a near-tie somewhere upstream
cannot move a later comparison.
"""

import numpy as np
import pytest

from oracle import kv, layer, layout, moe
from oracle.precision import bf16_round
from util import bf16_tensor, rel_err, to_f32

pytestmark = pytest.mark.gpu


def test_rms_norm_matches_oracle(cuda_device):
    from qk_b200 import _lib

    rng = np.random.default_rng(3)
    x = bf16_round(rng.normal(size=(7, 2048)).astype(np.float32) * 3)
    gamma = bf16_round(rng.uniform(0.5, 1.5, 2048).astype(np.float32))
    xd, gd = bf16_tensor(x, cuda_device), bf16_tensor(gamma, cuda_device)
    out = xd.clone()
    _lib.call("qk_rms_norm", _lib.ptr(xd), _lib.ptr(gd), 7, 2048, 1e-6, _lib.ptr(out), _lib.stream_handle(cuda_device))
    got, expected = to_f32(out), layer.rms(x, gamma, 1e-6)
    assert np.mean(got == expected) > 0.99
    assert rel_err(got, expected)[0] < 1e-2


def test_qk_norm_rope_matches_oracle(cuda_device):
    import torch

    from qk_b200 import _lib

    rng = np.random.default_rng(4)
    B, hq, kvh, hd, rot = 3, 16, 2, 256, 64
    qkv = bf16_round(rng.normal(size=(B, (2 * hq + 2 * kvh) * hd)).astype(np.float32))
    qn = bf16_round(rng.uniform(0.5, 1.5, hd).astype(np.float32))
    kn = bf16_round(rng.uniform(0.5, 1.5, hd).astype(np.float32))
    pos = np.array([0, 17, 8191], np.int32)
    inv = layer.inv_freq(rot, 1e7)
    outs = [torch.empty((B, h, hd), dtype=torch.bfloat16, device=cuda_device) for h in (hq, hq, kvh, kvh)]
    # device inputs stay referenced until the kernel has run (the caching allocator would
    # otherwise hand a freed input's memory to the next one)
    ins = [bf16_tensor(qkv, cuda_device), bf16_tensor(qn, cuda_device), bf16_tensor(kn, cuda_device),
           torch.from_numpy(inv).to(cuda_device), torch.from_numpy(pos).to(cuda_device)]
    _lib.call("qk_qk_norm_rope", *[_lib.ptr(t) for t in ins], B, hq, kvh, hd, rot, 1e-6,
              *[_lib.ptr(o) for o in outs], _lib.stream_handle(cuda_device))
    torch.cuda.synchronize(cuda_device)
    expected = layer.qk_norm_rope(qkv, qn, kn, pos, hq, kvh, hd, rot, 1e7, 1e-6)
    for name, got, exp in zip(("q", "gate", "k", "v"), outs, expected):
        got = to_f32(got)
        if name in ("gate", "v"):
            np.testing.assert_array_equal(got, exp)
        else:
            assert np.mean(got == exp) > 0.98, name
            assert rel_err(got, exp)[0] < 1e-2, name


def test_residual_add_and_shared_route(cuda_device):
    import torch

    from qk_b200 import _lib

    rng = np.random.default_rng(5)
    x = bf16_round(rng.normal(size=(5, 512)).astype(np.float32))
    y = bf16_round(rng.normal(size=(5, 512)).astype(np.float32))
    xd, yd = bf16_tensor(x, cuda_device), bf16_tensor(y, cuda_device)
    _lib.call("qk_residual_add", _lib.ptr(xd), _lib.ptr(yd), x.size, _lib.ptr(xd), _lib.stream_handle(cuda_device))
    np.testing.assert_array_equal(to_f32(xd), bf16_round(x + y))
    ids = rng.integers(0, 64, (5, 4)).astype(np.int32)
    w = bf16_round(rng.uniform(0, 1, (5, 4)).astype(np.float32))
    wsr = bf16_round(rng.normal(0, 0.05, 512).astype(np.float32))
    ids_out = torch.empty((5, 5), dtype=torch.int32, device=cuda_device)
    w_out = torch.empty((5, 5), dtype=torch.bfloat16, device=cuda_device)
    ins = [torch.from_numpy(ids).to(cuda_device), bf16_tensor(w, cuda_device), bf16_tensor(x, cuda_device),
           bf16_tensor(wsr, cuda_device)]
    _lib.call("qk_append_shared_route", _lib.ptr(ins[0]), _lib.ptr(ins[1]), 5, 4, _lib.ptr(ins[2]),
              _lib.ptr(ins[3]), 512, 64, _lib.ptr(ids_out), _lib.ptr(w_out), _lib.stream_handle(cuda_device))
    got_ids, got_w = ids_out.cpu().numpy(), to_f32(w_out)
    np.testing.assert_array_equal(got_ids[:, :4], ids)
    assert (got_ids[:, 4] == 64).all()
    np.testing.assert_array_equal(got_w[:, :4], w)
    gate = layer.shared_gate(x, wsr)
    assert np.max(np.abs(got_w[:, 4] - gate)) <= 2 ** -8  # one BF16 step of a value in (0, 1)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_checked_argmax(cuda_device, dtype):
    import torch

    from qk_b200.decoder import checked_argmax

    rng = np.random.default_rng(6)
    V = 151936
    logits = bf16_round(rng.normal(size=(6, V)).astype(np.float32))
    logits[1, [5, 70000, 151935]] = 9.0            # tied maximum: the first one
    logits[2, 1234] = np.nan                        # a NaN is the maximum
    logits[2, 99] = np.inf
    logits[3, :] = np.nan                           # all NaN: index 0, V non-finite
    logits[4, :] = -np.inf                          # all -inf: index 0
    logits[5, [7, 8]] = [np.inf, np.inf]            # +inf ties
    t = torch.from_numpy(logits).to(cuda_device)
    got = checked_argmax(t.bfloat16() if dtype == "bf16" else t).cpu().numpy()
    np.testing.assert_array_equal(got, layer.checked_argmax(logits))
    assert got[3].tolist() == [0, V] and got[1, 0] == 5 and got[2].tolist() == [1234, 2]


def _np(t):
    return to_f32(t) if t.dtype == __import__("torch").bfloat16 else t.float().cpu().numpy()


@pytest.mark.parametrize("qtype,down_qtype", [("Q6_K", None), ("Q4_K", None), ("Q6_K", "Q8_0")])
def test_one_decoder_layer_stage_by_stage(cuda_device, qtype, down_qtype):
    import torch

    from qk_b200.decoder import StackConfig, SyntheticDecoder

    cfg = StackConfig(layers=1, hidden=512, intermediate=256, experts=8, top_k=2, query_heads=8, kv_heads=2,
                      head_dim=128, rotary_dim=32, context=256, page=16, qtype=qtype, down_qtype=down_qtype)
    model = SyntheticDecoder(cfg, cuda_device, seed=11)
    state = model.state(3, seed=12)
    L = model.layers[0]
    cache0 = {n: (state.caches[0][n].cpu().numpy() if n in ("k", "v") else to_f32(state.caches[0][n]))
              for n in ("k", "v", "k_scale", "v_scale")}
    x0 = to_f32(state.x)
    state.step()
    torch.cuda.synchronize(cuda_device)
    hq, kvh, hd, H = cfg.query_heads, cfg.kv_heads, cfg.head_dim, cfg.hidden
    pos = state.positions.cpu().numpy()
    idx = state.indices.cpu().numpy()

    # attention half
    qkv = to_f32(state.qkv)
    mx, _ = rel_err(qkv, layer.linear(layer.rms(x0, _np(L.attn_norm), cfg.eps), _np(L.w_qkv)))
    assert mx < 1e-2, ("qkv", mx)
    q, gate, k, v = layer.qk_norm_rope(qkv, _np(L.q_norm), _np(L.k_norm), pos, hq, kvh, hd, cfg.rotary_dim,
                                       cfg.rope_theta, cfg.eps)
    assert rel_err(to_f32(state.q), q)[0] < 1e-2 and rel_err(to_f32(state.k), k)[0] < 1e-2
    np.testing.assert_array_equal(to_f32(state.gate), gate)
    kv.write_quantized(cache0, to_f32(state.k), to_f32(state.v), pos, np.ones(3, bool), kvh, hd)
    for n in ("k", "v"):
        np.testing.assert_array_equal(state.caches[0][n].cpu().numpy(), cache0[n])
    keys = kv.read_quantized(cache0["k"], cache0["k_scale"], idx, kvh, hd)
    values = kv.read_quantized(cache0["v"], cache0["v_scale"], idx, kvh, hd)
    o = kv.attention(to_f32(state.q), keys, values, np.arange(cfg.context)[None, :] <= pos[:, None],
                     to_f32(state.gate))
    mx, l2 = rel_err(to_f32(state.o), o)
    assert mx < 1e-2 and l2 < 5e-3, ("attention", mx, l2)
    a = to_f32(state.a)
    assert rel_err(a, layer.linear(to_f32(state.o).reshape(3, -1), _np(L.w_o)))[0] < 1e-2
    x1 = bf16_round((x0 + a).astype(np.float32))

    # MoE half
    h2 = to_f32(state.h)
    assert rel_err(h2, layer.rms(x1, _np(L.ffn_norm), cfg.eps))[0] < 1e-2
    ids_all = state.ids_all[0].cpu().numpy()
    w_all = to_f32(state.w_all)
    ids, w, _ = moe.routes(h2, _np(L.router), cfg.top_k)
    np.testing.assert_array_equal(ids_all[:, :cfg.top_k], ids)
    np.testing.assert_array_equal(w_all[:, :cfg.top_k], w)
    assert (ids_all[:, cfg.top_k] == cfg.experts).all()
    assert np.max(np.abs(w_all[:, cfg.top_k] - layer.shared_gate(h2, _np(L.shared_router)))) <= 2 ** -8
    raw = {}
    down_qtype = down_qtype or qtype
    for kind in ("gate", "up", "down"):
        rows, width = (H, cfg.intermediate) if kind == "down" else (cfg.intermediate, H)
        t = L.experts[kind].cpu().numpy()
        kt = down_qtype if kind == "down" else qtype
        raw[kind] = np.stack([layout.untile(t[e], kt, rows, width).reshape(-1) for e in range(t.shape[0])])
    y = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], h2, ids_all, w_all, gate_type=qtype, up_type=qtype,
                       down_type=down_qtype, hidden=H, intermediate=cfg.intermediate)
    mx, l2 = rel_err(to_f32(state.y), y)
    assert mx < 1e-2 and l2 < 5e-3, ("experts", mx, l2)
    np.testing.assert_array_equal(to_f32(state.x), bf16_round((x1 + to_f32(state.y)).astype(np.float32)))


def test_stack_step_in_a_cuda_graph_is_finite_and_repeatable(cuda_device):
    import torch

    from qk_b200.decoder import StackConfig, SyntheticDecoder

    cfg = StackConfig(layers=3, experts=64, top_k=4, context=1024)
    model = SyntheticDecoder(cfg, cuda_device, seed=21)
    state = model.state(8, seed=22)
    x0 = state.x.clone()
    state.step()
    eager = state.x.clone()
    graph = torch.cuda.CUDAGraph()
    state.x.copy_(x0)
    torch.cuda.synchronize(cuda_device)
    with torch.cuda.graph(graph):
        state.step()
    state.x.copy_(x0)
    graph.replay()
    torch.cuda.synchronize(cuda_device)
    assert torch.isfinite(state.x.float()).all()
    assert torch.equal(state.x.view(torch.int16), eager.view(torch.int16))
    nbytes, distinct = state.step_bytes()
    assert len(distinct) == 3 and all(1 <= d <= 65 for d in distinct) and nbytes > 0


def test_expert_parallel_shared_route_renumbers_the_routed_experts(cuda_device):
    """qk_append_shared_route_ep: routed expert e -> (e / per) * (per + 1) + e % per (each rank's
    slice followed by its copy of the shared expert), the shared route names this rank's copy,
    and the gate weight is the one qk_append_shared_route computes."""
    import torch

    from qk_b200 import _lib

    rng = np.random.default_rng(12)
    B, k, H, per, rank = 9, 10, 2048, 64, 3
    ids = np.stack([rng.choice(8 * per, k, replace=False) for _ in range(B)]).astype(np.int32)
    w = bf16_round(rng.uniform(0.01, 0.2, (B, k)).astype(np.float32))
    h = bf16_round(rng.normal(size=(B, H)).astype(np.float32))
    wsr = bf16_round(rng.normal(0, 0.02, H).astype(np.float32))
    idd, wd = torch.from_numpy(ids).to(cuda_device), bf16_tensor(w, cuda_device)
    hd, wsd = bf16_tensor(h, cuda_device), bf16_tensor(wsr, cuda_device)
    st = _lib.stream_handle(cuda_device)
    outs = {}
    for name, extra in (("plain", (8 * per,)), ("ep", (per, rank))):
        ids_all = torch.empty((B, k + 1), dtype=torch.int32, device=cuda_device)
        w_all = torch.empty((B, k + 1), dtype=torch.bfloat16, device=cuda_device)
        fn = "qk_append_shared_route" if name == "plain" else "qk_append_shared_route_ep"
        _lib.call(fn, _lib.ptr(idd), _lib.ptr(wd), B, k, _lib.ptr(hd), _lib.ptr(wsd), H, *extra,
                  _lib.ptr(ids_all), _lib.ptr(w_all), st)
        outs[name] = (ids_all.cpu().numpy(), to_f32(w_all))
    ids_ep, w_ep = outs["ep"]
    np.testing.assert_array_equal(ids_ep[:, :k], (ids // per) * (per + 1) + ids % per)
    np.testing.assert_array_equal(ids_ep[:, k], rank * (per + 1) + per)
    np.testing.assert_array_equal(w_ep, outs["plain"][1])


def test_residual_rms_norm_is_residual_add_then_rms_norm(cuda_device):
    """The fused launch gives the bits of qk_residual_add followed by qk_rms_norm, with x_out
    aliasing x as the decoder step uses it."""
    import torch

    from qk_b200 import _lib

    rng = np.random.default_rng(21)
    rows, width = 7, 2048
    x = bf16_round(rng.normal(size=(rows, width)).astype(np.float32))
    y = bf16_round(rng.normal(size=(rows, width)).astype(np.float32))
    g = bf16_round(rng.normal(1, 0.1, width).astype(np.float32))
    st = _lib.stream_handle(cuda_device)
    x1, yd, gd = bf16_tensor(x, cuda_device), bf16_tensor(y, cuda_device), bf16_tensor(g, cuda_device)
    h1 = torch.empty((rows, width), dtype=torch.bfloat16, device=cuda_device)
    _lib.call("qk_residual_add", _lib.ptr(x1), _lib.ptr(yd), rows * width, _lib.ptr(x1), st)
    _lib.call("qk_rms_norm", _lib.ptr(x1), _lib.ptr(gd), rows, width, 1e-6, _lib.ptr(h1), st)
    x2 = bf16_tensor(x, cuda_device)
    h2 = torch.empty_like(h1)
    _lib.call("qk_residual_rms_norm", _lib.ptr(x2), _lib.ptr(yd), _lib.ptr(gd), rows, width, 1e-6, _lib.ptr(x2),
              _lib.ptr(h2), st)
    assert torch.equal(x1.view(torch.int16), x2.view(torch.int16))
    assert torch.equal(h1.view(torch.int16), h2.view(torch.int16))


@pytest.mark.parametrize("per", [0, 64])
def test_router_select_shared_is_topk_then_shared_route(cuda_device, per):
    """qk_router_select_shared gives the bits of qk_router_topk_logits followed by
    qk_append_shared_route (per = 0) or its expert-parallel form (per > 0)."""
    import torch

    from qk_b200 import _lib

    rng = np.random.default_rng(22 + per)
    B, E, k, H, rank = 11, 512, 10, 2048, 3
    logits = torch.from_numpy(rng.normal(0, 1, (B, E)).astype(np.float32)).to(cuda_device)
    h = bf16_tensor(rng.normal(size=(B, H)).astype(np.float32), cuda_device)
    wsr = bf16_tensor(rng.normal(0, 0.02, H).astype(np.float32), cuda_device)
    st = _lib.stream_handle(cuda_device)
    ids = torch.empty((B, k), dtype=torch.int32, device=cuda_device)
    w = torch.empty((B, k), dtype=torch.bfloat16, device=cuda_device)
    _lib.call("qk_router_topk_logits", _lib.ptr(logits), None, B, E, k, _lib.ptr(ids), _lib.ptr(w), None, st)
    ref_ids = torch.empty((B, k + 1), dtype=torch.int32, device=cuda_device)
    ref_w = torch.empty((B, k + 1), dtype=torch.bfloat16, device=cuda_device)
    shared_id = E if per == 0 else rank * (per + 1) + per
    if per == 0:
        _lib.call("qk_append_shared_route", _lib.ptr(ids), _lib.ptr(w), B, k, _lib.ptr(h), _lib.ptr(wsr), H, E,
                  _lib.ptr(ref_ids), _lib.ptr(ref_w), st)
    else:
        _lib.call("qk_append_shared_route_ep", _lib.ptr(ids), _lib.ptr(w), B, k, _lib.ptr(h), _lib.ptr(wsr), H, per,
                  rank, _lib.ptr(ref_ids), _lib.ptr(ref_w), st)
    got_ids = torch.empty_like(ref_ids)
    got_w = torch.empty_like(ref_w)
    _lib.call("qk_router_select_shared", _lib.ptr(logits), None, B, E, k, _lib.ptr(h), _lib.ptr(wsr), H, shared_id,
              per, _lib.ptr(got_ids), _lib.ptr(got_w), st)
    assert torch.equal(got_ids, ref_ids)
    assert torch.equal(got_w.view(torch.int16), ref_w.view(torch.int16))


def _two_gpu_stack_rank(rank, world, port, path):
    import datetime
    import os

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from qk_b200.decoder import StackConfig, SyntheticDecoder

        cfg = StackConfig(layers=2, experts=64, top_k=4, context=512)
        model = SyntheticDecoder(cfg, dev, seed=1, group=dist.group.WORLD)
        state = model.state(3, seed=2)
        state.step()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            state.step()
        x0 = state.x.clone()
        graph.replay()
        graph.replay()
        torch.cuda.synchronize(dev)
        state.ep.check_status()
        x = state.x.float()
        np.save(f"{path}.{rank}.npy", np.array([bool(torch.isfinite(x).all()), not torch.equal(x0, state.x)]))
        del graph
        dist.barrier()
        state.close()
    finally:
        dist.destroy_process_group()


def test_expert_parallel_stack_on_two_gpus(tmp_path):
    """The decoder stack with its routed experts split over two ranks (each rank decodes its
    own sequences, tokens cross through peer memory) steps in a CUDA graph and stays finite."""
    import socket

    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = tmp_path / "stack2"
    mp.start_processes(_two_gpu_stack_rank, args=(2, port, str(path)), nprocs=2, start_method="spawn")
    for rank in range(2):
        assert np.load(f"{path}.{rank}.npy").all(), rank
