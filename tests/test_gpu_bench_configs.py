"""Parity at the exact configurations bench.py times.

* Config 2 (expert GEMM microbenchmark) at full shape: 128 experts, H 2048, I 512, the
  bench's own weights (N(0, 0.02), seed 1, this build's encoder) and its uniform top-1
  assignment of 128 * M rows, for M in {1, 16, 64, 256} (M = 256 takes the wide form) and
  Q6_K / Q4_K. A seeded sample of 64 output rows is compared with the oracle's routed FFN
  (experts.py:61-131 restated), which needs only the sampled rows' experts decoded.
* Config 3 (Q8 KV decode attention): the bench's six B x ctx inputs (16 q / 2 kv heads,
  head dim 256, a random permutation page table of 256-slot pages, every slot attended).
  Every row is compared with the oracle (attention_cache.py:152-170 restated) up to
  B = 32 x 4096 and B = 8 x 32768; at B = 32 x 32768 a seeded sample of 6 rows.
"""

import numpy as np
import pytest

from oracle import kv, moe
from oracle.precision import bf16_round
from util import bf16_tensor, rel_err, to_f32

pytestmark = pytest.mark.gpu

LAYER_TOL = 1e-2  # north-star layer tolerance: max relative error (BF16, FP32 accumulation)
SAMPLE_ROWS = 64


@pytest.fixture(scope="module")
def bench_module():
    import bench

    return bench


@pytest.fixture(scope="module", params=["Q6_K", "Q4_K"])
def config2_experts(request, bench_module, cuda_device):
    from qk_b200.parallel import put_expert_bytes

    qtype = request.param
    b = bench_module
    raw = b.synth_experts(qtype, b.EXPERTS)
    dev = {k: put_expert_bytes(v, k, qtype, b.HIDDEN, b.INTER, device=cuda_device) for k, v in raw.items()}
    return qtype, raw, dev


@pytest.mark.parametrize("m", [1, 16, 64, 256])
def test_config2_expert_gemm_full_shape_sampled_rows(cuda_device, bench_module, config2_experts, m):
    import torch

    from qk_b200.experts import expert_parallel

    b = bench_module
    qtype, raw, dev = config2_experts
    x, ids, weights = b.workload(m)
    fn = expert_parallel(gate_type=qtype, up_type=qtype, down_type=qtype, hidden=b.HIDDEN,
                         intermediate=b.INTER)
    out = fn(dev["gate"], dev["up"], dev["down"], bf16_tensor(x, cuda_device),
             torch.from_numpy(ids).to(cuda_device), bf16_tensor(weights, cuda_device))
    fn.check_status()
    got = to_f32(out)
    assert np.all(np.isfinite(got))
    rows = np.sort(np.random.default_rng(1000 + m).choice(x.shape[0], SAMPLE_ROWS, replace=False))
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x[rows], ids[rows], weights[rows],
                              gate_type=qtype, up_type=qtype, down_type=qtype, hidden=b.HIDDEN,
                              intermediate=b.INTER)
    mx, l2 = rel_err(got[rows], expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (qtype, m, mx, l2)


def _check_attention_rows(bench_module, device, batch, ctx, rows):
    b = bench_module
    inp = b.attention_inputs(device, batch, ctx)
    out = b.attention_call(inp)
    got = to_f32(out)
    assert np.all(np.isfinite(got))
    idx = inp["idx"].cpu().numpy()
    lengths = inp["lengths"].cpu().numpy()
    q = to_f32(inp["q"])
    worst = (0.0, 0.0)
    for r in rows:
        codes = {n: inp[n][r : r + 1].cpu().numpy() for n in ("k", "v")}
        planes = {n: to_f32(inp[n + "s"][r * 16 : (r + 1) * 16]) for n in ("k", "v")}
        sel = idx[r : r + 1]
        keys = kv.read_quantized(codes["k"], planes["k"], sel, 2, 256)
        values = kv.read_quantized(codes["v"], planes["v"], sel, 2, 256)
        mask = np.arange(ctx)[None, :] <= lengths[r]
        expected = kv.attention(q[r : r + 1], keys, values, mask)
        mx, l2 = rel_err(got[r : r + 1], expected)
        worst = (max(worst[0], mx), max(worst[1], l2))
    return worst


@pytest.mark.parametrize("batch,ctx", [(1, 4096), (8, 4096), (32, 4096), (1, 32768), (8, 32768), (32, 32768)])
def test_config3_decode_attention_bench_inputs(cuda_device, bench_module, batch, ctx):
    if batch * ctx > 8 * 32768:
        rows = np.sort(np.random.default_rng(batch + ctx).choice(batch, 6, replace=False))
    else:
        rows = np.arange(batch)
    mx, l2 = _check_attention_rows(bench_module, cuda_device, batch, ctx, rows)
    assert mx < 1e-2 and l2 < 5e-3, (batch, ctx, mx, l2)
