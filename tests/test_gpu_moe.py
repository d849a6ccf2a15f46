"""Routed expert FFN on the GPU against the pinned oracle and the reference's own golden."""

import numpy as np
import pytest

from oracle import gguf, moe
from oracle.precision import bf16_round
from util import bf16_tensor, random_blocks, rel_err, to_f32

pytestmark = pytest.mark.gpu

# North-star layer tolerance: max relative error 1e-2 (BF16 with FP32 accumulation).
LAYER_TOL = 1e-2


def make_experts(rng, count, hidden, intermediate, qtype, down_type=None):
    """Expert bytes: N(0, 0.02) weights encoded to Q6_K / Q4_K / Q8_0, or random blocks with
    finite scales for Q5_K / Q5_1 (no encoder of those types is needed)."""
    raw = {}
    for kind, (rows, width) in (("gate", (intermediate, hidden)), ("up", (intermediate, hidden)),
                                ("down", (hidden, intermediate))):
        t = (down_type or qtype) if kind == "down" else qtype
        if t in ("Q5_K", "Q5_1"):
            raw[kind] = random_blocks(rng, count * rows, width, t).reshape(count, -1)
            continue
        w = rng.normal(0, 0.02, (count, rows, width)).astype(np.float32)
        raw[kind] = gguf.encode(w, t).reshape(count, -1)
    return raw


def run_layer(device, raw, qtype, hidden, intermediate, x, ids, weights, down_type=None):
    import torch

    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes

    down_type = down_type or qtype
    dev = {k: put_expert_bytes(v, k, down_type if k == "down" else qtype, hidden, intermediate, device=device)
           for k, v in raw.items()}
    fn = expert_parallel(gate_type=qtype, up_type=qtype, down_type=down_type, hidden=hidden,
                         intermediate=intermediate)
    out = fn(dev["gate"], dev["up"], dev["down"], bf16_tensor(x, device),
             torch.from_numpy(np.asarray(ids, np.int32)).to(device), bf16_tensor(weights, device))
    fn.check_status()
    return to_f32(out), fn, dev


@pytest.mark.parametrize("label", ["mixed", "q6"])
def test_routed_ffn_matches_reference_numpy_oracle_golden(golden, cuda_device, label):
    """The reference's own routed-FFN case ("mixed": Q6_K gate/up, Q8_0 down, I = 32,
    routing_validation.py:193-243) and its Q6_K-down twin, against the reference oracle's
    BF16 outputs."""
    from make_golden import ROUTING_BATCHES, routing_inputs

    data = golden("routing_ffn.npz")
    packed, batches, down_type, hidden, intermediate, count = routing_inputs(label, gguf.encode_q8_0)
    flat = {k: v.reshape(count, -1) for k, v in packed.items()}
    for batch in ROUTING_BATCHES:
        ids, weights, source = batches[batch]
        got, _, _ = run_layer(cuda_device, flat, "Q6_K", hidden, intermediate, source, ids, weights,
                              down_type=down_type)
        expected = (data[f"{label}_b{batch}_bf16_bits"].astype(np.uint32) << 16).view(np.float32)
        # routing_validation.py:262 BF16 tolerance
        np.testing.assert_allclose(got, expected, atol=3e-3, rtol=3e-3)
        np.testing.assert_array_equal(got[np.all(weights == 0, axis=-1)], 0)


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K"])
def test_config1_layer_t8_top4_of_64(cuda_device, qtype):
    """T=8, H=2048, I=512, 64 experts, router top-4 (smaller E keeps the oracle fast)."""
    import torch

    from qk_b200.routing import routes

    hidden, intermediate, count, k = 2048, 512, 64, 4
    raw = make_experts(np.random.default_rng(1), count, hidden, intermediate, qtype)
    x = np.random.default_rng(0).normal(size=(8, hidden)).astype(np.float32)
    router = np.random.default_rng(2).normal(0, 0.02, (count, hidden)).astype(np.float32)
    ids, weights = routes(bf16_tensor(x, cuda_device), torch.from_numpy(router).to(cuda_device), k)
    ids, weights = ids.cpu().numpy(), to_f32(weights)
    got, _, _ = run_layer(cuda_device, raw, qtype, hidden, intermediate, x, ids, weights)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type=qtype,
                              up_type=qtype, down_type=qtype, hidden=hidden, intermediate=intermediate)
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)


@pytest.mark.parametrize("tokens_per_expert", [1, 9, 33, 70])
def test_many_tokens_per_expert_duplicates_and_finished_rows(cuda_device, tokens_per_expert):
    hidden, intermediate, count, k = 512, 256, 6, 2
    rng = np.random.default_rng(tokens_per_expert)
    raw = make_experts(rng, count, hidden, intermediate, "Q6_K")
    batch = tokens_per_expert * count // k + 1
    ids = rng.integers(0, count, (batch, k)).astype(np.int32)
    ids[:3, 1] = ids[:3, 0]  # duplicate routes of one token merge into one entry
    weights = bf16_round(rng.uniform(0.05, 1.0, (batch, k)).astype(np.float32))
    weights[::7] = 0  # finished rows contribute exactly zero
    x = rng.normal(size=(batch, hidden)).astype(np.float32)
    got, _, _ = run_layer(cuda_device, raw, "Q6_K", hidden, intermediate, x, ids, weights)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type="Q6_K",
                              up_type="Q6_K", down_type="Q6_K", hidden=hidden,
                              intermediate=intermediate)
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)
    np.testing.assert_array_equal(got[::7], 0)


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K"])
def test_wide_form_chunks_of_128_tokens(cuda_device, qtype):
    """Routes averaging 64 to 191 tokens per expert take the wide form (128-token chunks, one
    MMA issuer, N up to 128): 150 tokens per expert give chunks of 128 and a ragged last one;
    an expert with a single token shares the call."""
    hidden, intermediate, count, k = 512, 512, 5, 2
    rng = np.random.default_rng(300)
    raw = make_experts(rng, count, hidden, intermediate, qtype)
    batch = 150 * (count - 1) // k + 1
    ids = rng.integers(0, count - 1, (batch, k)).astype(np.int32)
    ids[0, 1] = count - 1            # the last expert: one token
    ids[1:4, 1] = ids[1:4, 0]        # duplicate routes merge
    weights = bf16_round(rng.uniform(0.05, 1.0, (batch, k)).astype(np.float32))
    weights[5::11] = 0
    x = rng.normal(size=(batch, hidden)).astype(np.float32)
    assert 64 * count <= batch * k < 192 * count   # the wide form
    got, _, _ = run_layer(cuda_device, raw, qtype, hidden, intermediate, x, ids, weights)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type=qtype,
                              up_type=qtype, down_type=qtype, hidden=hidden, intermediate=intermediate)
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)
    np.testing.assert_array_equal(got[5::11], 0)


@pytest.mark.parametrize("qtype,down_type,hidden,intermediate", [
    ("Q6_K", "Q6_K", 512, 512), ("Q4_K", "Q4_K", 768, 256), ("Q6_K", "Q8_0", 512, 640),
    ("Q4_K", "Q8_0", 256, 96)])
def test_prefill_form_chunks_of_256_tokens(cuda_device, qtype, down_type, hidden, intermediate):
    """Routes averaging >= 192 tokens per expert take the prefill form (256-token chunks,
    weights decoded into shared memory, both MMA operands in shared memory, 512 TMEM
    accumulator columns): 600 tokens per expert give chunks of 256, 256 and a ragged 88 (not a
    multiple of 16); an expert with one token, merged duplicate routes and finished rows share
    the call; I = 640 and 96 leave tile pairs and K blocks partly empty."""
    count, k = 5, 2
    rng = np.random.default_rng(600 + intermediate)
    raw = make_experts(rng, count, hidden, intermediate, qtype, down_type)
    batch = 600 * (count - 1) // k + 1
    ids = np.stack([rng.choice(count - 1, k, replace=False) for _ in range(batch)]).astype(np.int32)
    ids[0, 1] = count - 1            # the last expert: one token
    ids[1:4, 1] = ids[1:4, 0]        # duplicate routes merge
    weights = bf16_round(rng.uniform(0.05, 1.0, (batch, k)).astype(np.float32))
    weights[5::11] = 0
    x = rng.normal(size=(batch, hidden)).astype(np.float32)
    assert batch * k >= 192 * count  # the prefill form
    got, _, _ = run_layer(cuda_device, raw, qtype, hidden, intermediate, x, ids, weights, down_type=down_type)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type=qtype,
                              up_type=qtype, down_type=down_type, hidden=hidden, intermediate=intermediate)
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)
    np.testing.assert_array_equal(got[5::11], 0)


@pytest.mark.parametrize("batch", [300, 1200])
def test_top1_routes_zero_rows_and_fp32_output(cuda_device, batch):
    """Top-1 routes (config 2's routing): rows of tokens with a zero weight or an expert of
    another rank are zero; 300 tokens on 8 experts take the narrow form, 1200 the wide one.
    The FP32 output (the expert-parallel partial) rounds to the BF16 one bit for bit."""
    import torch

    hidden, intermediate, count = 512, 256, 8
    rng = np.random.default_rng(batch)
    raw = make_experts(rng, count, hidden, intermediate, "Q6_K")
    ids = rng.integers(0, count, (batch, 1)).astype(np.int32)
    ids[7::17, 0] = count + 2        # another rank's expert
    weights = bf16_round(rng.uniform(0.05, 1.0, (batch, 1)).astype(np.float32))
    weights[3::19] = 0
    x = rng.normal(size=(batch, hidden)).astype(np.float32)
    got, fn, dev = run_layer(cuda_device, raw, "Q6_K", hidden, intermediate, x, ids, weights)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type="Q6_K",
                              up_type="Q6_K", down_type="Q6_K", hidden=hidden, intermediate=intermediate)
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)
    np.testing.assert_array_equal(got[7::17], 0)
    np.testing.assert_array_equal(got[3::19], 0)
    ids_t = torch.from_numpy(ids).to(cuda_device)
    f32 = fn._run(dev["gate"], dev["up"], dev["down"], bf16_tensor(x, cuda_device), ids_t,
                  bf16_tensor(weights, cuda_device), 0, torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bf16_round(f32.cpu().numpy()), got)


@pytest.mark.parametrize("count,k,batch", [(6, 3, 6000), (512, 8, 2100)])
def test_many_routes_metadata_over_many_ctas(cuda_device, count, k, batch):
    """More than 16384 routes: the routing metadata comes from the count, tables and place
    kernels over many CTAs instead of one CTA. 6 experts x 3000 routes take the prefill form,
    512 experts x about 33 routes the narrow one; merged duplicate routes, zero weights and ids
    outside the rank's experts are in the same call."""
    hidden, intermediate = 256, 256
    rng = np.random.default_rng(count + batch)
    raw = make_experts(rng, count, hidden, intermediate, "Q6_K")
    ids = np.argsort(rng.random((batch, count)), axis=1)[:, :k].astype(np.int32)
    ids[1:40, 1] = ids[1:40, 0]      # duplicate routes merge
    ids[50:60, 2] = count + 3        # not an expert of this rank
    weights = bf16_round(rng.uniform(0.05, 1.0, (batch, k)).astype(np.float32))
    weights[5::13] = 0
    x = rng.normal(size=(batch, hidden)).astype(np.float32)
    assert batch * k > 16384
    got, _, _ = run_layer(cuda_device, raw, "Q6_K", hidden, intermediate, x, ids, weights)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type="Q6_K",
                              up_type="Q6_K", down_type="Q6_K", hidden=hidden, intermediate=intermediate)
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)
    np.testing.assert_array_equal(got[5::13], 0)


@pytest.mark.parametrize("qtype,intermediate,batch", [
    ("Q6_K", 512, 8), ("Q6_K", 640, 8), ("Q4_K", 96, 5), ("Q6_K", 640, 700)])
def test_q8_0_down_projection(cuda_device, qtype, intermediate, batch):
    """Q6_K/Q4_K gate and up with a Q8_0 down (the type mix of the reference's checkpoints):
    I a multiple of 256, ragged against the 256-value K blocks (640: two and a half, 96: a
    padded gate/up tile), and 700 tokens on 8 experts (the wide form)."""
    hidden, count, k = 512, 8, 2
    rng = np.random.default_rng(intermediate + batch)
    raw = make_experts(rng, count, hidden, intermediate, qtype, "Q8_0")
    ids = rng.integers(0, count, (batch, k)).astype(np.int32)
    weights = bf16_round(rng.uniform(0.05, 1.0, (batch, k)).astype(np.float32))
    x = rng.normal(size=(batch, hidden)).astype(np.float32)
    got, _, _ = run_layer(cuda_device, raw, qtype, hidden, intermediate, x, ids, weights, down_type="Q8_0")
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type=qtype,
                              up_type=qtype, down_type="Q8_0", hidden=hidden, intermediate=intermediate)
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)


@pytest.mark.parametrize("qtype,down_type,hidden,intermediate,batch", [
    ("Q4_K", "Q5_1", 512, 640, 8), ("Q5_K", "Q5_1", 512, 640, 8), ("Q5_K", "Q6_K", 512, 512, 300),
    ("Q4_K", "Q5_1", 256, 96, 700), ("Q5_K", "Q5_1", 512, 640, 1600)])
def test_q5_expert_types(cuda_device, qtype, down_type, hidden, intermediate, batch):
    """The reference Q4 checkpoint's expert types (checkpoints/q4.json: gate/up Q4_K or Q5_K,
    down Q5_1, intermediate 640): 8 tokens (narrow form), 300 and 700 (wide), 1600 on 8 experts
    top-2 (prefill form); I = 96 pads the gate/up tile and the down's K block."""
    count, k = 8, 2
    rng = np.random.default_rng(intermediate + batch)
    raw = make_experts(rng, count, hidden, intermediate, qtype, down_type)
    ids = np.argsort(rng.random((batch, count)), axis=1)[:, :k].astype(np.int32)
    weights = bf16_round(rng.uniform(0.05, 1.0, (batch, k)).astype(np.float32))
    x = rng.normal(size=(batch, hidden)).astype(np.float32)
    got, _, _ = run_layer(cuda_device, raw, qtype, hidden, intermediate, x, ids, weights, down_type=down_type)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type=qtype,
                              up_type=qtype, down_type=down_type, hidden=hidden, intermediate=intermediate)
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)


@pytest.mark.parametrize("qtype,hidden,intermediate,batch,k", [
    ("Q6_K", 512, 512, 8, 2), ("Q4_K", 512, 640, 40, 2), ("Q6_K", 256, 96, 300, 4), ("Q4_K", 2048, 512, 64, 4)])
def test_int8_q8_policy_w8a8_down(cuda_device, qtype, hidden, intermediate, batch, k):
    """compute="int8_q8" with a Q8_0 down (experts.py:85-107): the down projection is the W8A8
    integer dot (compute.py:20-34; tcgen05 kind::i8), checked against the oracle's restatement
    of the reference's numpy_q8_matmul inside the routed FFN. I = 640 and 96 leave a partial
    last K block (its padded groups are skipped); 300 tokens take several 32-token chunks per
    expert. The BF16 policy on the same experts differs from it by the activation rounding."""
    rng = np.random.default_rng(intermediate + batch + k)
    count = 8
    raw = make_experts(rng, count, hidden, intermediate, qtype, "Q8_0")
    ids = np.argsort(rng.random((batch, count)), axis=1)[:, :k].astype(np.int32)
    weights = bf16_round(rng.uniform(0.05, 1.0, (batch, k)).astype(np.float32))
    weights[3::7] = 0
    x = rng.normal(size=(batch, hidden)).astype(np.float32)
    import torch

    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes

    dev = {n: put_expert_bytes(v, n, "Q8_0" if n == "down" else qtype, hidden, intermediate, device=cuda_device)
           for n, v in raw.items()}
    args = (dev["gate"], dev["up"], dev["down"], bf16_tensor(x, cuda_device),
            torch.from_numpy(ids).to(cuda_device), bf16_tensor(weights, cuda_device))
    fn = expert_parallel(gate_type=qtype, up_type=qtype, down_type="Q8_0", hidden=hidden,
                         intermediate=intermediate, compute="int8_q8")
    got = to_f32(fn(*args))
    fn.check_status()
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type=qtype,
                              up_type=qtype, down_type="Q8_0", hidden=hidden, intermediate=intermediate,
                              compute="int8_q8")
    mx, l2 = rel_err(got, expected)
    assert mx < LAYER_TOL and l2 < 2e-3, (mx, l2)
    np.testing.assert_array_equal(got[3::7], 0)
    bf16 = expert_parallel(gate_type=qtype, up_type=qtype, down_type="Q8_0", hidden=hidden,
                           intermediate=intermediate)
    other = to_f32(bf16(*args))
    assert not np.array_equal(other, got)  # a different arithmetic ran
    assert rel_err(other, got)[1] < 0.05


def test_int8_q8_w8a8_dot_matches_reference_golden(golden, cuda_device):
    """The W8A8 projection (compute.py:20-34, q8_matmul) on the reference's integer-dot test
    (tests/test_qwen38_compute.py:81-100: a zero row, x20 outliers, a row of 127s) and a
    down-projection shape (K = 640, 20 groups), against the reference's own numpy_q8_matmul on
    its pack_q8 weights: FP32 within the reference's FP32 tolerance (atol 5e-4, rtol 2e-6), BF16
    within its BF16 tolerance (atol 0.5, rtol 0.004); the zero row stays zero."""
    import torch

    from qk_b200.packed import pack_rows, q8_matmul

    data = golden("w8a8.npz")
    for rows, width, outputs, _ in data["cases"]:
        key = f"{rows}_{width}_{outputs}"
        x, raw, expected = data[f"x_{key}"], data[f"raw_{key}"], data[f"expected_{key}"]
        packed = pack_rows(raw, int(width), "Q8_0", cuda_device)
        xd = bf16_tensor(x, cuda_device)
        got = q8_matmul(xd, packed, output_dtype=torch.float32).cpu().numpy()
        np.testing.assert_allclose(got, expected, atol=5e-4, rtol=2e-6)
        np.testing.assert_array_equal(got[0], 0)
        got16 = to_f32(q8_matmul(xd, packed))
        np.testing.assert_allclose(got16, bf16_round(expected), atol=0.5, rtol=0.004)
        np.testing.assert_array_equal(got16, bf16_round(got))


def test_zero_weights_give_zero_and_ids_outside_rank_are_ignored(cuda_device):
    hidden, intermediate, count = 256, 256, 4
    rng = np.random.default_rng(3)
    raw = make_experts(rng, count, hidden, intermediate, "Q6_K")
    x = rng.normal(size=(5, hidden)).astype(np.float32)
    ids = np.array([[0, 1]] * 5, np.int32)
    got, _, _ = run_layer(cuda_device, raw, "Q6_K", hidden, intermediate, x, ids,
                          np.zeros((5, 2), np.float32))
    np.testing.assert_array_equal(got, 0)
    ids = np.array([[7, 9]] * 5, np.int32)  # experts another rank would own
    got, _, _ = run_layer(cuda_device, raw, "Q6_K", hidden, intermediate, x, ids,
                          np.full((5, 2), 0.5, np.float32))
    np.testing.assert_array_equal(got, 0)


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K"])
def test_garbage_experts_do_not_leak_nan(cuda_device, qtype):
    """The NaN-isolation contract of test_qwen38_small_groups.py:227-264: an expert whose
    bytes decode to NaN (every byte 0xFF, so its FP16 block scales are NaN) must not reach
    the output when it is routed with weight 0 (a finished row) or not routed at all."""
    import torch

    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes

    hidden, intermediate, count = 256, 256, 4
    rng = np.random.default_rng(31)
    raw = make_experts(rng, count, hidden, intermediate, qtype)
    x = rng.normal(size=(6, hidden)).astype(np.float32)
    ids = np.array([[0, 3], [1, 3], [2, 3], [0, 1], [1, 2], [3, 0]], np.int32)
    w = bf16_round(rng.uniform(0.1, 1.0, (6, 2)).astype(np.float32))
    w[:3, 1] = 0.0   # rows 0-2 route to the garbage expert 3 with weight 0
    w[5, 0] = 0.0    # row 5 too
    clean, _, dev = run_layer(cuda_device, raw, qtype, hidden, intermediate, x, ids, w)
    for name in ("gate", "up", "down"):  # expert 3's tiles become 0xFF bytes on the device
        dev[name][3].fill_(0xFF)
    fn = expert_parallel(gate_type=qtype, up_type=qtype, down_type=qtype, hidden=hidden,
                         intermediate=intermediate)
    got = to_f32(fn(dev["gate"], dev["up"], dev["down"], bf16_tensor(x, cuda_device),
                    torch.from_numpy(ids).to(cuda_device), bf16_tensor(w, cuda_device)))
    fn.check_status()
    assert np.isfinite(got).all()
    np.testing.assert_array_equal(got, clean)
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, w, gate_type=qtype, up_type=qtype,
                              down_type=qtype, hidden=hidden, intermediate=intermediate)
    assert rel_err(got, expected)[0] < LAYER_TOL


def test_partial_sums_over_two_expert_ranges_add_up_to_the_layer(cuda_device):
    """The expert-parallel decomposition (per-rank FP32 partial + all-reduce) on one GPU."""
    import torch

    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes

    hidden, intermediate, count, k = 512, 256, 8, 3
    rng = np.random.default_rng(9)
    raw = make_experts(rng, count, hidden, intermediate, "Q6_K")
    x = rng.normal(size=(11, hidden)).astype(np.float32)
    ids = np.stack([rng.permutation(count)[:k] for _ in range(11)]).astype(np.int32)
    weights = bf16_round(rng.uniform(0.1, 1, (11, k)).astype(np.float32))
    fn = expert_parallel(gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=hidden,
                         intermediate=intermediate)
    xs, ids_t, w_t = bf16_tensor(x, cuda_device), torch.from_numpy(ids).to(cuda_device), bf16_tensor(weights, cuda_device)
    total = None
    for rank in range(2):
        dev = {kd: put_expert_bytes(v, kd, "Q6_K", hidden, intermediate, rank=rank, world=2,
                                    device=cuda_device) for kd, v in raw.items()}
        part = fn.partial(dev["gate"], dev["up"], dev["down"], xs, ids_t, w_t, first_expert=rank * 4)
        expected = moe.expert_ffn(raw["gate"][rank * 4:(rank + 1) * 4], raw["up"][rank * 4:(rank + 1) * 4],
                                  raw["down"][rank * 4:(rank + 1) * 4], x, ids, weights,
                                  gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=hidden,
                                  intermediate=intermediate, first_expert=rank * 4, partial=True)
        mx, _ = rel_err(part.cpu().numpy(), expected)
        assert mx < LAYER_TOL
        total = part if total is None else total + part
    full = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x, ids, weights, gate_type="Q6_K",
                          up_type="Q6_K", down_type="Q6_K", hidden=hidden, intermediate=intermediate)
    mx, _ = rel_err(bf16_round(total.cpu().numpy()), full)
    assert mx < LAYER_TOL


def test_contract_errors(cuda_device):
    from qk_b200.experts import expert_parallel

    with pytest.raises(ValueError, match="compute policy"):
        expert_parallel(gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=256,
                        intermediate=256, compute="fp8")
    with pytest.raises(ValueError, match="row tile"):
        expert_parallel(gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=256,
                        intermediate=256, row_tile=0)
    with pytest.raises(ValueError, match="gate and up"):
        expert_parallel(gate_type="Q6_K", up_type="Q4_K", down_type="Q6_K", hidden=256,
                        intermediate=256)
    with pytest.raises(ValueError, match="multiple of 256"):
        expert_parallel(gate_type="Q6_K", up_type="Q6_K", down_type="Q6_K", hidden=256,
                        intermediate=96)
