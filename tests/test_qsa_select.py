"""Sparse token selection (QSA indexer, attention_cache.py:84-125) feeding the decode attention.

CPU: the oracle's selection keeps the properties the reference's own test checks
(test_qwen38_compute.py:120-190): the selected count, no duplicates, every tail token, only
top-scoring blocks, no future token. GPU: the block scores against the oracle, the selection
from the GPU's own scores bit-exact against the oracle's (ties included), the selected
tokens through the Q8 decode attention, and whole select_tokens decode steps (key update,
query, selection) against the oracle.
"""

import numpy as np
import pytest

from oracle import kv
from oracle.precision import bf16_round
from util import bf16_tensor, rel_err, to_f32


def _inputs(rng, batch, blocks, heads=4, dim=128):
    q = bf16_round(rng.normal(size=(batch, heads, dim)).astype(np.float32))
    k = bf16_round(rng.normal(size=(batch, blocks, dim)).astype(np.float32))
    return q, k


def _check_properties(indices, valid, scores, lengths, ratio, budget):
    K = min(budget // ratio, scores.shape[1])
    for b in range(indices.shape[0]):
        n = (lengths[b] + 1) // ratio
        sel = indices[b, valid[b]]
        assert len(sel) == min(n, K) * ratio + (lengths[b] + 1) % ratio
        assert len(np.unique(sel)) == len(sel)
        assert set(range(n * ratio, lengths[b] + 1)).issubset(set(sel))
        assert sel.max(initial=0) <= lengths[b]
        chosen = sel[sel < n * ratio] // ratio
        if n > K:
            assert np.min(scores[b, chosen]) >= np.partition(scores[b, :n], n - K)[n - K]


def test_oracle_selection_keeps_the_reference_properties():
    rng = np.random.default_rng(33)
    ratio, budget = 4, 32
    for batch, blocks in ((2, 16), (3, 40)):
        q, k = _inputs(rng, batch, blocks)
        for lengths in (np.array([0, 3, 66, 159][:batch]), rng.integers(0, blocks * ratio, batch)):
            scores = kv.qsa_scores(q, k, lengths, ratio)
            indices, valid = kv.qsa_select(scores, lengths, ratio, budget)
            assert indices.shape == (batch, min(budget // ratio, blocks) * ratio + ratio - 1)
            _check_properties(indices, valid, scores, lengths, ratio, budget)
            assert (indices[~valid] == 0).all()


@pytest.mark.gpu
@pytest.mark.parametrize("batch,blocks,heads,dim,ratio,budget", [
    (2, 67, 4, 128, 4, 32),       # the reference's test shapes (small budget)
    (3, 2048, 4, 128, 4, 2048),   # context 8192, default budget: K = 512
    (1, 8192, 4, 128, 4, 2048),   # context 32768
    (4, 300, 8, 64, 2, 100),      # ratio 2, dim 64, K = 50
    (2, 1000, 2, 256, 4, 4096),   # K = 1000 = every block, dim 256
])
def test_scores_and_selection_match_oracle(cuda_device, batch, blocks, heads, dim, ratio, budget):
    import torch

    from qk_b200 import _lib
    from qk_b200.attention_cache import select_tokens_from_keys

    rng = np.random.default_rng(blocks + batch)
    q, k = _inputs(rng, batch, blocks, heads, dim)
    lengths = rng.integers(0, blocks * ratio, batch).astype(np.int32)
    lengths[0] = min(blocks * ratio - 1, 4 * ratio + 1)  # few complete blocks: masked selections
    qd, kd, ld = bf16_tensor(q, cuda_device), bf16_tensor(k, cuda_device), torch.from_numpy(lengths).to(cuda_device)
    scores = torch.empty((batch, blocks), dtype=torch.float32, device=cuda_device)
    _lib.call("qk_qsa_block_scores", _lib.ptr(qd), _lib.ptr(kd), _lib.ptr(ld), batch, heads, dim, blocks, ratio,
              _lib.ptr(scores), _lib.stream_handle(cuda_device))
    got_scores = scores.cpu().numpy()
    expected = kv.qsa_scores(q, k, lengths, ratio)
    finite = np.isfinite(expected)
    np.testing.assert_array_equal(np.isfinite(got_scores), finite)
    assert rel_err(got_scores[finite], expected[finite])[0] < 1e-5
    indices, valid = select_tokens_from_keys(qd, kd, ld, ratio=ratio, budget=budget)
    ref_i, ref_v = kv.qsa_select(got_scores, lengths, ratio, budget)  # the oracle on the GPU's scores
    np.testing.assert_array_equal(indices.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(valid.cpu().numpy(), ref_v)
    _check_properties(ref_i, ref_v, got_scores, lengths, ratio, budget)


@pytest.mark.gpu
def test_selection_ties_go_to_the_lower_block(cuda_device):
    import torch

    from qk_b200 import _lib

    rng = np.random.default_rng(5)
    batch, blocks, ratio, budget = 3, 4000, 4, 2048
    scores = rng.integers(0, 7, (batch, blocks)).astype(np.float32)  # heavy ties
    scores[1] = 0.0                                                   # all tied (index_q = 0)
    lengths = np.array([blocks * ratio - 1, blocks * ratio - 3, 1000], np.int32)
    count = (lengths + 1) // ratio
    scores = np.where(np.arange(blocks)[None, :] < count[:, None], scores, -np.inf).astype(np.float32)
    sd, ld = torch.from_numpy(scores).to(cuda_device), torch.from_numpy(lengths).to(cuda_device)
    K = budget // ratio
    indices = torch.empty((batch, K * ratio + ratio - 1), dtype=torch.int32, device=cuda_device)
    valid = torch.empty(indices.shape, dtype=torch.uint8, device=cuda_device)
    _lib.call("qk_qsa_select", _lib.ptr(sd), _lib.ptr(ld), batch, blocks, ratio, budget, _lib.ptr(indices),
              _lib.ptr(valid), _lib.stream_handle(cuda_device))
    ref_i, ref_v = kv.qsa_select(scores, lengths, ratio, budget)
    np.testing.assert_array_equal(indices.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(valid.cpu().numpy().astype(bool), ref_v)
    assert (ref_i[1, :K * ratio:ratio] == np.arange(K) * ratio).all()  # all tied: the first K blocks


@pytest.mark.gpu
def test_selected_tokens_through_decode_attention(cuda_device):
    import torch

    from qk_b200.attention_cache import CacheConfig, decode_attention, select_tokens_from_keys

    rng = np.random.default_rng(8)
    batch, T, ratio, budget = 2, 8192, 4, 2048
    blocks = T // ratio
    q_idx, k_idx = _inputs(rng, batch, blocks)
    lengths = np.array([T - 1, 5000], np.int32)
    indices, valid = select_tokens_from_keys(bf16_tensor(q_idx, cuda_device), bf16_tensor(k_idx, cuda_device),
                                             torch.from_numpy(lengths).to(cuda_device), ratio=ratio, budget=budget)
    c = CacheConfig(max_context=T)
    codes = {n: rng.integers(-127, 128, (batch, T, 512)).astype(np.int8) for n in ("k", "v")}
    planes = {n: bf16_round(rng.uniform(0.001, 0.021, (batch * 16, T)).astype(np.float32)) for n in ("k", "v")}
    cache = {n: torch.from_numpy(codes[n]).to(cuda_device) for n in ("k", "v")}
    cache.update({n + "_scale": bf16_tensor(planes[n], cuda_device) for n in ("k", "v")})
    q = bf16_round(rng.normal(size=(batch, 16, 256)).astype(np.float32))
    got = to_f32(decode_attention(bf16_tensor(q, cuda_device), cache, indices, c, valid=valid))
    idx, val = indices.cpu().numpy(), valid.cpu().numpy()
    keys = kv.read_quantized(codes["k"], planes["k"], idx, 2, 256)
    values = kv.read_quantized(codes["v"], planes["v"], idx, 2, 256)
    expected = kv.attention(q, keys, values, val)
    mx, l2 = rel_err(got, expected)
    assert mx < 1e-2 and l2 < 5e-3, (mx, l2)


@pytest.mark.gpu
def test_select_tokens_step_by_step_matches_oracle(cuda_device):
    """Decode steps through the whole select_tokens (attention_cache.py:84-125), as the
    reference's own test drives it (test_qwen38_compute.py:120-190): two rows, 67 steps,
    positions (t, t // 2, t % 7). Each step the tail and block start match the oracle's update
    on the same raw keys bit for bit, the block keys within the BF16 tolerance, and the
    selection keeps the reference test's properties under the oracle's query scores."""
    import torch

    from qk_b200.attention_cache import IndexerConfig, empty_index_cache, select_tokens

    ic = IndexerConfig(qsa_budget=32, indexer_heads=4, indexer_dim=64, indexer_compress=4, rotary_dim=32)
    B, H, steps, T = 2, 256, 67, 68
    rng = np.random.default_rng(33)
    inputs = bf16_round(rng.normal(size=(B, steps, H)).astype(np.float32))
    w = {"index_k": bf16_tensor(rng.normal(0, 0.1, (64, H)).astype(np.float32), cuda_device),
         "index_q": bf16_tensor(rng.normal(0, 0.1, (4 * 64, H)).astype(np.float32), cuda_device),
         "index_k_norm": bf16_tensor(rng.uniform(0.5, 1.5, 64).astype(np.float32), cuda_device),
         "index_q_norm": bf16_tensor(rng.uniform(0.5, 1.5, 64).astype(np.float32), cuda_device)}
    cache = empty_index_cache(B, T, ic, cuda_device)
    state = {"index_keys": np.zeros((B, T // 4, 64), np.float32), "index_tail": np.zeros((B, 4, 64), np.float32),
             "index_start": np.zeros((B, 3), np.int32)}
    inv, axis = (t.cpu().numpy() for t in ic.rope_tables("cpu"))
    kn, qn = to_f32(w["index_k_norm"]), to_f32(w["index_q_norm"])
    active = np.ones(B, bool)
    for step in range(steps):
        x = bf16_tensor(inputs[:, step], cuda_device)
        pos = np.broadcast_to(np.array([step, step // 2, step % 7], np.int32), (B, 3)).copy()
        lengths = np.full(B, step, np.int32)
        indices, valid, _ = select_tokens(x, w, cache, torch.from_numpy(lengths), torch.from_numpy(pos),
                                          torch.ones(B, dtype=torch.bool), ic)
        raw_k = to_f32(torch.matmul(x, w["index_k"].t()))
        kv.qsa_update(state, raw_k, lengths, pos, active, kn, ic.eps, inv, axis, 32, 4)
        np.testing.assert_array_equal(to_f32(cache["index_tail"]), state["index_tail"])
        np.testing.assert_array_equal(cache["index_start"].cpu().numpy(), state["index_start"])
        got_keys = to_f32(cache["index_keys"])
        assert rel_err(got_keys, state["index_keys"])[0] < 1e-2 if state["index_keys"].any() else True
        state["index_keys"] = got_keys.copy()  # the selection below scores the kernel's keys
        raw_q = to_f32(torch.matmul(x, w["index_q"].t())).reshape(B, 4, 64)
        query = kv.qsa_query(raw_q, pos, qn, ic.eps, inv, axis, 32)
        scores = kv.qsa_scores(query, got_keys, lengths, 4)
        n = (step + 1) // 4
        idx, val = indices.cpu().numpy(), valid.cpu().numpy()
        for row in range(B):
            sel = idx[row, val[row]]
            assert len(sel) == min(n, 8) * 4 + (step + 1) % 4
            assert len(np.unique(sel)) == len(sel)
            assert set(range(n * 4, step + 1)).issubset(set(sel))
            assert sel.max(initial=0) <= step
            chosen = sel[sel < n * 4] // 4
            if n > 8:
                assert np.min(scores[row, chosen]) >= np.partition(scores[row, :n], n - 8)[n - 8] - 1e-2
