"""Pin the CPU oracle to the reference's own outputs (golden fixtures) - no GPU needed."""

import hashlib

import numpy as np
import pytest

from oracle import gguf, kv, layout, moe
from oracle.precision import bf16_round


@pytest.mark.parametrize(
    "qtype",
    ["Q4_K", "Q5_K", "Q6_K", "Q8_0", "F16", "BF16", "F32", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "IQ4_NL"],
)
def test_decoders_match_reference_and_gguf_py_bit_for_bit(golden, qtype):
    data = golden("gguf_decode.npz")
    raw, width = data[f"{qtype}_raw"], int(data[f"{qtype}_width"])
    actual = gguf.dequantize_rows(raw, qtype, width)
    np.testing.assert_array_equal(actual.view(np.uint32), data[f"{qtype}_expected"].view(np.uint32))


def test_q6_k_extreme_scales_and_every_sub_scale_byte(golden):
    data = golden("q6_projection.npz")
    actual = bf16_round(gguf.dequantize_rows(data["extremes_raw"], "Q6_K", 256))
    np.testing.assert_array_equal(actual.view(np.uint32), data["extremes_bf16"].view(np.uint32))


def test_every_finite_fp16_scale_expands_exactly():
    bits = np.arange(65536, dtype=np.uint16)
    bits = bits[(bits & 0x7C00) != 0x7C00]
    raw = np.zeros((bits.size, 1, 34), np.uint8)
    raw[:, 0, 0:2] = bits.view(np.uint8).reshape(-1, 2)
    raw[:, 0, 2] = 1  # first code = 1 -> value = d
    decoded = gguf.dequantize_rows(raw, "Q8_0", 32)[:, 0]
    expected = bits.view(np.float16).astype(np.float32)
    np.testing.assert_array_equal(decoded.view(np.uint32), expected.view(np.uint32))


def test_packed_q6_projection_matches_reference_projection(golden):
    data = golden("q6_projection.npz")
    for batch, outputs, inputs in data["cases"]:
        key = f"{batch}_{outputs}_{inputs}"
        raw = gguf.legal_q6_k_fixture(int(outputs), int(inputs))
        digest = np.frombuffer(hashlib.sha256(raw.tobytes()).digest(), np.uint8)
        np.testing.assert_array_equal(digest, data[f"raw_sha256_{key}"])
        actual = moe.projection(data[f"x_{key}"], raw, int(inputs))
        np.testing.assert_array_equal(actual, data[f"expected_{key}"])


def test_bf16_rounding_ties_and_specials(golden):
    data = golden("q8_kv.npz")
    src, expected = data["bf16_source"], data["bf16_expected"]
    actual = bf16_round(src)
    finite = ~np.isnan(src)
    np.testing.assert_array_equal(actual[finite].view(np.uint32), expected[finite].view(np.uint32))
    assert np.isnan(actual[~finite]).all()


@pytest.mark.parametrize("width", [8, 256])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_q8_codec_matches_reference_oracle_and_rejects_unrounded_divisor(golden, width, dtype):
    data = golden("q8_kv.npz")
    tag = f"w{width}_{dtype}"
    codes, scale = kv.quantize(data[f"{tag}_x"], min(32, width))
    np.testing.assert_array_equal(codes, data[f"{tag}_codes"])
    np.testing.assert_array_equal(scale, data[f"{tag}_scale"])
    assert np.count_nonzero(data[f"{tag}_unrounded_codes"] != codes) > 0


def test_q8_cache_write_then_read_matches_reference_reconstruction(golden):
    data = golden("q8_kv.npz")
    source = data["read_source"]
    cache = {n: np.zeros((2, 32, 512), np.int8) for n in ("k", "v")}
    cache.update({n: np.zeros((32, 32), np.float32) for n in ("k_scale", "v_scale")})
    kv.write_quantized(cache, source, source, np.array([31, 8]), np.array([True, False]), 2, 256)
    indices = np.array([[31, 0, 31, 1], [8, 0, 8, 31]])
    actual = kv.read_quantized(cache["k"], cache["k_scale"], indices, 2, 256, dtype="f32")
    expected = np.zeros((2, 4, 2, 256), np.float32)
    expected[0, [0, 2]] = data["read_reconstructed"]
    np.testing.assert_array_equal(actual, expected)
    for name in ("k", "v", "k_scale", "v_scale"):
        np.testing.assert_array_equal(cache[name].reshape(2, -1)[1], 0)


@pytest.mark.parametrize("case", ["1_16_8", "2_4_32", "8_16_64"])
def test_scale_gather_wraps_negative_then_clamps(golden, case):
    data = golden("q8_kv.npz")
    batch, groups, time = map(int, case.split("_"))
    tag = f"gather_{case}"
    plane = data[f"{tag}_plane"]
    actual = kv.gather_scale_plane(plane, data[f"{tag}_indices"], groups)
    np.testing.assert_array_equal(actual, data[f"{tag}_expected"])


@pytest.mark.parametrize("label", ["mixed", "q6"])
def test_routed_ffn_oracle_matches_reference_numpy_oracle(golden, label):
    from make_golden import ROUTING_BATCHES, routing_inputs

    data = golden("routing_ffn.npz")
    packed, batches, down_type, hidden, intermediate, count = routing_inputs(
        label, gguf.encode_q8_0
    )
    for name, raw in packed.items():
        digest = np.frombuffer(hashlib.sha256(raw.tobytes()).digest(), np.uint8)
        np.testing.assert_array_equal(digest, data[f"{label}_{name}_sha256"])
    flat = {n: r.reshape(count, -1) for n, r in packed.items()}
    for batch in ROUTING_BATCHES:
        ids, weights, source = batches[batch]
        actual = moe.expert_ffn(
            flat["gate"], flat["up"], flat["down"], bf16_round(source), ids, bf16_round(weights),
            gate_type="Q6_K", up_type="Q6_K", down_type=down_type, hidden=hidden,
            intermediate=intermediate,
        )
        bits = data[f"{label}_b{batch}_bf16_bits"].astype(np.uint32) << 16
        expected = bits.view(np.float32)
        # routing_validation.py:262 tolerance for BF16 (the reference oracle's sigmoid
        # formula differs from numerics.sigmoid by FP32 ulps).
        np.testing.assert_allclose(actual, expected, atol=3e-3, rtol=3e-3)
        finished = np.all(weights == 0, axis=-1)
        np.testing.assert_array_equal(actual[finished], 0)


def test_router_top_k_ties_go_to_lower_index_and_weights_renormalise():
    logits = np.array([[1.0, 3.0, 3.0, 2.0, -1.0], [0.0, 0.0, 0.0, 0.0, 0.0]], np.float32)
    ids, weights, probs = moe.routes(None, None, 3, logits=logits)
    np.testing.assert_array_equal(ids, [[1, 2, 3], [0, 1, 2]])
    np.testing.assert_allclose(weights.sum(-1), 1, atol=1e-2)
    # independent fp64 formulation
    p = np.exp(logits.astype(np.float64) - logits.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    np.testing.assert_allclose(probs, p, rtol=1e-6)


def test_router_inactive_rows_get_zero_weight():
    rng = np.random.default_rng(5)
    x = rng.normal(size=(4, 64)).astype(np.float32)
    w = rng.normal(0, 0.02, (16, 64)).astype(np.float32)
    ids, weights, _ = moe.routes(x, w, 4, active=np.array([1, 0, 1, 0], bool))
    assert (weights[[1, 3]] == 0).all() and (weights[[0, 2]] > 0).all()


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K"])
def test_encoders_round_trip_through_reference_decoder_layout(qtype):
    rng = np.random.default_rng(1)
    w = rng.normal(0, 0.02, (48, 512)).astype(np.float32)
    raw = gguf.encode(w, qtype)
    decoded = gguf.dequantize_rows(raw, qtype, 512)
    rel = np.linalg.norm(decoded - w) / np.linalg.norm(w)
    assert rel < (0.02 if qtype == "Q6_K" else 0.08)
    tiled = layout.tile(raw, qtype)
    np.testing.assert_array_equal(layout.untile(tiled, qtype, 48, 512), raw)


@pytest.mark.parametrize("rows,width", [(1, 32), (48, 512), (70, 288)])
def test_q8_0_tiles_round_trip_and_place_codes_in_position_order(rows, width):
    rng = np.random.default_rng(rows + width)
    raw = gguf.encode(rng.normal(0, 0.02, (rows, width)).astype(np.float32), "Q8_0")
    tiled = layout.tile(raw, "Q8_0")
    assert tiled.size == layout.tiled_bytes("Q8_0", rows, width)
    np.testing.assert_array_equal(layout.untile(tiled, "Q8_0", rows, width), raw)
    nsup = (width + 255) // 256
    body = tiled.reshape(-1, nsup, 17, 64, 16)  # [row tile][column][chunk][row][16 B]
    r, j = rows - 1, raw.shape[1] - 1
    np.testing.assert_array_equal(body[r // 64, j // 8, 0, r % 64, 2 * (j % 8) : 2 * (j % 8) + 2], raw[r, j, :2])
    codes = body[r // 64, j // 8, 1:, r % 64].reshape(256)[32 * (j % 8) : 32 * (j % 8) + 32]
    np.testing.assert_array_equal(codes, raw[r, j, 2:])


@pytest.mark.parametrize("qtype,rows,width", [("Q5_K", 48, 512), ("Q5_K", 70, 300), ("Q5_1", 1, 32),
                                             ("Q5_1", 70, 288), ("Q5_1", 64, 640)])
def test_q5_tiles_round_trip_and_place_chunks(qtype, rows, width):
    """Q5_K tiles hold the GGUF bytes as [chunk][row][16 B]; Q5_1 super-blocks put each block's
    (d, m), high-bit word and nibbles into chunks h, 2 + h and 4 + block of its half h."""
    from util import random_blocks

    raw = random_blocks(np.random.default_rng(rows + width), rows, width, qtype)
    tiled = layout.tile(raw, qtype)
    assert tiled.size == layout.tiled_bytes(qtype, rows, width)
    np.testing.assert_array_equal(layout.untile(tiled, qtype, rows, width), raw)
    nsup = (width + 255) // 256
    c = layout.CHUNKS[qtype]
    body = tiled.reshape(-1, nsup, c, 64, 16)  # [row tile][column][chunk][row][16 B]
    r, j = rows - 1, raw.shape[1] - 1
    if qtype == "Q5_K":
        np.testing.assert_array_equal(body[r // 64, j, :, r % 64].reshape(-1), raw[r, j])
    else:
        blk, h = j % 8, (j % 8) // 4
        col = body[r // 64, j // 8, :, r % 64]
        np.testing.assert_array_equal(col[h, 4 * (blk % 4) : 4 * (blk % 4) + 4], raw[r, j, :4])
        np.testing.assert_array_equal(col[2 + h, 4 * (blk % 4) : 4 * (blk % 4) + 4], raw[r, j, 4:8])
        np.testing.assert_array_equal(col[4 + blk], raw[r, j, 8:])


def test_w8a8_dot_matches_reference_numpy_q8_matmul(golden):
    """``compute.py:52-65`` restated: bit-equal to the reference's own ``numpy_q8_matmul`` on
    its ``pack_q8`` weights, a zero row staying zero."""
    data = golden("w8a8.npz")
    for rows, width, outputs, _ in data["cases"]:
        key = f"{rows}_{width}_{outputs}"
        got = moe.q8_matmul(data[f"x_{key}"], data[f"raw_{key}"])
        np.testing.assert_array_equal(got.view(np.uint32), data[f"expected_{key}"].view(np.uint32))
        np.testing.assert_array_equal(got[0], 0)


def test_soa_restatement_inverts_the_reference_pack_q6(golden):
    """``oracle.layout.soa_to_rows`` against the reference's own ``pack_q6`` planes."""
    from oracle.layout import soa_to_rows

    data = golden("soa_q6.npz")
    for outputs, inputs in data["cases"]:
        key = f"{outputs}_{inputs}"
        raw = soa_to_rows(data[f"data_{key}"], data[f"scales_{key}"], int(outputs), int(inputs))
        assert np.array_equal(raw, data[f"raw_{key}"])
