"""GGUF decode, tiled repack and packed projection on the GPU against the pinned oracle."""

import hashlib

import numpy as np
import pytest

from oracle import gguf, layout, moe
from oracle.precision import bf16_round
from util import bf16_tensor, random_blocks, to_f32

pytestmark = pytest.mark.gpu

TYPES = ["Q4_K", "Q5_K", "Q6_K", "Q8_0", "F16", "BF16", "F32", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "IQ4_NL"]


@pytest.mark.parametrize("qtype", TYPES)
def test_dequantize_rows_bit_exact_against_reference_golden(golden, cuda_device, qtype):
    import torch

    from qk_b200.quant import dequantize_rows

    data = golden("gguf_decode.npz")
    raw, width = data[f"{qtype}_raw"], int(data[f"{qtype}_width"])
    expected = data[f"{qtype}_expected"]
    dev = torch.from_numpy(raw).to(cuda_device)
    got = dequantize_rows(dev, qtype, width).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), expected.view(np.uint32))
    got16 = to_f32(dequantize_rows(dev, qtype, width, dtype=torch.bfloat16))
    np.testing.assert_array_equal(got16.view(np.uint32), bf16_round(expected).view(np.uint32))


def test_q6_k_extreme_scales_every_sub_scale_bf16(golden, cuda_device):
    import torch

    from qk_b200.packed import dequantize_packed, pack_q6
    from qk_b200.quant import dequantize_rows

    data = golden("q6_projection.npz")
    raw = data["extremes_raw"]
    expected = data["extremes_bf16"]
    got = to_f32(dequantize_rows(torch.from_numpy(raw).to(cuda_device), "Q6_K", 256, torch.bfloat16))
    np.testing.assert_array_equal(got.view(np.uint32), expected.view(np.uint32))
    # the GEMM kernels' in-register fragment decoder gives the same bits
    tiled = to_f32(dequantize_packed(pack_q6(raw, 256, cuda_device)))
    np.testing.assert_array_equal(tiled.view(np.uint32), expected.view(np.uint32))


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K"])
@pytest.mark.parametrize("rows,width", [(1, 256), (17, 512), (65, 263), (512, 2048), (2048, 512)])
def test_repack_is_lossless_and_fragment_decode_is_bit_exact(cuda_device, qtype, rows, width):
    import torch

    from qk_b200.packed import dequantize_packed, pack_rows, unpack_rows

    rng = np.random.default_rng(rows * 7 + width)
    size = layout.BLOCK_BYTES[qtype]
    raw = rng.integers(0, 256, (rows, (width + 255) // 256, size), dtype=np.uint8)
    offs = (208,) if qtype == "Q6_K" else (0, 2)
    for off in offs:
        raw[..., off : off + 2] = rng.uniform(-0.05, 0.05, raw.shape[:2]).astype("<f2").view(
            np.uint8).reshape(*raw.shape[:2], 2)
    packed = pack_rows(raw, width, qtype, cuda_device)
    assert packed.data.numel() == layout.tiled_bytes(qtype, rows, width)
    np.testing.assert_array_equal(packed.data.cpu().numpy(), layout.tile(raw, qtype))
    np.testing.assert_array_equal(unpack_rows(packed).cpu().numpy(), raw)
    expected = bf16_round(gguf.dequantize_rows(raw, qtype, width))
    got = to_f32(dequantize_packed(packed, torch.bfloat16))
    np.testing.assert_array_equal(got.view(np.uint32), expected.view(np.uint32))
    # the fused form the GEMM kernels run: equal values (a zero may be -0 vs +0)
    fused = to_f32(dequantize_packed(packed, torch.bfloat16, fused=True))
    np.testing.assert_array_equal(fused, expected)


@pytest.mark.parametrize("rows,width", [(1, 32), (17, 96), (65, 263), (130, 2048), (64, 2080)])
def test_q8_0_repack_is_lossless_and_fragment_decode_is_bit_exact(cuda_device, rows, width):
    """Q8_0 rows (32-value blocks) in 256-value tile columns: ragged last columns are zero."""
    import torch

    from qk_b200.packed import dequantize_packed, pack_rows, unpack_rows

    rng = np.random.default_rng(rows * 5 + width)
    raw = rng.integers(0, 256, (rows, (width + 31) // 32, 34), dtype=np.uint8)
    raw[..., 0:2] = rng.uniform(-0.05, 0.05, raw.shape[:2]).astype("<f2").view(np.uint8).reshape(*raw.shape[:2], 2)
    raw[..., 2] = 0x80  # the code -128 in every block
    packed = pack_rows(raw, width, "Q8_0", cuda_device)
    assert packed.data.numel() == layout.tiled_bytes("Q8_0", rows, width)
    np.testing.assert_array_equal(packed.data.cpu().numpy(), layout.tile(raw, "Q8_0"))
    np.testing.assert_array_equal(unpack_rows(packed).cpu().numpy(), raw)
    expected = bf16_round(gguf.dequantize_rows(raw, "Q8_0", width))
    for dtype in (torch.bfloat16, torch.float32):  # FP32 out: the BF16 MMA operands, widened
        got = to_f32(dequantize_packed(packed, dtype))
        np.testing.assert_array_equal(got.view(np.uint32), expected.view(np.uint32))
        np.testing.assert_array_equal(to_f32(dequantize_packed(packed, dtype, fused=True)), expected)


@pytest.mark.parametrize("qtype,rows,width", [
    ("Q5_K", 1, 256), ("Q5_K", 17, 512), ("Q5_K", 65, 263), ("Q5_K", 512, 2048),
    ("Q5_1", 1, 32), ("Q5_1", 17, 96), ("Q5_1", 65, 263), ("Q5_1", 130, 2048), ("Q5_1", 64, 640)])
def test_q5_repack_is_lossless_and_fragment_decode_is_bit_exact(cuda_device, qtype, rows, width):
    """Q5_K (GGUF bytes, 11 chunks) and Q5_1 (8-block super-blocks, ragged last columns zero)
    tiles: byte-equal to the oracle's layout, lossless, and decoded bit-exactly by the
    fragment decoders the expert kernels run."""
    import torch

    from qk_b200.packed import dequantize_packed, pack_rows, unpack_rows

    raw = random_blocks(np.random.default_rng(rows * 3 + width), rows, width, qtype)
    packed = pack_rows(raw, width, qtype, cuda_device)
    assert packed.data.numel() == layout.tiled_bytes(qtype, rows, width)
    np.testing.assert_array_equal(packed.data.cpu().numpy(), layout.tile(raw, qtype))
    np.testing.assert_array_equal(unpack_rows(packed).cpu().numpy(), raw)
    expected = bf16_round(gguf.dequantize_rows(raw, qtype, width))
    for dtype in (torch.bfloat16, torch.float32):
        got = to_f32(dequantize_packed(packed, dtype))
        np.testing.assert_array_equal(got.view(np.uint32), expected.view(np.uint32))
        np.testing.assert_array_equal(to_f32(dequantize_packed(packed, dtype, fused=True)), expected)


@pytest.mark.parametrize("qtype,n,k", [("Q5_K", 200, 512), ("Q5_1", 130, 640)])
def test_q5_packed_projection(cuda_device, qtype, n, k):
    """The dense packed projection over Q5_K / Q5_1 tiles against an FP64 dot of the decoded
    BF16 weights (the projection tolerance of test_packed_q6.py:77-81)."""
    from qk_b200.packed import pack_rows, quant_matmul

    rng = np.random.default_rng(n + k)
    raw = random_blocks(rng, n, k, qtype)
    x = bf16_round(rng.normal(size=(9, k)).astype(np.float32))
    got = quant_matmul(bf16_tensor(x, cuda_device), pack_rows(raw, k, qtype, cuda_device)).cpu().numpy()
    w = bf16_round(gguf.dequantize_rows(raw, qtype, k)).astype(np.float64)
    np.testing.assert_allclose(got, x.astype(np.float64) @ w.T, rtol=2e-5, atol=2e-4)


@pytest.mark.parametrize("scale", [np.inf, -np.inf, np.nan])
def test_nonfinite_block_scale_rejected(cuda_device, scale):
    from qk_b200.packed import pack_q6

    raw = gguf.legal_q6_k_fixture(1, 256)
    raw[0, 0, 208:] = np.array([scale], dtype="<f2").view(np.uint8)
    with pytest.raises(ValueError, match="finite"):
        pack_q6(raw, 256, cuda_device)


def test_invalid_layout_or_projection_contract_rejected(cuda_device):
    import torch

    from qk_b200.packed import pack_q6, q6_matmul

    with pytest.raises(TypeError, match="uint8"):
        pack_q6(np.zeros((64, 1, 210)), 256, cuda_device)
    with pytest.raises(ValueError, match="Expected"):
        pack_q6(np.zeros((64, 1, 211), np.uint8), 256, cuda_device)
    packed = pack_q6(gguf.legal_q6_k_fixture(64, 256), 256, cuda_device)
    with pytest.raises(ValueError, match="BF16"):
        q6_matmul(torch.ones((1, 256), device=cuda_device), packed, output_features=64)
    with pytest.raises(ValueError, match="multiple of 8"):
        q6_matmul(torch.ones((1, 256), dtype=torch.bfloat16, device=cuda_device), packed,
                  output_features=64, batch_tile=1)
    with pytest.raises(ValueError, match="dtype/shape"):
        q6_matmul(torch.ones((1, 257), dtype=torch.bfloat16, device=cuda_device), packed,
                  output_features=64)


def test_packed_projection_matches_reference_fp64_dot(golden, cuda_device):
    from qk_b200.packed import pack_q6, q6_matmul

    data = golden("q6_projection.npz")
    for batch, outputs, inputs in data["cases"]:
        batch, outputs, inputs = int(batch), int(outputs), int(inputs)
        key = f"{batch}_{outputs}_{inputs}"
        raw = gguf.legal_q6_k_fixture(outputs, inputs)
        assert hashlib.sha256(raw.tobytes()).digest() == bytes(data[f"raw_sha256_{key}"])
        packed = pack_q6(raw, inputs, cuda_device)
        x = bf16_tensor(data[f"x_{key}"], cuda_device)
        got = q6_matmul(x, packed, output_features=outputs).cpu().numpy()
        assert got.dtype == np.float32 and got.shape == (batch, outputs)
        assert np.isfinite(got).all()
        # tests/test_packed_q6.py:81 tolerance
        np.testing.assert_allclose(got, data[f"expected_{key}"], rtol=2e-5, atol=2e-4)


@pytest.mark.parametrize("qtype", ["Q6_K", "Q4_K", "Q8_0"])
@pytest.mark.parametrize("m", [1, 5, 33, 70])
def test_quant_matmul_against_oracle(cuda_device, qtype, m):
    from qk_b200.packed import pack_rows, quant_matmul

    rng = np.random.default_rng(11 + m)
    w = rng.normal(0, 0.02, (96, 512)).astype(np.float32)
    raw = gguf.encode(w, qtype)
    x = rng.normal(size=(m, 512)).astype(np.float32)
    packed = pack_rows(raw, 512, qtype, cuda_device)
    got = quant_matmul(bf16_tensor(x, cuda_device), packed).cpu().numpy()
    wb = bf16_round(gguf.dequantize_rows(raw, qtype, 512))
    expected = (bf16_round(x).astype(np.float64) @ wb.astype(np.float64).T).astype(np.float32)
    np.testing.assert_allclose(got, expected, rtol=2e-5, atol=2e-4)


def test_accumulator_is_reset_between_row_and_token_tiles(cuda_device):
    import torch

    from qk_b200.packed import pack_q6, q6_matmul

    raw = gguf.legal_q6_k_fixture(128, 512)
    raw[64:] = raw[:64]
    packed = pack_q6(raw, 512, cuda_device)
    x = torch.ones((40, 512), dtype=torch.bfloat16, device=cuda_device)
    x[20:] = -1
    result = q6_matmul(x, packed, output_features=128).cpu().numpy()
    np.testing.assert_array_equal(result[:, :64], result[:, 64:])
    np.testing.assert_array_equal(result[:20], -result[20:])


def test_reference_soa_planes_restore_gguf_rows_and_project(golden, cuda_device):
    """The reference's ``PackedQ6`` planes (its own ``pack_q6`` output) through
    ``qk_q6_soa_to_rows`` give back the GGUF rows byte for byte, ``from_soa`` equals
    ``pack_q6`` of those rows, and ``q6_matmul(x, data, scales, ...)`` (the reference's call
    form, ``packed_q6/kernel.py:99``) equals the projection over this build's tiles."""
    import torch

    from qk_b200 import _lib
    from qk_b200.packed import from_soa, pack_q6, q6_matmul

    data = golden("soa_q6.npz")
    for outputs, inputs in data["cases"]:
        outputs, inputs = int(outputs), int(inputs)
        key = f"{outputs}_{inputs}"
        d = torch.from_numpy(data[f"data_{key}"]).to(cuda_device)
        sc = torch.from_numpy(data[f"scales_{key}"]).to(cuda_device)
        raw = torch.empty((outputs, (inputs + 255) // 256, 210), dtype=torch.uint8, device=cuda_device)
        _lib.call("qk_q6_soa_to_rows", _lib.ptr(d), _lib.ptr(sc), outputs, inputs, _lib.ptr(raw),
                  _lib.stream_handle(cuda_device))
        assert np.array_equal(raw.cpu().numpy(), data[f"raw_{key}"])
        mine = pack_q6(data[f"raw_{key}"], inputs, device=cuda_device)
        assert torch.equal(from_soa(data[f"data_{key}"], data[f"scales_{key}"], inputs, outputs,
                                    device=cuda_device).data, mine.data)
        x = torch.randn(9, inputs, generator=torch.Generator().manual_seed(outputs)).to(
            cuda_device, torch.bfloat16)
        want = q6_matmul(x, mine, output_features=outputs)
        got = q6_matmul(x, d, sc, output_features=outputs)
        assert torch.equal(got, want)
    with pytest.raises(ValueError, match="Packed Q6 dtype/shape"):
        q6_matmul(x, d[:-1], sc, output_features=outputs)
    with pytest.raises(ValueError, match="Packed Q6 scale dtype/shape"):
        q6_matmul(x, d, sc[:-512], output_features=outputs)
