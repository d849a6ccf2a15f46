"""Generate the golden fixtures in this directory from the reference's own NumPy code.

Run in a container that has the reference checkout (read-only) at REFERENCE_ROOT:

    python tests/golden/make_golden.py [REFERENCE_ROOT]

The fixtures are committed; tests never read the reference at run time. Sources:

* ``glm53_offload/gguf_quant.py`` ``dequantize_rows`` (numpy backend) and
  ``qwen38_tpu/quant.py`` ``dequantize_rows`` - decode golden for every block type;
* gguf-py 0.19.0 ``gguf.quants.dequantize`` - the third-party pin of the same decoders;
* ``packed_q6/reference.py`` ``fixture``, ``decode_reference``, ``projection_reference``
  - the packed-Q6 projection golden (``tests/test_packed_q6.py:51-81`` cases);
* ``packed_q6/layout.py`` ``pack_q6`` - the reference's SoA planes of fixture rows
  (``soa_q6.npz``), the input form ``qk_q6_soa_to_rows`` restores;
* ``compute.numpy_q8_matmul`` on ``compute.pack_q8`` weights - the W8A8 golden
  (``w8a8.npz``) of the ``int8_q8`` expert policy;
* pure-NumPy functions that live in modules importing JAX are executed from their own
  source text (extracted with ``ast``, no JAX needed): ``compute.pack_q8``,
  ``compute.numpy_q8_matmul`` and the test oracle ``scale_oracle``
  (``tests/test_qwen38_kv_gather.py:22-32``);
* the routed-FFN golden follows the reference's independent NumPy oracle
  ``routing_validation.py:193-243`` (seed 738) line by line, with the reference's
  ``dequantize_rows``;
* the Q8 codec golden evaluates the reference's ml_dtypes oracle expressions of
  ``validation.py:32-52`` (seed 118) and ``test_qwen38_kv_gather.py:69-94`` (seed 710).
"""

import ast
import hashlib
import os
import sys
from pathlib import Path

import ml_dtypes
import numpy as np

HERE = Path(__file__).resolve().parent
BF16 = ml_dtypes.bfloat16


def load_reference(root):
    kaggle = Path(root) / "kaggle"
    sys.path.insert(0, str(kaggle))
    from glm53_offload import gguf_quant
    from packed_q6 import layout as q6layout
    from packed_q6 import reference as q6ref
    from qwen38_tpu import quant

    def extract(path, name):
        tree = ast.parse(path.read_text())
        for node in tree.body:
            if isinstance(node, ast.FunctionDef) and node.name == name:
                scope = {"np": np}
                exec(compile(ast.Module([node], []), str(path), "exec"), scope)
                return scope[name]
        raise KeyError(name)

    compute = kaggle / "qwen38_tpu" / "compute.py"
    parallel = kaggle / "qwen38_tpu" / "parallel.py"
    funcs = {
        "split_expert_bytes": extract(parallel, "split_expert_bytes"),
        "pack_q8": extract(compute, "pack_q8"),
        "numpy_q8_matmul": extract(compute, "numpy_q8_matmul"),
        "scale_oracle": extract(kaggle / "tests" / "test_qwen38_kv_gather.py", "scale_oracle"),
        "pack_q6": q6layout.pack_q6,
    }
    return gguf_quant, quant, q6ref, funcs


def decode_golden(gguf_quant, quant):
    import gguf
    from gguf.quants import dequantize

    rng = np.random.default_rng(20261201)
    out = {}
    offsets = {"Q4_K": (0, 2), "Q5_K": (0, 2), "Q6_K": (208,), "Q8_0": (0,), "Q4_0": (0,),
               "Q4_1": (0, 2), "Q5_0": (0,), "Q5_1": (0, 2), "IQ4_NL": (0,)}
    for qtype, (values, size) in {
        "Q4_K": (256, 144), "Q5_K": (256, 176), "Q6_K": (256, 210), "Q8_0": (32, 34),
        "F16": (1, 2), "BF16": (1, 2), "F32": (1, 4), "Q4_0": (32, 18), "Q4_1": (32, 20),
        "Q5_0": (32, 22), "Q5_1": (32, 24), "IQ4_NL": (32, 18),
    }.items():
        nblk = 3 if values > 1 else 40
        raw = rng.integers(0, 256, (5, nblk, size), dtype=np.uint8)
        if qtype == "F16":
            raw = rng.uniform(-4, 4, (5, nblk)).astype("<f2").view(np.uint8).reshape(5, nblk, 2)
        elif qtype == "F32":
            raw = rng.uniform(-4, 4, (5, nblk)).astype("<f4").view(np.uint8).reshape(5, nblk, 4)
        for off in offsets.get(qtype, ()):
            scale = rng.uniform(-0.3, 0.3, (5, nblk)).astype("<f2")
            raw[..., off : off + 2] = scale.view(np.uint8).reshape(5, nblk, 2)
        width = nblk * values - (7 if values > 1 else 0)
        if qtype in ("Q4_0", "Q4_1", "Q5_0", "Q5_1", "IQ4_NL"):
            expected = quant.dequantize_rows(raw, qtype, width)
        else:
            expected = gguf_quant.dequantize_rows(raw, qtype, width)
        third = np.asarray(
            dequantize(raw.reshape(5, -1), gguf.GGMLQuantizationType[qtype]), np.float32
        )[:, :width]
        np.testing.assert_array_equal(expected, third)  # reference == gguf-py, bit for bit
        out[f"{qtype}_raw"] = raw
        out[f"{qtype}_width"] = np.int64(width)
        out[f"{qtype}_expected"] = np.asarray(expected, np.float32)
    np.savez_compressed(HERE / "gguf_decode.npz", **out)


def q6_golden(q6ref):
    out = {}
    # tests/test_packed_q6.py:27-39: FP16 extremes/subnormals and every sub-scale byte.
    raw = q6ref.fixture(64, 256)
    d = np.array([0, -0.0, 65504, -65504, 2**-24, -(2**-24), 2**-14, 1], dtype="<f2")
    raw[:8, 0, 208:] = d.view(np.uint8).reshape(8, 2)
    raw[..., 192:208] = np.arange(1024, dtype=np.uint16).astype(np.uint8).reshape(64, 1, 16)
    out["extremes_raw"] = raw
    out["extremes_bf16"] = q6ref.decode_reference(raw, 256).astype(BF16).astype(np.float32)
    # tests/test_packed_q6.py:51-81 projection cases, x from seed 721.
    cases = [(1, 1, 1), (2, 67, 255), (4, 128, 257), (8, 64, 512), (9, 65, 263),
             (1, 320, 2560), (8, 640, 2560)]
    out["cases"] = np.array(cases, np.int64)
    for batch, outputs, inputs in cases:
        raw = q6ref.fixture(outputs, inputs)
        x = np.random.default_rng(721).normal(size=(batch, inputs)).astype(np.float32)
        if batch > 1:
            x[0] = 0
        key = f"{batch}_{outputs}_{inputs}"
        out[f"raw_sha256_{key}"] = np.frombuffer(hashlib.sha256(raw.tobytes()).digest(), np.uint8)
        out[f"x_{key}"] = x
        out[f"expected_{key}"] = q6ref.projection_reference(x, raw)
    np.savez_compressed(HERE / "q6_projection.npz", **out)


ROUTING_CASES = (("mixed", "Q8_0", 32), ("q6", "Q6_K", 256))
ROUTING_BATCHES = (1, 17, 273)


def routing_inputs(label, pack_q8):
    """Inputs of routing_validation.py:193-218 (seed 738, EP8 -> 40 experts, tp=1).

    ``label`` "mixed" is the reference's own case (Q6_K gate/up, Q8_0 down, I=32);
    "q6" is the same generator with Q6_K down and I=256. Returns raw GGUF bytes per
    projection ``[count, bytes]`` and, per batch, ``(ids, weights, x)``.
    """
    down_type, intermediate = {k: (d, i) for k, d, i in ROUTING_CASES}[label]
    rng = np.random.default_rng(738)
    hidden, count = 256, 40
    packed = {}
    for name in ("gate", "up"):
        raw = rng.integers(0, 256, (count, intermediate, 1, 210), dtype=np.uint8)
        raw[..., 192:208] = rng.integers(1, 9, raw[..., 192:208].shape, dtype=np.uint8)
        raw[..., 208:210] = np.array([1 / 2048], "<f2").view(np.uint8)
        packed[name] = raw
    if down_type == "Q8_0":
        packed["down"] = pack_q8(
            rng.normal(0, 0.08, (count * hidden, intermediate)).astype(np.float32)
        ).reshape(count, hidden, intermediate // 32, 34)
    else:
        raw = rng.integers(0, 256, (count, hidden, intermediate // 256, 210), dtype=np.uint8)
        raw[..., 192:208] = rng.integers(1, 9, raw[..., 192:208].shape, dtype=np.uint8)
        raw[..., 208:210] = np.array([1 / 4096], "<f2").view(np.uint8)
        packed["down"] = raw
    batches = {}
    for batch in ROUTING_BATCHES:
        ids = np.stack((np.zeros(batch, np.int32), 1 + np.arange(batch) % (count - 1)), -1)
        ids[:8, 1] = 0  # duplicate routes combine, rather than overwrite
        weights = np.full(ids.shape, 0.5, np.float32)
        if batch > 1:
            weights[::37] = 0  # finished rows contribute zero
        source = np.random.default_rng(738 + batch).normal(0, 0.3, (batch, hidden))
        batches[batch] = (ids, weights, source.astype(np.float32))
    return packed, batches, down_type, hidden, intermediate, count


def routing_golden(quant, funcs):
    """Expected outputs of the reference's NumPy routed-FFN oracle (routing_validation.py:224-243)."""
    out = {}
    for label, _, _ in ROUTING_CASES:
        packed, batches, down_type, hidden, intermediate, count = routing_inputs(
            label, funcs["pack_q8"]
        )
        for name, raw in packed.items():
            out[f"{label}_{name}_sha256"] = np.frombuffer(
                hashlib.sha256(raw.tobytes()).digest(), np.uint8
            )
        for batch, (ids, weights, source) in batches.items():
            dtypes = (np.float32, np.dtype(BF16)) if label == "mixed" else (np.dtype(BF16),)
            for dtype in dtypes:
                x = source.astype(dtype)
                routing = weights.astype(dtype)
                expected = np.zeros((batch, hidden), np.float32)
                for expert in range(count):
                    route = np.sum(np.where(ids == expert, routing, 0).astype(np.float32), -1)

                    def project(value, name, expert=expert):
                        raw = packed[name][expert]
                        qtype = down_type if name == "down" else "Q6_K"
                        width = intermediate if name == "down" else hidden
                        matrix = quant.dequantize_rows(raw, qtype, width).astype(dtype)
                        return (value.astype(np.float32) @ matrix.astype(np.float32).T).astype(dtype)

                    gate = project(x, "gate").astype(np.float32)
                    activated = (gate / (1 + np.exp(-gate))).astype(dtype)
                    product = (
                        activated.astype(np.float32) * project(x, "up").astype(np.float32)
                    ).astype(dtype)
                    expected += project(product, "down").astype(np.float32) * route[:, None]
                expected = expected.astype(dtype).astype(np.float32)
                if dtype == np.float32:
                    out[f"{label}_b{batch}_f32_expected"] = expected
                else:
                    out[f"{label}_b{batch}_bf16_bits"] = (
                        expected.view(np.uint32) >> 16
                    ).astype(np.uint16)
    np.savez_compressed(HERE / "routing_ffn.npz", **out)


def q8_golden(funcs):
    out = {}
    # validation.py:32-52 (seed 118): codes/scales from ml_dtypes rounding, and the
    # unrounded-divisor codes of the v3 failure.
    rng = np.random.default_rng(118)
    for width in (8, 256):
        group = min(32, width)
        source = rng.normal(size=(2, 2, width)).astype(np.float32)
        source[0, 0, :group] = 0
        source[0, 1, :group] = np.linspace(-0.99, 0.99, group, dtype=np.float32)
        source[0, 1, 0] = 1
        stored = np.float32(1 / 127).astype(BF16).astype(np.float32)
        source[0, 1, 1] = np.float32(64.501) * stored
        for dtype in (np.float32, np.dtype(BF16)):
            host = source.astype(dtype)
            grouped = host.astype(np.float32).reshape(2, 2, -1, group)
            full = np.max(np.abs(grouped), -1) / np.float32(127)
            scale = full.astype(BF16)
            divisor = np.where(scale == 0, 1, scale.astype(np.float32))
            codes = np.clip(np.rint(grouped / divisor[..., None]), -127, 127).astype(np.int8)
            unrounded = np.clip(
                np.rint(grouped / np.where(full == 0, 1, full)[..., None]), -127, 127
            ).astype(np.int8)
            tag = f"w{width}_{'bf16' if dtype != np.float32 else 'f32'}"
            out[f"{tag}_x"] = host.astype(np.float32)
            out[f"{tag}_codes"] = codes.reshape(host.shape)
            out[f"{tag}_scale"] = scale.astype(np.float32)
            out[f"{tag}_unrounded_codes"] = unrounded.reshape(host.shape)
    # test_qwen38_kv_gather.py:69-94 (seed 710): full read of a written cache row.
    rng = np.random.default_rng(710)
    source = rng.normal(size=(2, 2, 256)).astype(BF16)
    source[0, 0, :32] = 0
    grouped = source[0].astype(np.float32).reshape(2, 8, 32)
    scale = (np.max(np.abs(grouped), -1) / 127).astype(BF16).astype(np.float32)
    codes = np.clip(np.rint(grouped / np.where(scale == 0, 1, scale)[..., None]), -127, 127)
    out["read_source"] = source.astype(np.float32)
    out["read_reconstructed"] = (codes * scale[..., None]).reshape(2, 256).astype(np.float32)
    # test_qwen38_kv_gather.py:35-53 (seed 629): scale gather with wrapped/clamped indices.
    oracle = funcs["scale_oracle"]
    for batch, groups, time in ((1, 16, 8), (2, 4, 32), (8, 16, 64)):
        rng = np.random.default_rng(629)
        plane = rng.normal(size=(batch * groups, time)).astype(BF16)
        plane[:, 0] = 0
        plane[:, 1] = -0.0
        indices = np.tile(
            np.array([0, 0, 1, time // 8, time - 1, -1, -time - 2, time + 3]), (batch, 1)
        )
        tag = f"gather_{batch}_{groups}_{time}"
        out[f"{tag}_plane"] = plane.view(np.uint16)
        out[f"{tag}_indices"] = indices.astype(np.int32)
        out[f"{tag}_expected"] = oracle(plane, indices, groups).view(np.uint16)
    # test_qwen38_gate_regression.py:15-28 (seed 49): BF16 RNE incl. ties and specials.
    rng = np.random.default_rng(49)
    random = rng.normal(size=1024).astype(np.float32)
    ties = np.array(
        [0.0, -0.0, 1.00390625, -1.00390625, 1.01171875, -1.01171875, np.inf, -np.inf, np.nan],
        np.float32,
    )
    src = np.concatenate((random, ties))
    out["bf16_source"] = src
    out["bf16_expected"] = src.astype(BF16).astype(np.float32)
    np.savez_compressed(HERE / "q8_kv.npz", **out)


SPLIT_CASES = (("Q6_K", 256, 512, 2), ("Q8_0", 64, 64, 2), ("Q4_K", 512, 256, 1))


def split_inputs(qtype, kind, hidden, inter, block):
    """Raw expert bytes [3, bytes] for one split case (seeded per case)."""
    values, size = block
    rows, width = (hidden, inter) if kind == "down" else (inter, hidden)
    seed = [101, hidden, inter, ("gate", "up", "down").index(kind), size]
    return np.random.default_rng(seed).integers(0, 256, (3, rows * (width // values) * size), dtype=np.uint8)


def split_golden(quant, funcs):
    """parallel.py:40-61 split_expert_bytes (its block_layout is quant's): sha256 + shape."""
    split = funcs["split_expert_bytes"]
    split.__globals__["block_layout"] = quant.block_layout
    out = {}
    for qtype, hidden, inter, tp in SPLIT_CASES:
        for kind in ("gate", "up", "down"):
            raw = split_inputs(qtype, kind, hidden, inter, quant.block_layout(qtype))
            result = np.ascontiguousarray(split(raw, kind, qtype, hidden, inter, tp))
            tag = f"{qtype}_{kind}_{tp}"
            out[f"{tag}_shape"] = np.array(result.shape, np.int64)
            out[f"{tag}_sha256"] = np.frombuffer(hashlib.sha256(result.tobytes()).digest(), np.uint8)
    np.savez_compressed(HERE / "split_experts.npz", **out)


SOA_CASES = ((64, 256), (70, 300), (130, 512))


def soa_golden(q6ref, funcs):
    """The reference's SoA planes (``packed_q6/layout.py:49-91``) of fixture rows."""
    out = {"cases": np.array(SOA_CASES, np.int64)}
    for outputs, inputs in SOA_CASES:
        raw = q6ref.fixture(outputs, inputs)
        packed = funcs["pack_q6"](raw, inputs)
        key = f"{outputs}_{inputs}"
        out[f"raw_{key}"] = raw
        out[f"data_{key}"] = np.asarray(packed.data)
        out[f"scales_{key}"] = np.asarray(packed.scales)
    np.savez_compressed(HERE / "soa_q6.npz", **out)


W8A8_CASES = ((8, 256, 64, 837), (24, 640, 256, 5))


def w8a8_golden(funcs):
    """The reference's W8A8 dot ``numpy_q8_matmul`` (``compute.py:52-65``) on weights packed by
    its ``pack_q8`` (``compute.py:41-49``): the integer-dot test of
    ``tests/test_qwen38_compute.py:81-100`` (seed 837: a zero row, x20 outliers on every 32nd
    value, a row of 127s), and a down-projection shape (I = 640, 20 groups)."""
    out = {"cases": np.array(W8A8_CASES, np.int64)}
    for rows, width, outputs, seed in W8A8_CASES:
        rng = np.random.default_rng(seed)
        x = rng.normal(size=(rows, width)).astype(np.float32)
        x[0] = 0
        x[1, ::32] *= 20
        x[2] = 127
        x = x.astype(BF16).astype(np.float32)  # the kernels take BF16 activations
        raw = funcs["pack_q8"](rng.normal(size=(outputs, width)).astype(np.float32))
        key = f"{rows}_{width}_{outputs}"
        out[f"x_{key}"] = x
        out[f"raw_{key}"] = raw.reshape(outputs, width // 32, 34)
        out[f"expected_{key}"] = funcs["numpy_q8_matmul"](x, raw.reshape(outputs, width // 32, 34))
    np.savez_compressed(HERE / "w8a8.npz", **out)


def main():
    args = [a for a in sys.argv[1:] if not a.startswith("--only=")]
    only = [a.split("=", 1)[1] for a in sys.argv[1:] if a.startswith("--only=")]
    root = args[0] if args else os.environ.get("QK_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_CHECKOUT [--only=NAME] (or set QK_REFERENCE_ROOT)")
    gguf_quant, quant, q6ref, funcs = load_reference(root)
    steps = {
        "decode": lambda: decode_golden(gguf_quant, quant),
        "q6": lambda: q6_golden(q6ref),
        "routing": lambda: routing_golden(quant, funcs),
        "q8": lambda: q8_golden(funcs),
        "split": lambda: split_golden(quant, funcs),
        "soa": lambda: soa_golden(q6ref, funcs),
        "w8a8": lambda: w8a8_golden(funcs),
    }
    for name, step in steps.items():
        if not only or name in only:
            step()
    for path in sorted(HERE.glob("*.npz")):
        print(f"{path.name}: {path.stat().st_size} bytes")


if __name__ == "__main__":
    main()
