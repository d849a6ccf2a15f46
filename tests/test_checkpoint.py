"""GGUF checkpoint access (``qk_b200.checkpoint``): the tensor table from a GGUF header and from
the reference's audit JSON form, range reads and their checks, and (GPU) the per-rank resident
experts, byte-equal to placing the same GGUF bytes directly.

Test files are written with gguf-py's ``GGUFWriter`` (an independent implementation of the
container format), and the parsed table is checked against gguf-py's ``GGUFReader``."""

import json

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

# I = 512: a tensor-parallel slice of 256 intermediate channels is one whole Q6_K / Q4_K
# down block, which the reference's split requires (qwen38_tpu/parallel.py:53-55)
H, I, E = 512, 512, 4


def finite_blocks(rng, shape, qtype):
    """Random GGUF blocks of ``qtype`` with finite FP16 block scales (the repack rejects others)."""
    raw = rng.integers(0, 256, size=shape, dtype=np.uint8)
    count = int(np.prod(shape[:-1]))
    d = rng.uniform(1e-3, 2e-3, count).astype(np.float16).view(np.uint8).reshape(shape[:-1] + (2,))
    if qtype == "Q6_K":
        raw[..., 208:210] = d
    elif qtype == "Q4_K":
        raw[..., 0:2] = d
        raw[..., 2:4] = rng.uniform(0, 1e-3, count).astype(np.float16).view(np.uint8).reshape(shape[:-1] + (2,))
    elif qtype == "Q8_0":
        raw[..., 0:2] = d
    return raw


def write_model(path, rng, layers=1, gate="Q6_K", down="Q6_K"):
    """A GGUF file with one MoE expert set per layer, a norm and an F16 tensor."""
    from qk_b200.quant import BLOCK_LAYOUTS

    t = gguf.GGMLQuantizationType
    w = gguf.GGUFWriter(str(path), "qwen4exp")
    w.add_uint32("qwen4exp.expert_count", E)
    w.add_array("qwen4exp.layer_multipliers", [3, 5, 7])
    w.add_string("general.name", "synthetic")
    raws = {}
    for layer in range(layers):
        for kind, qtype in (("gate", gate), ("up", gate), ("down", down)):
            rows, width = (H, I) if kind == "down" else (I, H)
            values, size = BLOCK_LAYOUTS[qtype]
            raw = finite_blocks(rng, (E, rows, width // values, size), qtype)
            name = f"blk.{layer}.ffn_{kind}_exps.weight"
            w.add_tensor(name, raw.reshape(E, rows, -1), raw_dtype=getattr(t, qtype))
            raws[name] = raw
    w.add_tensor("blk.0.attn_norm.weight", np.ones(H, np.float32))
    w.add_tensor("token_embd.weight", rng.standard_normal((8, H)).astype(np.float16))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return raws


@pytest.fixture()
def model(tmp_path):
    path = tmp_path / "model.gguf"
    raws = write_model(path, np.random.default_rng(5))
    return path, raws


def test_header_table_matches_gguf_reader(model):
    from qk_b200.checkpoint import read_gguf_header

    path, raws = model
    metadata, tensors = read_gguf_header(path)
    assert metadata["qwen4exp.expert_count"] == E
    assert metadata["qwen4exp.layer_multipliers"] == [3, 5, 7]
    assert metadata["general.name"] == "synthetic"
    reader = gguf.GGUFReader(str(path))
    assert {t.name for t in reader.tensors} == set(tensors)
    for t in reader.tensors:
        mine = tensors[t.name]
        assert mine["dims"] == [int(v) for v in t.shape]
        assert mine["type"] == t.tensor_type.name
        assert mine["data0"] + mine["offset"] == t.data_offset
        assert mine["nbytes"] == t.n_bytes


def test_reads_and_packed_shapes(model):
    from qk_b200.checkpoint import Checkpoint

    path, raws = model
    ckpt = Checkpoint.from_gguf(path, log=lambda *_: None)
    for name, raw in raws.items():
        assert ckpt.packed_shape(name) == raw.shape
        assert np.array_equal(ckpt.packed(name), raw)
    name = "blk.0.ffn_down_exps.weight"
    flat = raws[name].reshape(-1)
    assert ckpt.read(name, 1000, 77) == flat[1000:1077].tobytes()
    assert ckpt.expert_types(0) == ("Q6_K", "Q6_K", "Q6_K")
    with pytest.raises(ValueError, match="Read outside tensor"):
        ckpt.read(name, len(flat) - 4, 8)
    with pytest.raises(ValueError, match="Read outside tensor"):
        ckpt.read(name, -1, 4)


def test_audit_json_form_and_bounds(model, tmp_path):
    from qk_b200.checkpoint import Checkpoint, read_gguf_header

    path, raws = model
    _, tensors = read_gguf_header(path)
    audit = tmp_path / "audit.json"
    audit.write_text(json.dumps({"tensors": tensors,
                                 "files": [{"file": path.name, "file_bytes": path.stat().st_size}]}))
    ckpt = Checkpoint(audit, tmp_path, log=lambda *_: None)
    name = "blk.0.ffn_gate_exps.weight"
    assert np.array_equal(ckpt.packed(name), raws[name])
    # a table entry reaching past its file is refused before any read
    bad = dict(tensors)
    bad[name] = dict(tensors[name], offset=path.stat().st_size)
    audit.write_text(json.dumps({"tensors": bad}))
    with pytest.raises(ValueError, match="Tensor outside source shard"):
        Checkpoint(audit, tmp_path)
    # a byte count that does not match the dims and type
    bad[name] = dict(tensors[name], nbytes=tensors[name]["nbytes"] - 210)
    audit.write_text(json.dumps({"tensors": bad}))
    with pytest.raises(ValueError, match="Invalid quantized tensor size"):
        Checkpoint(audit, tmp_path)


def test_not_a_gguf_file(tmp_path):
    from qk_b200.checkpoint import read_gguf_header

    path = tmp_path / "x.gguf"
    path.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(ValueError, match="not a GGUF file"):
        read_gguf_header(path)


@pytest.mark.gpu
@pytest.mark.parametrize("gate,down", [("Q6_K", "Q6_K"), ("Q4_K", "Q8_0")])
def test_resident_experts_equal_direct_placement(tmp_path, cuda_device, gate, down):
    import torch

    from qk_b200.checkpoint import Checkpoint
    from qk_b200.parallel import put_expert_bytes

    path = tmp_path / "model.gguf"
    raws = write_model(path, np.random.default_rng(11), gate=gate, down=down)
    ckpt = Checkpoint.from_gguf(path, log=lambda *_: None)
    types = dict(gate=gate, up=gate, down=down)
    # one device; then every rank of a 2 (expert) x 2 (tensor) mesh placed by one process
    for rank, world, tp in ((0, 1, 1), (0, 4, 2), (1, 4, 2), (2, 4, 2), (3, 4, 2)):
        got = ckpt.resident_experts(0, tensor_parallel=tp, device=cuda_device, rank=rank, world=world)
        for kind in ("gate", "up", "down"):
            raw = raws[f"blk.0.ffn_{kind}_exps.weight"]
            want = put_expert_bytes(raw.reshape(E, -1), kind, types[kind], H, I, rank=rank // tp,
                                    world=world // tp, device=cuda_device, tensor_rank=rank % tp,
                                    tensor_parallel=tp)
            assert got[kind].shape == want.shape
            assert torch.equal(got[kind], want), (rank, world, kind)
