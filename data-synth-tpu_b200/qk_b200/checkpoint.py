"""GGUF expert tensors from local files into device-resident tiled experts.

Mirrors the part of ``qwen38_tpu/checkpoint.py`` that feeds the routed FFN: the tensor table
(``Checkpoint.__init__`` / ``validate`` bounds, ``checkpoint.py:34-46,168-176``), byte-range
reads (``read``, ``:178-196``), ``packed_shape`` / ``packed`` (``:183-192``) and
``resident_experts`` (``:225-261``), which places one layer's ``ffn_{gate,up,down}_exps``
on the devices with the expert (and tensor) split of ``parallel.py:40-87``.

The tensor table comes from either the reference's audit JSON (``{"tensors": {name:
{"file", "data0", "offset", "nbytes", "dims", "type"}}, "files": [...]}``) with a local
directory holding the files, or straight from a GGUF file's header
(:meth:`Checkpoint.from_gguf`, the public GGUF v2/v3 container format). Only local files are
read: the reference's HTTP range reader and its pinned-revision check belong to its
download path, which is out of scope here.

Per rank, only that rank's experts are read (one contiguous byte range per matrix, into
pinned host memory), copied to the device and repacked there into the B200 tile layout
(``put_expert_bytes``), so host staging is bounded by one rank's share of one matrix, as
in the reference (``checkpoint.py:247-252``).
"""

import json
import os
import struct
from pathlib import Path

import numpy as np
import torch

from .parallel import put_expert_bytes
from .quant import BLOCK_LAYOUTS, GGML_TYPE, normalize_qtype

_GGUF_MAGIC = b"GGUF"
# GGUF metadata value types: fixed-size scalars as struct formats; 8 = string, 9 = array.
_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
_STRING, _ARRAY = 8, 9


class _Reader:
    def __init__(self, f):
        self.f = f

    def take(self, n):
        data = self.f.read(n)
        if len(data) != n:
            raise ValueError("Truncated GGUF header")
        return data

    def scalar(self, fmt):
        return struct.unpack("<" + fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self):
        return self.take(self.scalar("Q")).decode("utf-8")

    def value(self, vtype):
        if vtype in _SCALAR:
            return self.scalar(_SCALAR[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, count = self.scalar("I"), self.scalar("Q")
            return [self.value(etype) for _ in range(count)]
        raise ValueError(f"Unknown GGUF metadata type {vtype}")


def read_gguf_header(path):
    """``(metadata, tensors)`` of a GGUF file.

    ``tensors[name] = {"file", "data0", "offset", "nbytes", "dims", "type"}``: the entry
    form of the reference's audit table, with ``dims`` innermost first (GGUF order) and
    ``type`` the GGML type name. Tensors of block types this library does not decode are
    left out of the table and listed under ``metadata["qk_b200.unsupported_tensors"]``."""
    path = Path(path)
    with path.open("rb") as f:
        r = _Reader(f)
        if r.take(4) != _GGUF_MAGIC:
            raise ValueError(f"{path.name}: not a GGUF file")
        version = r.scalar("I")
        if version not in (2, 3):
            raise ValueError(f"{path.name}: unsupported GGUF version {version}")
        n_tensors, n_kv = r.scalar("Q"), r.scalar("Q")
        metadata = {}
        for _ in range(n_kv):
            key = r.string()
            metadata[key] = r.value(r.scalar("I"))
        infos = []
        for _ in range(n_tensors):
            name = r.string()
            dims = [r.scalar("Q") for _ in range(r.scalar("I"))]
            gtype, offset = r.scalar("I"), r.scalar("Q")
            infos.append((name, dims, gtype, offset))
        alignment = int(metadata.get("general.alignment", 32))
        end = f.tell()
    data0 = (end + alignment - 1) // alignment * alignment
    tensors, other = {}, {}
    for name, dims, gtype, offset in infos:
        try:
            qtype = normalize_qtype(gtype)
        except ValueError:  # a block type this library does not decode: listed, never read
            other[name] = dict(dims=list(dims), ggml_type=gtype, offset=offset)
            continue
        values, size = BLOCK_LAYOUTS[qtype]
        count = int(np.prod(dims, dtype=np.int64)) if dims else 1
        if dims and dims[0] % values:
            raise ValueError(f"{name}: GGUF rows do not divide into quant blocks")
        tensors[name] = dict(file=path.name, data0=data0, offset=offset,
                             nbytes=count // values * size, dims=list(dims), type=qtype)
    if other:
        metadata = dict(metadata, **{"qk_b200.unsupported_tensors": other})
    return metadata, tensors


class Checkpoint:
    """Audited access to local GGUF tensors (``qwen38_tpu/checkpoint.py:34``)."""

    def __init__(self, audit_path=None, local_dir=None, log=print, *, tensors=None, files=None):
        if tensors is None:
            if audit_path is None:
                raise ValueError("give an audit file or a tensor table")
            audit = json.loads(Path(audit_path).read_text())
            tensors = audit["tensors"]
            files = {f["file"]: int(f["file_bytes"]) for f in audit.get("files", [])}
        if local_dir is None:
            raise ValueError("a local directory holding the GGUF files is required")
        self.local_dir = Path(local_dir)
        self.tensors = tensors
        self.log = log
        self.files = dict(files or {})
        for t in tensors.values():
            if t["file"] not in self.files:
                self.files[t["file"]] = os.path.getsize(self.local_dir / t["file"])
        self.bytes_read = 0
        self.metadata = {}
        self._check_bounds()

    @classmethod
    def from_gguf(cls, path, log=print):
        """A checkpoint of one local GGUF file, its tensor table read from the header."""
        path = Path(path)
        metadata, tensors = read_gguf_header(path)
        ckpt = cls(local_dir=path.parent, log=log, tensors=tensors,
                   files={path.name: path.stat().st_size})
        ckpt.metadata = metadata
        return ckpt

    def _check_bounds(self):
        """The source-bound and size checks of ``checkpoint.py:168-176``."""
        for key, t in self.tensors.items():
            if (t["data0"] + t["offset"] + t["nbytes"] > self.files[t["file"]]
                    or min(t["data0"], t["offset"], t["nbytes"]) < 0):
                raise ValueError(f"Tensor outside source shard: {key}")
            values, size = BLOCK_LAYOUTS[normalize_qtype(t["type"])]
            width = t["dims"][0]
            if width % values or int(np.prod(t["dims"], dtype=np.int64)) // values * size != t["nbytes"]:
                raise ValueError(f"Invalid quantized tensor size: {key}")

    def _range(self, name, offset, length):
        t = self.tensors[name]
        length = t["nbytes"] - offset if length is None else length
        if offset < 0 or length < 0 or offset + length > t["nbytes"]:
            raise ValueError("Read outside tensor")
        return t, t["data0"] + t["offset"] + offset, length

    def read_into(self, name, out, offset=0):
        """Read ``len(out)`` bytes of tensor ``name`` from ``offset`` into the writable
        buffer ``out`` (a NumPy array or pinned host tensor's NumPy view) without a copy."""
        view = memoryview(out).cast("B")
        t, absolute, length = self._range(name, offset, len(view))
        fd = os.open(self.local_dir / t["file"], os.O_RDONLY)
        try:
            done = 0
            while done < length:  # preadv may return short counts on large ranges
                n = os.preadv(fd, [view[done:]], absolute + done)
                if n <= 0:
                    raise OSError("Truncated local tensor")
                done += n
        finally:
            os.close(fd)
        self.bytes_read += length
        return out

    def read(self, name, offset=0, length=None):
        """Bytes ``[offset, offset + length)`` of tensor ``name`` (``checkpoint.py:178``)."""
        _, _, length = self._range(name, offset, length)
        return self.read_into(name, np.empty(length, np.uint8), offset).tobytes()

    def packed_shape(self, name):
        """``(*outer dims reversed, blocks per row, bytes per block)`` (``checkpoint.py:183``)."""
        t = self.tensors[name]
        width, *others = t["dims"]
        values, size = BLOCK_LAYOUTS[normalize_qtype(t["type"])]
        if width % values:
            raise ValueError(f"{name}: GGUF rows do not divide into quant blocks")
        return tuple(reversed(others)) + (width // values, size)

    def packed(self, name):
        t = self.tensors[name]
        return self.read_into(name, np.empty(t["nbytes"], np.uint8)).reshape(self.packed_shape(name))

    def resident_experts(self, layer, group=None, *, tensor_parallel=1, device=None, rank=None,
                         world=None):
        """This rank's experts of layer ``layer``: ``{"gate"|"up"|"down": uint8[E_local,
        tiled bytes]}`` on ``device`` (``checkpoint.py:225-261``).

        Ranks of ``group`` (a ``torch.distributed`` group, or None for one device) form the
        reference's ("expert", "tensor") mesh: rank = e * tensor_parallel + t
        (``parallel.py:28-33``). Rank e·tp + t holds experts ``[e·E/ep, (e+1)·E/ep)``, cut
        to tensor slice t of the intermediate channels. The tensors feed
        ``expert_parallel(...)`` / ``ExpertAllToAll`` directly. ``rank``/``world`` stand in
        for a group (one process placing the share of a given rank)."""
        if group is not None:
            import torch.distributed as dist
            rank, world = dist.get_rank(group), dist.get_world_size(group)
        elif rank is None or world is None:
            rank, world = 0, 1
        if not 0 <= rank < world:
            raise ValueError("rank must lie in [0, world)")
        if world % tensor_parallel:
            raise ValueError("Expert group size must divide into tensor parallel size")
        ep, e_rank, t_rank = world // tensor_parallel, rank // tensor_parallel, rank % tensor_parallel
        device = torch.device(device or "cuda")
        result = {}
        for kind in ("gate", "up", "down"):
            name = f"blk.{layer}.ffn_{kind}_exps.weight"
            t = self.tensors[name]
            count = self.packed_shape(name)[0]
            if count % ep:
                raise ValueError("Expert count does not divide into expert groups")
            stride = t["nbytes"] // count
            dims = t["dims"]
            hidden, intermediate = (dims[1], dims[0]) if kind == "down" else (dims[0], dims[1])
            per = count // ep
            staging = torch.empty(per * stride, dtype=torch.uint8, pin_memory=True)
            self.read_into(name, staging.numpy(), e_rank * per * stride)
            result[kind] = put_expert_bytes(
                staging.view(per, stride), kind, t["type"], hidden, intermediate, device=device,
                tensor_rank=t_rank, tensor_parallel=tensor_parallel)
            self.log(f"expert_load layer={layer} matrix={kind} bytes={per * stride}")
        return result

    def expert_types(self, layer):
        """``(gate_type, up_type, down_type)`` of a layer, for ``expert_parallel``."""
        return tuple(normalize_qtype(self.tensors[f"blk.{layer}.ffn_{k}_exps.weight"]["type"])
                     for k in ("gate", "up", "down"))


__all__ = ["Checkpoint", "read_gguf_header", "GGML_TYPE"]
