"""Safetensors checkpoints straight into HBM-resident matrices.

The reference reads expert weights from safetensors shards on demand and keeps a bounded LRU of
decoded experts (src/storage/safetensors.rs, src/storage/weight.rs:118-477, expert stores such
as src/models/glm/runtime/expert.rs:199-265).  Here every matrix is read once and uploaded to
the GPU, where it stays resident: the same file layouts and sidecar rules as
``inspect_weight_matrix`` (src/storage/weight.rs:118-310), without the cache.

Layouts recognised for a ``[rows, cols]`` matrix ``name``:

* plain F32 / F16 / BF16 ``[rows, cols]`` (no scale sidecar);
* MXFP4: packed E2M1 nibbles, low nibble = even column, ``[rows, ceil(cols/2)]`` as I8 with an
  F8_E8M0 sidecar, or as U8 ``<prefix>.weight_packed`` with a U8 sidecar; sidecar
  ``[rows, ceil(cols/32)]``;
* MXFP8: F8_E4M3 ``[rows, cols]`` with an E8M0 sidecar of ``[ceil(rows/32), ceil(cols/32)]``
  (32x32 blocks), ``[ceil(rows/128), ceil(cols/128)]`` (128x128 blocks) as F8_E8M0, or
  ``[rows, ceil(cols/32)]`` as U8 (ModelOpt 1x32).
Sidecar names: ``<prefix>.weight_scale`` when present for ``<prefix>.weight`` (ModelOpt), else
``<prefix>.weight_packed`` -> ``<prefix>.weight_scale`` and ``<prefix>.weight`` ->
``<prefix>.scale`` (src/storage/weight.rs:636-653).  More than one candidate sidecar is an
error, as in the reference.

Consolidated experts (Hy4 layout, src/models/hy4/expert.rs:436-560): ``<stem>.gate_up_proj``
F8_E4M3 ``[experts, 2 * inter, hidden]`` with U8 1x32 scales ``<stem>.gate_up_proj_scale``, and
``<stem>.down_proj`` ``[experts, hidden, inter]`` with ``<stem>.down_proj_scale``; gate is the
first ``inter`` rows of an expert's gate_up slice, up the rest.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import Bf16Matrix, DenseMatrix, GatedMlp, MxFp4Matrix, MxFp8Matrix

_ELEMENT_BYTES = {
    "BOOL": 1, "U8": 1, "I8": 1, "F8_E4M3": 1, "F8_E5M2": 1, "F8_E8M0": 1,
    "U16": 2, "I16": 2, "F16": 2, "BF16": 2,
    "U32": 4, "I32": 4, "F32": 4,
    "U64": 8, "I64": 8, "F64": 8,
}
_DTYPE_ALIASES = {"F8_E4M3FN": "F8_E4M3", "F8_E8M0FNU": "F8_E8M0"}  # safetensors.rs:223-242


class CheckpointError(Exception):
    """A checkpoint that does not hold the requested matrix in a supported layout.  ``kind``
    follows the reference's WeightLoadError / SafetensorError variants: "Missing",
    "InvalidShape", "Unsupported", "InvalidHeader"."""

    def __init__(self, kind: str, message: str):
        self.kind = kind
        super().__init__("%s: %s" % (kind, message))


@dataclass
class TensorInfo:
    name: str
    path: str
    dtype: str
    shape: Tuple[int, ...]
    begin: int          # absolute byte offset in the shard file
    data_len: int


class SafetensorIndex:
    """The tensors of a checkpoint directory: one ``*.safetensors`` file, or shards listed by
    ``model.safetensors.index.json`` (or every ``*.safetensors`` file in the directory)."""

    def __init__(self, model_dir: str):
        self.model_dir = model_dir
        index_json = os.path.join(model_dir, "model.safetensors.index.json")
        if os.path.exists(index_json):
            weight_map = json.load(open(index_json))["weight_map"]
            shards = sorted(set(weight_map.values()))
        else:
            shards = sorted(f for f in os.listdir(model_dir) if f.endswith(".safetensors"))
        if not shards:
            raise CheckpointError("Missing", "no safetensors shards in %r" % model_dir)
        self.tensors: Dict[str, TensorInfo] = {}
        for shard in shards:
            self._read_header(os.path.join(model_dir, shard))

    def _read_header(self, path: str):
        size = os.path.getsize(path)
        with open(path, "rb") as f:
            raw = f.read(8)
            if len(raw) != 8:
                raise CheckpointError("InvalidHeader", "%r is shorter than its header length" % path)
            n = struct.unpack("<Q", raw)[0]
            if n > size - 8:
                raise CheckpointError("InvalidHeader", "%r header length exceeds the file" % path)
            try:
                header = json.loads(f.read(n))
            except ValueError as e:
                raise CheckpointError("InvalidHeader", "%r header is not JSON: %s" % (path, e))
        start = 8 + n
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            dtype = _DTYPE_ALIASES.get(meta["dtype"], meta["dtype"])
            shape = tuple(int(d) for d in meta["shape"])
            b, e = (int(v) for v in meta["data_offsets"])
            if not (0 <= b <= e and start + e <= size):
                raise CheckpointError("InvalidHeader", "tensor %r lies outside %r" % (name, path))
            elem = _ELEMENT_BYTES.get(dtype)
            if elem is None:
                raise CheckpointError("Unsupported", "tensor %r has dtype %s" % (name, dtype))
            if int(np.prod(shape, dtype=np.int64)) * elem != e - b:
                raise CheckpointError("InvalidHeader",
                                      "tensor %r: %d bytes for shape %s" % (name, e - b, shape))
            if name in self.tensors:
                raise CheckpointError("InvalidHeader", "tensor %r appears in two shards" % name)
            self.tensors[name] = TensorInfo(name, path, dtype, shape, start + b, e - b)

    def get(self, name: str) -> Optional[TensorInfo]:
        return self.tensors.get(name)

    def require(self, name: str) -> TensorInfo:
        t = self.tensors.get(name)
        if t is None:
            raise CheckpointError("Missing", "tensor %r is not in the checkpoint" % name)
        return t

    def read(self, name: str, begin: int = 0, length: Optional[int] = None) -> np.ndarray:
        """Raw bytes of a tensor (or of a byte range inside it) as a read-only uint8 view."""
        t = self.require(name)
        length = t.data_len - begin if length is None else length
        if begin < 0 or begin + length > t.data_len:
            raise CheckpointError("InvalidShape", "byte range outside tensor %r" % name)
        return np.memmap(t.path, dtype=np.uint8, mode="r", offset=t.begin + begin, shape=(length,))


@dataclass
class WeightLayout:
    format: str            # "f32" | "f16" | "bf16" | "mxfp4" | "mxfp8"
    scale_name: Optional[str] = None
    block_rows: int = 1
    block_cols: int = 32


def _native_scale_name(name: str) -> str:
    if name.endswith(".weight_packed"):
        return name[: -len(".weight_packed")] + ".weight_scale"
    if name.endswith(".weight"):
        return name[: -len(".weight")] + ".scale"
    return name + ".scale"


def _find_native_scale_name(index: SafetensorIndex, name: str) -> str:
    if name.endswith(".weight"):
        modelopt = name[: -len(".weight")] + ".weight_scale"
        if index.get(modelopt) is not None:
            return modelopt
    return _native_scale_name(name)


def inspect_weight_matrix(index: SafetensorIndex, name: str, rows: int, cols: int) -> WeightLayout:
    """The layout of matrix ``name`` (src/storage/weight.rs:118-310, MX and plain formats)."""
    if rows <= 0 or cols <= 0:
        raise CheckpointError("InvalidShape", "rows and columns must be non-zero")
    t = index.require(name)
    mx_name = _find_native_scale_name(index, name)
    mx = index.get(mx_name)
    others = [n for n in (name + ".qs", name[:-len(".weight")] + ".weight_scale_inv"
                          if name.endswith(".weight") else name + "_scale_inv")
              if index.get(n) is not None]
    if mx is not None and others:
        raise CheckpointError("Unsupported", "tensor %r has conflicting scale sidecars: %s"
                              % (name, ", ".join([mx_name] + others)))
    if others:
        raise CheckpointError("Unsupported", "tensor %r: %s sidecars are not MX scales" % (name, others[0]))
    if t.dtype in ("F32", "F16", "BF16") and mx is None:
        if t.shape != (rows, cols):
            raise CheckpointError("InvalidShape", "plain tensor %r must be [%d,%d]" % (name, rows, cols))
        return WeightLayout(t.dtype.lower())
    if t.dtype == "F8_E4M3":
        if mx is None:
            raise CheckpointError("Unsupported", "MX tensor has no required E8M0 sidecar %r" % mx_name)
        shapes = {(-(-rows // 32), -(-cols // 32)): (32, 32, "F8_E8M0"),
                  (-(-rows // 128), -(-cols // 128)): (128, 128, "F8_E8M0"),
                  (rows, -(-cols // 32)): (1, 32, "U8")}
        for shape, (br, bc, dt) in shapes.items():
            if mx.shape == shape and mx.dtype == dt:
                if t.shape != (rows, cols):
                    raise CheckpointError("InvalidShape", "MXFP8 tensor %r must be [%d,%d]"
                                          % (name, rows, cols))
                return WeightLayout("mxfp8", mx_name, br, bc)
        raise CheckpointError("InvalidShape", "MXFP8 tensor %r: unsupported scale %s %s"
                              % (name, mx.dtype, mx.shape))
    native_mxfp4 = t.dtype == "I8" or (t.dtype == "U8" and name.endswith(".weight_packed"))
    if native_mxfp4 and mx is not None:
        want_dtype = "U8" if t.dtype == "U8" else "F8_E8M0"
        if (t.shape != (rows, -(-cols // 2)) or mx.dtype != want_dtype
                or mx.shape != (rows, -(-cols // 32))):
            raise CheckpointError("InvalidShape",
                                  "MXFP4 tensor %r needs packed weight [%d,%d] and %s E8M0 scale [%d,%d]"
                                  % (name, rows, -(-cols // 2), want_dtype, rows, -(-cols // 32)))
        return WeightLayout("mxfp4", mx_name, 1, 32)
    raise CheckpointError("Unsupported", "tensor %r has dtype %s without a supported sidecar"
                          % (name, t.dtype))


def load_weight_matrix(ctx, index: SafetensorIndex, name: str, rows: int, cols: int):
    """Reads matrix ``name`` and uploads it (validated: 0xFF scales are rejected on upload)."""
    lay = inspect_weight_matrix(index, name, rows, cols)
    data = np.asarray(index.read(name))
    if lay.format == "mxfp4":
        return MxFp4Matrix.from_packed(rows, cols, 32, data, np.asarray(index.read(lay.scale_name)),
                                       ctx=ctx)
    if lay.format == "mxfp8":
        return MxFp8Matrix.from_packed(rows, cols, lay.block_rows, lay.block_cols, data,
                                       np.asarray(index.read(lay.scale_name)), ctx=ctx)
    if lay.format == "bf16":
        return Bf16Matrix.from_bits(rows, cols, data.view(np.uint16), ctx=ctx)
    values = data.view(np.float16).astype(np.float32) if lay.format == "f16" else data.view(np.float32)
    return DenseMatrix.new(rows, cols, values, ctx=ctx)


def _rank3(index: SafetensorIndex, name: str, dtype: str, shape: Tuple[int, int, int]) -> TensorInfo:
    t = index.require(name)
    if t.dtype != dtype or t.shape != shape:
        raise CheckpointError("InvalidShape", "tensor %r is %s %s; expected %s %s"
                              % (name, t.dtype, list(t.shape), dtype, list(shape)))
    return t


def load_consolidated_mxfp8_expert(ctx, index: SafetensorIndex, stem: str, expert: int,
                                   experts: int, hidden: int, inter: int) -> GatedMlp:
    """One expert of a consolidated MXFP8 checkpoint (Hy4 layout): gate / up from the expert's
    slice of ``<stem>.gate_up_proj``, down from ``<stem>.down_proj``, 1x32 U8 E8M0 scales."""
    if not 0 <= expert < experts:
        raise CheckpointError("InvalidShape", "expert %d is outside 0..%d" % (expert, experts))
    sc_h, sc_i = -(-hidden // 32), -(-inter // 32)
    gu = _rank3(index, stem + ".gate_up_proj", "F8_E4M3", (experts, 2 * inter, hidden))
    _rank3(index, stem + ".gate_up_proj_scale", "U8", (experts, 2 * inter, sc_h))
    _rank3(index, stem + ".down_proj", "F8_E4M3", (experts, hidden, inter))
    _rank3(index, stem + ".down_proj_scale", "U8", (experts, hidden, sc_i))
    del gu
    vals = np.asarray(index.read(stem + ".gate_up_proj", expert * 2 * inter * hidden, 2 * inter * hidden))
    scl = np.asarray(index.read(stem + ".gate_up_proj_scale", expert * 2 * inter * sc_h, 2 * inter * sc_h))
    gate = MxFp8Matrix.from_packed(inter, hidden, 1, 32, vals[: inter * hidden], scl[: inter * sc_h], ctx=ctx)
    up = MxFp8Matrix.from_packed(inter, hidden, 1, 32, vals[inter * hidden:], scl[inter * sc_h:], ctx=ctx)
    dv = np.asarray(index.read(stem + ".down_proj", expert * hidden * inter, hidden * inter))
    ds = np.asarray(index.read(stem + ".down_proj_scale", expert * hidden * sc_i, hidden * sc_i))
    down = MxFp8Matrix.from_packed(hidden, inter, 1, 32, dv, ds, ctx=ctx)
    return GatedMlp(gate, up, down)


def write_safetensors(path: str, tensors: Dict[str, Tuple[str, Tuple[int, ...], np.ndarray]]):
    """Writes ``{name: (dtype, shape, array)}`` as one safetensors file (test fixtures and
    conversion tools)."""
    header, blobs, off = {}, [], 0
    for name, (dtype, shape, arr) in tensors.items():
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


__all__: List[str] = ["SafetensorIndex", "TensorInfo", "WeightLayout", "CheckpointError",
                      "inspect_weight_matrix", "load_weight_matrix",
                      "load_consolidated_mxfp8_expert", "write_safetensors"]
