"""urbilateria_b200 — B200-native routed-expert (MoE) hot path of Urbilateria.

The product is the C-ABI library liburb_moe.so (include/urb_moe.h; CUDA kernels for sm_100a).
This package is its Python host mirror: the class and method names, argument meaning and
error variants follow the reference's Rust API so that code written against
``MxFp4Matrix::matvec`` / ``GatedMlp::forward`` / ``route_noaux_tc`` /
``RuntimeMoeLayer::forward`` reads the same here.  Every call runs on the GPU; nothing falls
back to the CPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import native
from .native import MoeGeometry as _CGeometry

__all__ = [
    "UrbError", "MxError", "Context", "MxFp4Matrix", "MxFp8Matrix", "Bf16Matrix", "DenseMatrix",
    "GatedMlp", "RouteChoice", "MoeGeometry", "route_noaux_tc", "route_softmax_top_k",
    "group_routes", "RuntimeMoeLayer", "default_context", "simulate_e4m3_activation",
    "route_sqrt_softplus", "simulate_finegrained_e4m3_activation", "linear_bf16_fp32_lanes",
]


class UrbError(Exception):
    """A non-zero urb_status.  ``kind`` is the reference error variant name."""

    def __init__(self, code: int, message: str = ""):
        self.code = code
        self.kind = native.STATUS_NAMES.get(code, str(code))
        super().__init__("%s%s" % (self.kind, (": " + message) if message else ""))


MxError = UrbError  # MxError::{Shape, InvalidScale, NonFinite} map onto UrbError.kind


def _ptr(a: Optional[np.ndarray]) -> int:
    return 0 if a is None else a.ctypes.data


class Context:
    """One CUDA device and stream (urb_ctx)."""

    def __init__(self, device: int = 0):
        self.lib = native.load()
        h = ctypes.c_void_p()
        rc = self.lib.urb_ctx_create(device, ctypes.byref(h))
        if rc != native.OK:
            raise UrbError(rc, "urb_ctx_create(device=%d)" % device)
        self.h = h
        self.device = device

    def check(self, rc: int):
        if rc != native.OK:
            buf = ctypes.create_string_buffer(512)
            self.lib.urb_last_error(self.h, buf, 512)
            raise UrbError(rc, buf.value.decode(errors="replace"))

    def synchronize(self):
        self.check(self.lib.urb_ctx_synchronize(self.h))

    @property
    def stream(self) -> int:
        return self.lib.urb_ctx_stream(self.h) or 0

    def set_stream(self, stream: int):
        self.check(self.lib.urb_ctx_set_stream(self.h, ctypes.c_void_p(stream)))

    def close(self):
        if getattr(self, "h", None):
            self.lib.urb_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default = None


def default_context() -> Context:
    global _default
    if _default is None:
        _default = Context(0)
    return _default


class _Matrix:
    """Common WeightMatrix surface (src/model/weight.rs:69-320)."""

    fmt = -1

    def __init__(self, ctx: Context, handle: ctypes.c_void_p, rows: int, cols: int):
        self.ctx, self.h, self._rows, self._cols = ctx, handle, rows, cols

    def rows(self) -> int:
        return self._rows

    def cols(self) -> int:
        return self._cols

    def resident_bytes(self) -> int:
        v = ctypes.c_size_t()
        self.ctx.check(self.ctx.lib.urb_mat_info(self.h, None, None, None, ctypes.byref(v)))
        return v.value

    def transpose_rows_matvec(self, start: int, x) -> np.ndarray:
        """WeightMatrix::transpose_rows_matvec (src/model/weight.rs:332-343): rows
        start..start+len(x) of the matrix, transposed, times x -> [cols]."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        y = np.empty(self._cols, dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_transpose_rows_matvec(
            self.ctx.h, self.h, start, _ptr(x) if x.size else None, x.size, _ptr(y)))
        return y

    def transpose_matvec(self, x) -> np.ndarray:
        """WeightMatrix::transpose_matvec: all rows, transposed, times x [rows]."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        if x.size != self._rows:
            raise UrbError(native.ERR_SHAPE, "transpose input length %d != %d rows" % (x.size, self._rows))
        return self.transpose_rows_matvec(0, x)

    def write_rows(self, start: int, count: int) -> np.ndarray:
        """WeightMatrix::write_row for rows start..start+count -> [count, cols] f32."""
        out = np.empty((count, self._cols), dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_mat_write_rows(self.ctx.h, self.h, start, count,
                                                       _ptr(out) if count else None))
        return out

    def row(self, row: int) -> np.ndarray:
        """WeightMatrix::row (src/model/weight.rs:388-392): one decoded row."""
        return self.write_rows(row, 1)[0]

    def matvec_rows(self, start: int, count: int, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        y = np.empty(count, dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_matvec_rows(self.ctx.h, self.h, start, count, _ptr(x),
                                                    x.size, _ptr(y)))
        return y

    def matvec(self, x) -> np.ndarray:
        return self.matvec_rows(0, self._rows, x)

    def matmul_rows(self, x, batch: int) -> np.ndarray:
        """x [batch, cols] (flat or 2-D) -> [batch, rows] token-major."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        y = np.empty((batch, self._rows), dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_matmul_rows(self.ctx.h, self.h, _ptr(x), batch, x.size,
                                                    _ptr(y)))
        return y

    def matmul_row_range(self, start: int, count: int, x, batch: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        y = np.empty((batch, count), dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_matmul_row_range(self.ctx.h, self.h, start, count,
                                                         _ptr(x), batch, x.size, _ptr(y)))
        return y

    def matmul_rows_fp32_accum(self, x, batch: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        y = np.empty((batch, self._rows), dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_matmul_rows_fp32_accum(self.ctx.h, self.h, _ptr(x),
                                                               batch, x.size, _ptr(y)))
        return y

    def matvec_fp32_accum(self, x) -> np.ndarray:
        return self.matmul_rows_fp32_accum(x, 1)[0]

    def matmul_rows_device(self, d_x: int, batch: int, d_y: int, d_status: int = 0):
        """Device pointers (e.g. torch tensor.data_ptr()); stream-ordered, no host sync."""
        self.ctx.check(self.ctx.lib.urb_matmul_rows_device(self.ctx.h, self.h, d_x, batch, d_y,
                                                           d_status or None))

    def free(self):
        # A closed context has already ended every call on its objects; freeing through it
        # would touch released state, so the handle is dropped instead.
        if self.h and self.ctx.h:
            self.ctx.lib.urb_mat_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class MxFp4Matrix(_Matrix):
    """MxFp4Matrix (src/math/mxfp.rs:1363-1847), resident in HBM."""

    fmt = native.FMT_MXFP4

    @classmethod
    def from_packed(cls, rows: int, cols: int, group_size: int, packed, scale_bytes,
                    ctx: Optional[Context] = None):
        ctx = ctx or default_context()
        packed = np.ascontiguousarray(packed, dtype=np.uint8).ravel()
        scales = np.ascontiguousarray(scale_bytes, dtype=np.uint8).ravel()
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.urb_mxfp4_upload(ctx.h, rows, cols, group_size, _ptr(packed),
                                           packed.size, _ptr(scales), scales.size,
                                           ctypes.byref(h)))
        return cls(ctx, h, rows, cols)


    @classmethod
    def from_device(cls, rows: int, cols: int, group_size: int, d_packed: int, packed_len: int,
                    d_scales: int, scales_len: int, ctx: Optional[Context] = None):
        """from_packed with the packed nibbles and scale bytes already in device memory (device
        pointers; urb_mxfp4_upload accepts host or device memory).  The source buffers may be
        released once this returns."""
        ctx = ctx or default_context()
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.urb_mxfp4_upload(ctx.h, rows, cols, group_size, ctypes.c_void_p(d_packed),
                                           packed_len, ctypes.c_void_p(d_scales), scales_len,
                                           ctypes.byref(h)))
        return cls(ctx, h, rows, cols)


class MxFp8Matrix(_Matrix):
    """MxFp8Matrix with E8M0 block scales (src/math/mxfp.rs:321-877), resident in HBM."""

    fmt = native.FMT_MXFP8

    @classmethod
    def from_packed(cls, rows: int, cols: int, block_rows: int, block_cols: int, values,
                    scale_bytes, ctx: Optional[Context] = None):
        ctx = ctx or default_context()
        values = np.ascontiguousarray(values, dtype=np.uint8).ravel()
        scales = np.ascontiguousarray(scale_bytes, dtype=np.uint8).ravel()
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.urb_mxfp8_upload(ctx.h, rows, cols, block_rows, block_cols,
                                           _ptr(values), values.size, _ptr(scales), scales.size,
                                           ctypes.byref(h)))
        return cls(ctx, h, rows, cols)


class Bf16Matrix(_Matrix):
    """Bf16Matrix (src/model/bf16.rs): bf16 bit patterns as uint16, row-major."""

    fmt = native.FMT_BF16

    @classmethod
    def from_bits(cls, rows: int, cols: int, bits, ctx: Optional[Context] = None):
        ctx = ctx or default_context()
        bits = np.ascontiguousarray(bits, dtype=np.uint16).ravel()
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.urb_bf16_upload(ctx.h, rows, cols, _ptr(bits), bits.size,
                                          ctypes.byref(h)))
        return cls(ctx, h, rows, cols)


class DenseMatrix(_Matrix):
    """DenseMatrix (src/model/matrix.rs), f32 row-major."""

    fmt = native.FMT_F32

    @classmethod
    def new(cls, rows: int, cols: int, data, ctx: Optional[Context] = None):
        ctx = ctx or default_context()
        data = np.ascontiguousarray(data, dtype=np.float32).ravel()
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.urb_f32_upload(ctx.h, rows, cols, _ptr(data), data.size,
                                         ctypes.byref(h)))
        return cls(ctx, h, rows, cols)


class Int8Matrix(_Matrix):
    """Int8Matrix (src/math/quant.rs:355-573): two's-complement bytes [rows, cols] with one f32
    scale per row (WeightMatrix::Int8PerRow), resident in HBM."""

    fmt = native.FMT_INT8

    @classmethod
    def from_packed(cls, rows: int, cols: int, data, scales, ctx: Optional[Context] = None):
        ctx = ctx or default_context()
        data = np.ascontiguousarray(data).view(np.uint8).ravel()
        scales = np.ascontiguousarray(scales, dtype=np.float32).ravel()
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.urb_int8_upload(ctx.h, rows, cols, _ptr(data), data.size, _ptr(scales),
                                          scales.size, ctypes.byref(h)))
        return cls(ctx, h, rows, cols)


class Int4Matrix(_Matrix):
    """Int4Matrix (src/math/quant.rs:28-350): low-nibble-first codes (value code - 8) with f32
    scales per group of `group_size` columns (WeightMatrix::Int4), resident in HBM."""

    fmt = native.FMT_INT4

    def __init__(self, ctx: Context, handle: ctypes.c_void_p, rows: int, cols: int,
                 group_size: int = 0):
        super().__init__(ctx, handle, rows, cols)
        self._group = group_size or cols

    def group_size(self) -> int:
        return self._group

    @classmethod
    def from_packed(cls, rows: int, cols: int, group_size: int, packed, scales,
                    ctx: Optional[Context] = None):
        ctx = ctx or default_context()
        packed = np.ascontiguousarray(packed, dtype=np.uint8).ravel()
        scales = np.ascontiguousarray(scales, dtype=np.float32).ravel()
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.urb_int4_upload(ctx.h, rows, cols, group_size, _ptr(packed), packed.size,
                                          _ptr(scales), scales.size, ctypes.byref(h)))
        return cls(ctx, h, rows, cols, group_size)

    @classmethod
    def quantize_grouped(cls, rows: int, cols: int, group_size: int, values,
                         ctx: Optional[Context] = None):
        """Int4Matrix::quantize_grouped (quant.rs:46-90), computed on the device."""
        ctx = ctx or default_context()
        values = np.ascontiguousarray(values, dtype=np.float32).ravel()
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.urb_int4_quantize_grouped(ctx.h, rows, cols, group_size, _ptr(values),
                                                    values.size, ctypes.byref(h)))
        return cls(ctx, h, rows, cols, group_size)

    @classmethod
    def quantize_per_row(cls, rows: int, cols: int, values, ctx: Optional[Context] = None):
        """Int4Matrix::quantize_per_row (quant.rs:42-44): one group per row."""
        return cls.quantize_grouped(rows, cols, cols, values, ctx)

    def packed(self) -> np.ndarray:
        p = np.empty(self._rows * ((self._cols + 1) // 2), dtype=np.uint8)
        s = np.empty(self._rows * ((self._cols + self._group - 1) // self._group), dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_int4_payload(self.ctx.h, self.h, _ptr(p), _ptr(s)))
        self._scales_cache = s
        return p

    def scales(self) -> np.ndarray:
        self.packed()
        return self._scales_cache


class GatedMlp:
    """GatedMlp (src/model/mlp.rs:38-99): down(silu(gate x) * (up x))."""

    def __init__(self, gate: _Matrix, up: _Matrix, down: _Matrix):
        if gate.rows() != up.rows() or gate.cols() != up.cols():
            raise UrbError(native.ERR_SHAPE, "gate and up shapes differ")
        if down.cols() != gate.rows() or down.rows() != gate.cols():
            raise UrbError(native.ERR_SHAPE, "down must map intermediate back to hidden")
        self.gate, self.up, self.down = gate, up, down
        self.ctx = gate.ctx

    def hidden_size(self) -> int:
        return self.gate.cols()

    def intermediate_size(self) -> int:
        return self.gate.rows()

    def resident_bytes(self) -> int:
        return self.gate.resident_bytes() + self.up.resident_bytes() + self.down.resident_bytes()

    def forward_batch(self, x, tokens: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.empty((tokens, self.hidden_size()), dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_gated_mlp_forward(self.ctx.h, self.gate.h, self.up.h,
                                                          self.down.h, _ptr(x), tokens,
                                                          _ptr(out)))
        return out

    def forward(self, x) -> np.ndarray:
        return self.forward_batch(x, 1)[0]


@dataclass
class RouteChoice:
    """RouteChoice (src/math/routing.rs:8-15)."""
    expert: int
    weight: float
    selection_score: float


@dataclass
class MoeGeometry:
    top_k: int = 8
    n_group: int = 1
    topk_group: int = 1
    normalize: bool = True
    routed_scaling_factor: float = 1.0

    def c(self) -> _CGeometry:
        return _CGeometry(self.top_k, self.n_group, self.topk_group, int(self.normalize),
                          self.routed_scaling_factor)


def route_noaux_tc(logits, correction_bias, top_k: int, n_group: int, topk_group: int,
                   normalize: bool, routed_scaling_factor: float,
                   ctx: Optional[Context] = None):
    """route_noaux_tc (src/math/routing.rs:38-155).  1-D logits -> List[RouteChoice];
    2-D [tokens, experts] -> (experts, weights, scores) arrays [tokens, top_k]."""
    ctx = ctx or default_context()
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    single = lg.ndim == 1
    lg2 = lg.reshape(1, -1) if single else lg
    bias = np.ascontiguousarray(correction_bias, dtype=np.float32).ravel()
    t, e = lg2.shape
    if bias.size != e:
        raise UrbError(native.ERR_SHAPE, "%d logits but %d bias values" % (e, bias.size))
    geo = MoeGeometry(top_k, n_group, topk_group, normalize, routed_scaling_factor).c()
    k = max(top_k, 1)
    ids = np.empty((t, k), dtype=np.int32)
    w = np.empty((t, k), dtype=np.float32)
    s = np.empty((t, k), dtype=np.float32)
    ctx.check(ctx.lib.urb_route_noaux_tc(ctx.h, _ptr(lg2), _ptr(bias), t, e, ctypes.byref(geo),
                                         _ptr(ids), _ptr(w), _ptr(s)))
    if single:
        return [RouteChoice(int(ids[0, i]), float(w[0, i]), float(s[0, i])) for i in range(top_k)]
    return ids, w, s


def route_softmax_top_k(logits, top_k: int, ctx: Optional[Context] = None):
    """route_softmax_top_k (src/models/qwen3_8/moe.rs:91-159)."""
    ctx = ctx or default_context()
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    single = lg.ndim == 1
    lg2 = lg.reshape(1, -1) if single else lg
    t, e = lg2.shape
    ids = np.empty((t, max(top_k, 1)), dtype=np.int32)
    w = np.empty((t, max(top_k, 1)), dtype=np.float32)
    ctx.check(ctx.lib.urb_route_softmax_top_k(ctx.h, _ptr(lg2), t, e, top_k, _ptr(ids),
                                              _ptr(w)))
    if single:
        return [(int(ids[0, i]), float(w[0, i])) for i in range(top_k)]
    return ids, w


def route_sqrt_softplus(logits, correction_bias, hash_experts, top_k: int,
                        routed_scaling_factor: float, ctx: Optional[Context] = None):
    """route_sqrt_softplus (src/models/deepseek_v4/math.rs:451-516) on the device for one or
    more rows of logits: (expert ids, weights, selection scores) [tokens, top_k]."""
    ctx = ctx or default_context()
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    if lg.ndim == 1:
        lg = lg[None, :]
    t, e = lg.shape
    b = None if correction_bias is None else np.ascontiguousarray(correction_bias, dtype=np.float32)
    h = None if hash_experts is None else np.ascontiguousarray(hash_experts, dtype=np.int32)
    ids = np.empty((t, top_k), dtype=np.int32)
    w = np.empty((t, top_k), dtype=np.float32)
    s = np.empty((t, top_k), dtype=np.float32)
    ctx.check(ctx.lib.urb_route_sqrt_softplus(ctx.h, _ptr(lg), _ptr(b), t, e, _ptr(h), top_k,
                                              routed_scaling_factor, _ptr(ids), _ptr(w), _ptr(s)))
    return ids, w, s


def simulate_e4m3_activation(values, block_size: int, ctx: Optional[Context] = None) -> np.ndarray:
    """simulate_e4m3_activation (src/math/mxfp.rs:82-115) on the device."""
    ctx = ctx or default_context()
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    out = np.empty_like(v)
    ctx.check(ctx.lib.urb_simulate_e4m3_activation(ctx.h, _ptr(v) if v.size else None, v.size,
                                                   block_size, _ptr(out) if v.size else None))
    return out


def simulate_finegrained_e4m3_activation(values, block_size: int,
                                         ctx: Optional[Context] = None) -> np.ndarray:
    """simulate_finegrained_e4m3_activation (src/math/mxfp.rs:122-149) on the device."""
    ctx = ctx or default_context()
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    out = np.empty_like(v)
    ctx.check(ctx.lib.urb_simulate_finegrained_e4m3_activation(
        ctx.h, _ptr(v) if v.size else None, v.size, block_size, _ptr(out) if v.size else None))
    return out


def linear_bf16_fp32_lanes(matrix: "Bf16Matrix", x, tokens: int) -> np.ndarray:
    """The Qwen3.6 BF16 linear (qwen3_8/math.rs:10-26, dot_bf16_fp32_avx2_fma of
    src/model/bf16.rs:591-613, rounded to BF16) of x [tokens, cols]: [tokens, rows]."""
    ctx = matrix.ctx
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty((tokens, matrix.rows()), dtype=np.float32)
    ctx.check(ctx.lib.urb_linear_bf16_fp32_lanes(ctx.h, matrix.h, _ptr(x), tokens, _ptr(out)))
    return out


def group_routes(expert_ids, experts: int, ctx: Optional[Context] = None):
    """Ragged grouping (src/models/qwen3_6/runtime.rs:1083-1132): experts ascending, tokens
    ascending.  Returns (counts, offsets, perm_token, perm_slot)."""
    ctx = ctx or default_context()
    ids = np.ascontiguousarray(expert_ids, dtype=np.int32)
    t, k = ids.shape
    counts = np.empty(experts, dtype=np.int32)
    offsets = np.empty(experts + 1, dtype=np.int32)
    pt = np.empty(max(t * k, 1), dtype=np.int32)
    ps = np.empty(max(t * k, 1), dtype=np.int32)
    ctx.check(ctx.lib.urb_group_routes(ctx.h, _ptr(ids), t, k, experts, _ptr(counts),
                                       _ptr(offsets), _ptr(pt), _ptr(ps)))
    return counts, offsets, pt[:t * k], ps[:t * k]


_NUMERICS = {"glm": native.NUMERICS_GLM, "deepseek_v4": native.NUMERICS_DEEPSEEK_V4,
             "qwen36": native.NUMERICS_QWEN36}


class RuntimeMoeLayer:
    """RuntimeMoeLayer (src/models/glm/runtime/moe.rs:73-176), all experts resident in HBM.

    With ``expert_range=(begin, count)`` the layer is one expert-parallel shard: ``experts``
    holds the ``count`` experts starting at ``begin`` (router and bias still cover all
    experts), and it runs through :class:`urbilateria_b200.expert_parallel.ExpertParallelMoeLayer`.
    """

    def __init__(self, router: _Matrix, correction_bias, experts: Sequence[GatedMlp],
                 shared: Optional[GatedMlp], geometry: MoeGeometry,
                 expert_range: Optional[Tuple[int, int]] = None):
        self.ctx = router.ctx
        self.router = router
        self.bias = np.ascontiguousarray(correction_bias, dtype=np.float32).ravel()
        self.experts = list(experts)
        self.shared = shared
        self.geometry = geometry
        n = len(self.experts)
        arr = lambda ms: (ctypes.c_void_p * n)(*[m.h.value for m in ms])
        self._g = arr([e.gate for e in self.experts])
        self._u = arr([e.up for e in self.experts])
        self._d = arr([e.down for e in self.experts])
        self._geo = geometry.c()
        h = ctypes.c_void_p()
        sg = shared.gate.h if shared else None
        su = shared.up.h if shared else None
        sd = shared.down.h if shared else None
        self.expert_range = (0, n) if expert_range is None else tuple(expert_range)
        if expert_range is None:
            self.ctx.check(self.ctx.lib.urb_moe_layer_create(
                self.ctx.h, router.h, _ptr(self.bias), n, self._g, self._u, self._d, sg, su, sd,
                ctypes.byref(self._geo), ctypes.byref(h)))
        else:
            begin, count = self.expert_range
            if count != n:
                raise UrbError(native.ERR_SHAPE, "expert_range count %d != %d experts given" % (count, n))
            self.ctx.check(self.ctx.lib.urb_moe_layer_create_sharded(
                self.ctx.h, router.h, _ptr(self.bias), self.bias.size, begin, count, self._g,
                self._u, self._d, sg, su, sd, ctypes.byref(self._geo), ctypes.byref(h)))
        self.h = h

    def set_shared_expert_gate(self, gate: Optional[_Matrix]) -> None:
        """Attach the Qwen3.6 shared_expert_gate, a [1, hidden] BF16 matrix (kept alive by the
        layer), or detach it with None."""
        self.ctx.check(self.ctx.lib.urb_moe_layer_set_shared_expert_gate(
            self.ctx.h, self.h, gate.h if gate is not None else None))
        self._shared_expert_gate = gate

    def hidden_size(self) -> int:
        return self.router.cols()

    def expert_count(self) -> int:
        return self.router.rows()

    def forward_batch(self, x, tokens: int, details: bool = False):
        """x [tokens, hidden] -> (out [tokens, hidden], expert ids, weights[, extras])."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        H, E, K = self.hidden_size(), self.expert_count(), self.geometry.top_k
        out = np.empty((tokens, H), dtype=np.float32)
        ids = np.empty((tokens, K), dtype=np.int32)
        w = np.empty((tokens, K), dtype=np.float32)
        s = np.empty((tokens, K), dtype=np.float32)
        extra = {}
        logits = counts = pt = ps = None
        if details:
            logits = np.empty((tokens, E), dtype=np.float32)
            counts = np.empty(E, dtype=np.int32)
            pt = np.empty(tokens * K, dtype=np.int32)
            ps = np.empty(tokens * K, dtype=np.int32)
            extra = dict(router_logits=logits, counts=counts, perm_token=pt, perm_slot=ps)
        self.ctx.check(self.ctx.lib.urb_moe_forward(
            self.ctx.h, self.h, _ptr(x), tokens, _ptr(out), _ptr(ids), _ptr(w), _ptr(s),
            _ptr(logits), _ptr(counts), _ptr(pt), _ptr(ps)))
        extra["selection_score"] = s
        return out, ids, w, extra

    def forward_routed(self, x, tokens: int, expert_ids, weights, numerics: str = "glm",
                       swiglu_limit: float = 0.0) -> np.ndarray:
        """Experts half of the forward for caller-chosen routes ([tokens, top_k] ids and
        weights, e.g. from route_softmax_top_k): grouped SwiGLU experts + combine.  numerics
        "glm" (f64 combine in route order), "deepseek_v4" or "qwen36" (urb_moe_numerics)."""
        K = self.geometry.top_k
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        ids = np.ascontiguousarray(expert_ids, dtype=np.int32).reshape(tokens, K)
        w = np.ascontiguousarray(weights, dtype=np.float32).reshape(tokens, K)
        out = np.empty((tokens, self.hidden_size()), dtype=np.float32)
        num = native.Numerics(_NUMERICS[numerics], swiglu_limit)
        self.ctx.check(self.ctx.lib.urb_moe_forward_routed_ex(
            self.ctx.h, self.h, _ptr(x), tokens, _ptr(ids), _ptr(w), ctypes.byref(num),
            _ptr(out)))
        return out

    def forward_ex(self, x, tokens: int, numerics: str = "glm", swiglu_limit: float = 0.0,
                   hash_experts=None):
        """The layer forward with checkpoint numerics (urb_moe_forward_ex): "glm",
        "deepseek_v4" (route_sqrt_softplus routing, or fixed `hash_experts` [tokens, top_k],
        and the DeepSeek-V4 expert numerics) or "qwen36" (BF16 router, softmax top-k with
        BF16 weights, the Qwen3.6 expert numerics and the gated shared expert).  Returns (out,
        expert ids, weights)."""
        K = self.geometry.top_k
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.empty((tokens, self.hidden_size()), dtype=np.float32)
        ids = np.empty((tokens, K), dtype=np.int32)
        w = np.empty((tokens, K), dtype=np.float32)
        h = None if hash_experts is None else np.ascontiguousarray(hash_experts, dtype=np.int32)
        num = native.Numerics(_NUMERICS[numerics], swiglu_limit)
        self.ctx.check(self.ctx.lib.urb_moe_forward_ex(
            self.ctx.h, self.h, _ptr(x), tokens, ctypes.byref(num), _ptr(h), _ptr(out), _ptr(ids),
            _ptr(w)))
        return out, ids, w

    def forward(self, x):
        """Single token: (Vec<f32>, Vec<RouteChoice>) as in the reference."""
        out, ids, w, extra = self.forward_batch(x, 1)
        s = extra["selection_score"]
        routes = [RouteChoice(int(ids[0, i]), float(w[0, i]), float(s[0, i]))
                  for i in range(self.geometry.top_k)]
        return out[0], routes

    def forward_device(self, d_x: int, tokens: int, d_out: int, d_ids: int = 0, d_w: int = 0,
                       d_status: int = 0):
        self.ctx.check(self.ctx.lib.urb_moe_forward_device(
            self.ctx.h, self.h, d_x, tokens, d_out, d_ids or None, d_w or None,
            d_status or None))

    def free(self):
        if getattr(self, "h", None) and self.ctx.h:  # see Matrix.free
            self.ctx.lib.urb_moe_layer_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
