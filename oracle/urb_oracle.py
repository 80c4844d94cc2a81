"""ctypes wrapper of the CPU oracle (oracle/liburb_oracle.so).

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
import this module to check or time the CUDA path.  The product package ``urbilateria_b200``
never imports it.  The C++ it wraps restates Urbilateria v0.2.4's CPU arithmetic
(src/math/mxfp.rs, src/model/bf16.rs, src/math/routing.rs, src/model/mlp.rs,
src/models/glm/runtime/moe.rs, src/models/qwen3_6/runtime.rs); see urb_oracle.h.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liburb_oracle.so")

F32, BF16, MXFP8, MXFP4, INT8, INT4 = 0, 1, 2, 3, 4, 5
OK, ERR_SHAPE, ERR_INVALID_SCALE, ERR_NONFINITE, ERR_INVALID_GEOMETRY = 0, 1, 2, 3, 4
ERR_INVALID_GROUP = 11


class OracleMatrix(ctypes.Structure):
    _fields_ = [
        ("format", ctypes.c_int32),
        ("rows", ctypes.c_size_t),
        ("cols", ctypes.c_size_t),
        ("group_size", ctypes.c_size_t),
        ("block_rows", ctypes.c_size_t),
        ("block_cols", ctypes.c_size_t),
        ("values", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("fscales", ctypes.c_void_p),
    ]


class OracleMoeLayer(ctypes.Structure):
    _fields_ = [
        ("router", ctypes.POINTER(OracleMatrix)),
        ("bias", ctypes.c_void_p),
        ("experts", ctypes.c_size_t),
        ("gate", ctypes.POINTER(OracleMatrix)),
        ("up", ctypes.POINTER(OracleMatrix)),
        ("down", ctypes.POINTER(OracleMatrix)),
        ("shared_gate", ctypes.POINTER(OracleMatrix)),
        ("shared_up", ctypes.POINTER(OracleMatrix)),
        ("shared_down", ctypes.POINTER(OracleMatrix)),
        ("top_k", ctypes.c_size_t),
        ("n_group", ctypes.c_size_t),
        ("topk_group", ctypes.c_size_t),
        ("normalize", ctypes.c_int),
        ("routed_scaling_factor", ctypes.c_float),
    ]


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.urbo_decode_e8m0.restype = ctypes.c_float
        _lib.urbo_decode_e4m3fn.restype = ctypes.c_float
        _lib.urbo_decode_e2m1.restype = ctypes.c_float
        _lib.urbo_encode_e4m3fn.restype = ctypes.c_uint8
        _lib.urbo_encode_e4m3fn.argtypes = [ctypes.c_float]
        _lib.urbo_expf.restype = ctypes.c_float
        _lib.urbo_expf.argtypes = [ctypes.c_float]
        _lib.urbo_silu.restype = ctypes.c_float
        _lib.urbo_silu.argtypes = [ctypes.c_float]
        _lib.urbo_route_noaux_tc.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
            ctypes.c_size_t, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p]
        _lib.urbo_route_softmax_top_k.argtypes = [
            ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
        _lib.urbo_matvec_rows.argtypes = [
            ctypes.POINTER(OracleMatrix), ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_int]
        _lib.urbo_mxfp4_matvec_rows_fp32.argtypes = _lib.urbo_matvec_rows.argtypes
        _lib.urbo_transpose_rows_matvec.argtypes = [
            ctypes.POINTER(OracleMatrix), ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
            ctypes.c_void_p]
        _lib.urbo_matmul_rows.argtypes = [
            ctypes.POINTER(OracleMatrix), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
            ctypes.c_int]
        _lib.urbo_validate.argtypes = [ctypes.POINTER(OracleMatrix)]
        _lib.urbo_int4_quantize_grouped.argtypes = [
            ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p]
        _lib.urbo_write_row.argtypes = [ctypes.POINTER(OracleMatrix), ctypes.c_size_t,
                                        ctypes.c_void_p]
        _lib.urbo_gated_mlp_forward.argtypes = [
            ctypes.POINTER(OracleMatrix), ctypes.POINTER(OracleMatrix),
            ctypes.POINTER(OracleMatrix), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        _lib.urbo_group_routes.argtypes = [
            ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib.urbo_moe_layer_forward.argtypes = [
            ctypes.POINTER(OracleMoeLayer), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        _lib.urbo_power_of_two_ceiling.restype = ctypes.c_float
        _lib.urbo_power_of_two_ceiling.argtypes = [ctypes.c_float]
        _lib.urbo_simulate_e4m3_activation.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                                       ctypes.c_size_t]
        _lib.urbo_round_bf16.restype = ctypes.c_float
        _lib.urbo_round_bf16.argtypes = [ctypes.c_float]
        _lib.urbo_bounded_swiglu.restype = ctypes.c_float
        _lib.urbo_bounded_swiglu.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float]
        _lib.urbo_route_sqrt_softplus.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
            ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib.urbo_moe_deepseek_layer_forward.argtypes = [
            ctypes.POINTER(OracleMoeLayer), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
            ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        _lib.urbo_dot_bf16_fp32_lanes.restype = ctypes.c_float
        _lib.urbo_dot_bf16_fp32_lanes.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        _lib.urbo_simulate_finegrained_e4m3.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                                        ctypes.c_size_t]
        _lib.urbo_moe_qwen_layer_forward.argtypes = [
            ctypes.POINTER(OracleMoeLayer), ctypes.POINTER(OracleMatrix), ctypes.c_void_p,
            ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        _lib.urbo_deepseek_expert_forward.argtypes = [
            ctypes.POINTER(OracleMatrix), ctypes.POINTER(OracleMatrix), ctypes.POINTER(OracleMatrix),
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p,
            ctypes.c_int]
        _lib.urbo_moe_deepseek_forward.argtypes = [
            ctypes.POINTER(OracleMoeLayer), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p, ctypes.c_int]
    return _lib


def default_threads() -> int:
    return max(1, os.cpu_count() or 1)


class OracleError(Exception):
    def __init__(self, code: int):
        super().__init__({1: "Shape", 2: "InvalidScale", 3: "NonFinite",
                          4: "InvalidGeometry"}.get(code, str(code)))
        self.code = code


def _check(rc: int):
    if rc != OK:
        raise OracleError(rc)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Matrix:
    """One reference WeightMatrix held as numpy arrays (keeps the buffers alive)."""

    def __init__(self, fmt, rows, cols, values, scales=None, group_size=32, block_rows=1,
                 block_cols=32, validate=True):
        self.fmt, self.rows, self.cols = fmt, rows, cols
        self.values = np.ascontiguousarray(values)
        # MX formats carry E8M0 scale bytes; Int8Matrix / Int4Matrix carry f32 scales.
        sdt = np.float32 if fmt in (INT8, INT4) else np.uint8
        self.scales = None if scales is None else np.ascontiguousarray(scales, dtype=sdt)
        self.group_size, self.block_rows, self.block_cols = group_size, block_rows, block_cols
        sp = 0 if self.scales is None else _ptr(self.scales)
        self.c = OracleMatrix(fmt, rows, cols, group_size, block_rows, block_cols,
                              _ptr(self.values), 0 if fmt in (INT8, INT4) else sp,
                              sp if fmt in (INT8, INT4) else 0)
        if validate:
            _check(lib().urbo_validate(ctypes.byref(self.c)))

    # WeightMatrix::matvec_rows
    def matvec_rows(self, start, count, x, threads=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.size != self.cols:
            raise OracleError(ERR_SHAPE)
        y = np.empty(count, dtype=np.float32)
        _check(lib().urbo_matvec_rows(ctypes.byref(self.c), start, count, _ptr(x), _ptr(y),
                                      threads or default_threads()))
        return y

    def matvec(self, x, threads=None):
        return self.matvec_rows(0, self.rows, x, threads)

    def transpose_rows_matvec(self, start, x):
        """WeightMatrix::transpose_rows_matvec (src/model/weight.rs:332-343): rows
        start..start+len(x) transposed times x -> [cols]."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        y = np.empty(self.cols, dtype=np.float32)
        _check(lib().urbo_transpose_rows_matvec(ctypes.byref(self.c), start, _ptr(x), x.size,
                                                _ptr(y)))
        return y

    def write_row(self, row):
        """WeightMatrix::write_row (src/model/weight.rs:347-392): one decoded f32 row."""
        y = np.empty(self.cols, dtype=np.float32)
        _check(lib().urbo_write_row(ctypes.byref(self.c), row, _ptr(y)))
        return y

    def matvec_fp32(self, x, start=0, count=None, threads=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        count = self.rows if count is None else count
        y = np.empty(count, dtype=np.float32)
        _check(lib().urbo_mxfp4_matvec_rows_fp32(ctypes.byref(self.c), start, count, _ptr(x),
                                                 _ptr(y), threads or default_threads()))
        return y

    # WeightMatrix::matmul_rows: x [batch, cols] -> [batch, rows]
    def matmul_rows(self, x, batch, threads=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.size != batch * self.cols:
            raise OracleError(ERR_SHAPE)
        y = np.empty((batch, self.rows), dtype=np.float32)
        _check(lib().urbo_matmul_rows(ctypes.byref(self.c), _ptr(x), batch, _ptr(y),
                                      threads or default_threads()))
        return y


def int4_quantize_grouped(rows, cols, group_size, values):
    """Int4Matrix::quantize_grouped (src/math/quant.rs:46-90) -> (packed u8, scales f32)."""
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    if v.size != rows * cols:
        raise OracleError(ERR_SHAPE)
    packed = np.empty(rows * ((cols + 1) // 2), dtype=np.uint8)
    scales = np.empty(rows * ((cols + group_size - 1) // group_size if group_size else 1),
                      dtype=np.float32)
    _check(lib().urbo_int4_quantize_grouped(rows, cols, group_size, _ptr(v), _ptr(packed),
                                            _ptr(scales)))
    return packed, scales


def route_noaux_tc(logits, bias, top_k, n_group=1, topk_group=1, normalize=True, scaling=1.0):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    e = np.empty(top_k, dtype=np.int32)
    w = np.empty(top_k, dtype=np.float32)
    s = np.empty(top_k, dtype=np.float32)
    _check(lib().urbo_route_noaux_tc(_ptr(logits), _ptr(bias), logits.size, top_k, n_group,
                                     topk_group, int(normalize), scaling, _ptr(e), _ptr(w),
                                     _ptr(s)))
    return e, w, s


def route_softmax_top_k(logits, top_k):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    e = np.empty(top_k, dtype=np.int32)
    w = np.empty(top_k, dtype=np.float32)
    _check(lib().urbo_route_softmax_top_k(_ptr(logits), logits.size, top_k, _ptr(e), _ptr(w)))
    return e, w


def gated_mlp_forward(gate: Matrix, up: Matrix, down: Matrix, x, threads=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(down.rows, dtype=np.float32)
    _check(lib().urbo_gated_mlp_forward(ctypes.byref(gate.c), ctypes.byref(up.c),
                                        ctypes.byref(down.c), _ptr(x), _ptr(y),
                                        threads or default_threads()))
    return y


def group_routes(expert_ids: np.ndarray, experts: int):
    ids = np.ascontiguousarray(expert_ids, dtype=np.int32)
    tokens, top_k = ids.shape
    counts = np.empty(experts, dtype=np.int32)
    offsets = np.empty(experts + 1, dtype=np.int32)
    perm_token = np.empty(tokens * top_k, dtype=np.int32)
    perm_slot = np.empty(tokens * top_k, dtype=np.int32)
    _check(lib().urbo_group_routes(_ptr(ids), tokens, top_k, experts, _ptr(counts),
                                   _ptr(offsets), _ptr(perm_token), _ptr(perm_slot)))
    return counts, offsets, perm_token, perm_slot


class MoeLayer:
    """GLM RuntimeMoeLayer composition (glm/runtime/moe.rs:138-176) over oracle matrices."""

    def __init__(self, router: Matrix, bias, gates, ups, downs, shared, top_k=8, n_group=1,
                 topk_group=1, normalize=True, scaling=2.5):
        self.router, self.bias = router, np.ascontiguousarray(bias, dtype=np.float32)
        self.experts = router.rows
        self._g = (OracleMatrix * self.experts)(*[m.c for m in gates])
        self._u = (OracleMatrix * self.experts)(*[m.c for m in ups])
        self._d = (OracleMatrix * self.experts)(*[m.c for m in downs])
        self._keep = (gates, ups, downs, shared)
        self.hidden = router.cols
        self.top_k = top_k
        self.c = OracleMoeLayer(
            ctypes.pointer(router.c), _ptr(self.bias), self.experts,
            ctypes.cast(self._g, ctypes.POINTER(OracleMatrix)),
            ctypes.cast(self._u, ctypes.POINTER(OracleMatrix)),
            ctypes.cast(self._d, ctypes.POINTER(OracleMatrix)),
            ctypes.pointer(shared[0].c), ctypes.pointer(shared[1].c), ctypes.pointer(shared[2].c),
            top_k, n_group, topk_group, int(normalize), scaling)

    def forward(self, x, threads=None):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.hidden)
        t = x.shape[0]
        out = np.empty_like(x)
        e = np.empty((t, self.top_k), dtype=np.int32)
        w = np.empty((t, self.top_k), dtype=np.float32)
        s = np.empty((t, self.top_k), dtype=np.float32)
        logits = np.empty((t, self.experts), dtype=np.float32)
        _check(lib().urbo_moe_layer_forward(ctypes.byref(self.c), _ptr(x), t, _ptr(out), _ptr(e),
                                            _ptr(w), _ptr(s), _ptr(logits),
                                            threads or default_threads()))
        return out, e, w, s, logits


# ---- checkpoint numerics (DeepSeek-V4) -------------------------------------------------------

def power_of_two_ceiling(value: float) -> float:
    """src/math/mxfp.rs:300-319."""
    return lib().urbo_power_of_two_ceiling(value)


def simulate_e4m3_activation(values, block: int) -> np.ndarray:
    """src/math/mxfp.rs:91-115 (E4M3 round trip with a power-of-two scale per block)."""
    v = np.array(values, dtype=np.float32).ravel()
    _check(lib().urbo_simulate_e4m3_activation(_ptr(v), v.size, block))
    return v


def round_bf16(value: float) -> float:
    """deepseek_v4/math.rs:90-101 (finite inputs)."""
    return lib().urbo_round_bf16(value)


def bounded_swiglu(gate: float, up: float, limit: float) -> float:
    """deepseek_v4/math.rs:518-549, one element."""
    return lib().urbo_bounded_swiglu(gate, up, limit)


def moe_deepseek_forward(layer: "MoeLayer", x, expert_ids, weights, limit: float, threads=None):
    """The DeepSeek-V4 MoE composition for given routes (deepseek_v4/runtime.rs:2500-2700)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, layer.hidden)
    t = x.shape[0]
    ids = np.ascontiguousarray(expert_ids, dtype=np.int32).reshape(t, layer.top_k)
    w = np.ascontiguousarray(weights, dtype=np.float32).reshape(t, layer.top_k)
    out = np.empty_like(x)
    _check(lib().urbo_moe_deepseek_forward(ctypes.byref(layer.c), _ptr(x), t, _ptr(ids), _ptr(w),
                                           limit, _ptr(out), threads or default_threads()))
    return out


def deepseek_expert_forward(gate: Matrix, up: Matrix, down: Matrix, x, limit: float,
                            route_weight=None, threads=None):
    """DeepExpert::forward_with_mx_input (deepseek_v4/runtime.rs:3081-3104) of one token: MX
    projections see x simulated as E4M3 per 128 values, plain ones see x itself."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    mx = simulate_e4m3_activation(x, 128)
    y = np.empty(down.rows, np.float32)
    w = None if route_weight is None else np.array([route_weight], np.float32)
    _check(lib().urbo_deepseek_expert_forward(ctypes.byref(gate.c), ctypes.byref(up.c),
                                              ctypes.byref(down.c), _ptr(x), _ptr(mx),
                                              None if w is None else _ptr(w),
                                              limit, _ptr(y), threads or default_threads()))
    return y


def route_sqrt_softplus(logits, bias, hash_experts, top_k, scaling):
    """deepseek_v4/math.rs:451-516 for one row: (ids, weights, selection scores)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    h = None if hash_experts is None else np.ascontiguousarray(hash_experts, dtype=np.int32)
    e = np.empty(top_k, dtype=np.int32)
    w = np.empty(top_k, dtype=np.float32)
    s = np.empty(top_k, dtype=np.float32)
    _check(lib().urbo_route_sqrt_softplus(_ptr(lg), None if b is None else _ptr(b), lg.size,
                                          None if h is None else _ptr(h), top_k, scaling,
                                          _ptr(e), _ptr(w), _ptr(s)))
    return e, w, s


def moe_deepseek_layer_forward(layer: "MoeLayer", x, limit: float, hash_experts=None,
                               threads=None):
    """DeepSeek-V4 MoeWeights::forward (router, route_sqrt_softplus, expert numerics)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, layer.hidden)
    t = x.shape[0]
    h = None if hash_experts is None else np.ascontiguousarray(hash_experts, dtype=np.int32)
    out = np.empty_like(x)
    e = np.empty((t, layer.top_k), dtype=np.int32)
    w = np.empty((t, layer.top_k), dtype=np.float32)
    _check(lib().urbo_moe_deepseek_layer_forward(ctypes.byref(layer.c), _ptr(x), t,
                                                 None if h is None else _ptr(h), limit, _ptr(out),
                                                 _ptr(e), _ptr(w), threads or default_threads()))
    return out, e, w


# ---- checkpoint numerics (Qwen3.6) -----------------------------------------------------------

def dot_bf16_fp32_lanes(row_bits, x) -> float:
    """src/model/bf16.rs:591-613 (eight FMA lanes)."""
    r = np.ascontiguousarray(row_bits, dtype=np.uint16)
    v = np.ascontiguousarray(x, dtype=np.float32)
    return lib().urbo_dot_bf16_fp32_lanes(_ptr(r), _ptr(v), v.size)


def simulate_finegrained_e4m3(values, block: int) -> np.ndarray:
    """src/math/mxfp.rs:122-149 (exact scale max|v| / 448 per block)."""
    v = np.array(values, dtype=np.float32).ravel()
    _check(lib().urbo_simulate_finegrained_e4m3(_ptr(v), v.size, block))
    return v


def moe_qwen_layer_forward(layer: "MoeLayer", shared_gate_vec: Matrix, x, threads=None):
    """Qwen3.6 execute_batched_moe composition (qwen3_6/runtime.rs:1067-1215)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, layer.hidden)
    t = x.shape[0]
    out = np.empty_like(x)
    e = np.empty((t, layer.top_k), dtype=np.int32)
    w = np.empty((t, layer.top_k), dtype=np.float32)
    _check(lib().urbo_moe_qwen_layer_forward(ctypes.byref(layer.c), ctypes.byref(shared_gate_vec.c),
                                             _ptr(x), t, _ptr(out), _ptr(e), _ptr(w),
                                             threads or default_threads()))
    return out, e, w
