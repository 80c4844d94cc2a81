"""ctypes binding of liburb_moe.so (include/urb_moe.h).

The library is built in-tree by ``urbilateria_b200.build``.  Loading fails loudly when it is
missing: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "liburb_moe.so")

OK = 0
ERR_SHAPE = 1
ERR_INVALID_SCALE = 2
ERR_NONFINITE = 3
ERR_INVALID_GEOMETRY = 4
ERR_CUDA = 5
ERR_TIMEOUT = 6
ERR_NCCL = 7
ERR_UNSUPPORTED = 8
ERR_INVALID_ARGUMENT = 9
ERR_PEER = 10
ERR_INVALID_GROUP = 11

FMT_F32, FMT_BF16, FMT_MXFP8, FMT_MXFP4, FMT_INT8, FMT_INT4 = 0, 1, 2, 3, 4, 5

# urb_kernel_kind
(K_ROW_SHIFT, K_ROUTER_LOGITS, K_ROUTE, K_PERMUTE, K_GATE_UP, K_DOWN, K_COMBINE, K_PRODUCT,
 K_PREP, K_GROUP_BUILD, K_EXCHANGE) = range(11)
KERNEL_NAMES = ["row_shift", "router_logits", "route", "permute", "gate_up", "down", "combine",
                "product", "prep", "group_build", "exchange"]

EP_MAX_WORLD = 8
EP_HANDLE_BYTES = 256

STATUS_NAMES = {
    ERR_SHAPE: "Shape", ERR_INVALID_SCALE: "InvalidScale", ERR_NONFINITE: "NonFinite",
    ERR_INVALID_GEOMETRY: "InvalidGeometry", ERR_CUDA: "Cuda", ERR_TIMEOUT: "Timeout",
    ERR_NCCL: "Nccl", ERR_UNSUPPORTED: "Unsupported", ERR_INVALID_ARGUMENT: "InvalidArgument",
    ERR_PEER: "Peer", ERR_INVALID_GROUP: "InvalidGroupSize",
}


NUMERICS_GLM, NUMERICS_DEEPSEEK_V4, NUMERICS_QWEN36 = 0, 1, 2


class Numerics(ctypes.Structure):
    """urb_moe_numerics."""
    _fields_ = [("mode", ctypes.c_int32), ("swiglu_limit", ctypes.c_float)]


class MoeGeometry(ctypes.Structure):
    """urb_moe_geometry, the MoeGeometry of src/models/glm/moe_geometry.rs:1-9."""
    _fields_ = [("top_k", ctypes.c_uint32), ("n_group", ctypes.c_uint32),
                ("topk_group", ctypes.c_uint32), ("normalize", ctypes.c_int32),
                ("routed_scaling_factor", ctypes.c_float)]


# (name, restype, argtypes) of every exported entry point.
P = ctypes.c_void_p
SZ = ctypes.c_size_t
I32 = ctypes.c_int
U32 = ctypes.c_uint32
PP = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = [
    ("urb_ctx_create", I32, [I32, PP]),
    ("urb_ctx_destroy", I32, [P]),
    ("urb_ctx_set_stream", I32, [P, P]),
    ("urb_ctx_stream", P, [P]),
    ("urb_last_error", I32, [P, ctypes.c_char_p, SZ]),
    ("urb_ctx_synchronize", I32, [P]),
    ("urb_mxfp4_upload", I32, [P, SZ, SZ, SZ, P, SZ, P, SZ, PP]),
    ("urb_mxfp8_upload", I32, [P, SZ, SZ, SZ, SZ, P, SZ, P, SZ, PP]),
    ("urb_bf16_upload", I32, [P, SZ, SZ, P, SZ, PP]),
    ("urb_f32_upload", I32, [P, SZ, SZ, P, SZ, PP]),
    ("urb_mat_free", I32, [P]),
    ("urb_mat_info", I32, [P, P, P, P, P]),
    ("urb_matvec_rows", I32, [P, P, SZ, SZ, P, SZ, P]),
    ("urb_matmul_rows", I32, [P, P, P, SZ, SZ, P]),
    ("urb_matmul_row_range", I32, [P, P, SZ, SZ, P, SZ, SZ, P]),
    ("urb_matmul_rows_fp32_accum", I32, [P, P, P, SZ, SZ, P]),
    ("urb_matmul_rows_device", I32, [P, P, P, SZ, P, P]),
    ("urb_gated_mlp_forward", I32, [P, P, P, P, P, SZ, P]),
    ("urb_gated_mlp_forward_device", I32, [P, P, P, P, P, SZ, P, P]),
    ("urb_gated_mlp_forward_device_noalloc", I32, [P, P, P, P, P, SZ, P, P]),
    ("urb_route_noaux_tc", I32, [P, P, P, SZ, SZ, ctypes.POINTER(MoeGeometry), P, P, P]),
    ("urb_route_softmax_top_k", I32, [P, P, SZ, SZ, U32, P, P]),
    ("urb_group_routes", I32, [P, P, SZ, U32, SZ, P, P, P, P]),
    ("urb_moe_layer_create", I32, [P, P, P, SZ, P, P, P, P, P, P,
                                   ctypes.POINTER(MoeGeometry), PP]),
    ("urb_moe_layer_free", I32, [P]),
    ("urb_moe_forward", I32, [P, P, P, SZ, P, P, P, P, P, P, P, P]),
    ("urb_moe_forward_device", I32, [P, P, P, SZ, P, P, P, P]),
    ("urb_moe_forward_routed", I32, [P, P, P, SZ, P, P, P]),
    ("urb_moe_forward_routed_device", I32, [P, P, P, SZ, P, P, P, P]),
    ("urb_moe_forward_routed_ex", I32, [P, P, P, SZ, P, P, P, P]),
    ("urb_moe_forward_routed_ex_device", I32, [P, P, P, SZ, P, P, P, P, P]),
    ("urb_simulate_e4m3_activation", I32, [P, P, SZ, SZ, P]),
    ("urb_simulate_finegrained_e4m3_activation", I32, [P, P, SZ, SZ, P]),
    ("urb_transpose_rows_matvec", I32, [P, P, SZ, P, SZ, P]),
    ("urb_mat_write_rows", I32, [P, P, SZ, SZ, P]),
    ("urb_int8_upload", I32, [P, SZ, SZ, P, SZ, P, SZ, PP]),
    ("urb_int4_upload", I32, [P, SZ, SZ, SZ, P, SZ, P, SZ, PP]),
    ("urb_int4_quantize_grouped", I32, [P, SZ, SZ, SZ, P, SZ, PP]),
    ("urb_int4_payload", I32, [P, P, P, P]),
    ("urb_linear_bf16_fp32_lanes", I32, [P, P, P, SZ, P]),
    ("urb_moe_forward_ex", I32, [P, P, P, SZ, P, P, P, P, P]),
    ("urb_route_sqrt_softplus", I32, [P, P, P, SZ, SZ, P, U32, ctypes.c_float, P, P, P]),
    ("urb_moe_layer_set_shared_expert_gate", I32, [P, P, P]),
    ("urb_moe_layer_create_sharded", I32, [P, P, P, SZ, SZ, SZ, P, P, P, P, P, P,
                                           ctypes.POINTER(MoeGeometry), PP]),
    ("urb_ep_create", I32, [P, P, I32, I32, SZ, U32, PP]),
    ("urb_ep_export", I32, [P, P]),
    ("urb_ep_connect", I32, [P, P]),
    ("urb_ep_forward", I32, [P, P, P, SZ, P, P, P]),
    ("urb_ep_forward_device", I32, [P, P, P, SZ, P, P, P, P]),
    ("urb_ep_free", I32, [P]),
    ("urb_status_read", I32, [P, P, P]),
    ("urb_profile_enable", I32, [P, I32]),
    ("urb_profile_read", I32, [P, I32, P, P]),
    ("urb_profile_reset", I32, [P]),
]

_lib = None


def load():
    """Loads liburb_moe.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                "liburb_moe.so is not built (run `python -m urbilateria_b200.build`); "
                "there is no CPU fallback")
        lib = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
