"""Expert-parallel MoE layer across the GPUs of one node: one process per GPU.

The reference runs every expert of a layer in one process (RuntimeMoeLayer::forward,
src/models/glm/runtime/moe.rs:138-176, rows split over Rayon workers).  Here rank g of a group
of ``world`` processes holds the routed experts ``shard_range(experts, world, g)`` (a sharded
:class:`~urbilateria_b200.RuntimeMoeLayer`) plus the replicated router and shared expert, and
owns the tokens it passes to :meth:`ExpertParallelMoeLayer.forward_batch`.  Token rows and expert
outputs cross NVLink inside the library's kernels (peer loads of the owners' rows, peer stores
of the experts' outputs); the only host-side exchange is the one-time all-gather of the ranks'
window handles, done over the caller's ``torch.distributed`` process group (any backend).
Outputs are bit-identical to the single-GPU layer.

``forward_batch`` is collective: every rank calls it for every forward, in the same order, with
its own (possibly zero) token count.
"""
from __future__ import annotations

import ctypes
from typing import Callable, List, Optional, Tuple

import numpy as np

from . import native
from . import RuntimeMoeLayer, UrbError, _ptr


def shard_range(experts: int, world: int, rank: int) -> Tuple[int, int]:
    """(begin, count) of the routed experts held by ``rank``: contiguous ranges whose sizes
    differ by at most one, the first ``experts % world`` ranks holding the larger ones."""
    if not (1 <= world <= experts) or not (0 <= rank < world):
        raise ValueError("need 1 <= world <= experts and 0 <= rank < world")
    base, extra = divmod(experts, world)
    begin = rank * base + min(rank, extra)
    return begin, base + (1 if rank < extra else 0)


def token_range(tokens: int, world: int, rank: int) -> Tuple[int, int]:
    """(begin, count) of a batch's tokens owned by ``rank`` (data-parallel split; ranks past
    the token count own none)."""
    if not (0 <= rank < world):
        raise ValueError("rank out of range")
    base, extra = divmod(tokens, world)
    begin = rank * base + min(rank, extra)
    return begin, base + (1 if rank < extra else 0)


def all_gather_bytes(blob: bytes, group=None) -> List[bytes]:
    """All-gathers one byte string per rank over a torch.distributed group, in rank order."""
    import torch.distributed as dist
    out: List[Optional[bytes]] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, blob, group=group)
    return [bytes(b) for b in out]


class ExpertParallelMoeLayer:
    """This rank's member of an expert-parallel group over ``layer`` (urb_ep_*).

    ``exchange`` all-gathers the ranks' handle blobs (default: :func:`all_gather_bytes` over
    the default process group); with ``world == 1`` no exchange happens."""

    def __init__(self, layer: RuntimeMoeLayer, world: int, rank: int, max_tokens: int,
                 exchange: Optional[Callable[[bytes], List[bytes]]] = None,
                 timeout_ms: int = 0):
        self.layer = layer
        self.ctx = layer.ctx
        self.world, self.rank, self.max_tokens = world, rank, max_tokens
        lib = self.ctx.lib
        h = ctypes.c_void_p()
        self.ctx.check(lib.urb_ep_create(self.ctx.h, layer.h, world, rank, max_tokens,
                                         timeout_ms, ctypes.byref(h)))
        self.h = h
        blob = (ctypes.c_uint8 * native.EP_HANDLE_BYTES)()
        self.ctx.check(lib.urb_ep_export(h, ctypes.cast(blob, ctypes.c_void_p)))
        mine = bytes(blob)
        blobs = [mine] if world == 1 else (exchange or all_gather_bytes)(mine)
        if len(blobs) != world or any(len(b) != native.EP_HANDLE_BYTES for b in blobs):
            self.free()
            raise UrbError(native.ERR_INVALID_ARGUMENT, "handle exchange returned %d blobs" % len(blobs))
        if blobs[rank] != mine:
            self.free()
            raise UrbError(native.ERR_INVALID_ARGUMENT, "handle exchange is not in rank order")
        joined = (ctypes.c_uint8 * (world * native.EP_HANDLE_BYTES)).from_buffer_copy(b"".join(blobs))
        rc = lib.urb_ep_connect(h, ctypes.cast(joined, ctypes.c_void_p))
        if rc != native.OK:
            try:
                self.ctx.check(rc)
            finally:
                self.free()

    def forward_batch(self, x, tokens: int):
        """x [tokens, hidden] of this rank -> (out [tokens, hidden], expert ids, weights)."""
        H, K = self.layer.hidden_size(), self.layer.geometry.top_k
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(tokens, H)
        out = np.empty((tokens, H), dtype=np.float32)
        ids = np.empty((tokens, K), dtype=np.int32)
        w = np.empty((tokens, K), dtype=np.float32)
        self.ctx.check(self.ctx.lib.urb_ep_forward(self.ctx.h, self.h, _ptr(x) if tokens else None,
                                                   tokens, _ptr(out) if tokens else None,
                                                   _ptr(ids) if tokens else None,
                                                   _ptr(w) if tokens else None))
        return out, ids, w

    def forward_device(self, d_x: int, tokens: int, d_out: int, d_status: int, d_ids: int = 0,
                       d_w: int = 0):
        self.ctx.check(self.ctx.lib.urb_ep_forward_device(
            self.ctx.h, self.h, d_x or None, tokens, d_out or None, d_ids or None, d_w or None,
            d_status))

    def free(self):
        if getattr(self, "h", None) and self.ctx.h:  # a closed context: drop the handle
            self.ctx.lib.urb_ep_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
