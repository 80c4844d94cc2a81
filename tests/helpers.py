"""Test helpers: build the same weights as a device matrix and an oracle matrix, and the
tolerance check of the parity bar (relative L2 <= 1e-3 and max-abs <= 2e-2 on outputs scaled
to unit RMS; see rel_err)."""
import numpy as np

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

REL_L2 = 1e-3
MAX_ABS = 2e-2


def rel_err(got, want):
    """(relative L2, max-abs error after dividing both by the reference RMS)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    d = got - want
    nrm = np.linalg.norm(want)
    rms = nrm / np.sqrt(max(want.size, 1))
    rel = np.linalg.norm(d) / nrm if nrm > 0 else np.linalg.norm(d)
    mx = np.abs(d).max() / rms if rms > 0 else np.abs(d).max()
    return rel, mx


def assert_close(got, want, rel=REL_L2, mx=MAX_ABS):
    r, m = rel_err(got, want)
    assert r <= rel and m <= mx, "relL2=%.3e max_abs(normalised)=%.3e" % (r, m)


def mxfp4_pair(oracle, ctx, g, rows, cols, group=32, lo=119, hi=127):
    packed, scales = syn.mxfp4_matrix(g, rows, cols, lo, hi, group)
    dev = urb.MxFp4Matrix.from_packed(rows, cols, group, packed, scales, ctx=ctx)
    orc = oracle.Matrix(oracle.MXFP4, rows, cols, packed, scales, group_size=group)
    return dev, orc


def mxfp8_pair(oracle, ctx, g, rows, cols, block_rows=1, block_cols=32, lo=117, hi=123):
    values = syn.encode_e4m3fn(g.standard_normal((rows, cols), dtype=np.float32))
    ns = (-(-rows // block_rows), -(-cols // block_cols))
    scales = g.integers(lo, hi + 1, size=ns, dtype=np.uint8)
    dev = urb.MxFp8Matrix.from_packed(rows, cols, block_rows, block_cols, values, scales, ctx=ctx)
    orc = oracle.Matrix(oracle.MXFP8, rows, cols, values, scales, block_rows=block_rows,
                        block_cols=block_cols)
    return dev, orc


def bf16_pair(oracle, ctx, g, rows, cols, std=0.02):
    bits = syn.bf16_normal(g, (rows, cols), std)
    dev = urb.Bf16Matrix.from_bits(rows, cols, bits, ctx=ctx)
    orc = oracle.Matrix(oracle.BF16, rows, cols, bits)
    return dev, orc


def memory_state(device: int):
    """(bytes in use from the device's default stream-ordered pool, bytes that pool reserves,
    free device memory): what a cudaMallocAsync or a cudaMalloc inside the library would move."""
    from cuda.bindings import runtime as rt
    err, pool = rt.cudaDeviceGetDefaultMemPool(device)
    assert err == rt.cudaError_t.cudaSuccess
    err, used = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent)
    assert err == rt.cudaError_t.cudaSuccess
    err, reserved = rt.cudaMemPoolGetAttribute(
        pool, rt.cudaMemPoolAttr.cudaMemPoolAttrReservedMemCurrent)
    assert err == rt.cudaError_t.cudaSuccess
    err, free, _ = rt.cudaMemGetInfo()
    assert err == rt.cudaError_t.cudaSuccess
    return int(used), int(reserved), int(free)


def profiled_kinds(ctx, fn):
    """Runs fn() with the library's per-launch profiler on; the kernel kinds it launched."""
    import ctypes
    from urbilateria_b200 import native
    ctx.lib.urb_profile_reset(ctx.h)
    ctx.lib.urb_profile_enable(ctx.h, 1)
    try:
        fn()
    finally:
        ctx.lib.urb_profile_enable(ctx.h, 0)
    kinds = {}
    for k, name in enumerate(native.KERNEL_NAMES):
        t, n = ctypes.c_double(), ctypes.c_int64()
        ctx.lib.urb_profile_read(ctx.h, k, ctypes.byref(t), ctypes.byref(n))
        if n.value:
            kinds[name] = n.value
    return kinds
