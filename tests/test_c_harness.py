"""The boundary a Rust crate links: tests/c_harness/urb_harness.c built with gcc against the
static liburb_moe.a, the static CUDA runtime and libstdc++ / rt / pthread / dl (the link line of
the build.rs in INTEGRATION.md), with no Python or ctypes in the process.

On the CPU the harness must compile and link.  On a GPU it uploads a small MXFP4 MoE layer,
runs urb_moe_forward (RuntimeMoeLayer::forward, src/models/glm/runtime/moe.rs:138-176) and
urb_matvec_rows, checks a 0xFF-scale upload is rejected with InvalidScale and a message, and
its outputs are compared with the oracle: routes bit-exact, outputs within the parity bar."""
import os
import subprocess
import tempfile

import numpy as np
import pytest

from urbilateria_b200 import synthetic as syn

from helpers import assert_close

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build_harness(out_dir: str) -> str:
    import urbilateria_b200.build as b
    b.build()
    exe = os.path.join(out_dir, "urb_harness")
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "c_harness", "urb_harness.c"),
           b.AR, "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart_static", "-lstdc++", "-lrt",
           "-lpthread", "-ldl", "-lm", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_harness_links_against_static_library():
    with tempfile.TemporaryDirectory() as d:
        exe = build_harness(d)
        assert os.path.getsize(exe) > 0


@pytest.mark.gpu
def test_harness_layer_forward_matches_oracle(oracle):
    H, I, E, K, T, scale = 512, 256, 16, 4, 5, 2.5
    g = syn.rng(9100)
    router = syn.bf16_normal(g, (E, H), 0.02)
    bias = syn.normal_f32(g, E, 0.01)
    mlps = [[syn.mxfp4_matrix(g, r, c) for r, c in ((I, H), (I, H), (H, I))] for _ in range(E + 1)]
    x = syn.normal_bf16_as_f32(g, (T, H))
    with tempfile.TemporaryDirectory() as d:
        exe = build_harness(d)
        inp, outp = os.path.join(d, "in.bin"), os.path.join(d, "out.bin")
        with open(inp, "wb") as f:
            f.write(np.array([H, I, E, K, T], np.uint32).tobytes())
            f.write(np.array([scale], np.float32).tobytes())
            f.write(router.tobytes())
            f.write(bias.tobytes())
            for mlp in mlps:
                for p, s in mlp:
                    f.write(p.tobytes())
                    f.write(s.tobytes())
            f.write(x.tobytes())
        r = subprocess.run([exe, inp, outp], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0 and r.stdout.strip() == "OK", r.stdout + r.stderr
        raw = open(outp, "rb").read()
    out = np.frombuffer(raw, np.float32, T * H).reshape(T, H)
    ids = np.frombuffer(raw, np.int32, T * K, offset=T * H * 4).reshape(T, K)
    w = np.frombuffer(raw, np.float32, T * K, offset=(T * H + T * K) * 4).reshape(T, K)
    y = np.frombuffer(raw, np.float32, 64, offset=(T * H + 2 * T * K) * 4)

    om = [tuple(oracle.Matrix(oracle.MXFP4, r_, c_, p, s, group_size=32)
                for (p, s), (r_, c_) in zip(m, ((I, H), (I, H), (H, I)))) for m in mlps]
    orouter = oracle.Matrix(oracle.BF16, E, H, router)
    layer = oracle.MoeLayer(orouter, bias, [m[0] for m in om[:E]], [m[1] for m in om[:E]],
                            [m[2] for m in om[:E]], om[E], K, 1, 1, True, scale)
    o_out, o_ids, o_w = layer.forward(x)[:3]
    assert np.array_equal(ids, o_ids)
    assert np.array_equal(w.view(np.uint32), o_w.view(np.uint32))
    assert_close(out, o_out)
    assert_close(y, om[0][0].matvec_rows(5, 64, x[0]))
