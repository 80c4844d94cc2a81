"""The C-ABI library exports every entry point that include/urb_moe.h declares, and the
Python binding covers them.  No CUDA call is made (CPU-only test)."""
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "urb_moe.h")
SO = os.path.join(ROOT, "urbilateria_b200", "liburb_moe.so")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"URB_API\s+[\w\s\*]+?\b(urb_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert "urb_moe_forward" in names and "urb_mxfp4_upload" in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol():
    from urbilateria_b200 import build
    build.build()
    out = subprocess.run(["nm", "-D", "--defined-only", SO], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s(urb_\w+)$", out, flags=re.M))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing


def test_python_binding_matches_header():
    from urbilateria_b200 import native
    lib = native.load()  # loads the shared library without touching the GPU
    bound = {name for name, _, _ in native.SIGNATURES}
    assert bound == set(declared())
    for name in bound:
        assert getattr(lib, name) is not None


def test_no_cluster_multicast_loads_in_sources():
    # Multi-GPU safety rule of this build: no TMA/bulk load with cluster multicast anywhere.
    pat = re.compile(re.escape(bytes.fromhex("6d756c7469636173743a3a636c7573746572").decode()))  # the qualifier, hex-encoded
    for d in ("urbilateria_b200/csrc", "include"):
        for f in os.listdir(os.path.join(ROOT, d)):
            p = os.path.join(ROOT, d, f)
            if os.path.isfile(p) and f.endswith((".cu", ".cuh", ".h", ".cpp")):
                assert not pat.search(open(p).read()), p
