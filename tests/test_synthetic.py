"""Host-side generators: the vectorised E4M3 encoder equals the reference encoder
(src/math/mxfp.rs:247-275, restated in the oracle) on every float8 boundary region, and the
bf16 rounding is round-to-nearest-even."""
import numpy as np

from urbilateria_b200 import synthetic as syn


def test_e4m3_encoder_matches_oracle(oracle):
    lib = oracle.lib()
    g = np.random.default_rng(0)
    v = np.concatenate([
        g.standard_normal(20000).astype(np.float32),
        g.standard_normal(5000).astype(np.float32) * np.float32(300),
        g.standard_normal(5000).astype(np.float32) * np.float32(2 ** -8),
        np.array([0.0, -0.0, 448.0, -448.0, 1e9, -1e9, 2 ** -6, 2 ** -9, 2 ** -10, 464.0], np.float32),
    ])
    # Every midpoint between adjacent representable E4M3 magnitudes (ties to even).
    mags = np.array([lib.urbo_decode_e4m3fn(c) for c in range(0x7F)], np.float32)
    mids = ((mags[:-1].astype(np.float64) + mags[1:]) / 2).astype(np.float32)
    v = np.concatenate([v, mids, -mids])
    got = syn.encode_e4m3fn(v)
    want = np.array([lib.urbo_encode_e4m3fn(float(x)) for x in v], np.uint8)
    assert np.array_equal(got, want)


def test_bf16_round_to_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 3.0e38], np.float32)
    bits = syn.f32_to_bf16_bits(x)
    assert list(bits) == [0x3F80, 0x3F80, 0x3F82, 0xC020, 0x7F62]
    back = syn.bf16_bits_to_f32(bits)
    assert back[0] == 1.0 and back[3] == -2.5


def test_zipf_routes_are_distinct_and_seeded():
    a = syn.zipf_routes(syn.rng(1), 64, 128, 8)
    b = syn.zipf_routes(syn.rng(1), 64, 128, 8)
    assert np.array_equal(a, b)
    assert all(len(set(r)) == 8 for r in a)
    counts = np.bincount(a.ravel(), minlength=128)
    assert counts.max() > 4 * np.median(counts[counts > 0])  # skewed popularity
