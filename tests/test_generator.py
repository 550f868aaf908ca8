"""The seeded counter-based input generator (csrc/generator.cpp)."""
import numpy as np

import sparsemoe_b200 as sm


def test_deterministic_and_prefix_stable():
    a = sm.normal16(100_000, 7, 3, 1.0, False)
    b = sm.normal16(100_000, 7, 3, 1.0, False)
    assert np.array_equal(a, b)
    # value i depends only on (seed, stream, i): a longer (multi-threaded) fill has the same prefix
    c = sm.normal16(300_000, 7, 3, 1.0, False)
    assert np.array_equal(a, c[:100_000])
    assert not np.array_equal(a, sm.normal16(100_000, 8, 3, 1.0, False))
    assert not np.array_equal(a, sm.normal16(100_000, 7, 4, 1.0, False))


def test_moments():
    x = sm.normal_f32(1 << 20, 0, 0, 1.0)
    assert abs(x.mean()) < 5e-3 and abs(x.std() - 1.0) < 5e-3
    y = sm.normal16(1 << 20, 0, 0, 0.02, True).astype(np.uint32) << 16
    y = y.view(np.float32)
    assert abs(y.std() - 0.02) < 2e-4


def test_f16_matches_f32_rounding():
    f = sm.normal_f32(50_000, 3, 9, 0.5)
    h = sm.normal16(50_000, 3, 9, 0.5, False).view(np.float16)
    assert np.array_equal(h, f.astype(np.float16))
    b = sm.normal16(50_000, 3, 9, 0.5, True)
    # bf16 = round-to-nearest-even of the f32 value
    u = f.view(np.uint32).astype(np.uint64)
    rne = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    assert np.array_equal(b, rne)


def test_zipf_bias():
    b = sm.zipf_bias(8, 1.1)
    assert b[0] == 0 and np.all(np.diff(b) < 0)
    np.testing.assert_allclose(b, -1.1 * np.log1p(np.arange(8)), rtol=1e-6)
    p = sm.zipf_bias(64, 1.0, 1.0, seed=5)
    assert sorted(np.round(p, 5)) == sorted(np.round(sm.zipf_bias(64, 1.0), 5))
