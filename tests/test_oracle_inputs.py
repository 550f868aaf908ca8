"""The reference arm's host-side input builder (oracle/inputs.py) restates the
library's host quantisers: checked bit for bit on random weights, including a
constant group, an all-zero group and ties, so the reference arm's workload is
in exactly the formats the product reads."""
import numpy as np
import pytest

import sparsemoe_b200 as sm
from oracle import inputs as I


@pytest.fixture(scope="module")
def weights():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((2, 256, 256)) * 0.05).astype(np.float32)
    w[1, :128, 3] = 0.25          # constant INT4 group
    w[0, 16:32, 5] = 0.0          # all-zero NVFP4 group
    return (w.view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("name", ["quantize_int8_channel", "quantize_fp8_blocks", "quantize_int4_g128",
                                  "quantize_nvfp4"])
def test_quantiser_matches_library(weights, name):
    ours = getattr(sm, name)(weights, bf16=True)
    host = getattr(I, name)(weights, True)
    for a, b in zip(ours, host):
        assert np.array_equal(a, b)


def test_per_tensor_matches_library():
    h = np.float16(np.random.default_rng(1).standard_normal(5000)).view(np.uint16)
    q0, s0 = sm.quantize_per_tensor(h)
    q1, s1 = I.quantize_per_tensor(h)
    assert np.array_equal(q0, q1) and s0 == s1


def test_zipf_bias_matches_library():
    assert np.array_equal(sm.zipf_bias(256, 1.0), I.zipf_bias(256, 1.0))


def test_make_inputs_shapes_and_keys():
    cfg = sm.LayerConfig(1, 8, 256, 256, 8, 2, 1.0, dtype=sm.DTYPE_NVFP4, router_f32=True, zipf_s=1.0)
    a, b = sm.make_inputs(cfg, 0), I.make_inputs(cfg, 0)
    assert set(a) == set(b)
    for k in a:
        if isinstance(a[k], np.ndarray):
            assert a[k].shape == b[k].shape and a[k].dtype == b[k].dtype, k
