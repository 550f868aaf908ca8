"""GPU parity of the stages either side of the layer (MoeDims.norm_* and
residual): the pre-MoE RMSNorm written to norm_out must equal the oracle's
restatement bit for bit (it feeds the router, so routing stays bit-exact),
and the residual added in the combine must keep the output within the
format's bar of the oracle's ((r + w0*y0) + w1*y1) + ... ."""
import numpy as np
import pytest

import sparsemoe_b200 as sm
from oracle import oracle as O

from test_layer_gpu import TOL_16, check_routing, max_abs_rel, run

pytestmark = pytest.mark.gpu


def _gamma(d, bf16, seed=3):
    v = (1.0 + 0.1 * np.random.default_rng(seed).standard_normal(d)).astype(np.float32)
    return (v.view(np.uint32) >> 16).astype(np.uint16) if bf16 else v.astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("dtype,E", [(sm.DTYPE_F16, 8), (sm.DTYPE_BF16, 64)], ids=["f16_E8", "bf16_E64"])
def test_norm_and_residual_match_oracle(gpu, dtype, E):
    cfg = sm.LayerConfig(2, 192, 512, 256, E, 2, 1.0, dtype=dtype, zipf_s=1.0 if E == 64 else 0.0)
    inp = sm.make_inputs(cfg, 6)
    inp = {**inp, "norm_w": _gamma(cfg.d_model, cfg.act_bf16), "norm_eps": 1e-5, "residual": inp["x"]}
    L = run(cfg, inp, gpu)
    xn = O.rmsnorm(inp["x"], inp["norm_w"], 1e-5, cfg.act_bf16)
    got = L.xn.view(__import__("torch").int16).cpu().numpy().view(np.uint16)[: cfg.T]
    assert np.array_equal(got, xn), "normalised rows differ from the oracle"
    ref = O.forward(inp, cfg)
    check_routing(L, ref, cfg)
    assert max_abs_rel(L.out.cpu().numpy()[: cfg.T], ref["out"]) <= TOL_16
    if L.out16 is not None:
        assert max_abs_rel(L.out16.float().cpu().numpy()[: cfg.T], ref["out"]) <= TOL_16


def test_residual_alone_passes_dropped_tokens_through(gpu):
    """Tokens whose routes were all dropped get exactly the residual row."""
    cfg = sm.LayerConfig(1, 256, 256, 256, 16, 2, 0.25, zipf_s=2.0)
    inp = sm.make_inputs(cfg, 1)
    inp = {**inp, "residual": inp["x"]}
    L = run(cfg, inp, gpu)
    ref = O.forward(inp, cfg)
    check_routing(L, ref, cfg)
    slots = ref["route_slot"].reshape(cfg.T, cfg.top_k)
    dropped = np.nonzero((slots < 0).all(axis=1))[0]
    assert dropped.size > 0
    x = inp["x"].view(np.float16).astype(np.float32)
    assert np.array_equal(L.out.cpu().numpy()[dropped], x[dropped])
    assert max_abs_rel(L.out.cpu().numpy()[: cfg.T], ref["out"]) <= TOL_16


def test_norm_needs_an_output_buffer(gpu):
    import ctypes
    cfg = sm.LayerConfig(1, 64, 256, 256, 8, 2, 1.0)
    inp = sm.make_inputs(cfg, 0)
    L = sm.MoeLayer(cfg, gpu).load({**inp, "norm_w": _gamma(256, False)})
    a, dm = L.args(), L.dims()
    dm.norm_out = None
    assert sm.lib.moe_solve_v2(ctypes.byref(a), ctypes.byref(dm), None) == sm.MOE_ERR_INVALID_ARG
    assert "norm_out" in sm.last_error()
