"""GPU parity of the reference's own int4 and fp8 formats, the two paths its
drivers/main.cu selects with --kernel=capacity_int4_ptx and
--kernel=capacity_fp8_ptx:

* MOE_DTYPE_INT4_PTX (kernels/capacity_int4_ptx.cu): per-tensor int4 weights
  packed transposed ([N/2][K] bytes per expert, inputs/data.cu:89-140),
  activations and h quantised to int4 values (clamp +-7), exact s32 GEMMs;
* MOE_DTYPE_FP8 (kernels/capacity_fp8_ptx.cu): e4m3 weights by direct cast,
  activations and h e4m3(clamp(v / s, +-448)), f32 accumulation.

Bars: routing bit-exact; output max-abs-rel 6e-2 (4-bit) and 3e-2 (8-bit)
against the oracle's restatement on the same quantised operands, through
moe_solve_v2 and through the legacy solve()."""
import ctypes

import numpy as np
import pytest

import sparsemoe_b200 as sm
from oracle import oracle as O

from test_layer_gpu import check_routing, max_abs_rel, run

pytestmark = pytest.mark.gpu

TOL = {sm.DTYPE_INT4_PTX: 6e-2, sm.DTYPE_FP8: 3e-2}


def ref_check(cfg, gpu, seed=0):
    inp = sm.make_inputs(cfg, seed)
    L = run(cfg, inp, gpu)
    ref = O.forward(inp, cfg)
    check_routing(L, ref, cfg)
    err = max_abs_rel(L.out.cpu().numpy()[: cfg.T], ref["out"])
    assert float(np.abs(ref["out"]).max()) > 0, "degenerate case: zero output"
    assert err <= TOL[cfg.dtype], err
    return L, ref, err


@pytest.mark.parametrize("dtype", [sm.DTYPE_INT4_PTX, sm.DTYPE_FP8], ids=["int4_ptx", "fp8"])
def test_small(gpu, dtype):
    ref_check(sm.LayerConfig(1, 512, 512, 768, 16, 4, 1.25, dtype=dtype, act_scale=0.3, mid_scale=0.1), gpu)


@pytest.mark.parametrize("dtype", [sm.DTYPE_INT4_PTX, sm.DTYPE_FP8], ids=["int4_ptx", "fp8"])
def test_drops_ragged(gpu, dtype):
    cfg = sm.LayerConfig(2, 300, 1024, 384, 32, 8, 1.0, dtype=dtype, zipf_s=1.2, act_scale=0.3, mid_scale=0.05)
    L, ref, _ = ref_check(cfg, gpu, seed=4)
    assert (ref["route_slot"] < 0).any()


def test_fp8_placeholder_scales(gpu):
    """The reference builder's scales (all 1.0, inputs/data.cu:368-372)."""
    ref_check(sm.LayerConfig(1, 256, 1024, 1024, 8, 2, 1.25, dtype=sm.DTYPE_FP8), gpu, seed=2)


def test_int4_placeholder_scales(gpu):
    """The reference builder's activation scales (1.0, inputs/data.cu:320-322):
    x ~ N(0,1) rounds to the integers in [-7, 7]."""
    ref_check(sm.LayerConfig(1, 256, 512, 512, 8, 2, 1.25, dtype=sm.DTYPE_INT4_PTX), gpu, seed=3)


@pytest.mark.parametrize("dtype", [sm.DTYPE_INT4_PTX, sm.DTYPE_FP8], ids=["int4_ptx", "fp8"])
def test_legacy_solve_picks_the_format(gpu, dtype, capfd):
    """solve(MoEArgs) (reference kernels/launcher.h:21) chooses the path from
    the weight fields the allocator filled: same result as moe_solve_v2."""
    cfg = sm.LayerConfig(2, 256, 512, 512, 16, 4, 0.8, dtype=dtype, act_scale=0.3, mid_scale=0.1)
    L = run(cfg, sm.make_inputs(cfg, 1), gpu)
    ref_out = L.out.clone()
    L.out.zero_()
    old = sm.MoeDims()
    sm.lib.moe_get_solve_dims(ctypes.byref(old))
    dims = cfg.dims()
    dims.dtype = sm.DTYPE_F16                   # solve() must not need the dtype: the fields decide
    sm.check(sm.lib.moe_set_solve_dims(ctypes.byref(dims)))
    try:
        sm.lib.solve(L.args())
    finally:
        sm.lib.moe_set_solve_dims(ctypes.byref(old))
    assert "Total duration via cudaEventRecord:" in capfd.readouterr().out
    assert bool((L.out == ref_out).all())
