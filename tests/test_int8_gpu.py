"""GPU parity of the int8 path (reference kernels/capacity_int8_ptx.cu
semantics: per-tensor int8 weights and activations, s32 tensor-core GEMMs,
dequant/SiLU/requant epilogue) against the CPU oracle's exact integer GEMMs.
Bar: routing bit-exact, output max-abs-rel 3e-2 (BASELINE tolerance for
INT8); in practice only SiLU's exp differs, flipping rare requant roundings."""
import ctypes

import pytest

import sparsemoe_b200 as sm
from oracle import oracle as O

from test_layer_gpu import check_routing, max_abs_rel, run

pytestmark = pytest.mark.gpu

TOL_8 = 3e-2


def int8_check(cfg, gpu, seed=0):
    inp = sm.make_inputs(cfg, seed)
    L = run(cfg, inp, gpu)
    ref = O.forward(inp, cfg)
    check_routing(L, ref, cfg)
    err = max_abs_rel(L.out.cpu().numpy()[: cfg.T], ref["out"])
    assert err <= TOL_8, err
    return L, ref, err


def test_int8_config1_shape(gpu):
    int8_check(sm.LayerConfig(1, 512, 1024, 2048, 8, 2, 1.25, dtype=sm.DTYPE_INT8), gpu)


def test_int8_drops_and_many_experts(gpu):
    cfg = sm.LayerConfig(2, 384, 512, 384, 64, 6, 1.0, dtype=sm.DTYPE_INT8, zipf_s=1.1)
    L, ref, _ = int8_check(cfg, gpu, seed=3)
    assert (ref["route_slot"] < 0).any()


def test_int8_calibrated_scales(gpu):
    """Non-placeholder activation scales (s_in = max|x|/127, s_mid = 1/16)."""
    cfg = sm.LayerConfig(1, 256, 512, 512, 16, 4, 1.0, dtype=sm.DTYPE_INT8, act_scale=4.5 / 127,
                         mid_scale=1.0 / 16)
    int8_check(cfg, gpu, seed=5)


def test_int8_solve_selects_int8_path(gpu, capfd):
    """solve() with the int8 allocator's fields picks the int8 kernels
    (reference: built with KERNEL=capacity_int8_ptx)."""
    cfg = sm.LayerConfig(1, 256, 512, 256, 16, 2, 1.0, dtype=sm.DTYPE_INT8)
    inp = sm.make_inputs(cfg, 2)
    L = run(cfg, inp, gpu)
    ref_out = L.out.clone()
    L.out.zero_()
    old = sm.MoeDims()
    sm.lib.moe_get_solve_dims(ctypes.byref(old))
    dims = cfg.dims()
    sm.check(sm.lib.moe_set_solve_dims(ctypes.byref(dims)))
    try:
        sm.lib.solve(L.args())
    finally:
        sm.lib.moe_set_solve_dims(ctypes.byref(old))
    assert "Total duration via cudaEventRecord:" in capfd.readouterr().out
    assert bool((L.out == ref_out).all())
