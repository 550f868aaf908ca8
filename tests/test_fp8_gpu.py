"""GPU parity of the FP8 block-scaled path (BASELINE config 4 format): e4m3
weights with f32 scales per 128x128 block, activations and h quantised per
1x128 block on the device, f32 accumulation with per-K-block promotion.
Bar: routing bit-exact, output max-abs-rel 3e-2 vs the oracle's restatement."""
import pytest

import sparsemoe_b200 as sm
from oracle import oracle as O

from test_layer_gpu import check_routing, max_abs_rel, run

pytestmark = pytest.mark.gpu

TOL_8 = 3e-2


def fp8_check(cfg, gpu, seed=0, t_end=None):
    inp = sm.make_inputs(cfg, seed)
    L = run(cfg, inp, gpu)
    ref = O.forward(inp, cfg, 0, t_end)
    check_routing(L, ref, cfg)
    n = ref["out"].shape[0]
    err = max_abs_rel(L.out.cpu().numpy()[:n], ref["out"])
    assert err <= TOL_8, err
    return L, ref, err


def test_fp8_small(gpu):
    fp8_check(sm.LayerConfig(1, 512, 512, 768, 16, 4, 1.25, dtype=sm.DTYPE_FP8_BLOCK), gpu)


def test_fp8_drops_ragged(gpu):
    cfg = sm.LayerConfig(2, 300, 1024, 384, 32, 8, 1.0, dtype=sm.DTYPE_FP8_BLOCK, zipf_s=1.2)
    L, ref, _ = fp8_check(cfg, gpu, seed=4)
    assert (ref["route_slot"] < 0).any()


def test_fp8_config4_shape_token_sample(gpu):
    """BASELINE config 4 shape (T=32768, d=2048, f=768, E=128, k=8, cf=1.25):
    routing of all tokens bit-exact, output checked on the first 256 tokens."""
    cfg = sm.LayerConfig(1, 32768, 2048, 768, 128, 8, 1.25, dtype=sm.DTYPE_FP8_BLOCK)
    L, ref, err = fp8_check(cfg, gpu, t_end=256)
    assert L.cap == 2560
