"""moe_solve_v2_noalloc: the layer with its scratch in a fixed static device
array, for callers that cannot let the library allocate device memory (an
engine that owns every byte through its own pre-planned pool, or a serving
loop that cannot afford the device synchronisation of cudaMalloc/cudaFree).

Checked through the C ABI against moe_solve_v2 on the same buffers, two calls
in a row (the array keeps the previous call's contents).  Both entry points
run the same deterministic kernels on the same inputs, so the outputs must be
bit-identical (stricter than the 1e-2 / 3e-2 bars the formats' own parity
tests hold against the oracle); a stale table left in the shared array would
show as a difference.  The FP8 case also exercises the per-row activation and
h scale regions that the dynamic formats carve from the array.  This file is
collected last so that a stop-at-first-failure run has run every other test
before it.
"""
import ctypes

import numpy as np
import pytest

import sparsemoe_b200 as sm

pytestmark = pytest.mark.gpu


def _call_noalloc(layer):
    import torch
    a, dm = layer.args(), layer.dims()
    s = torch.cuda.current_stream(layer.device)
    rc = sm.lib.moe_solve_v2_noalloc(ctypes.byref(a), ctypes.byref(dm), ctypes.c_void_p(s.cuda_stream))
    sm.check(rc)
    layer.sync_check()


@pytest.mark.parametrize("cfg", [
    sm.LayerConfig(1, 512, 1024, 2048, 8, 2, 1.25),
    sm.LayerConfig(2, 384, 256, 256, 64, 6, 1.0, zipf_s=1.1, dtype=sm.DTYPE_BF16),
    sm.LayerConfig(1, 512, 512, 768, 16, 4, 1.25, dtype=sm.DTYPE_FP8_BLOCK),
], ids=["f16_cfg1", "bf16_zipf_drops", "fp8_block"])
def test_noalloc_matches_allocating_entry(gpu, cfg):
    inp = sm.make_inputs(cfg, 11)
    layer = sm.MoeLayer(cfg, gpu).load(inp)
    dims = layer.dims()
    assert sm.lib.moe_workspace_bytes(ctypes.byref(dims)) <= sm.lib.moe_noalloc_scratch_bytes()
    layer.forward()
    layer.sync_check()
    ref_out = layer.out.cpu().numpy().copy()
    ref_idx = layer.idx.cpu().numpy().copy()
    ref_counts = layer.counts.cpu().numpy().copy()
    for _ in range(2):                      # two calls in a row share the static array
        layer.out.fill_(float("nan"))
        layer.counts.fill_(-1)
        _call_noalloc(layer)
        assert np.array_equal(layer.idx.cpu().numpy(), ref_idx)
        assert np.array_equal(layer.counts.cpu().numpy(), ref_counts)
        assert np.array_equal(layer.out.cpu().numpy(), ref_out)


def test_noalloc_rejects_oversized_call(gpu):
    cfg = sm.LayerConfig(1, 600000, 256, 128, 8, 2, 1.25)   # 1.2M routes: > 4 MiB of scratch
    dims = cfg.dims()
    assert sm.lib.moe_workspace_bytes(ctypes.byref(dims)) > sm.lib.moe_noalloc_scratch_bytes()
    a = sm.MoEArgs()
    for name, _ in sm.MoEArgs._fields_[:-3]:
        if name not in ("scale_up_w", "scale_gate_w", "scale_down_w", "scale_input_act", "scale_mid_act"):
            setattr(a, name, 256)           # non-null placeholders: the size check comes first
    rc = sm.lib.moe_solve_v2_noalloc(ctypes.byref(a), ctypes.byref(dims), None)
    assert rc == sm.MOE_ERR_UNSUPPORTED
    assert "static array" in sm.last_error()


def test_noalloc_rejects_caller_scratch(gpu):
    """A caller with scratch of its own uses moe_solve_v2; here it is refused."""
    import torch
    cfg = sm.LayerConfig(1, 64, 256, 128, 8, 2, 1.25)
    layer = sm.MoeLayer(cfg, gpu).load(sm.make_inputs(cfg, 0))
    buf = torch.empty(1 << 20, dtype=torch.uint8, device=gpu)
    a, dm = layer.args(), layer.dims()
    dm.scratch, dm.scratch_bytes = buf.data_ptr(), buf.numel()
    rc = sm.lib.moe_solve_v2_noalloc(ctypes.byref(a), ctypes.byref(dm), None)
    assert rc == sm.MOE_ERR_INVALID_ARG
    assert "scratch must be null" in sm.last_error()
