"""Expert weight files (.bin): every format's router and expert weights
round-trip bit-exactly through moe_weights_write / _read_*, and damaged files
are rejected (no GPU needed)."""
import numpy as np
import pytest

import sparsemoe_b200 as sm

FORMATS = [sm.DTYPE_F16, sm.DTYPE_BF16, sm.DTYPE_INT8, sm.DTYPE_INT8_CHANNEL, sm.DTYPE_FP8_BLOCK, sm.DTYPE_W4A16,
           sm.DTYPE_NVFP4]


@pytest.mark.parametrize("dtype", FORMATS)
def test_round_trip(tmp_path, dtype):
    cfg = sm.LayerConfig(1, 8, 256, 256, 8, 2, 1.25, dtype=dtype, zipf_s=1.0,
                         router_f32=dtype in (sm.DTYPE_W4A16, sm.DTYPE_NVFP4))
    inp = sm.make_inputs(cfg, 3)
    path = tmp_path / "layer.bin"
    sm.save_weights(path, cfg, inp)
    info, back = sm.load_weights(path)
    assert info == {"dtype": dtype, "router_dtype": sm.ROUTER_F32 if cfg.router_f32 else sm.ROUTER_SAME,
                    "num_experts": 8, "d_model": 256, "d_ff": 256}
    expect = {k: v for k, v in inp.items() if k != "x" and v is not None}
    assert set(back) == set(expect)
    for k, v in expect.items():
        if isinstance(v, np.ndarray):
            assert back[k].dtype == v.dtype and back[k].shape == v.shape, k
            assert np.array_equal(back[k].view(np.uint8), np.ascontiguousarray(v).view(np.uint8)), k
        else:
            assert back[k] == pytest.approx(v, rel=0, abs=0) or np.float32(back[k]) == np.float32(v), k


def test_damaged_files_rejected(tmp_path):
    cfg = sm.LayerConfig(1, 8, 256, 256, 8, 2, 1.25, dtype=sm.DTYPE_W4A16)
    path = tmp_path / "layer.bin"
    sm.save_weights(path, cfg, sm.make_inputs(cfg, 0))
    raw = path.read_bytes()
    (tmp_path / "short.bin").write_bytes(raw[: len(raw) - 100])        # truncated data
    (tmp_path / "magic.bin").write_bytes(b"XXXXXXXX" + raw[8:])          # wrong magic
    (tmp_path / "tiny.bin").write_bytes(raw[:64])                        # truncated header
    for name in ("short.bin", "magic.bin", "tiny.bin", "missing.bin"):
        with pytest.raises(sm.MoeError):
            sm.load_weights(tmp_path / name)
