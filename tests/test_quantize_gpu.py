"""Device weight quantisers (moe_quantize_*_device) against their host twins:
the same formats must come out bit-identical, for bf16 and fp16 sources,
with all-zero columns / groups and outliers included."""
import ctypes

import numpy as np
import pytest
import torch

import sparsemoe_b200 as sm

pytestmark = pytest.mark.gpu


def _weights(E, K, N, bf16, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((E, K, N)) / np.sqrt(K)).astype(np.float32)
    w[0, :, 3] = 0.0                          # a zero column
    w[-1, :16, :8] = 0.0                      # a zero 16-row group
    w[-1, 5, 9] = 40.0                        # an outlier
    if bf16:
        return (w.view(np.uint32) >> 16).astype(np.uint16)
    return w.astype(np.float16).view(np.uint16)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("bf16", [True, False])
def test_int8_channel_device(gpu, bf16):
    E, K, N = 3, 256, 384
    w = _weights(E, K, N, bf16, 1)
    q_h = np.empty((E, K, N), np.int8)
    s_h = np.empty((E, N), np.float32)
    sm.lib.moe_quantize_int8_channel(w.ctypes.data, E, K, N, int(bf16), q_h.ctypes.data, s_h.ctypes.data)
    q_d = torch.empty(E, K, N, dtype=torch.int8, device="cuda")
    s_d = torch.empty(E, N, dtype=torch.float32, device="cuda")
    assert sm.lib.moe_quantize_int8_channel_device(_ptr(_dev(w)), E, K, N, int(bf16), _ptr(q_d), _ptr(s_d),
                                                   _stream()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(q_d.cpu().numpy(), q_h)
    assert np.array_equal(s_d.cpu().numpy().view(np.uint32), s_h.view(np.uint32))


@pytest.mark.parametrize("bf16", [True, False])
def test_fp8_blocks_device(gpu, bf16):
    E, K, N = 2, 256, 384
    w = _weights(E, K, N, bf16, 2)
    q_h, s_h = sm.quantize_fp8_blocks(w, bf16=bf16)
    q_d = torch.empty(E, K, N, dtype=torch.uint8, device="cuda")
    s_d = torch.empty(E, K // 128, N // 128, dtype=torch.float32, device="cuda")
    assert sm.lib.moe_quantize_fp8_blocks_device(_ptr(_dev(w)), E, K, N, int(bf16), _ptr(q_d), _ptr(s_d),
                                                 _stream()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(q_d.cpu().numpy(), q_h)
    assert np.array_equal(s_d.cpu().numpy().view(np.uint32), s_h.view(np.uint32))


@pytest.mark.parametrize("bf16", [True, False])
def test_int4_g128_device(gpu, bf16):
    E, K, N = 3, 256, 256
    w = _weights(E, K, N, bf16, 3)
    p_h, s_h, z_h = sm.quantize_int4_g128(w, bf16=bf16)
    p_d = torch.empty(E, K, N // 2, dtype=torch.uint8, device="cuda")
    s_d = torch.empty(E, K // 128, N, dtype=torch.int16, device="cuda")
    z_d = torch.empty_like(s_d)
    assert sm.lib.moe_quantize_int4_g128_device(_ptr(_dev(w)), E, K, N, int(bf16), _ptr(p_d), _ptr(s_d), _ptr(z_d),
                                                _stream()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(p_d.cpu().numpy(), p_h)
    assert np.array_equal(s_d.cpu().numpy().view(np.uint16), s_h)
    assert np.array_equal(z_d.cpu().numpy().view(np.uint16), z_h)


@pytest.mark.parametrize("bf16", [True, False])
def test_nvfp4_device(gpu, bf16):
    E, K, N = 3, 256, 256
    w = _weights(E, K, N, bf16, 4)
    p_h, s_h, g_h = sm.quantize_nvfp4(w, bf16=bf16)
    p_d = torch.empty(E, K, N // 2, dtype=torch.uint8, device="cuda")
    s_d = torch.empty(E, K // 16, N, dtype=torch.uint8, device="cuda")
    g_d = torch.empty(E, dtype=torch.float32, device="cuda")
    assert sm.lib.moe_quantize_nvfp4_device(_ptr(_dev(w)), E, K, N, int(bf16), _ptr(p_d), _ptr(s_d), _ptr(g_d),
                                            _stream()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(g_d.cpu().numpy().view(np.uint32), g_h.view(np.uint32))
    assert np.array_equal(s_d.cpu().numpy(), s_h)
    assert np.array_equal(p_d.cpu().numpy(), p_h)
