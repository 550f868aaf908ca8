"""Host-side mirror of the B200 MoE layer's C ABI (include/sparsemoe_b200.h).

The product is libsparsemoe_b200.so: hand-written sm_100a CUDA behind the
reference's C++ host API (`MoEArgs`, `solve()`, the input builder of
MattJBorowski1991/SparseMoE).  This module binds that library with ctypes and
uses PyTorch only for device memory and streams.  There is no CPU fallback:
importing the module fails if the library is missing.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
# the in-tree build; SPARSEMOE_B200_LIB may name another build of the same library
LIB_PATH = Path(os.environ["SPARSEMOE_B200_LIB"]) if os.environ.get("SPARSEMOE_B200_LIB") else \
    _PKG / "libsparsemoe_b200.so"

from .config import (  # noqa: F401  (re-exported)
    MOE_OK, MOE_ERR_INVALID_ARG, MOE_ERR_UNSUPPORTED, MOE_ERR_CUDA, MOE_ERR_TIMEOUT, MOE_ERR_NO_KERNEL,
    DTYPE_F16, DTYPE_BF16, DTYPE_INT8, DTYPE_FP8_BLOCK, DTYPE_W4A16, DTYPE_INT8_CHANNEL, DTYPE_NVFP4,
    DTYPE_INT4_PTX, DTYPE_FP8, ROUTER_SAME, ROUTER_F32, MoeError, MoEArgs, MoeDims, MoeWeightArray,
    MoeWeightFile, LayerConfig, _p)
from . import config as _config


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python sparsemoe_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
    sig = {
        "solve": (None, [MoEArgs]),
        "moe_solve_v2": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p]),
        "moe_check_device_status": (ctypes.c_int, [_p]),
        "moe_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_int64, _p]),
        "moe_set_solve_dims": (ctypes.c_int, [ctypes.POINTER(MoeDims)]),
        "moe_get_solve_dims": (ctypes.c_int, [ctypes.POINTER(MoeDims)]),
        "moe_capacity": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float]),
        "moe_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(MoeDims)]),
        "moe_release": (None, []),
        "moe_stage_route": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p]),
        "moe_stage_expert_ffn": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p, _p, _p,
                                                ctypes.c_int, ctypes.c_int64, _p]),
        "moe_stage_combine": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p]),
        "moe_stage_route_counts": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p, _p]),
        "moe_stage_route_finish": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p]),
        "moe_ffn_scratch_bytes": (ctypes.c_size_t, [ctypes.POINTER(MoeDims), ctypes.c_int64]),
        "moe_stage_expert_ffn_peer": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p, _p, _p,
                                                      _p, _p, ctypes.c_int, ctypes.c_int64, _p, ctypes.c_int, _p]),
        "moe_weights_write": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(MoeWeightFile), _p]),
        "moe_weights_read_header": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(MoeWeightFile)]),
        "moe_weights_read_array": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(MoeWeightFile), ctypes.c_int,
                                                   _p, ctypes.c_size_t]),
        "moe_ep_plan": (ctypes.c_int, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _p, _p]),
        "moe_stage_dispatch_peer": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p, _p, _p,
                                                    ctypes.c_int, _p]),
        "moe_stage_expert_ffn_planned": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p,
                                                         ctypes.c_int, ctypes.c_int64, _p, ctypes.c_int, _p]),
        "moe_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _p]),
        "moe_peer_open": (ctypes.c_int, [_p, ctypes.POINTER(ctypes.c_void_p)]),
        "moe_peer_close": (ctypes.c_int, [_p]),
        "moe_peer_free": (ctypes.c_int, [_p]),
        "moe_memcpy_async": (ctypes.c_int, [_p, _p, ctypes.c_size_t, _p]),
        "moe_solve_v2_noalloc": (ctypes.c_int, [ctypes.POINTER(MoEArgs), ctypes.POINTER(MoeDims), _p]),
        "moe_noalloc_scratch_bytes": (ctypes.c_size_t, []),
        "moe_set_stage_events": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]),
        "moe_last_error": (ctypes.c_char_p, []),
        "moe_fill_normal_16": (None, [_p, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float,
                                      ctypes.c_int]),
        "moe_quantize_per_tensor": (ctypes.c_float, [_p, ctypes.c_size_t, _p, ctypes.c_float]),
        "moe_pack_int4_transposed": (None, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _p]),
        "moe_cast_e4m3": (None, [_p, ctypes.c_size_t, _p]),
        "moe_quantize_int4_g128": (None, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _p, _p, _p]),
        "moe_quantize_fp8_blocks": (None, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _p, _p]),
        "moe_quantize_int8_channel": (None, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _p, _p]),
        "moe_quantize_nvfp4": (None, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _p, _p, _p]),
        "moe_quantize_int8_channel_device": (ctypes.c_int, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                             _p, _p, _p]),
        "moe_quantize_fp8_blocks_device": (ctypes.c_int, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                           _p, _p, _p]),
        "moe_quantize_int4_g128_device": (ctypes.c_int, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                          _p, _p, _p, _p]),
        "moe_quantize_nvfp4_device": (ctypes.c_int, [_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                      _p, _p, _p, _p]),
        "moe_fill_normal_f32": (None, [_p, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float]),
        "moe_zipf_bias": (None, [_p, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_uint64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    return lib.moe_last_error().decode()


def check(rc: int) -> None:
    if rc != MOE_OK:
        raise MoeError(rc, last_error())


def capacity(tokens: int, top_k: int, num_experts: int, cf: float) -> int:
    """CAP = round_up(ceilf(N*k/E*cf), 16) (reference inputs/data.cu:392-398)."""
    return lib.moe_capacity(tokens, top_k, num_experts, ctypes.c_float(cf))


_config.set_capacity_fn(capacity)


# ---- seeded generator -------------------------------------------------------
def normal16(n: int, seed: int, stream: int, std: float, bf16: bool) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib.moe_fill_normal_16(out.ctypes.data, n, seed, stream, ctypes.c_float(std), int(bf16))
    return out


def normal_f32(n: int, seed: int, stream: int, std: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib.moe_fill_normal_f32(out.ctypes.data, n, seed, stream, ctypes.c_float(std))
    return out


def zipf_bias(num_experts: int, s: float, scale: float = 1.0, seed: int = 0) -> np.ndarray:
    out = np.empty(num_experts, dtype=np.float32)
    lib.moe_zipf_bias(out.ctypes.data, num_experts, ctypes.c_float(s), ctypes.c_float(scale), seed)
    return out


def make_inputs(cfg: LayerConfig, seed: int = 0) -> dict:
    """Seeded host inputs (streams: x 0, router 1, gate 2, up 3, down 4).

    x ~ N(0,1); router ~ N(0,0.02); gate/up ~ N(0,1/sqrt(d)); down ~ N(0,1/sqrt(f)).
    16-bit tensors are returned as uint16 bit patterns.
    """
    d, f, E = cfg.d_model, cfg.d_ff, cfg.num_experts
    b16 = cfg.act_bf16
    out = {
        "x": normal16(cfg.T * d, seed, 0, 1.0, b16).reshape(cfg.T, d),
        "wg": normal16(E * d * f, seed, 2, 1.0 / np.sqrt(d), b16).reshape(E, d, f),
        "wu": normal16(E * d * f, seed, 3, 1.0 / np.sqrt(d), b16).reshape(E, d, f),
        "wd": normal16(E * f * d, seed, 4, 1.0 / np.sqrt(f), b16).reshape(E, f, d),
    }
    if cfg.router_f32:
        out["wr"] = normal_f32(d * E, seed, 1, 0.02).reshape(d, E)
    else:
        out["wr"] = normal16(d * E, seed, 1, 0.02, b16).reshape(d, E)
    if cfg.nvfp4:
        for n in ("wg", "wu", "wd"):
            q, sc, gl = quantize_nvfp4(out[n], bf16=True)
            out[n + "_q"], out[n + "_s"], out[n + "_g"] = q, sc, gl
    elif cfg.w4:
        for n in ("wg", "wu", "wd"):
            q, sc, zr = quantize_int4_g128(out[n], bf16=True)
            out[n + "_q"], out[n + "_s"], out[n + "_z"] = q, sc, zr
    if cfg.fp8:
        for n, key in (("wg", "sg"), ("wu", "su"), ("wd", "sd")):
            q, sc = quantize_fp8_blocks(out[n], bf16=True)
            out[n + "_q"], out[key] = q, sc
    if cfg.int8ch:
        for n, key in (("wg", "sg"), ("wu", "su"), ("wd", "sd")):
            q, sc = quantize_int8_channel(out[n], bf16=True)
            out[n + "_q"], out[key] = q, sc
    out["bias"] = zipf_bias(E, cfg.zipf_s) if cfg.zipf_s > 0 else None
    if cfg.per_tensor:
        # reference inputs/data.cu:275-390: per-tensor int8 (max/127) or int4 (max/7, packed
        # transposed) weights, or a direct e4m3 cast with unit scales; activation scales from cfg
        # (the reference's placeholders are 1.0)
        for n in ("wg", "wu", "wd"):
            name = "s_" + {"wg": "gate", "wu": "up", "wd": "down"}[n]
            if cfg.fp8pt:
                q = np.empty(out[n].size, np.uint8)
                lib.moe_cast_e4m3(out[n].ctypes.data, out[n].size, q.ctypes.data)
                out[n + "_q"], out[name] = q.reshape(out[n].shape), 1.0
                continue
            q = np.empty(out[n].size, np.int8)
            scale = lib.moe_quantize_per_tensor(out[n].ctypes.data, out[n].size, q.ctypes.data,
                                                7.0 if cfg.int4ptx else 127.0)
            q = q.reshape(out[n].shape)
            out[name] = float(scale)
            if cfg.int4ptx:
                E_, K_, N_ = q.shape
                packed = np.empty((E_, N_ // 2, K_), np.uint8)
                lib.moe_pack_int4_transposed(q.ctypes.data, E_, K_, N_, packed.ctypes.data)
                out[n + "_i4"] = q                  # the unpacked int4 values (for checks)
                q = packed
            out[n + "_q"] = q
        out["s_in"] = float(np.float32(cfg.act_scale))
        out["s_mid"] = float(np.float32(cfg.mid_scale))
    return out


_KIND = {"u": 0, "i": 1, "f": 2}
_INT8_SCALES = ("s_in", "s_gate", "s_up", "s_mid", "s_down")


def save_weights(path: str, cfg: LayerConfig, inputs: dict) -> None:
    """Writes the router and expert weights of `inputs` (a make_inputs() dict,
    or one with the same keys) in the library's .bin format: every array but
    the tokens `x`, the per-tensor int8 scales as one f32 array."""
    arrays = {k: np.ascontiguousarray(v) for k, v in inputs.items()
              if k not in ("x",) + _INT8_SCALES and v is not None and isinstance(v, np.ndarray)}
    if cfg.per_tensor:
        arrays["int8_scales"] = np.array([inputs[k] for k in _INT8_SCALES], np.float32)
    if len(arrays) > 16:
        raise ValueError("more than 16 arrays")
    h = MoeWeightFile()
    h.dtype, h.router_dtype = cfg.dtype, ROUTER_F32 if cfg.router_f32 else ROUTER_SAME
    h.num_experts, h.d_model, h.d_ff, h.num_arrays = cfg.num_experts, cfg.d_model, cfg.d_ff, len(arrays)
    ptrs = (ctypes.c_void_p * len(arrays))()
    for i, (name, a) in enumerate(arrays.items()):
        d = h.arrays[i]
        d.name = name.encode()
        d.elem_bytes, d.kind, d.ndim = a.dtype.itemsize, _KIND[a.dtype.kind], a.ndim
        for j, n in enumerate(a.shape):
            d.shape[j] = n
        ptrs[i] = a.ctypes.data
    check(lib.moe_weights_write(str(path).encode(), ctypes.byref(h), ptrs))


def load_weights(path: str) -> tuple[dict, dict]:
    """Reads a .bin weight file: (info: dtype, router_dtype, num_experts,
    d_model, d_ff; arrays by name, with the int8 scales back as floats)."""
    h = MoeWeightFile()
    check(lib.moe_weights_read_header(str(path).encode(), ctypes.byref(h)))
    out = {}
    for i in range(h.num_arrays):
        d = h.arrays[i]
        dt = np.dtype(f"{'uif'[d.kind]}{d.elem_bytes}")
        a = np.empty(tuple(d.shape[j] for j in range(d.ndim)), dt)
        check(lib.moe_weights_read_array(str(path).encode(), ctypes.byref(h), i, a.ctypes.data, a.nbytes))
        out[d.name.decode()] = a
    if "int8_scales" in out:
        for k, v in zip(_INT8_SCALES, out.pop("int8_scales")):
            out[k] = float(v)
    info = {"dtype": h.dtype, "router_dtype": h.router_dtype, "num_experts": h.num_experts,
            "d_model": h.d_model, "d_ff": h.d_ff}
    return info, out


def quantize_int4_g128(w16: np.ndarray, bf16: bool = True):
    """INT4 asymmetric, group 128 along K, fp16 scale and zero per (group,
    column); returns (packed [E, K, N/2] uint8, scales, zeros [E, K/128, N]
    as fp16 bit patterns).  w16: [E, K, N] 16-bit bit patterns."""
    E, K, N = w16.shape
    w16 = np.ascontiguousarray(w16, np.uint16)
    q = np.empty((E, K, N // 2), np.uint8)
    sc = np.empty((E, K // 128, N), np.uint16)
    zr = np.empty((E, K // 128, N), np.uint16)
    lib.moe_quantize_int4_g128(w16.ctypes.data, E, K, N, int(bf16), q.ctypes.data, sc.ctypes.data, zr.ctypes.data)
    return q, sc, zr


def quantize_nvfp4(w16: np.ndarray, bf16: bool = True):
    """NVFP4: e2m1 nibbles (packed like quantize_int4_g128), one e4m3 scale per
    16 K-rows and column, one f32 global scale per expert matrix.  w16: [E, K,
    N] 16-bit bit patterns.  Returns (packed [E, K, N/2] uint8, scales [E,
    K/16, N] uint8 e4m3 codes, globals [E] f32)."""
    E, K, N = w16.shape
    w16 = np.ascontiguousarray(w16, np.uint16)
    q = np.empty((E, K, N // 2), np.uint8)
    sc = np.empty((E, K // 16, N), np.uint8)
    gl = np.empty(E, np.float32)
    lib.moe_quantize_nvfp4(w16.ctypes.data, E, K, N, int(bf16), q.ctypes.data, sc.ctypes.data, gl.ctypes.data)
    return q, sc, gl


def quantize_fp8_blocks(w16: np.ndarray, bf16: bool = True):
    """e4m3 weights with f32 scales per 128x128 block of each [K, N] expert
    matrix (s = amax/448).  w16: [E, K, N] 16-bit bit patterns."""
    E, K, N = w16.shape
    w16 = np.ascontiguousarray(w16, np.uint16)
    q = np.empty((E, K, N), np.uint8)
    sc = np.empty((E, K // 128, N // 128), np.float32)
    lib.moe_quantize_fp8_blocks(w16.ctypes.data, E, K, N, int(bf16), q.ctypes.data, sc.ctypes.data)
    return q, sc


def quantize_int8_channel(w16: np.ndarray, bf16: bool = True):
    """Symmetric int8 weights with one f32 scale per output column of each
    [K, N] expert matrix (s = amax/127).  w16: [E, K, N] 16-bit bit patterns.
    Returns (q [E, K, N] int8, scales [E, N] f32)."""
    E, K, N = w16.shape
    w16 = np.ascontiguousarray(w16, np.uint16)
    q = np.empty((E, K, N), np.int8)
    sc = np.empty((E, N), np.float32)
    lib.moe_quantize_int8_channel(w16.ctypes.data, E, K, N, int(bf16), q.ctypes.data, sc.ctypes.data)
    return q, sc


def quantize_per_tensor(w16: np.ndarray, qmax: float = 127.0):
    """Reference inputs/data.cu:13-57 per-tensor quantiser; returns (int8 values, scale)."""
    w16 = np.ascontiguousarray(w16, np.uint16)
    q = np.empty(w16.size, np.int8)
    scale = lib.moe_quantize_per_tensor(w16.ctypes.data, w16.size, q.ctypes.data, ctypes.c_float(qmax))
    return q.reshape(w16.shape), float(scale)


from .layer import MoeLayer  # noqa: E402  (needs `lib` above)

__all__ = ["MoEArgs", "MoeDims", "LayerConfig", "MoeLayer", "make_inputs", "capacity", "lib", "check",
           "MoeError", "normal16", "normal_f32", "zipf_bias", "quantize_per_tensor", "DTYPE_F16", "DTYPE_BF16",
           "DTYPE_INT8", "DTYPE_FP8_BLOCK", "quantize_fp8_blocks",
           "DTYPE_W4A16", "quantize_int4_g128", "DTYPE_INT8_CHANNEL", "quantize_int8_channel",
           "DTYPE_NVFP4", "quantize_nvfp4", "DTYPE_INT4_PTX", "DTYPE_FP8", "save_weights", "load_weights", "MoeWeightFile", "MoeWeightArray"]
