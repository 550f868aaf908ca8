"""Seeded synthetic layer inputs built on the host without the product library.

TEST INFRASTRUCTURE ONLY: the benchmark's reference arm (`bench.py --impl
reference`) draws its workload here so that the timed CPU transcription of the
reference never loads libsparsemoe_b200.so, and tests/ check these quantisers
against the library's host quantisers bit for bit.

Distributions are the BASELINE ones (x ~ N(0,1), router ~ N(0,0.02), gate/up ~
N(0,1/sqrt(d)), down ~ N(0,1/sqrt(f))), drawn with torch's CPU generator
straight into the 16-bit type; the values differ from the product arm's
device-drawn ones, the distributions and shapes do not.  The quantisers
restate the formats:
  * per-tensor int8: the reference's inputs/data.cu:13-57 (scale = max|w|/127,
    nearbyint of the clamped quotient);
  * int8 per output channel (amax over K / 127);
  * FP8 e4m3 per 128x128 block (amax / 448, satfinite round-to-nearest-even);
  * INT4 asymmetric g128 (fp16 scale (max-min)/15 and zero -min/scale);
  * NVFP4 (global amax/(448*6), e4m3 scale per 16 K-rows, e2m1 codes, ties to
    the even code);
with the 4-bit codes in the kernels' layout: [E, K, N/2] bytes, 8 columns per
32-bit word, column pair (2p, 2p+1) at bits 4p and 16+4p.
"""
from __future__ import annotations

import numpy as np

_E2M1_MIDS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)


def _u16(t) -> np.ndarray:
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _to_f32(u16: np.ndarray, bf16: bool) -> np.ndarray:
    if bf16:
        return (u16.astype(np.uint32) << 16).view(np.float32)
    return u16.view(np.float16).astype(np.float32)


def _e4m3(v: np.ndarray) -> np.ndarray:
    """f32 -> e4m3 codes, round-to-nearest-even, saturating at +-448."""
    import torch
    t = torch.from_numpy(np.clip(v, -448.0, 448.0).astype(np.float32))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def _e4m3_value(code: np.ndarray) -> np.ndarray:
    import torch
    return torch.from_numpy(np.ascontiguousarray(code, np.uint8)).view(torch.float8_e4m3fn).float().numpy()


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """[E, K, N] 4-bit codes -> [E, K, N/2] bytes in the kernels' layout."""
    E, K, N = codes.shape
    c = codes.astype(np.uint8).reshape(E, K, N // 8, 4, 2)      # (word, pair p, column 2p + j)
    lo, hi = c[..., 0], c[..., 1]                                # bits 4p (byte p//2) and 16 + 4p
    out = np.zeros((E, K, N // 8, 4), np.uint8)
    for p in range(4):
        sh = 4 * (p & 1)
        out[..., p >> 1] |= (lo[..., p] << sh).astype(np.uint8)
        out[..., 2 + (p >> 1)] |= (hi[..., p] << sh).astype(np.uint8)
    return out.reshape(E, K, N // 2)


def quantize_per_tensor(w16: np.ndarray, qmax: float = 127.0):
    """fp16 bit patterns -> (int8, scale); reference inputs/data.cu:13-57."""
    v = w16.view(np.float16).astype(np.float32)
    m = np.float32(np.abs(v).max()) if v.size else np.float32(0)
    scale = np.float32(m / np.float32(qmax)) if m > 0 else np.float32(1)
    q = np.rint(np.clip(v / scale, -qmax, qmax)).astype(np.int8)
    return q, float(scale)


def quantize_int8_channel(w16: np.ndarray, bf16: bool = True):
    E, K, N = w16.shape
    q = np.empty((E, K, N), np.int8)
    sc = np.empty((E, N), np.float32)
    for e in range(E):
        v = _to_f32(w16[e], bf16)
        m = np.abs(v).max(axis=0)
        s = np.where(m > 0, m / np.float32(127), np.float32(1)).astype(np.float32)
        sc[e] = s
        q[e] = np.clip(np.rint(v / s), -127, 127).astype(np.int8)
    return q, sc


def quantize_fp8_blocks(w16: np.ndarray, bf16: bool = True):
    E, K, N = w16.shape
    q = np.empty((E, K, N), np.uint8)
    sc = np.empty((E, K // 128, N // 128), np.float32)
    for e in range(E):
        v = _to_f32(w16[e], bf16).reshape(K // 128, 128, N // 128, 128)
        m = np.abs(v).max(axis=(1, 3))
        s = np.where(m > 0, m / np.float32(448), np.float32(1)).astype(np.float32)
        sc[e] = s
        q[e] = _e4m3(v / s[:, None, :, None]).reshape(K, N)
    return q, sc


def quantize_int4_g128(w16: np.ndarray, bf16: bool = True):
    E, K, N = w16.shape
    codes = np.empty((E, K, N), np.uint8)
    sc = np.empty((E, K // 128, N), np.uint16)
    zr = np.empty((E, K // 128, N), np.uint16)
    for e in range(E):
        v = _to_f32(w16[e], bf16).reshape(K // 128, 128, N)
        mn, mx = v.min(axis=1), v.max(axis=1)
        s = ((mx - mn) / np.float32(15)).astype(np.float32)
        s = np.where(s > 0, s, np.float32(1)).astype(np.float32)
        sh = s.astype(np.float16)
        zh = (-mn / sh.astype(np.float32)).astype(np.float16)
        sc[e], zr[e] = sh.view(np.uint16), zh.view(np.uint16)
        qv = np.rint(v / sh.astype(np.float32)[:, None, :] + zh.astype(np.float32)[:, None, :])
        codes[e] = np.clip(qv, 0, 15).astype(np.uint8).reshape(K, N)
    return pack_nibbles(codes), sc, zr


def _e2m1(v: np.ndarray) -> np.ndarray:
    a = np.abs(v)
    lo = np.searchsorted(_E2M1_MIDS, a, side="left")
    hi = np.searchsorted(_E2M1_MIDS, a, side="right")
    code = np.where(lo == hi, lo, np.where(lo % 2 == 0, lo, lo + 1))   # on a midpoint: the even code
    code = np.where(a >= 6, 7, code)
    return (code | np.where(v < 0, 8, 0)).astype(np.uint8)


def quantize_nvfp4(w16: np.ndarray, bf16: bool = True):
    E, K, N = w16.shape
    codes = np.empty((E, K, N), np.uint8)
    sc = np.empty((E, K // 16, N), np.uint8)
    gl = np.empty(E, np.float32)
    for e in range(E):
        v = _to_f32(w16[e], bf16)
        amax = np.float32(np.abs(v).max())
        g = np.float32(amax / np.float32(448.0 * 6.0)) if amax > 0 else np.float32(1)
        gl[e] = g
        vb = v.reshape(K // 16, 16, N)
        m = np.abs(vb).max(axis=1)
        s = _e4m3(m / (np.float32(6) * g))
        s = np.where((s & 0x7F) == 0, np.uint8(1), s).astype(np.uint8)
        s = np.where(m > 0, s, np.uint8(0x38)).astype(np.uint8)
        sc[e] = s
        div = (_e4m3_value(s) * g).astype(np.float32)
        codes[e] = _e2m1(vb / div[:, None, :]).reshape(K, N)
    return pack_nibbles(codes), sc, gl


def zipf_bias(num_experts: int, s: float, scale: float = 1.0) -> np.ndarray:
    """Zipf(s) popularity bias over expert index: logit bias -scale*s*log(1+e),
    so expert e is picked about (1+e)^-s as often (the library's
    moe_zipf_bias with seed 0)."""
    b = -np.float64(scale) * np.float64(np.float32(s)) * np.log(1.0 + np.arange(num_experts, dtype=np.float64))
    return b.astype(np.float32)


def make_inputs(cfg, seed: int = 0) -> dict:
    """Host inputs with the keys of the library's make_inputs() for a
    LayerConfig-like `cfg` (fields and format flags of sparsemoe_b200's
    LayerConfig), drawn with torch's CPU generator."""
    import torch
    g = torch.Generator().manual_seed(seed)
    d, f, E = cfg.d_model, cfg.d_ff, cfg.num_experts
    t16 = torch.bfloat16 if cfg.act_bf16 else torch.float16

    def normal(n, std, dt=t16):
        return torch.empty(n, dtype=dt).normal_(0.0, std, generator=g)
    out = {"x": _u16(normal(cfg.T * d, 1.0)).reshape(cfg.T, d)}
    out["wr"] = (normal(d * E, 0.02, torch.float32).numpy() if cfg.router_f32 else
                 _u16(normal(d * E, 0.02))).reshape(d, E)
    for n, (K, N) in (("wg", (d, f)), ("wu", (d, f)), ("wd", (f, d))):
        out[n] = _u16(normal(E * K * N, K ** -0.5)).reshape(E, K, N)
    if cfg.nvfp4:
        for n in ("wg", "wu", "wd"):
            out[n + "_q"], out[n + "_s"], out[n + "_g"] = quantize_nvfp4(out[n], True)
    elif cfg.w4:
        for n in ("wg", "wu", "wd"):
            out[n + "_q"], out[n + "_s"], out[n + "_z"] = quantize_int4_g128(out[n], True)
    if cfg.fp8:
        for n, key in (("wg", "sg"), ("wu", "su"), ("wd", "sd")):
            out[n + "_q"], out[key] = quantize_fp8_blocks(out[n], True)
    if cfg.int8ch:
        for n, key in (("wg", "sg"), ("wu", "su"), ("wd", "sd")):
            out[n + "_q"], out[key] = quantize_int8_channel(out[n], True)
    if cfg.int8:
        for n, nm in (("wg", "gate"), ("wu", "up"), ("wd", "down")):
            out[n + "_q"], out["s_" + nm] = quantize_per_tensor(out[n])
        out["s_in"] = float(np.float32(cfg.act_scale))
        out["s_mid"] = float(np.float32(cfg.mid_scale))
    out["bias"] = zipf_bias(E, cfg.zipf_s) if cfg.zipf_s > 0 else None
    return out
