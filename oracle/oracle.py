"""ctypes binding of the CPU oracle (oracle/moe_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline arm as the checker; the product never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libmoe_oracle.so"


def build() -> Path:
    src = HERE / "moe_oracle.cpp"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        I = ctypes.c_int
        L.oracle_capacity.restype = I
        L.oracle_capacity.argtypes = [I, I, I, ctypes.c_float]
        L.oracle_route.restype = None
        L.oracle_route.argtypes = [P, P, I, P, I, I, I, I, I, I, I, P, P, P, P, P, P, P, I]
        L.oracle_ffn_combine.restype = None
        L.oracle_ffn_combine.argtypes = [P, P, P, P, I, I, I, I, I, I, I, P, P, P, ctypes.c_int64,
                                         ctypes.c_int64, P, I]
        L.oracle_ffn_combine_int8.restype = None
        F = ctypes.c_float
        L.oracle_ffn_combine_int8.argtypes = [P, P, P, P, F, F, F, F, F, I, I, I, I, P, P, P, ctypes.c_int64,
                                              ctypes.c_int64, P, I]
        for name in ("oracle_ffn_combine_int4ptx", "oracle_ffn_combine_fp8pt"):
            fn = getattr(L, name)
            fn.restype = None
            fn.argtypes = [P, P, P, P, F, F, F, F, F, I, I, I, I, P, P, P, ctypes.c_int64, ctypes.c_int64, P, I]
        L.oracle_ffn_combine_fp8.restype = None
        L.oracle_ffn_combine_fp8.argtypes = [P, P, P, P, P, P, P, I, I, I, I, P, P, P, ctypes.c_int64,
                                             ctypes.c_int64, P, I]
        L.oracle_ffn_combine_int8ch.restype = None
        L.oracle_ffn_combine_int8ch.argtypes = [P, P, P, P, P, P, P, I, I, I, I, P, P, P, ctypes.c_int64,
                                                ctypes.c_int64, P, I]
        L.oracle_ffn_combine_nvfp4.restype = None
        L.oracle_ffn_combine_nvfp4.argtypes = [P] * 10 + [I, I, I, I, P, P, P, ctypes.c_int64, ctypes.c_int64, P, I]
        L.oracle_e4m3.restype = ctypes.c_uint8
        L.oracle_e4m3.argtypes = [ctypes.c_float]
        L.oracle_e4m3_decode.restype = ctypes.c_float
        L.oracle_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.oracle_set_residual.restype = None
        L.oracle_set_residual.argtypes = [P, I]
        L.oracle_rmsnorm.restype = None
        L.oracle_rmsnorm.argtypes = [P, P, ctypes.c_int64, I, F, I, P]
        L.oracle_ffn_combine_w4.restype = None
        L.oracle_ffn_combine_w4.argtypes = [P] * 10 + [I, I, I, I, P, P, P, ctypes.c_int64, ctypes.c_int64, P, I]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data


def threads() -> int:
    return int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1))


def capacity(tokens: int, top_k: int, num_experts: int, cf: float) -> int:
    return lib().oracle_capacity(tokens, top_k, num_experts, ctypes.c_float(cf))


def route(x, wr, bias, B, N, d, E, k, cap, bf16, router_f32=False, nthreads=None):
    """Stages 1-3.  Returns dict(logits, idx, w, counts, token_ids, token_weights, route_slot)."""
    T = B * N
    x = np.ascontiguousarray(x, dtype=np.uint16)
    wr = np.ascontiguousarray(wr, dtype=np.float32 if router_f32 else np.uint16)
    out = {
        "logits": np.empty((T, E), np.float32), "idx": np.empty((T, k), np.int32),
        "w": np.empty((T, k), np.float32), "counts": np.empty((B, E), np.int32),
        "token_ids": np.full((B, E, max(cap, 0)), -1, np.int32),
        "token_weights": np.zeros((B, E, max(cap, 0)), np.float32),
        "route_slot": np.empty((T * k,), np.int32),
    }
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().oracle_route(_ptr(x), _ptr(wr), int(router_f32), _ptr(b), B, N, d, E, k, cap, int(bf16),
                       _ptr(out["logits"]), _ptr(out["idx"]), _ptr(out["w"]), _ptr(out["counts"]),
                       _ptr(out["token_ids"]), _ptr(out["token_weights"]), _ptr(out["route_slot"]),
                       nthreads or threads())
    return out


def ffn_combine(x, wg, wu, wd, B, N, d, f, E, k, bf16, idx, w, route_slot, t_begin=0, t_end=None,
                nthreads=None):
    """Stages 4-5 for tokens [t_begin, t_end); returns the [t_end - t_begin, d] f32 output rows."""
    T = B * N
    t_end = T if t_end is None else t_end
    out = np.zeros((T, d), np.float32)
    args = [np.ascontiguousarray(a, dtype=np.uint16) for a in (x, wg, wu, wd)]
    lib().oracle_ffn_combine(*(_ptr(a) for a in args), B, N, d, f, E, k, int(bf16),
                             _ptr(np.ascontiguousarray(idx, np.int32)), _ptr(np.ascontiguousarray(w, np.float32)),
                             _ptr(np.ascontiguousarray(route_slot, np.int32)), t_begin, t_end, _ptr(out),
                             nthreads or threads())
    return out[t_begin:t_end]


def ffn_combine_int8(x, q, cfg, idx, w, route_slot, t_begin=0, t_end=None, nthreads=None):
    """int8 path (reference capacity_int8_ptx.cu) for tokens [t_begin, t_end).
    `q` holds wg_q/wu_q/wd_q (int8) and the scales s_in, s_gate, s_up, s_mid, s_down."""
    T = cfg.T
    t_end = T if t_end is None else t_end
    out = np.zeros((T, cfg.d_model), np.float32)
    ws = [np.ascontiguousarray(q[n], np.int8) for n in ("wg_q", "wu_q", "wd_q")]
    lib().oracle_ffn_combine_int8(_ptr(np.ascontiguousarray(x, np.uint16)), *(_ptr(a) for a in ws),
                                  q["s_in"], q["s_gate"], q["s_up"], q["s_mid"], q["s_down"], cfg.d_model,
                                  cfg.d_ff, cfg.num_experts, cfg.top_k,
                                  _ptr(np.ascontiguousarray(idx, np.int32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                  _ptr(np.ascontiguousarray(route_slot, np.int32)), t_begin, t_end, _ptr(out),
                                  nthreads or threads())
    return out[t_begin:t_end]


def ffn_combine_per_tensor(x, q, cfg, idx, w, route_slot, t_begin=0, t_end=None, nthreads=None):
    """The reference's int4 (capacity_int4_ptx.cu: packed-transposed weights,
    clamps at +-7) or fp8 (capacity_fp8_ptx.cu: e4m3 operands) format for
    tokens [t_begin, t_end).  `q` holds wg_q/wu_q/wd_q and the five scales."""
    T = cfg.T
    t_end = T if t_end is None else t_end
    out = np.zeros((T, cfg.d_model), np.float32)
    ws = [np.ascontiguousarray(q[n], np.uint8) for n in ("wg_q", "wu_q", "wd_q")]
    fn = lib().oracle_ffn_combine_int4ptx if cfg.int4ptx else lib().oracle_ffn_combine_fp8pt
    fn(_ptr(np.ascontiguousarray(x, np.uint16)), *(_ptr(a) for a in ws), q["s_in"], q["s_gate"], q["s_up"],
       q["s_mid"], q["s_down"], cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k,
       _ptr(np.ascontiguousarray(idx, np.int32)), _ptr(np.ascontiguousarray(w, np.float32)),
       _ptr(np.ascontiguousarray(route_slot, np.int32)), t_begin, t_end, _ptr(out), nthreads or threads())
    return out[t_begin:t_end]


def ffn_combine_fp8(x, q, cfg, idx, w, route_slot, t_begin=0, t_end=None, nthreads=None):
    """FP8 block-scaled path for tokens [t_begin, t_end); q holds wg_q/wu_q/wd_q
    (e4m3 bytes) and sg/su/sd (block scales)."""
    T = cfg.T
    t_end = T if t_end is None else t_end
    out = np.zeros((T, cfg.d_model), np.float32)
    ws = [np.ascontiguousarray(q[n], np.uint8) for n in ("wg_q", "wu_q", "wd_q")]
    ss = [np.ascontiguousarray(q[n], np.float32) for n in ("sg", "su", "sd")]
    lib().oracle_ffn_combine_fp8(_ptr(np.ascontiguousarray(x, np.uint16)), *(_ptr(a) for a in ws),
                                 *(_ptr(a) for a in ss), cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k,
                                 _ptr(np.ascontiguousarray(idx, np.int32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                 _ptr(np.ascontiguousarray(route_slot, np.int32)), t_begin, t_end, _ptr(out),
                                 nthreads or threads())
    return out[t_begin:t_end]


def ffn_combine_int8ch(x, q, cfg, idx, w, route_slot, t_begin=0, t_end=None, nthreads=None):
    """int8 per-channel / per-token path for tokens [t_begin, t_end); q holds
    wg_q/wu_q/wd_q (int8) and sg/su/sd (per-output-channel scales)."""
    T = cfg.T
    t_end = T if t_end is None else t_end
    out = np.zeros((T, cfg.d_model), np.float32)
    ws = [np.ascontiguousarray(q[n], np.int8) for n in ("wg_q", "wu_q", "wd_q")]
    ss = [np.ascontiguousarray(q[n], np.float32) for n in ("sg", "su", "sd")]
    lib().oracle_ffn_combine_int8ch(_ptr(np.ascontiguousarray(x, np.uint16)), *(_ptr(a) for a in ws),
                                    *(_ptr(a) for a in ss), cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k,
                                    _ptr(np.ascontiguousarray(idx, np.int32)),
                                    _ptr(np.ascontiguousarray(w, np.float32)),
                                    _ptr(np.ascontiguousarray(route_slot, np.int32)), t_begin, t_end, _ptr(out),
                                    nthreads or threads())
    return out[t_begin:t_end]


def ffn_combine_nvfp4(x, q, cfg, idx, w, route_slot, t_begin=0, t_end=None, nthreads=None):
    """NVFP4 weight path for tokens [t_begin, t_end): exact e2m1 * e4m3 * g weights."""
    T = cfg.T
    t_end = T if t_end is None else t_end
    out = np.zeros((T, cfg.d_model), np.float32)
    arrs = [np.ascontiguousarray(q[n], np.uint8) for n in ("wg_q", "wu_q", "wd_q", "wg_s", "wu_s", "wd_s")]
    arrs += [np.ascontiguousarray(q[n], np.float32) for n in ("wg_g", "wu_g", "wd_g")]
    lib().oracle_ffn_combine_nvfp4(_ptr(np.ascontiguousarray(x, np.uint16)), *(_ptr(a) for a in arrs),
                                   cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k,
                                   _ptr(np.ascontiguousarray(idx, np.int32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                   _ptr(np.ascontiguousarray(route_slot, np.int32)), t_begin, t_end, _ptr(out),
                                   nthreads or threads())
    return out[t_begin:t_end]


def ffn_combine_w4(x, q, cfg, idx, w, route_slot, t_begin=0, t_end=None, nthreads=None):
    """4-bit weight path for tokens [t_begin, t_end): exact (q - z) * s weights."""
    T = cfg.T
    t_end = T if t_end is None else t_end
    out = np.zeros((T, cfg.d_model), np.float32)
    arrs = [np.ascontiguousarray(q[n], np.uint8) for n in ("wg_q", "wu_q", "wd_q")]
    arrs += [np.ascontiguousarray(q[n], np.uint16) for n in ("wg_s", "wu_s", "wd_s", "wg_z", "wu_z", "wd_z")]
    lib().oracle_ffn_combine_w4(_ptr(np.ascontiguousarray(x, np.uint16)), *(_ptr(a) for a in arrs), cfg.d_model,
                                cfg.d_ff, cfg.num_experts, cfg.top_k, _ptr(np.ascontiguousarray(idx, np.int32)),
                                _ptr(np.ascontiguousarray(w, np.float32)),
                                _ptr(np.ascontiguousarray(route_slot, np.int32)), t_begin, t_end, _ptr(out),
                                nthreads or threads())
    return out[t_begin:t_end]


def rmsnorm(x, g, eps: float, bf16: bool) -> np.ndarray:
    """Pre-MoE RMSNorm in the GPU kernel's order: [T, d] 16-bit rows -> 16-bit rows."""
    x = np.ascontiguousarray(x, np.uint16)
    out = np.empty_like(x)
    lib().oracle_rmsnorm(_ptr(x), _ptr(np.ascontiguousarray(g, np.uint16)), x.shape[0], x.shape[1],
                         ctypes.c_float(eps), int(bf16), _ptr(out))
    return out


def forward(inputs: dict, cfg, t_begin=0, t_end=None, nthreads=None):
    """Whole layer on the CPU for a sparsemoe_b200.LayerConfig and make_inputs() dict.
    Optional keys: "norm_w" ([d] 16-bit gamma; "norm_eps") runs the pre-MoE
    RMSNorm on x first; "residual" ([T, d] 16-bit) is added in the combine."""
    cap = cfg.capacity()
    act_bf16 = getattr(cfg, "act_bf16", cfg.bf16)
    if inputs.get("norm_w") is not None:
        inputs = {**inputs, "x": rmsnorm(inputs["x"], inputs["norm_w"], inputs.get("norm_eps", 1e-6), act_bf16)}
    res = inputs.get("residual")
    res = None if res is None else np.ascontiguousarray(res, np.uint16)
    lib().oracle_set_residual(_ptr(res), int(act_bf16))
    try:
        return _forward(inputs, cfg, cap, act_bf16, t_begin, t_end, nthreads)
    finally:
        lib().oracle_set_residual(None, 0)


def _forward(inputs, cfg, cap, act_bf16, t_begin, t_end, nthreads):
    r = route(inputs["x"], inputs["wr"], inputs.get("bias"), cfg.num_batches, cfg.tokens, cfg.d_model,
              cfg.num_experts, cfg.top_k, cap, act_bf16, cfg.router_f32, nthreads)
    if getattr(cfg, "nvfp4", False):
        r["out"] = ffn_combine_nvfp4(inputs["x"], inputs, cfg, r["idx"], r["w"], r["route_slot"], t_begin, t_end,
                                     nthreads)
    elif getattr(cfg, "w4", False):
        r["out"] = ffn_combine_w4(inputs["x"], inputs, cfg, r["idx"], r["w"], r["route_slot"], t_begin, t_end,
                                  nthreads)
    elif getattr(cfg, "fp8", False):
        r["out"] = ffn_combine_fp8(inputs["x"], inputs, cfg, r["idx"], r["w"], r["route_slot"], t_begin, t_end,
                                   nthreads)
    elif getattr(cfg, "int8ch", False):
        r["out"] = ffn_combine_int8ch(inputs["x"], inputs, cfg, r["idx"], r["w"], r["route_slot"], t_begin, t_end,
                                      nthreads)
    elif getattr(cfg, "int4ptx", False) or getattr(cfg, "fp8pt", False):
        r["out"] = ffn_combine_per_tensor(inputs["x"], inputs, cfg, r["idx"], r["w"], r["route_slot"], t_begin,
                                          t_end, nthreads)
    elif getattr(cfg, "int8", False):
        r["out"] = ffn_combine_int8(inputs["x"], inputs, cfg, r["idx"], r["w"], r["route_slot"], t_begin, t_end,
                                    nthreads)
    else:
        r["out"] = ffn_combine(inputs["x"], inputs["wg"], inputs["wu"], inputs["wd"], cfg.num_batches, cfg.tokens,
                               cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k, cfg.bf16, r["idx"], r["w"],
                               r["route_slot"], t_begin, t_end, nthreads)
    return r
