"""Quantisation-accuracy report: every weight format of the layer against the
16-bit layer on the same seeded tokens, router and weights.

    python -m sparsemoe_b200.quant_report [--tokens T] [--d D] [--f F] [--experts E] [--topk K]

All bf16-activation formats (BF16 baseline, INT8_CHANNEL, FP8_BLOCK, W4A16
INT4-g128, NVFP4) start from the same seeded bf16 weights and tokens, so they
route identically; the reference's per-tensor INT8 format runs on fp16
activations and is compared with the F16 layer.  Capacity is unlimited (no
drops) so every format computes the same routes.  For each format: max-abs
and max-abs-rel error of the f32 output against the 16-bit layer, cosine
similarity over the whole output, and whether the routing matched.  One JSON
line per format.
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def compare(out: np.ndarray, ref: np.ndarray) -> dict:
    diff = out.astype(np.float64) - ref.astype(np.float64)
    denom = float(np.abs(ref).max()) or 1.0
    cos = float(np.dot(out.ravel().astype(np.float64), ref.ravel().astype(np.float64)) /
                (np.linalg.norm(out.astype(np.float64)) * np.linalg.norm(ref.astype(np.float64)) or 1.0))
    return {"max_abs": float(np.abs(diff).max()), "max_abs_rel": float(np.abs(diff).max()) / denom, "cosine": cos}


def run_format(cfg, device, seed, want_layer=False):
    import sparsemoe_b200 as sm
    layer = sm.MoeLayer(cfg, device).load(sm.make_inputs(cfg, seed))
    layer.forward()
    layer.sync_check()
    res = (layer.out.cpu().numpy()[: cfg.T], layer.idx.cpu().numpy()[: cfg.T])
    return res + (layer,) if want_layer else res


def report(tokens=2048, d=2048, f=1024, experts=16, topk=4, seed=0, device="cuda:0"):
    import sparsemoe_b200 as sm
    shape = dict(num_batches=1, tokens=tokens, d_model=d, d_ff=f, num_experts=experts, top_k=topk,
                 capacity_factor=1.0, cap=-1)
    rows = []
    base_out, base_idx = run_format(sm.LayerConfig(**shape, dtype=sm.DTYPE_BF16), device, seed)
    for name, dt in (("int8_channel_token", sm.DTYPE_INT8_CHANNEL), ("fp8_e4m3_block", sm.DTYPE_FP8_BLOCK),
                     ("int4_g128", sm.DTYPE_W4A16), ("nvfp4_g16", sm.DTYPE_NVFP4)):
        out, idx = run_format(sm.LayerConfig(**shape, dtype=dt), device, seed)
        rows.append({"format": name, "baseline": "bf16 layer", **compare(out, base_out),
                     "routing_identical": bool(np.array_equal(idx, base_idx))})
    f16_out, f16_idx, f16 = run_format(sm.LayerConfig(**shape, dtype=sm.DTYPE_F16), device, seed, want_layer=True)
    # the reference's per-tensor format with activation scales calibrated on this batch
    # (amax / 127 of x and of the f16 layer's h); the reference itself ships placeholders of 1.0
    rows_used = int(f16.counts.sum().item())
    s_in = float(f16.x[:tokens].float().abs().max().item()) / 127.0
    s_mid = float(f16.h_rows[:rows_used].float().abs().max().item()) / 127.0
    out, idx = run_format(sm.LayerConfig(**shape, dtype=sm.DTYPE_INT8, act_scale=s_in, mid_scale=s_mid), device, seed)
    rows.append({"format": "int8_per_tensor (reference format, calibrated scales)",
                 "baseline": "f16 layer", **compare(out, f16_out),
                 "routing_identical": bool(np.array_equal(idx, f16_idx))})
    for r in rows:
        r["shape"] = {k: v for k, v in shape.items() if k != "cap"}
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--d", type=int, default=2048)
    ap.add_argument("--f", type=int, default=1024)
    ap.add_argument("--experts", type=int, default=16)
    ap.add_argument("--topk", type=int, default=4)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    for r in report(a.tokens, a.d, a.f, a.experts, a.topk, a.seed):
        print(json.dumps(r))


if __name__ == "__main__":
    main()
