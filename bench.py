#!/usr/bin/env python
"""Benchmark of the capacity-routed MoE layer (BASELINE metric: MoE-layer tokens/s).

Default workload (fits one B200): Mixtral-8x7B-shape layer
in bf16, num_batches=8 x N=2048 tokens (T=16384), d_model=4096, d_ff=14336,
E=8, top-2, capacity_factor=1.25 (CAP=640 per batch).  One step = one full
layer call (router, top-k, dispatch, up/gate GEMM + SwiGLU, down GEMM,
combine) over the T tokens.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N>1 runs under torchrun: every rank runs its own replica of the layer on its
own tokens (no collective on the data path), value = all tokens / max-over-
ranks time.  `--impl reference` times the CPU transcription of the reference's
five stages (oracle/, rank 0 only) on a bounded token sample.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
STAGES = ["router_topk", "dispatch", "expert_up_gate_gemm", "expert_down_gemm", "combine"]
def kernels_per_step(cfg) -> int:
    """Kernels one layer call launches: router (+ the block fold / top-k pass of
    the many-expert routers, E >= 64), dispatch x4 (count, scan, assign,
    gather), up/gate GEMM, down GEMM, combine."""
    blocked = cfg.num_experts >= 64 and cfg.num_experts % 32 == 0
    return 8 + (1 if blocked else 0)


# workloads whose batches are split over the ranks under expert parallelism (global CAP)
GLOBAL_BATCH = {"ds3_int4_decode", "ds3_int4_prefill", "ds3_nvfp4_decode", "ds3_nvfp4_prefill"}


def load_config_module():
    """sparsemoe_b200/config.py loaded by path: LayerConfig and the format
    codes without importing the package (which loads libsparsemoe_b200.so).
    CAP comes from the CPU oracle's restatement of the reference formula."""
    import importlib.util
    from oracle import oracle as O
    spec = importlib.util.spec_from_file_location("_smoe_config", ROOT / "sparsemoe_b200" / "config.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod            # dataclasses resolve annotations through sys.modules
    spec.loader.exec_module(mod)
    mod.set_capacity_fn(O.capacity)
    return mod


def workload(name: str, sm=None):
    """The named workload as a LayerConfig of `sm` (default: the package)."""
    if sm is None:
        import sparsemoe_b200 as sm
    table = {
        "mixtral_bf16": sm.LayerConfig(8, 2048, 4096, 14336, 8, 2, 1.25, dtype=sm.DTYPE_BF16),
        "mixtral_fp16": sm.LayerConfig(8, 2048, 4096, 14336, 8, 2, 1.25, dtype=sm.DTYPE_F16),
        "small_fp16": sm.LayerConfig(1, 512, 1024, 2048, 8, 2, 1.25, dtype=sm.DTYPE_F16),
        # Mixtral weights with one 2048-token batch: the small case for ncu captures.
        "mixtral_t2048": sm.LayerConfig(1, 2048, 4096, 14336, 8, 2, 1.25, dtype=sm.DTYPE_BF16),
        # BASELINE configs[2] shape in the reference's int8 format (per-tensor int8 weights and
        # activations, kernels/capacity_int8_ptx.cu), Zipf(1.1) router bias so hot experts drop routes.
        "int8_cfg3": sm.LayerConfig(1, 16384, 2048, 1408, 64, 6, 1.0, dtype=sm.DTYPE_INT8, zipf_s=1.1),
        # BASELINE configs[2] in its own format: per-output-channel int8 weights, per-token int8 x
        # (h per token and 128-feature block), same shape and Zipf(1.1) bias.
        "int8ch_cfg3": sm.LayerConfig(1, 16384, 2048, 1408, 64, 6, 1.0, dtype=sm.DTYPE_INT8_CHANNEL, zipf_s=1.1),
        # FP8 e4m3, 128x128 weight / 1x128 activation block scales.
        "fp8_cfg4": sm.LayerConfig(1, 32768, 2048, 768, 128, 8, 1.25, dtype=sm.DTYPE_FP8_BLOCK),
        # BASELINE configs[4], one GPU's share under 8-way expert parallelism: 32 experts, top-8 over them
        # gives the same per-GPU routes and CAP as the global 256-expert routing (decode 160, prefill 2560).
        "w4_cfg5_decode": sm.LayerConfig(1, 512, 7168, 2048, 32, 8, 1.25, dtype=sm.DTYPE_W4A16, router_f32=True,
                                         zipf_s=1.0),
        "w4_cfg5_prefill": sm.LayerConfig(1, 8192, 7168, 2048, 32, 8, 1.25, dtype=sm.DTYPE_W4A16, router_f32=True,
                                          zipf_s=1.0),
        # the same two shapes with config 5's other weight format, NVFP4 (e2m1, e4m3 scale per 16 K-rows)
        "nvfp4_cfg5_decode": sm.LayerConfig(1, 512, 7168, 2048, 32, 8, 1.25, dtype=sm.DTYPE_NVFP4,
                                            router_f32=True, zipf_s=1.0),
        "nvfp4_cfg5_prefill": sm.LayerConfig(1, 8192, 7168, 2048, 32, 8, 1.25, dtype=sm.DTYPE_NVFP4,
                                             router_f32=True, zipf_s=1.0),
        # BASELINE configs[4] as the whole expert-parallel layer: E = 256 over the GPUs, 512 (decode) or
        # 8192 (prefill) tokens per GPU; under torchrun the batch of N x tokens is split over the ranks
        # and CAP / drops are global (GLOBAL_BATCH).  On one GPU: all 256 experts, its own tokens.
        "ds3_int4_decode": sm.LayerConfig(1, 512, 7168, 2048, 256, 8, 1.25, dtype=sm.DTYPE_W4A16,
                                          router_f32=True, zipf_s=1.0),
        "ds3_int4_prefill": sm.LayerConfig(1, 8192, 7168, 2048, 256, 8, 1.25, dtype=sm.DTYPE_W4A16,
                                           router_f32=True, zipf_s=1.0),
        # the reference's own include/config.h shape (4 batches x 256 tokens, d=4096, d_ff=16384, E=32,
        # top-4, cf=0.8, CAP=32) in its four kernels' formats, with seeded data and the builder's scales
        "refcfg_fp16": sm.LayerConfig(4, 256, 4096, 16384, 32, 4, 0.8, dtype=sm.DTYPE_F16),
        "refcfg_int8": sm.LayerConfig(4, 256, 4096, 16384, 32, 4, 0.8, dtype=sm.DTYPE_INT8),
        "refcfg_int4": sm.LayerConfig(4, 256, 4096, 16384, 32, 4, 0.8, dtype=sm.DTYPE_INT4_PTX),
        "refcfg_fp8": sm.LayerConfig(4, 256, 4096, 16384, 32, 4, 0.8, dtype=sm.DTYPE_FP8),
        "ds3_nvfp4_decode": sm.LayerConfig(1, 512, 7168, 2048, 256, 8, 1.25, dtype=sm.DTYPE_NVFP4,
                                           router_f32=True, zipf_s=1.0),
        "ds3_nvfp4_prefill": sm.LayerConfig(1, 8192, 7168, 2048, 256, 8, 1.25, dtype=sm.DTYPE_NVFP4,
                                            router_f32=True, zipf_s=1.0),
    }
    return table[name]


def profiled_traffic(config: str):
    """DRAM bytes of one up/gate launch for this workload from the ncu table in
    profiles/traffic.md (None when no capture exists)."""
    tf = ROOT / "profiles" / "traffic.md"
    if not tf.exists():
        return None
    for line in tf.read_text().splitlines():
        cells = [c.strip() for c in line.strip().strip("|").split("|")]
        if len(cells) >= 3 and cells[0] == config:
            try:
                return float(cells[2])
            except ValueError:
                return None
    return None


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


_PEAK8_CACHE: dict = {}


def measure_8bit_peak(kind: str, dev=None):
    """Dense 8-bit tensor TFLOP/s measured here the way the bf16 figures are
    (a cuBLAS GEMM, M = N = K = 8192): `kind` "e4m3" runs torch._scaled_mm on
    e4m3 operands, "int8" torch._int_mm.  Returns (burst, sustained, note):
    burst = best of 10 trials of 10 back-to-back GEMMs, sustained = one ~1 s
    loop.  Measured once per process; None figures if the library refuses
    the shape."""
    if kind in _PEAK8_CACHE:
        return _PEAK8_CACHE[kind]
    import torch
    dev = dev or torch.device("cuda", torch.cuda.current_device())
    n = 8192
    g = torch.Generator(device=dev).manual_seed(0)
    try:
        if kind == "e4m3":
            a = torch.randn(n, n, device=dev, generator=g).to(torch.float8_e4m3fn)
            b = torch.randn(n, n, device=dev, generator=g).to(torch.float8_e4m3fn).t()   # column-major
            one = torch.ones((), device=dev)
            op = lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)  # noqa: E731
            what = "cuBLAS e4m3 GEMM (torch._scaled_mm, bf16 out)"
        else:
            a = torch.randint(-127, 128, (n, n), device=dev, dtype=torch.int8, generator=g)
            b = torch.randint(-127, 128, (n, n), device=dev, dtype=torch.int8, generator=g).t()
            op = lambda: torch._int_mm(a, b)  # noqa: E731
            what = "cuBLAS int8 GEMM (torch._int_mm, s32 out)"
        for _ in range(3):
            op()
        torch.cuda.synchronize(dev)
        flop = 2.0 * n ** 3
        best = 0.0
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                op()
            e1.record()
            e1.synchronize()
            best = max(best, 10 * flop / (e0.elapsed_time(e1) * 1e-3) / 1e12)
        reps = max(10, int(1.0 / (flop / (best * 1e12))))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            op()
        e1.record()
        e1.synchronize()
        sus = reps * flop / (e0.elapsed_time(e1) * 1e-3) / 1e12
        res = (best, sus, f"measured in this process: {what} at {n}^3, burst best of 10 x 10 launches, "
                          f"sustained one {reps}-launch loop")
        del a, b
    except Exception as e:   # noqa: BLE001 (no 8-bit GEMM in this build of the library)
        res = (None, None, f"8-bit GEMM not measurable here ({type(e).__name__}: {str(e)[:80]})")
    _PEAK8_CACHE[kind] = res
    return res


def eight_bit_kind(cfg):
    """The tensor-core kind an 8-bit format runs on: "e4m3" (kind::f8f6f4) or
    "int8" (kind::i8); None for the 16-bit MMAs."""
    if cfg.fp8 or cfg.fp8pt:
        return "e4m3"
    if cfg.int8 or cfg.int8ch or cfg.int4ptx:
        return "int8"
    return None


def tensor_peaks(peaks, eight_bit, dev=None):
    """(burst, sustained, note) dense tensor TFLOP/s for the roofline: the
    driver-measured bf16 figures for the 16-bit MMAs; for an 8-bit kind
    ("e4m3" / "int8") the cuBLAS 8-bit GEMM measured here, or twice the bf16
    figures if that cannot run."""
    burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    sus = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    if not eight_bit:
        return burst, sus, "bf16_tflops (cuBLAS bf16 burst)"
    kind = eight_bit if isinstance(eight_bit, str) else "e4m3"
    b8, s8, note = measure_8bit_peak(kind, dev)
    if b8:
        return b8, s8, note
    return 2 * burst, 2 * sus, f"2 x bf16_tflops burst ({note})"


def dtype_name(cfg):
    if cfg.nvfp4:
        return "nvfp4_g16_weights_bf16_act"
    if cfg.w4:
        return "int4_g128_weights_bf16_act"
    if cfg.int8ch:
        return "int8_channel_token"
    if cfg.int4ptx:
        return "int4_per_tensor"
    if cfg.fp8pt:
        return "fp8_e4m3_per_tensor"
    return "int8" if cfg.int8 else ("fp8_e4m3_block" if cfg.fp8 else ("bf16" if cfg.bf16 else "f16"))


def cfg_json(name, cfg, cap):
    wb = 0.5 if (cfg.w4 or cfg.int4ptx) else (1 if (cfg.int8 or cfg.int8ch or cfg.fp8 or cfg.fp8pt) else 2)
    xb = cfg.T * cfg.d_model * 2 / 1e6
    wmb = 3 * cfg.num_experts * cfg.d_model * cfg.d_ff * wb / 1e9
    return {"workload": name, "num_batches": cfg.num_batches, "tokens_per_batch": cfg.tokens,
            "tokens": cfg.T, "d_model": cfg.d_model, "d_ff": cfg.d_ff, "experts": cfg.num_experts,
            "top_k": cfg.top_k, "capacity_factor": cfg.capacity_factor, "cap": cap, "zipf_s": cfg.zipf_s,
            "l2": (f"inputs larger than L2 (x {xb:.0f} MB, weights {wmb:.2f} GB; no flush needed)"
                   if xb + wmb * 1e3 > 126 else
                   f"inputs smaller than L2 (x {xb:.0f} MB, weights {wmb * 1e3:.0f} MB): L2-resident between "
                   f"steps, not flushed")}


def parallelism_desc(args, cfg, ws, cap, mode) -> str:
    """config.parallelism of a run (the same text on both arms)."""
    if ws == 1:
        return "single GPU"
    if mode != "ep":
        return f"{ws} independent replicas (no data-path collective)"
    glob = args.config in GLOBAL_BATCH
    placement = "strided" if glob and args.ep_transport == "peer" else "contiguous"
    return (f"ep{ws} (expert parallel, {cfg.num_experts // ws} experts per GPU, "
            + ("rows over NVLink peer memory: gather kernels store the rows into the owners, down-GEMM "
               "epilogue stores the results into the senders' buffers; " if args.ep_transport == "peer" else
               f"NCCL all-to-all dispatch/return on a second stream, {args.ep_chunks} pipelined batch chunks; ")
            + f"{cfg.T} tokens per GPU"
            + (f"; each batch split over the {ws} ranks, global CAP {cap}, {placement} expert ownership)"
               if glob else ", per-rank batches)"))


def run_cap(args, cfg, ws, mode) -> int:
    """CAP of the run: per batch, or of the whole split batch under EP with global batches."""
    if ws > 1 and mode == "ep" and args.config in GLOBAL_BATCH and cfg.cap == 0:
        from oracle import oracle as O
        return O.capacity(cfg.tokens * ws, cfg.top_k, cfg.num_experts, cfg.capacity_factor)
    return cfg.capacity()


# ---------------------------------------------------------------------------
def init_dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl" if os.environ.get("BENCH_BACKEND", "nccl") == "nccl" else "gloo")
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, ws: int, device) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.f is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
def quantise_weights(cfg, dev, g, E, wdict):
    """Seeded 16-bit weights (gate/up ~ N(0,1/sqrt(d)), down ~ N(0,1/sqrt(f)))
    generated on the device and quantised there by the library's device
    quantisers (bit-identical to the host ones).  Fills wdict with the
    quantised tensors: wg/wu/wd plus w_scale (FP8 / int8 per channel), w4
    (INT4 scales+zeros, NVFP4 scales) and fp4g (NVFP4 globals)."""
    import torch
    import sparsemoe_b200 as sm
    d, f = cfg.d_model, cfg.d_ff
    t16 = torch.bfloat16 if cfg.act_bf16 else torch.float16
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    ws, w4s, w4z, fp4g = [], [], [], []
    for name, (K, N) in (("wg", (d, f)), ("wu", (d, f)), ("wd", (f, d))):
        w16 = torch.empty(E, K, N, dtype=t16, device=dev).normal_(0.0, K ** -0.5, generator=g)
        bf = int(cfg.act_bf16)
        if not (cfg.fp8 or cfg.int8ch or cfg.w4):
            wdict[name] = w16
            continue
        if cfg.fp8:
            q = torch.empty(E, K, N, dtype=torch.uint8, device=dev)
            sc = torch.empty(E, K // 128, N // 128, dtype=torch.float32, device=dev)
            rc = sm.lib.moe_quantize_fp8_blocks_device(p(w16), E, K, N, bf, p(q), p(sc), st)
            ws.append(sc)
        elif cfg.int8ch:
            q = torch.empty(E, K, N, dtype=torch.int8, device=dev)
            sc = torch.empty(E, N, dtype=torch.float32, device=dev)
            rc = sm.lib.moe_quantize_int8_channel_device(p(w16), E, K, N, bf, p(q), p(sc), st)
            ws.append(sc)
        elif cfg.nvfp4:
            q = torch.empty(E, K, N // 2, dtype=torch.uint8, device=dev)
            sc = torch.empty(E, K // 16, N, dtype=torch.uint8, device=dev)
            gl = torch.empty(E, dtype=torch.float32, device=dev)
            rc = sm.lib.moe_quantize_nvfp4_device(p(w16), E, K, N, bf, p(q), p(sc), p(gl), st)
            w4s.append(sc)
            fp4g.append(gl)
        else:
            q = torch.empty(E, K, N // 2, dtype=torch.uint8, device=dev)
            sc = torch.empty(E, K // 128, N, dtype=torch.int16, device=dev)
            zr = torch.empty_like(sc)
            rc = sm.lib.moe_quantize_int4_g128_device(p(w16), E, K, N, bf, p(q), p(sc), p(zr), st)
            w4s.append(sc)
            w4z.append(zr)
        sm.check(rc)
        wdict[name] = q
        del w16
    if ws:
        wdict["w_scale"] = ws
    if w4s:
        wdict["w4"] = w4s + w4z
    if fp4g:
        wdict["fp4g"] = fp4g
    torch.cuda.synchronize(dev)


def device_inputs(layer, seed: int):
    """Seeded synthetic inputs generated on the device: x ~ N(0,1), router
    ~ N(0,0.02) (+ the Zipf popularity bias), weights as quantise_weights."""
    import torch
    import sparsemoe_b200 as sm
    cfg = layer.cfg
    if cfg.per_tensor:
        # the reference's per-tensor formats (int8, packed int4, e4m3): host generator + host quantisers
        layer.host_inputs = sm.make_inputs(cfg, seed)
        layer.load(layer.host_inputs)
        return
    g = torch.Generator(device=layer.device)
    g.manual_seed(seed)
    layer.x.normal_(0.0, 1.0, generator=g)
    layer.wr.normal_(0.0, 0.02, generator=g)
    if cfg.zipf_s > 0:
        layer.bias = torch.from_numpy(sm.zipf_bias(cfg.num_experts, cfg.zipf_s)).to(layer.device)
    wd = {}
    quantise_weights(cfg, layer.device, g, cfg.num_experts, wd)
    for n in ("wg", "wu", "wd"):
        getattr(layer, n).copy_(wd[n].view(getattr(layer, n).dtype))
    if "w_scale" in wd:
        layer.wscale = wd["w_scale"]
    if "w4" in wd:
        layer.w4sz = wd["w4"]
    if "fp4g" in wd:
        layer.fp4g = wd["fp4g"]
    layer.host_inputs = None


def host_inputs_from_device(layer) -> dict:
    """The layer's device inputs as the host dict the oracle reads."""
    import numpy as np
    import torch
    cfg = layer.cfg
    u16 = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    inp = {"x": u16(layer.x)[: cfg.T], "wr": layer.wr.cpu().numpy() if cfg.router_f32 else u16(layer.wr),
           "bias": None if layer.bias is None else layer.bias.cpu().numpy()}
    quant = cfg.fp8 or cfg.int8ch or cfg.w4
    for n in ("wg", "wu", "wd"):
        t = getattr(layer, n)
        inp[n + ("_q" if quant else "")] = t.cpu().numpy() if quant else u16(t)
    if cfg.channel_scaled:
        inp["sg"], inp["su"], inp["sd"] = (t.cpu().numpy() for t in layer.wscale)
    if cfg.nvfp4:
        inp["wg_s"], inp["wu_s"], inp["wd_s"] = (t.cpu().numpy() for t in layer.w4sz)
        inp["wg_g"], inp["wu_g"], inp["wd_g"] = (t.cpu().numpy() for t in layer.fp4g)
    elif cfg.w4:
        v = [t.cpu().numpy().view(np.uint16) for t in layer.w4sz]
        inp["wg_s"], inp["wu_s"], inp["wd_s"], inp["wg_z"], inp["wu_z"], inp["wd_z"] = v
    return inp


def pipelined_e2e(layer, stream, x_host, out_host, K, warmup, dev, set_io=None) -> float:
    """ms per step of K layer calls with every step's tokens copied in from
    pinned host memory and its 16-bit output copied back, the copies on a
    second stream with two device buffers each, so that step i's compute
    overlaps step i+1's input copy and step i-1's output copy.  The timed
    region starts before the first input copy and ends after the last output
    copy."""
    import torch
    copy = torch.cuda.Stream(dev)
    xs = [layer.x, torch.empty_like(layer.x)]
    outs = [layer.out16, torch.empty_like(layer.out16)]
    hosts = [out_host, torch.empty_like(out_host).pin_memory()]
    x0, o0 = layer.x, layer.out16
    if set_io is None:
        def set_io(xb, ob):
            layer.x, layer.out16 = xb, ob

    def run(n, e_start=None, e_end=None):
        h2d_done = [torch.cuda.Event(), torch.cuda.Event()]
        fwd_done = [torch.cuda.Event(), torch.cuda.Event()]
        if e_start is not None:
            e_start.record(stream)
        copy.wait_stream(stream)
        for b in range(min(2, n)):                     # the first two steps' tokens
            with torch.cuda.stream(copy):
                xs[b].copy_(x_host, non_blocking=True)
            h2d_done[b].record(copy)
        for i in range(n):
            b = i & 1
            stream.wait_event(h2d_done[b])
            set_io(xs[b], outs[b])
            layer.forward(stream)
            fwd_done[b].record(stream)
            copy.wait_event(fwd_done[b])
            with torch.cuda.stream(copy):
                hosts[b].copy_(outs[b], non_blocking=True)
                if i + 2 < n:                          # step i+2's tokens into the buffer step i read
                    xs[b].copy_(x_host, non_blocking=True)
            h2d_done[b].record(copy)
        stream.wait_stream(copy)
        if e_end is not None:
            e_end.record(stream)

    run(max(warmup, 1))
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run(K, e0, e1)
    torch.cuda.synchronize(dev)
    set_io(x0, o0)
    return e0.elapsed_time(e1) / K


def oracle_measure(inp: dict, cfg, cap: int, sample_tokens: int, nthreads: int):
    """The oracle (CPU transcription of the reference's five stages) on a
    bounded sample of host inputs: routing of all T tokens, expert FFN +
    combine of the first S tokens.  tokens/s = S / (t_ffn(S) + t_route(T) * S / T).
    Returns (tokens/s, t_route, t_ffn, S)."""
    from oracle import oracle as O
    t0 = time.perf_counter()
    r = O.route(inp["x"], inp["wr"], inp.get("bias"), cfg.num_batches, cfg.tokens, cfg.d_model, cfg.num_experts,
                cfg.top_k, cap, cfg.act_bf16, cfg.router_f32, nthreads)
    t_route = time.perf_counter() - t0
    S = min(sample_tokens, cfg.T)
    fn = O.ffn_combine_fp8 if cfg.fp8 else (O.ffn_combine_int8 if cfg.int8 else
                                            (O.ffn_combine_nvfp4 if cfg.nvfp4 else
                                             O.ffn_combine_w4 if cfg.w4 else
                                             (O.ffn_combine_int8ch if cfg.int8ch else
                                              (O.ffn_combine_per_tensor if (cfg.int4ptx or cfg.fp8pt) else None))))
    t0 = time.perf_counter()
    if fn is not None:
        fn(inp["x"], inp, cfg, r["idx"], r["w"], r["route_slot"], 0, S, nthreads)
    else:
        O.ffn_combine(inp["x"], inp["wg"], inp["wu"], inp["wd"], cfg.num_batches, cfg.tokens, cfg.d_model,
                      cfg.d_ff, cfg.num_experts, cfg.top_k, cfg.bf16, r["idx"], r["w"], r["route_slot"], 0, S,
                      nthreads)
    t_ffn = time.perf_counter() - t0
    return S / (t_ffn + t_route * S / max(cfg.T, 1)), t_route, t_ffn, S


def cpu_measure(layer, sample_tokens: int, nthreads: int):
    """cpu_baseline of our own line: the oracle on this layer's own inputs."""
    if getattr(layer, "host_inputs", None) is None:
        layer.host_inputs = host_inputs_from_device(layer)
    return oracle_measure(layer.host_inputs, layer.cfg, layer.cap, sample_tokens, nthreads)


# other BASELINE configs measured after the headline line (one GPU, device time)
OTHER_CONFIGS = ("small_fp16,int8_cfg3,int8ch_cfg3,fp8_cfg4,w4_cfg5_prefill,nvfp4_cfg5_prefill,w4_cfg5_decode,"
                 "ds3_int4_decode")


def measure_other_configs(names, dev, stream, steps: int = 5, warmup: int = 3) -> dict:
    """Device-time of one layer call for each named workload (seeded inputs as
    the headline line; warm-up calls, then `steps` timed calls bracketed by
    CUDA events on the launching stream), with the per-stage split and the
    dominant GEMM's fraction of the measured tensor peak.  A config that fails
    is reported with its error instead of a time."""
    import torch
    import sparsemoe_b200 as sm
    peaks, _ = load_peaks()
    out = {}
    for name in names:
        try:
            cfg = workload(name)
            layer = sm.MoeLayer(cfg, dev, want_logits=True, want_out16=True)
            device_inputs(layer, seed=1000)
            for _ in range(warmup):
                layer.forward(stream)
            layer.sync_check(stream)
            kept = int(layer.counts.sum().item())
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(steps)]
            for row in evs:
                for e in row:
                    e.record(stream)
            torch.cuda.synchronize(dev)
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for i in range(steps):
                arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in evs[i]])
                sm.lib.moe_set_stage_events(arr, 6)
                layer.forward(stream)
            t1.record(stream)
            sm.lib.moe_set_stage_events(None, 0)
            torch.cuda.synchronize(dev)
            layer.sync_check(stream)
            ms = t0.elapsed_time(t1) / steps
            stages = {st: statistics.mean(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(steps))
                      for j, st in enumerate(STAGES)}
            burst, _sus, _note = tensor_peaks(peaks, eight_bit_kind(cfg), dev)
            flop_up = 4.0 * cfg.d_model * cfg.d_ff * kept
            out[name] = {"ms_per_step": ms, "tokens_per_s": cfg.T / (ms * 1e-3), "stages_ms": stages,
                         "dtype": dtype_name(cfg), "kept_routes": kept,
                         "up_gate_frac_of_tensor_burst": flop_up / (stages["expert_up_gate_gemm"] * 1e-3) / 1e12 / burst}
            del layer
            torch.cuda.empty_cache()
        except Exception as e:   # noqa: BLE001 (report and go on to the next config)
            out[name] = {"error": f"{type(e).__name__}: {e}"}
    return out


def run_reference_arm(args, ws, rank, local):
    """`--impl reference`: the reference has no CPU implementation and its GPU
    kernels are not this arm; the CPU transcription of its five stages (oracle/)
    is timed on the host cores, rank 0 only.  Nothing of the product is loaded:
    the workload is described by sparsemoe_b200/config.py (loaded by path),
    drawn and quantised on the host by oracle/inputs.py, and CAP comes from the
    oracle."""
    if rank != 0:
        return
    from oracle import inputs as OI
    cm = load_config_module()
    cfg = workload(args.config, cm)
    mode = args.parallel if args.parallel != "auto" else ("ep" if ws > 1 else "single")
    nthreads = os.cpu_count() or 1
    cap = cfg.capacity()
    inp = OI.make_inputs(cfg, 0)
    for _ in range(args.warmup):
        oracle_measure(inp, cfg, cap, args.ref_sample_tokens, nthreads)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, _, _, S = oracle_measure(inp, cfg, cap, args.ref_sample_tokens, nthreads)
        vals.append(v)
    wall = time.perf_counter() - t0
    value = statistics.mean(vals)
    sample = (f"routing of all {cfg.T} tokens + expert FFN/combine of {S} tokens per step, "
              f"scaled to tokens/s")
    print(json.dumps({
        "impl": "reference", "metric": f"MoE-layer tokens/s ({args.config})", "value": value,
        "unit": "tokens/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * wall / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype_name(cfg),
        "data": "synthetic (seeded normal: x N(0,1), router N(0,0.02), W N(0,1/sqrt(fan_in)); host-drawn)",
        "config": {**cfg_json(args.config, cfg, run_cap(args, cfg, ws, mode)),
                   "parallelism": parallelism_desc(args, cfg, ws, run_cap(args, cfg, ws, mode), mode)},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---------------------------------------------------------------------------
def ep_parity(layer, cfg, ws, rank, dev, glob, int8_full=None):
    """Checks the expert-parallel layer's last call against the single-GPU
    layer on the same tokens and weights: every rank's tokens, router and
    experts are all-gathered, rank 0 runs one MoeLayer over all of them
    (all E experts, all ranks' tokens, the same batches and CAP) and compares
    each rank's expert indices and f32 output rows.  Runs after the timed
    region.  Returns {"idx_equal", "out_equal", "max_abs_rel", ...} on rank 0."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import sparsemoe_b200 as sm

    def gather(t):
        t = t.contiguous()
        b = t.view(torch.uint8)                 # as bytes: NCCL has no int16 (the INT4 scales / zeros)
        out = torch.empty((ws,) + tuple(b.shape), dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(out, b)
        return out.view(t.dtype)

    def experts(t):
        """[e_loc, ...] per rank -> [E, ...] in global expert order."""
        g = gather(t)
        if layer.placement == "strided":        # rank q holds experts q, q + P, ...
            g = g.transpose(0, 1)
        return g.reshape((cfg.num_experts,) + tuple(t.shape[1:]))

    B, N = cfg.num_batches, cfg.tokens
    xs, outs, idxs = gather(layer.x[: cfg.T]), gather(layer.out[: cfg.T]), gather(layer.idx[: cfg.T])
    wts = {n: experts(getattr(layer, n)) for n in ("wg", "wu", "wd")}
    extra = {k: [experts(t) for t in layer.weights[k]] for k in ("w_scale", "w4", "fp4g") if layer.weights.get(k)}
    if rank != 0:
        torch.cuda.synchronize(dev)
        return None
    if glob:     # every batch of P*N tokens split over the ranks in token order
        full = sm.LayerConfig(B, N * ws, cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k, cfg.capacity_factor,
                              cfg.dtype, cfg.router_f32, cfg.zipf_s, layer.cap, cfg.act_scale, cfg.mid_scale)
        order = lambda t: t.reshape(ws, B, N, -1).transpose(0, 1).reshape(B * ws * N, -1)  # noqa: E731
    else:        # per-rank batches, rank-major
        full = sm.LayerConfig(B * ws, N, cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k, cfg.capacity_factor,
                              cfg.dtype, cfg.router_f32, cfg.zipf_s, cfg.cap, cfg.act_scale, cfg.mid_scale)
        order = lambda t: t.reshape(ws * B * N, -1)  # noqa: E731
    single = sm.MoeLayer(full, dev, want_logits=False, want_out16=False)
    if cfg.per_tensor:
        single.load({**int8_full, "x": np.zeros((0, cfg.d_model), np.uint16)} if full.T == 0 else
                    {**int8_full, "x": order(xs).view(torch.int16).cpu().numpy().view(np.uint16)})
    else:
        single.x.copy_(order(xs))
        single.wr.copy_(layer.wr)
        for n in ("wg", "wu", "wd"):
            getattr(single, n).copy_(wts[n])
        single.bias = layer.bias
        if "w_scale" in extra:
            single.wscale = extra["w_scale"]
        if "w4" in extra:
            single.w4sz = extra["w4"]
        if "fp4g" in extra:
            single.fp4g = extra["fp4g"]
    single.forward()
    single.sync_check()
    a, b = order(outs), single.out[: full.T]
    idx_equal = bool(torch.equal(order(idxs), single.idx[: full.T]))
    out_equal = bool(torch.equal(a, b))
    err = float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))
    return {"idx_equal": idx_equal, "out_equal": out_equal, "max_abs_rel": err, "ranks_checked": ws,
            "tokens_checked": full.T,
            "how": "all ranks' tokens and experts gathered; one single-GPU MoeLayer over them on rank 0; "
                   "expert indices and f32 output rows of every rank compared"}


# ---------------------------------------------------------------------------
def run_ep(args, cfg, ws, rank, local, dev):
    """Expert parallelism: every rank holds E/P experts and routes its own T
    tokens (weak scaling); rows cross NVLink twice per layer (NCCL all-to-all)."""
    import torch
    import torch.distributed as dist
    from sparsemoe_b200.ep import ExpertParallelLayer
    import sparsemoe_b200 as sm
    glob = args.config in GLOBAL_BATCH
    # the DeepSeek-V3 workloads own experts strided, so the Zipf-popular low-index experts spread over the ranks
    placement = "strided" if glob and args.ep_transport == "peer" else "contiguous"
    layer = ExpertParallelLayer(cfg, dev, chunks=args.ep_chunks, global_batch=glob, transport=args.ep_transport,
                                placement=placement)
    full = None
    if cfg.per_tensor:
        # the reference's per-tensor formats: host generator + host quantiser (all experts; each
        # rank keeps its own), this rank's tokens
        full = sm.make_inputs(cfg, 5)
        layer.load({**full, "x": sm.make_inputs(cfg, 100 + rank)["x"]})
    else:
        g = torch.Generator(device=dev)
        g.manual_seed(1000 + rank)
        layer.x.normal_(0.0, 1.0, generator=g)
        g.manual_seed(7)                                   # router replicated on every rank
        layer.wr.normal_(0.0, 0.02, generator=g)
        if cfg.zipf_s > 0:
            layer.bias = torch.from_numpy(sm.zipf_bias(cfg.num_experts, cfg.zipf_s)).to(dev)
        g.manual_seed(2000 + rank)                         # this rank's experts, quantised on the device
        quantise_weights(cfg, dev, g, layer.e_loc, layer.weights)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        layer.forward(stream)
    layer.sync_check(stream)
    K = args.steps
    timings = [dict() for _ in range(K)]
    owner_rows = []
    torch.cuda.synchronize(dev)
    barrier(ws)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        for i in range(K):
            layer.forward(stream, timing=timings[i])
        torch.cuda.synchronize(dev)
    barrier(ws)

    def span(tm, a, b):
        return tm[a][0].elapsed_time(tm[b][0])
    ms_local = statistics.mean(span(tm, "start", "end") for tm in timings)
    ms = max_over_ranks(ms_local, ws, dev)
    ffn_ms = statistics.mean(sum(tm["ffn"][2 * j].elapsed_time(tm["ffn"][2 * j + 1])
                                 for j in range(len(tm["ffn"]) // 2)) for tm in timings)
    phase_ms = {"route": statistics.mean(span(tm, "start", "routed") for tm in timings),
                "expert_ffn_compute": ffn_ms,
                "combine_tail": statistics.mean(tm["combine"][-1].elapsed_time(tm["end"][0]) for tm in timings)}
    phase_ms["exposed_exchange"] = ms_local - phase_ms["route"] - ffn_ms - phase_ms["combine_tail"]
    phase_ms["expert_ffn_compute_slowest_rank"] = max_over_ranks(ffn_ms, ws, dev)
    if timings[0].get("dispatch"):    # peer transport: the gather into the owners, part of the exchange
        phase_ms["dispatch_gather"] = statistics.mean(tm["dispatch"][0].elapsed_time(tm["dispatch"][1])
                                                      for tm in timings)
    layer.sync_check(stream)
    # end-to-end: host x in, 16-bit output out, per step
    x_host = torch.empty_like(layer.x, device="cpu").pin_memory()
    x_host.copy_(layer.x)
    out_host = torch.empty_like(layer.out16, device="cpu").pin_memory()
    for _ in range(args.warmup):
        layer.x.copy_(x_host, non_blocking=True)
        layer.forward(stream)
        out_host.copy_(layer.out16, non_blocking=True)
    torch.cuda.synchronize(dev)
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        layer.x.copy_(x_host, non_blocking=True)
        layer.forward(stream)
        out_host.copy_(layer.out16, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(ws)
    serial_ms = max_over_ranks(e0.elapsed_time(e1) / K, ws, dev)

    # the same double-buffered copy stream as the one-GPU line: step i+1's
    # tokens arrive and step i-1's output leaves while step i computes
    def ep_set_io(xb, ob):
        layer.x, layer.out16 = xb, ob
        if layer.n_chunks == 1:
            layer.chunks[0].x, layer.chunks[0].out16 = xb[: cfg.T], ob[: cfg.T]
    barrier(ws)
    pipe_ms = pipelined_e2e(layer, stream, x_host, out_host, K, args.warmup, dev, set_io=ep_set_io)
    e2e_ms = max_over_ranks(pipe_ms, ws, dev)
    barrier(ws)
    # the last call's output against one GPU running all experts on all ranks' tokens (untimed)
    parity = ep_parity(layer, cfg, ws, rank, dev, glob, full)
    barrier(ws)
    peaks, peak_src = load_peaks()
    eight_bit = eight_bit_kind(cfg)
    peak_tf, peak_sus, peak_what = tensor_peaks(peaks, eight_bit, dev)
    owner_rows.append(layer.owner_rows())   # the same tokens every step
    flop_ffn = 6.0 * cfg.d_model * cfg.d_ff * statistics.mean(owner_rows)
    ach = flop_ffn / (phase_ms["expert_ffn_compute"] * 1e-3) / 1e12
    ach_min = max_over_ranks(-ach, ws, dev) * -1.0      # slowest rank
    h2d = x_host.numel() * x_host.element_size()
    d2h = out_host.numel() * out_host.element_size()
    result = {
        "metric": f"MoE-layer tokens/s ({args.config})", "value": ws * cfg.T / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": ws, "steps": K, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype_name(cfg),
        "data": "synthetic (seeded torch normal: x N(0,1), router N(0,0.02), W N(0,1/sqrt(fan_in)))",
        "config": {**cfg_json(args.config, cfg, layer.cap),
                   "parallelism": parallelism_desc(args, cfg, ws, layer.cap, "ep")},
        "roofline": {"bound": "tensor", "achieved": ach_min, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": ach_min / peak_tf, "frac_of_sustained": ach_min / peak_sus, "traffic": None,
                     "kernel": "expert_ffn phase (up/gate + down tcgen05 GEMMs), slowest rank",
                     "peak_source": peak_what if eight_bit else f"{peak_src} {peak_what}"},
        "phases_ms": phase_ms,
        "e2e": {"value": ws * cfg.T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "serial_ms_per_step": serial_ms,
                "path": "ExpertParallelLayer.forward (moe_stage_route / moe_stage_expert_ffn / moe_stage_combine) "
                        "each step, pinned host x in and 16-bit output out every step on a copy stream, "
                        "double-buffered (serial_ms_per_step: copy in, layer, copy out on one stream)"},
        "gpu_launches": kernels_per_step(cfg) * K,
        "clocks": clocks.summary(),
        "ep_parity": parity,
    }
    if rank == 0:
        print(json.dumps(result))
    layer.close()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="mixtral_bf16")
    ap.add_argument("--cpu-sample-tokens", type=int, default=1024)
    ap.add_argument("--ref-sample-tokens", type=int, default=512)
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline measurement")
    ap.add_argument("--also", default=None,
                    help="comma-separated workloads measured after the headline (one GPU); default: the other "
                         "BASELINE configs for the default workload, none otherwise ('' for none)")
    ap.add_argument("--graph", action="store_true",
                    help="also time the layer captured as one CUDA graph (the decode path)")
    ap.add_argument("--parallel", default="auto", choices=["auto", "ep", "replicas"],
                    help="N>1: expert parallelism over NCCL (default) or independent replicas")
    ap.add_argument("--ep-chunks", type=int, default=1, help="pipelined batch chunks in EP mode")
    ap.add_argument("--ep-transport", default="peer", choices=["peer", "nccl"],
                    help="EP rows over NVLink peer memory (copy engines + down-GEMM epilogue stores) or NCCL all-to-all")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.also is None:
        args.also = OTHER_CONFIGS if args.config == "mixtral_bf16" else ""

    ws, rank, local = init_dist()
    if args.impl == "reference":
        run_reference_arm(args, ws, rank, local)
        return

    import torch
    import sparsemoe_b200 as sm
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    cfg = workload(args.config)
    mode = args.parallel if args.parallel != "auto" else ("ep" if ws > 1 else "single")
    if ws > 1 and mode == "ep":
        run_ep(args, cfg, ws, rank, local, dev)
        return
    layer = sm.MoeLayer(cfg, dev, want_logits=True, want_out16=True)
    device_inputs(layer, seed=1000 + rank)
    stream = torch.cuda.current_stream(dev)

    # warm-up (also checks the device status word once)
    for _ in range(args.warmup):
        layer.forward(stream)
    layer.sync_check(stream)
    kept = int(layer.counts.sum().item())

    # ---- device-resident timing with per-stage events ----------------------
    K = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for row in evs:            # torch creates the CUDA event on its first record
        for e in row:
            e.record(stream)
    torch.cuda.synchronize(dev)
    barrier(ws)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(K):
            arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in evs[i]])
            sm.lib.moe_set_stage_events(arr, 6)
            layer.forward(stream)
        end.record(stream)
        sm.lib.moe_set_stage_events(None, 0)
        torch.cuda.synchronize(dev)
    barrier(ws)
    ms_local = start.elapsed_time(end) / K
    ms = max_over_ranks(ms_local, ws, dev)
    stage_ms = {name: statistics.mean(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(K))
                for j, name in enumerate(STAGES)}
    layer.sync_check(stream)

    # ---- end-to-end through the public API with host buffers ---------------
    x_host = torch.empty_like(layer.x, device="cpu").pin_memory()
    x_host.copy_(layer.x)
    out_host = torch.empty_like(layer.out16, device="cpu").pin_memory()
    h2d = x_host.numel() * x_host.element_size()
    d2h = out_host.numel() * out_host.element_size()
    # (a) serial: copy in, layer, copy out, one after the other on one stream
    for _ in range(args.warmup):
        layer.x.copy_(x_host, non_blocking=True)
        layer.forward(stream)
        out_host.copy_(layer.out16, non_blocking=True)
    torch.cuda.synchronize(dev)
    barrier(ws)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        layer.x.copy_(x_host, non_blocking=True)
        layer.forward(stream)
        out_host.copy_(layer.out16, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(ws)
    serial_ms = max_over_ranks(e0.elapsed_time(e1) / K, ws, dev)
    # (b) pipelined: double-buffered x / output on a copy stream, so step i+1's
    # tokens arrive and step i-1's output leaves while step i computes
    pipe_ms = pipelined_e2e(layer, stream, x_host, out_host, K, args.warmup, dev)
    e2e_ms = max_over_ranks(pipe_ms, ws, dev)

    # ---- optional: the layer as one CUDA graph (decode path) ----------------
    graph = None
    if args.graph:
        gstream = torch.cuda.Stream(dev)
        layer.capture(gstream)
        with torch.cuda.stream(gstream):
            for _ in range(args.warmup):
                layer.replay()
            torch.cuda.synchronize(dev)
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(gstream)
            for _ in range(K):
                layer.replay()
            g1.record(gstream)
            torch.cuda.synchronize(dev)
            gms = max_over_ranks(g0.elapsed_time(g1) / K, ws, dev)
            t0 = time.perf_counter()
            for _ in range(K):
                layer.x.copy_(x_host, non_blocking=True)
                layer.replay()
                out_host.copy_(layer.out16, non_blocking=True)
            torch.cuda.synchronize(dev)
            gwall = (time.perf_counter() - t0) * 1e3 / K
        graph = {"ms_per_step": gms, "value": ws * cfg.T / (gms * 1e-3), "unit": "tokens/s",
                 "e2e_wall_ms_per_step": gwall,
                 "path": "MoeLayer.capture -> CUDAGraph.replay (one launch per layer)"}
        layer.sync_check(gstream)

    # ---- roofline of the dominant kernel (up/gate GEMM with fused SwiGLU) --
    peaks, peak_src = load_peaks()
    eight_bit = eight_bit_kind(cfg)
    peak_tf, peak_sus, peak_what = tensor_peaks(peaks, eight_bit, dev)
    peak_note = (f"{peak_src} bf16_tflops (cuBLAS bf16 burst; the timed region is ~20 steps, not a seconds-long "
                 f"loop)" if not eight_bit else peak_what)
    d, f = cfg.d_model, cfg.d_ff
    flop_up = 4.0 * d * f * kept            # gate + up, kept routes only
    flop_down = 2.0 * d * f * kept
    flop_router = 2.0 * cfg.T * d * cfg.num_experts
    ach_up = flop_up / (stage_ms["expert_up_gate_gemm"] * 1e-3) / 1e12
    ach_down = flop_down / (stage_ms["expert_down_gemm"] * 1e-3) / 1e12
    traffic = profiled_traffic(args.config)

    result = {
        "metric": f"MoE-layer tokens/s ({args.config})", "value": ws * cfg.T / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": ws, "steps": K, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype_name(cfg),
        "data": "synthetic (seeded normal: x N(0,1), router N(0,0.02), W N(0,1/sqrt(fan_in)))",
        "config": {**cfg_json(args.config, cfg, layer.cap),
                   "parallelism": parallelism_desc(args, cfg, ws, layer.cap, mode)},
        "roofline": {"bound": "tensor", "achieved": ach_up, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": ach_up / peak_tf, "frac_of_sustained": ach_up / peak_sus, "traffic": traffic,
                     "kernel": "expert_up_gate_gemm (tcgen05, fused SwiGLU)",
                     "peak_source": peak_note},
        "stages_ms": stage_ms,
        "stage_tflops": {"expert_up_gate_gemm": ach_up, "expert_down_gemm": ach_down,
                         "layer_alg": (flop_up + flop_down + flop_router) / (ms * 1e-3) / 1e12},
        "kept_routes": kept,
        "e2e": {"value": ws * cfg.T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "serial_ms_per_step": serial_ms,
                "path": "MoeLayer.forward -> moe_solve_v2 each step, pinned host x in and 16-bit output out "
                        "every step on a copy stream, double-buffered so transfers overlap the neighbouring "
                        "steps' compute (serial_ms_per_step: copy in, layer, copy out on one stream)"},
        "gpu_launches": kernels_per_step(cfg) * K,
        "clocks": clocks.summary(),
    }
    if graph is not None:
        result["graph"] = graph
    if rank == 0 and ws == 1 and not args.no_cpu:
        nthreads = os.cpu_count() or 1
        v, t_route, t_ffn, S = cpu_measure(layer, args.cpu_sample_tokens, nthreads)
        result["cpu_baseline"] = {
            "value": v, "unit": "tokens/s", "cores": nthreads, "kind": "port",
            "sample": f"oracle: routing of all {cfg.T} tokens ({t_route:.2f} s, scaled by S/T) + expert "
                      f"FFN/combine of S={S} tokens ({t_ffn:.2f} s)"}
    if ws == 1 and args.also:
        del layer
        torch.cuda.empty_cache()
        result["other_configs"] = measure_other_configs(args.also.split(","), dev, stream)
    if rank == 0:
        print(json.dumps(result))
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
