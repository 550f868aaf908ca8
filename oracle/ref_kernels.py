"""The reference's own fused kernels on a B200 (test infrastructure; needs the
binaries oracle/build_ref_kernels.sh builds into oracle/_ref/).

  python -m oracle.ref_kernels time [--warmups 5 --runs 20]   -> JSON line
  python -m oracle.ref_kernels pin                            -> JSON line

`time`: the reference's program (drivers/main.cu + inputs/data.cu +
kernels/<kernel>.cu at its own include/config.h shape: 4 batches x 256
tokens, d=4096, d_ff=16384, E=32, top-4, cf 0.8, all-zero data) for
capacity, capacity_int8_ptx, capacity_int4_ptx and capacity_fp8_ptx, and the
same driver linked against libsparsemoe_b200.so (oracle/_ref/profile_b200)
with the same --kernel flag.  Both print the reference launcher's
"Total duration via cudaEventRecord" line per solve() call (kernels/launcher.h:
event before the launch, after cudaDeviceSynchronize); the median of the
timed runs is reported.  The reference's fused kernels compute only part of
the layer (their grids cover N rows and d_model columns of every GEMM), so
their times are for that partial work.

`pin`: each fused kernel at a one-thread-block shape (oracle/ref_pin.cu:
N=16, d=f=64, E=16, top-1, CAP=16; every token forced to expert 0 by a large
first feature) on seeded inputs in its format, against the oracle's
restatement of that format on the same quantised operands, over the 8 tokens
the kernel routes.  Result per kernel: max-abs-rel and "pinned" (within the
format's bar: 1e-2 fp16, 3e-2 int8 / fp8, 6e-2 int4) or "refuted".
"""
from __future__ import annotations

import argparse
import json
import re
import statistics
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = HERE / "_ref"
KERNELS = ["capacity", "capacity_int8_ptx", "capacity_int4_ptx", "capacity_fp8_ptx"]
_DUR = re.compile(r"Total duration via cudaEventRecord: ([0-9.]+) ms")


def _durations(cmd, timeout=900):
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    ms = [float(m) for m in _DUR.findall(r.stdout)]
    return r.returncode, ms, (r.stdout + r.stderr)[-600:]


def time_kernels(warmups: int, runs: int) -> dict:
    out = {}
    for kern in KERNELS:
        row = {}
        for arm, exe in (("reference", REF / f"ref_{kern}"), ("sparsemoe_b200", REF / "profile_b200")):
            if not exe.exists():
                row[arm] = {"unavailable": f"{exe.name} not built"}
                continue
            rc, ms, tail = _durations([str(exe), f"--kernel={kern}", f"--warmups={warmups}", f"--runs={runs}"])
            timed = ms[warmups:]
            row[arm] = ({"rc": rc, "ms_median": statistics.median(timed), "ms_min": min(timed), "runs": len(timed)}
                        if rc == 0 and timed else {"rc": rc, "tail": tail})
        if "ms_median" in row.get("reference", {}) and "ms_median" in row.get("sparsemoe_b200", {}):
            row["speedup"] = row["reference"]["ms_median"] / row["sparsemoe_b200"]["ms_median"]
        out[kern] = row
    return {"what": "reference fused kernels vs this library, same unmodified drivers/main.cu, reference "
                    "include/config.h shape (B=4, N=256, d=4096, f=16384, E=32, k=4, cf=0.8, zero data)",
            "warmups": warmups, "runs": runs, "kernels": out}


def pin_kernels() -> dict:
    sys.path.insert(0, str(HERE.parent))
    import sparsemoe_b200 as sm
    from oracle import oracle as O
    dtypes = {"capacity": sm.DTYPE_F16, "capacity_int8_ptx": sm.DTYPE_INT8, "capacity_int4_ptx": sm.DTYPE_INT4_PTX,
              "capacity_fp8_ptx": sm.DTYPE_FP8}
    scales = {"capacity": (1.0, 1.0), "capacity_int8_ptx": (0.05, 0.02), "capacity_int4_ptx": (0.6, 0.1),
              "capacity_fp8_ptx": (1.0, 1.0)}
    tol = {"capacity": 1e-2, "capacity_int8_ptx": 3e-2, "capacity_int4_ptx": 6e-2, "capacity_fp8_ptx": 3e-2}
    res = {}
    for kern in KERNELS:
        exe = REF / f"ref_pin_{kern}"
        if not exe.exists():
            res[kern] = {"unavailable": f"{exe.name} not built"}
            continue
        s_in, s_mid = scales[kern]
        cfg = sm.LayerConfig(1, 16, 64, 64, 16, 1, 16.0, dtype=dtypes[kern], act_scale=s_in, mid_scale=s_mid)
        inp = sm.make_inputs(cfg, 7)
        x = inp["x"].copy()
        x[:, 0] = np.float16(4.0).view(np.uint16)          # a large first feature ...
        wr = inp["wr"].copy()
        wr[0, :] = 0
        wr[0, 0] = np.float16(1.0).view(np.uint16)         # ... that only expert 0 reads
        inp["x"], inp["wr"] = x, wr
        with tempfile.TemporaryDirectory() as td:
            tin, tout = Path(td) / "in", Path(td) / "out"
            tin.mkdir()
            tout.mkdir()
            x.tofile(tin / "x.bin")
            wr.tofile(tin / "wr.bin")
            for n in ("wg", "wu", "wd"):
                if cfg.dtype == sm.DTYPE_F16:
                    inp[n].tofile(tin / f"{n}.bin")
                elif cfg.int8:
                    inp[n + "_q"].tofile(tin / f"{n}_i8.bin")
                elif cfg.int4ptx:
                    inp[n + "_q"].tofile(tin / f"{n}_i4.bin")
                else:
                    inp[n + "_q"].tofile(tin / f"{n}_f8.bin")
            if cfg.per_tensor:
                np.array([inp["s_up"], inp["s_gate"], inp["s_down"], inp["s_in"], inp["s_mid"]],
                         np.float32).tofile(tin / "scales.bin")
            r = subprocess.run([str(exe), str(tin), str(tout)], capture_output=True, text=True, timeout=300)
            if r.returncode != 0:
                res[kern] = {"rc": r.returncode, "tail": (r.stdout + r.stderr)[-400:]}
                continue
            idx = np.fromfile(tout / "idx.bin", np.int32)
            ids = np.fromfile(tout / "token_ids.bin", np.int32).reshape(16, 16)
            counts = np.fromfile(tout / "counts.bin", np.int32)
            out = np.fromfile(tout / "out.bin", np.float32).reshape(16, 64)
        ref = O.forward(inp, cfg)
        toks = sorted(int(t) for t in ids[0, : counts[0]] if 0 <= t < 16)
        a, b = out[toks], ref["out"][toks]
        err = float(np.abs(a - b).max() / max(float(np.abs(b).max()), 1e-30))
        res[kern] = {"tokens_compared": toks, "routed_to_expert0": bool((idx[:8] == 0).all()),
                     "max_abs_rel": err, "tolerance": tol[kern],
                     "verdict": "pinned" if err <= tol[kern] and len(toks) == 8 else "refuted"}
    return {"what": "reference fused kernel vs the oracle's restatement, one-thread-block shape N=16 d=f=64 E=16 "
                    "top-1 CAP=16, the 8 tokens the kernel routes", "kernels": res}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["time", "pin"])
    ap.add_argument("--warmups", type=int, default=5)
    ap.add_argument("--runs", type=int, default=20)
    a = ap.parse_args()
    print(json.dumps(time_kernels(a.warmups, a.runs) if a.mode == "time" else pin_kernels()))


if __name__ == "__main__":
    main()
