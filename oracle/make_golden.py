"""Golden vectors from the reference's own GPU code (test infrastructure).

On a B200 box (the binaries were built from the reference sources by
oracle/build_ref.sh and travel in oracle/_ref/):

    python oracle/make_golden.py <out_dir>

For each config below it generates the seeded inputs with the library's
generator, runs oracle/_ref/ref_unfused_<name> (the reference's
kernels/unfused.cu multi-launch path: no capacity drop, fp16, --use_fast_math)
and writes <out_dir>/ref_unfused_<name>.npz with the reference's logits,
top-k indices and weights, expert counts and a strided subset of output rows.
The .npz files are committed under tests/golden/.
"""
from __future__ import annotations

import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

# name: (B, N, d, f, E, k, seed, output-row stride)
CONFIGS = {
    "k2": (2, 256, 512, 1024, 16, 2, 0, 4),
    "k4": (2, 128, 256, 1024, 32, 4, 1, 1),
}


def layer_config(name):
    import sparsemoe_b200 as sm
    B, N, d, f, E, k, seed, stride = CONFIGS[name]
    return sm.LayerConfig(B, N, d, f, E, k, 1.0, cap=-1), seed, stride


def run(name: str, out_dir: Path) -> Path:
    import sparsemoe_b200 as sm
    cfg, seed, stride = layer_config(name)
    inp = sm.make_inputs(cfg, seed)
    exe = ROOT / "oracle" / "_ref" / f"ref_unfused_{name}"
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        for key, fn in (("x", "x"), ("wr", "wr"), ("wg", "wg"), ("wu", "wu"), ("wd", "wd")):
            np.ascontiguousarray(inp[key]).tofile(td / f"{fn}.bin")
        r = subprocess.run([str(exe), str(td), str(td)], capture_output=True, text=True, timeout=120)
        if r.returncode != 0:
            raise RuntimeError(f"{exe.name} failed: {r.stdout}\n{r.stderr}")
        T, E, k, d = cfg.T, cfg.num_experts, cfg.top_k, cfg.d_model
        out = np.fromfile(td / "out.bin", np.float32).reshape(T, d)
        rows = np.arange(0, T, stride)
        res = {
            "logits": np.fromfile(td / "logits.bin", np.float32).reshape(T, E),
            "idx": np.fromfile(td / "idx.bin", np.int32).reshape(T, k),
            "w": np.fromfile(td / "w.bin", np.float32).reshape(T, k),
            "counts": np.fromfile(td / "counts.bin", np.int32).reshape(cfg.num_batches, E),
            "out_rows": rows.astype(np.int32),
            "out": out[rows],
            "meta": np.array(CONFIGS[name], np.int64),
            "stdout": np.array(r.stdout),
        }
    out_dir.mkdir(parents=True, exist_ok=True)
    path = out_dir / f"ref_unfused_{name}.npz"
    np.savez_compressed(path, **res)
    return path


if __name__ == "__main__":
    od = Path(sys.argv[1] if len(sys.argv) > 1 else "golden_out")
    for n in CONFIGS:
        print(run(n, od))
