"""C-ABI checks that need no GPU: the library loads, exports every function
include/*.h declares, and struct MoEArgs has the reference's byte layout."""
import ctypes
import json
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))

import sparsemoe_b200 as sm  # noqa: E402


def declared_c_functions():
    text = (ROOT / "include" / "sparsemoe_b200.h").read_text()
    text = re.sub(r"//[^\n]*", "", text)
    return sorted(set(re.findall(r"^\s*(?:[A-Za-z_][\w\s\*]*?[\s\*])([a-z_][a-z0-9_]*)\s*\(", text, re.M)))


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(sm.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_library_loads_without_gpu():
    assert sm.LIB_PATH.exists()
    assert sm.capacity(512, 2, 8, 1.25) == 160


def test_every_declared_c_symbol_is_exported():
    names = declared_c_functions()
    assert "solve" in names and "moe_solve_v2" in names and "moe_solve_v2_noalloc" in names
    syms = exported()
    missing = [n for n in names if n not in syms]
    assert not missing, f"declared but not exported: {missing}"
    for n in names:
        getattr(sm.lib, n)   # and resolvable through ctypes


def test_builder_cxx_symbols_are_exported():
    """inputs/data.h functions (C++ linkage, the reference's signatures)."""
    out = subprocess.run(["nm", "-DC", "--defined-only", str(sm.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    text = (ROOT / "include" / "data.h").read_text()
    for name in re.findall(r"^(?:MoEArgs|void)\s+(\w+)\(", text, re.M):
        assert re.search(rf"\b{name}\(", out), f"{name} not exported"


def test_moeargs_layout_matches_reference():
    import make_layout
    golden = json.loads((ROOT / "tests" / "golden" / "moe_args_layout.json").read_text())
    ours = make_layout.layout(ROOT / "include")
    assert ours == golden
    # and the ctypes mirror agrees
    assert ctypes.sizeof(sm.MoEArgs) == golden["sizeof"]
    for name, off, size in golden["fields"]:
        assert getattr(sm.MoEArgs, name).offset == off, name
        assert getattr(sm.MoEArgs, name).size == size, name


def test_invalid_dims_rejected_on_cpu():
    d = sm.LayerConfig(1, 64, 200, 128, 8, 2, 1.25).dims()
    assert sm.lib.moe_workspace_bytes(ctypes.byref(d)) == 0
    a = sm.MoEArgs()
    assert sm.lib.moe_solve_v2(ctypes.byref(a), ctypes.byref(d), None) == sm.MOE_ERR_UNSUPPORTED
    d = sm.LayerConfig(1, 64, 256, 128, 8, 9, 1.25).dims()    # top_k > E
    assert sm.lib.moe_solve_v2(ctypes.byref(a), ctypes.byref(d), None) == sm.MOE_ERR_INVALID_ARG
    assert "top_k" in sm.last_error()


def test_null_buffers_rejected():
    d = sm.LayerConfig(1, 64, 256, 128, 8, 2, 1.25).dims()
    a = sm.MoEArgs()
    assert sm.lib.moe_solve_v2(ctypes.byref(a), ctypes.byref(d), None) == sm.MOE_ERR_INVALID_ARG
    assert sm.lib.moe_solve_v2_noalloc(ctypes.byref(a), ctypes.byref(d), None) == sm.MOE_ERR_INVALID_ARG


def test_solve_dims_roundtrip_defaults_to_reference_config():
    d = sm.MoeDims()
    assert sm.lib.moe_get_solve_dims(ctypes.byref(d)) == 0
    # reference include/config.h: N=256, d_model=4096, B=4, E=32, k=4, up_proj_dim=4, cf=0.8
    assert (d.num_batches, d.tokens, d.d_model, d.d_ff, d.num_experts, d.top_k) == (4, 256, 4096, 16384, 32, 4)
    assert abs(d.capacity_factor - 0.8) < 1e-7


@pytest.mark.parametrize("N,k,E,cf,cap", [
    (256, 4, 32, 0.8, 32),        # reference include/config.h -> CAP 32
    (512, 2, 8, 1.25, 160),       # config 1
    (2048, 2, 8, 1.25, 640),      # Mixtral, per batch
    (16384, 6, 64, 1.0, 1536),    # INT8 config
    (32768, 8, 128, 1.25, 2560),  # FP8 config
    (4096, 8, 256, 1.25, 160),    # DeepSeek-V3 decode (global)
    (65536, 8, 256, 1.25, 2560),  # DeepSeek-V3 prefill (global)
    (1, 1, 8, 1.0, 16),
    (0, 2, 8, 1.0, 0),
])
def test_capacity_formula(N, k, E, cf, cap):
    """inputs/data.cu:392-398: round_up((int)ceilf((float)N*(float)k/(float)E*cf), 16)."""
    import numpy as np
    v = np.float32(np.float32(np.float32(N) * np.float32(k)) / np.float32(E)) * np.float32(cf)
    expect = ((int(np.ceil(np.float32(v))) + 15) // 16) * 16
    assert expect == cap
    assert sm.capacity(N, k, E, cf) == cap
