"""Drop-in check: the reference's unmodified drivers/main.cu, linked against
libsparsemoe_b200.so (oracle/build_ref_driver.sh), runs its own workload (its
include/config.h shape, all-zero data) through our solve() and builder."""
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

EXE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "profile_b200"


def test_reference_driver_runs_unchanged(gpu):
    if not EXE.exists():
        pytest.skip("reference driver not built (needs the reference sources at build time)")
    r = subprocess.run([str(EXE), "--kernel=capacity", "--warmups=1", "--runs=2"], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("Total duration via cudaEventRecord:") == 3
    assert "Profiling is complete." in r.stdout


@pytest.mark.parametrize("kernel", ["capacity_int8_ptx", "capacity_int4_ptx", "capacity_fp8_ptx"])
def test_reference_driver_quantised_kernels(gpu, kernel):
    """The driver's other KERNEL variants (drivers/main.cu:84-106 picks their
    allocators): solve() takes the int8, packed-transposed int4 and e4m3
    weight fields those allocators fill."""
    if not EXE.exists():
        pytest.skip("reference driver not built (needs the reference sources at build time)")
    r = subprocess.run([str(EXE), f"--kernel={kernel}", "--warmups=1", "--runs=2"], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("Total duration via cudaEventRecord:") == 3
    assert "Profiling is complete." in r.stdout
