"""CPU test: the library still compiles for sm_100a with each documented compile-time
alternative switched (the forms that were measured against the defaults and are
kept for re-measurement): plain launches instead of programmatic dependent launch,
one prologue CTA per token, two-tile attention CTAs on small grids, and part of the
exponentials on the FMA pipe.  Compile only (-c), in parallel, into a temporary
directory; nothing is loaded or run."""
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "dirktensor_b200", "csrc", "capi.cu")
VARIANTS = ["-DDT_PDL=0", "-DDT_PROLOGUE_PERSISTENT=0", "-DDT_FLASH_SMALL_GRID_ONE_TILE=0", "-DDT_FLASH_EMU_PAIRS=2"]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    return None


@pytest.mark.timeout(600)
def test_documented_compile_options_build(tmp_path):
    nvcc = _nvcc()
    if nvcc is None:
        pytest.skip("nvcc not found")

    def build(flag):
        out = tmp_path / (flag.strip("-D").replace("=", "_") + ".o")
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
               "--expt-relaxed-constexpr", flag, "-c", "-o", str(out), SRC]
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=500)
        return flag, r.returncode, r.stderr[-1500:]

    with ThreadPoolExecutor(max_workers=len(VARIANTS)) as ex:
        results = list(ex.map(build, VARIANTS))
    failed = [(f, err) for f, rc, err in results if rc != 0]
    assert not failed, failed
