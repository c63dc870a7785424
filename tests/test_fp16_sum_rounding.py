"""The exact attention kernel sums its softmax weights with one fp16 addition
per step (attention.cu add_hh); the reference rounds each step's sum to float
and then to fp16 (templates/attention_op.c.j2).  This test compiles and runs an
exhaustive CPU check that the two agree for every pair of fp16 values."""
import os
import platform
import shutil
import subprocess
import tempfile
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.mark.skipif(platform.machine() not in ("x86_64", "AMD64") or shutil.which("gcc") is None,
                    reason="needs gcc and x86-64 F16C conversions")
def test_fp16_sum_single_rounding_equals_double_rounding():
    with tempfile.TemporaryDirectory() as d:
        exe = Path(d) / "fp16_sum_check"
        flags = ["-O2", "-mf16c", "-fopenmp"]
        r = subprocess.run(["gcc", *flags, str(HERE / "fp16_sum_rounding_check.c"), "-o", str(exe), "-lm"],
                           capture_output=True, text=True)
        if r.returncode != 0:  # no OpenMP runtime: the single-threaded build is the same check
            flags.remove("-fopenmp")
            subprocess.run(["gcc", *flags, str(HERE / "fp16_sum_rounding_check.c"), "-o", str(exe), "-lm"],
                           check=True)
        out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600,
                             env={**os.environ, "OMP_NUM_THREADS": str(os.cpu_count() or 1)})
        checked, bad = map(int, out.stdout.split())
        assert checked == 63490 * 63491 // 2  # unordered pairs of the 65536 - 2 * 1023 non-NaN encodings
        assert bad == 0 and out.returncode == 0
