"""The reference's own tests for the NF4 path, run unmodified against this package.

``tests/_reference_alias.py`` maps ``stratum.upload`` / ``assign`` / ``stage`` /
``pipeline`` / ``host_staging`` / ``grad_hooks`` / ``nf4_linear`` /
``scheduler`` / ``runtime`` / ``layer_transfer`` to the ``stratum_b200`` modules
that replace them, and the reference's test files run in a child pytest with
that alias loaded.  The checkout is found through ``STRATUM_REFERENCE_DIR``, or
as a ``reference`` directory beside this repository; without one (e.g. on a GPU
box) the test is skipped.  Nothing is written into the checkout (no bytecode,
no pytest cache, a temporary rootdir).

Deselected, by design: the three ``PrepareNF4Tests`` run ``prepare_nf4`` on a
CPU-only machine with bitsandbytes replaced by a fake; this build quantizes
with its own CUDA kernels and has no CPU fallback (the same cases pass on a
GPU through ``tests/test_upload_gpu.py``).  The reference itself skips its
CUDA round-trip test without a GPU.
"""

import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
FILES = [
    "tests/test_upload.py",
    "tests/test_assign.py",
    "tests/test_host_staging.py",
    "tests/test_pipeline_prefetch.py",
    "tests/test_bwd_prefetch.py",
]
CPU_QUANTIZE = [  # prepare_nf4 on the CPU: this build's quantizer is CUDA-only
    "tests/test_upload.py::PrepareNF4Tests::test_prepare_nf4_3d_source_bytes_correct",
    "tests/test_upload.py::PrepareNF4Tests::test_prepare_nf4_stages_2d_frozen_param",
    "tests/test_upload.py::PrepareNF4Tests::test_prepare_nf4_stages_3d_stacked_param_with_original_shape",
]


def _reference_dir():
    cands = []
    if os.environ.get("STRATUM_REFERENCE_DIR"):
        cands.append(Path(os.environ["STRATUM_REFERENCE_DIR"]))
    cands.append(ROOT.parent / "reference")
    for c in cands:
        if (c / "stratum" / "upload.py").is_file() and all((c / f).is_file() for f in FILES):
            return c
    return None


def test_reference_tests_pass_against_this_package(tmp_path):
    ref = _reference_dir()
    if ref is None:
        pytest.skip("no reference checkout (set STRATUM_REFERENCE_DIR)")
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=os.pathsep.join([str(ROOT / "tests"), str(ROOT)]))
    cmd = [sys.executable, "-m", "pytest", "-p", "_reference_alias", "-p", "no:cacheprovider",
           f"--rootdir={tmp_path}", "-q", "-rs", *[str(ref / f) for f in FILES]]
    import torch

    if not torch.cuda.is_available():  # files outside the child's rootdir get node ids "::Class::test"
        cmd += [f"--deselect=::{d.split('::', 1)[1]}" for d in CPU_QUANTIZE]
    r = subprocess.run(cmd, cwd=tmp_path, env=env, capture_output=True, text=True, timeout=900)
    tail = (r.stdout[-4000:] + r.stderr[-2000:])
    assert r.returncode == 0, tail
    passed = re.search(r"(\d+) passed", r.stdout)
    assert passed and int(passed.group(1)) >= 45, tail
    assert " failed" not in r.stdout.splitlines()[-1], tail
