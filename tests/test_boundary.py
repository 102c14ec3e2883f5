"""The drop-in boundary compiled against the reference's own GraphIR.

tests/boundary/cuda_lowering.cpp builds reference ir::Graph steps
(KvAppend -> CausalGqa, DeltaUpdate; prefill and decode), lowers every op
through the C ABI as a CudaExecutionPlan would (the sibling of
MetalExecutionPlan.cpp:511-549 and :663-676), and checks dispatch names,
state effects and costs against the reference; with --run it executes the
lowered calls on the GPU and checks them against the oracle.  The binary is
built from the reference tree by tests/boundary/Makefile into oracle/_ref/
(it travels to GPU hosts prebuilt, where the reference tree is absent).
"""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
BINARY = ROOT / "oracle" / "_ref" / "cuda_lowering_test"
REFERENCE = Path(os.environ.get("LLMI_REFERENCE_TREE", "/root/reference"))


def binary() -> Path:
    if (REFERENCE / "lib" / "GraphIR").is_dir():
        subprocess.run(["make", "-s", "-C", str(ROOT / "tests" / "boundary"),
                        f"REFERENCE={REFERENCE}"], check=True, capture_output=True)
    if not BINARY.exists():
        pytest.skip("no reference tree to build the boundary check from, and no prebuilt binary")
    return BINARY


def test_lowering_matches_reference_graph():
    run = subprocess.run([str(binary())], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "boundary: ok" in run.stdout
    assert run.stdout.count("effects and costs match") == 5


@pytest.mark.gpu
def test_lowered_calls_match_oracle_on_gpu():
    run = subprocess.run([str(binary()), "--run"], capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "boundary: ok (executed on the GPU)" in run.stdout
