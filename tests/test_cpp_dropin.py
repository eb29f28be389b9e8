"""The C++ drop-in boundary at the linker (CPU only): a program written
against the reference's call sequence (tests/cpp/model_step.cpp: Model::forward
of src/model.cu through kernels::embedding, rmsnorm, matmul, rope, attention,
add, fused_silu_mul, bf16_to_fp32 and orin_kv_append) compiles against
include/orin_kernels.h and links against liborin_b200.so with every symbol
resolved."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "orininfer_b200")
CUDA = "/usr/local/cuda"


@pytest.mark.skipif(shutil.which("g++") is None or not os.path.isdir(f"{CUDA}/include"),
                    reason="needs g++ and the CUDA headers")
def test_reference_call_sequence_links_against_the_library(tmp_path):
    exe = tmp_path / "model_step"
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
           "-I", f"{CUDA}/include", os.path.join(ROOT, "tests", "cpp", "model_step.cpp"),
           "-o", str(exe), "-L", LIBDIR, "-lorin_b200", f"-Wl,-rpath,{LIBDIR}",
           "-Wl,--no-undefined", "-L", f"{CUDA}/lib64", "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-2000:]
    assert exe.exists()
