"""The C ABI from plain C: tests/c_abi/consumer.c is compiled with gcc against
include/*.h, linked with libphysis_b200.so and libcudart, and run -- host-only validation on
the CPU, one fused prep on device buffers (checked against the C restatement in oracle/c)
on a GPU.  No Python or torch sits between the consumer and the library."""
import subprocess
from pathlib import Path

import pytest

from physisserve_b200 import _lib
from physisserve_b200.build import INCLUDE, build

ROOT = Path(__file__).resolve().parents[1]
CUDA = Path("/usr/local/cuda")


@pytest.fixture(scope="module")
def consumer(tmp_path_factory):
    build()
    if not (CUDA / "include" / "cuda_runtime_api.h").exists():
        pytest.skip("CUDA toolkit headers are not installed")
    exe = tmp_path_factory.mktemp("c_abi") / "consumer"
    lib_dir = _lib.LIB_PATH.parent
    cmd = ["gcc", "-std=c11", "-O2", "-ffp-contract=off", "-Wall", "-Wextra", "-Werror",
           "-I", str(INCLUDE), "-I", str(ROOT / "oracle" / "c"), "-I", str(CUDA / "include"),
           str(ROOT / "tests" / "c_abi" / "consumer.c"), str(ROOT / "oracle" / "c" / "prep_ref.c"),
           "-L", str(lib_dir), "-lphysis_b200", "-L", str(CUDA / "lib64"), "-lcudart", "-lm",
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_consumer_validates_without_a_gpu(consumer):
    out = subprocess.run([str(consumer), "validate"], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert "validate: ok" in out.stdout


@pytest.mark.gpu
def test_c_consumer_runs_the_fused_prep(consumer):
    out = subprocess.run([str(consumer), "run"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "rotated K exact, V exact" in out.stdout and out.stdout.strip().endswith("ok")
