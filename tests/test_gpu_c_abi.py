"""GPU: the C ABI from a plain C program (tests/c_abi_ffn.c), compiled with
gcc against include/wamffn.h and the in-tree libwamffn.so and the CUDA
runtime: pack, plan (tuned), FFN run and status, checked in C against a CPU
restatement of the prepared FFN, an invalid plan rejected with a message, and
the masked attention with a padded-prompt mask against a CPU softmax."""

import os
import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def test_c_program_runs_the_ffn_through_the_abi(cuda_device, tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    from waminfer_b200 import _lib

    _lib.lib()  # the library exists (built in-tree)
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    exe = tmp_path / "c_abi_ffn"
    lib_dir = ROOT / "waminfer_b200"
    subprocess.run([gcc, "-O2", "-std=c11", str(ROOT / "tests" / "c_abi_ffn.c"), "-I", str(ROOT / "include"),
                    "-I", str(cuda / "include"), "-L", str(lib_dir), "-l:libwamffn.so", "-L", str(cuda / "lib64"),
                    "-lcudart", "-lm", f"-Wl,-rpath,{lib_dir}:{cuda / 'lib64'}", "-o", str(exe)],
                   check=True, capture_output=True, text=True, timeout=120)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "ffn: 0 of" in run.stdout and "attention: 0 of" in run.stdout
