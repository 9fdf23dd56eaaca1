"""The int8-operand prefill GEMM (tcgen05.mma kind::i8, LLMRS_PREFILL_BF16=0).

The switch is read once per process, so the prefill GEMM parity tests and the
model-level prefill tests run again in a child process with it set.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_int8_operand_prefill_path():
    env = dict(os.environ, LLMRS_PREFILL_BF16="0")
    r = subprocess.run(
        [sys.executable, "-m", "pytest", os.path.join(HERE, "test_gpu_ops.py"), os.path.join(HERE, "test_gpu_prefill.py"),
         "-m", "gpu", "-x", "-q", "-p", "no:cacheprovider", "-k", "prefill"],
        env=env, cwd=os.path.dirname(HERE), capture_output=True, text=True, timeout=1200)
    tail = "\n".join((r.stdout + r.stderr).splitlines()[-30:])
    assert r.returncode == 0, tail
    assert " passed" in r.stdout, tail
