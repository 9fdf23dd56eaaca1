"""Parity of the opt-in persistent decode-step kernel (LLMRS_STEP_KERNEL=1).

The switch is read once per process, so the model parity tests run again in a
child process with it set: same seeded inputs, same oracle comparisons (greedy
tokens bit-exact, logits within the tolerances of test_gpu_model.py).
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_model_parity_through_step_kernel():
    env = dict(os.environ, LLMRS_STEP_KERNEL="1")
    sel = "small_model or config1 or config3 or f32_scale or q8_weights or generate"
    r = subprocess.run(
        [sys.executable, "-m", "pytest", os.path.join(HERE, "test_gpu_model.py"),
         "-m", "gpu", "-x", "-q", "-p", "no:cacheprovider", "-k", sel],
        env=env, cwd=os.path.dirname(HERE), capture_output=True, text=True, timeout=1200)
    tail = "\n".join((r.stdout + r.stderr).splitlines()[-30:])
    assert r.returncode == 0, tail
    assert " passed" in r.stdout, tail
