"""A tensor-parallel peer that stops answering, on 2 GPUs (tests/tp_failure_worker.py).

The fault is made on the host: between two steps, rank 1 does not launch the
next one.  Rank 0's decode-step kernels then wait for rank 1's partial sums
with a bounded wait (the model's peer timeout, 200 ms here), give up, set the
device error word and finish, so the step returns LLMRS_ETIMEDOUT and the
context stays usable; after resync_tensor_parallel both ranks re-run the last
two steps and get the tokens of the undisturbed run.  NVLS is off and the
kernels use plain peer stores and loads (no multicast)."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def n_gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_peer_timeout_then_resync_two_gpus(llmrs):
    if n_gpus() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000, max_seq=32,
               rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=0, scale_dtype=0)
    spec = dict(cfg=cfg, seed=23, token=321, timeout_ms=200)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "tests", "tp_failure_worker.py"), json.dumps(spec)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-4000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("TPFAIL ")]
    assert line, r.stdout[-2000:]
    r0, r1 = json.loads(line[0][len("TPFAIL "):])
    assert r0["tokens"] == r1["tokens"]                           # undisturbed steps agree
    assert r0["fault"] == llmrs.ETIMEDOUT, r0                     # the bounded wait ran out
    assert r0["fault_seconds"] < 3.0, r0                          # within the short limit, not 5 s
    assert r0["epoch_after_fault"] == r0["epoch_before"] + 1      # rank 0 finished its (failed) step
    assert r1["epoch_after_fault"] == r1["epoch_before"]          # rank 1 never ran it
    assert r0["agreed"] == r1["agreed"] == r0["epoch_after_fault"]
    assert r0["resumed"] == r1["resumed"] == r0["tokens"][1:]     # same tokens as before the fault
