"""The N > 1 path on CPU: two and four gloo ranks (tests/tp_cpu_worker.py) check the
IPC-handle exchange helper and that the tensor-parallel partition of the model
-- the one the CUDA path implements -- reproduces the unsharded oracle (logits
to rounding, greedy tokens identical)."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CFG2 = dict(n_layers=2, hidden=256, n_heads=8, n_kv_heads=2, head_dim=32, ffn=512, vocab=1000, max_seq=16,
            rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=1)
# four ranks: one KV head and four query heads each
CFG4 = dict(CFG2, hidden=512, n_heads=16, n_kv_heads=4, ffn=1024)


@pytest.mark.parametrize("world,cfg", [(2, CFG2), (4, CFG4)])
def test_tensor_parallel_partition_gloo_ranks(orc, world, cfg):
    seed = 31
    om = orc.Model(cfg)
    om.init_synthetic(seed)
    tokens = [orc.synth_token(seed, i, cfg["vocab"]) for i in range(4)]
    ref = [om.forward([t], i) for i, t in enumerate(tokens)]
    spec = dict(cfg=cfg, seed=seed, tokens=tokens)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(world),
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "tests", "tp_cpu_worker.py"), json.dumps(spec)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-4000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("TPCPU ")]
    assert line, r.stdout[-2000:]
    got = json.loads(line[0][len("TPCPU "):])
    for g, o in zip(got, ref):
        g = np.asarray(g, np.float32)
        assert orc.argmax(g) == orc.argmax(o)
        rel = float(np.linalg.norm((g - o).astype(np.float64)) / np.linalg.norm(o.astype(np.float64)))
        assert rel < 1e-3, rel


def run_resync_worker(mode, timeout):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "tests", "tp_resync_cpu_worker.py"), mode]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)


def test_resync_after_a_rank_skipped_a_step_gloo():
    """A rank that sat out one step (host-side fault) is one completed step
    behind; resync_tensor_parallel agrees on the larger count on every rank."""
    r = run_resync_worker("skip", 120)
    assert r.returncode == 0, r.stderr[-4000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESYNC ")]
    assert line, r.stdout[-2000:]
    res = json.loads(line[0][len("RESYNC "):])
    assert [x["agreed"] for x in res] == [10, 10]          # max(7 + 3, 7 + 2)
    assert [x["epoch"] for x in res] == [10, 10]
    assert [x["resyncs"] for x in res] == [[10], [10]]     # one call each, same value


def test_resync_with_a_vanished_rank_ends_with_an_error_gloo():
    """A rank that exits instead of joining the resync makes the other rank's
    resync fail within the process group's timeout (5 s), not wait for good,
    and no tp_resync is applied on a partial agreement."""
    r = run_resync_worker("vanish", 120)
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("VANISH ")]
    assert line, r.stdout[-2000:] + r.stderr[-2000:]
    out = json.loads(line[0][len("VANISH "):])
    assert out["error"] is not None and out["seconds"] < 60, out
    assert out["resyncs"] == [], out
