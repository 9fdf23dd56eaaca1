"""Tensor-parallel decode on 2, 4 and 8 GPUs (one process per GPU, shards
connected over CUDA IPC / NVLink) against the single-device CPU oracle, on a
small model and on 2-layer models of the 8B and 70B shapes (configs 3 and 5).  The
o_proj and down_proj sums are split across ranks and added in rank order, so
logits agree to rounding (same bounds as the single-GPU parity tests); greedy
tokens must match (teacher-forced).  Each case is skipped on boxes with fewer
GPUs than its ranks."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LOGIT_ABS, LOGIT_REL_L2, LOGIT_SCALE_REF = 2e-2, 1e-3, 100.0


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


def run_tp(world, spec):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(world),
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "tests", "tp_worker.py"), json.dumps(spec)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("TPRESULT ")]
    assert line, r.stdout[-2000:] + r.stderr[-2000:]
    return json.loads(line[0][len("TPRESULT "):])


def oracle_run(orc, cfg, seed, prompt, n_decode, kv):
    om = orc.Model(cfg)
    om.init_synthetic(seed)
    if kv:
        om.kv_fill_synthetic(seed, kv)
    out = [om.forward(prompt, kv)]
    pos = kv + len(prompt)
    forced = []
    for _ in range(n_decode):
        t = orc.argmax(out[-1])
        forced.append(int(t))
        out.append(om.forward([t], pos))
        pos += 1
    return out, forced


def test_tensor_parallel_checkpoint_ingest(orc, tmp_path):
    """Every rank loads the same safetensors checkpoint (llmrs_model_load_weight
    keeps its own shard); the ranks together match the oracle holding the
    reference loader's quantised weights."""
    world = 2
    if n_gpus() < world:
        pytest.skip("needs %d GPUs" % world)
    from test_gpu_ingest import CFG, make_checkpoint, reference_tensors, write_safetensors
    cfg = dict(CFG)
    stored, seen = make_checkpoint(cfg, 5, "BF16")
    path = str(tmp_path / "tp.safetensors")
    write_safetensors(path, stored)
    om = orc.Model(cfg)
    om.init_synthetic(0)
    for layer, which, codes, scales in reference_tensors(orc, cfg, seen):
        om.set_tensor(layer, which, codes, scales)
    prompt, n_dec = [5, 17, 900, 3], 4
    ref = [om.forward(prompt, 0)]
    forced, pos = [], len(prompt)
    for _ in range(n_dec):
        forced.append(int(orc.argmax(ref[-1])))
        ref.append(om.forward([forced[-1]], pos))
        pos += 1
    om.close()
    got = run_tp(world, dict(cfg=cfg, seed=0, prompt=prompt, forced=forced, kv=0, ckpt=path))
    assert len(got) == len(ref)
    for step, (g, o) in enumerate(zip(got, ref)):
        gl = np.asarray(g["logits"], np.float32)
        assert len(set(g["tokens"])) == 1 and (g["tokens"][0] == orc.argmax(o) or orc.top2_margin(o) < 1e-3)
        rel = float(np.linalg.norm((gl - o).astype(np.float64)) / np.linalg.norm(o.astype(np.float64)))
        assert float(np.abs(gl - o).max()) < LOGIT_ABS and rel < LOGIT_REL_L2, (step, rel)


@pytest.mark.parametrize("world,shape", [(2, "small"), (2, "8b2"), (4, "8b2"), (8, "8b2"), (2, "70b2"), (4, "70b2"),
                                         (8, "70b2")])
def test_tensor_parallel_decode_matches_oracle(orc, world, shape):
    if n_gpus() < world:
        pytest.skip("needs %d GPUs" % world)
    if shape == "small":
        cfg = dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000,
                   max_seq=96, rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=1, scale_dtype=0)
        seed, prompt, n_dec, kv = 21, [5, 17, 900, 3], 6, 0
    elif shape == "8b2":
        cfg = dict(n_layers=2, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
                   max_seq=4352, rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=0, scale_dtype=0)
        seed, prompt, n_dec, kv = 3, [orc.synth_token(3, 0, 128256)], 3, 4096
    else:  # the 70B shape (config 5): hidden 8192, 64 query / 8 KV heads, FFN 28672, KV 2048
        cfg = dict(n_layers=2, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=128256,
                   max_seq=2176, rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=0, scale_dtype=0)
        seed, prompt, n_dec, kv = 5, [orc.synth_token(5, 0, 128256)], 3, 2048
    ref, forced = oracle_run(orc, cfg, seed, prompt, n_dec, kv)
    got = run_tp(world, dict(cfg=cfg, seed=seed, prompt=prompt, forced=forced, kv=kv))
    assert len(got) == len(ref)
    for step, (g, o) in enumerate(zip(got, ref)):
        gl = np.asarray(g["logits"], np.float32)
        assert len(set(g["tokens"])) == 1, g["tokens"]          # every rank agrees
        assert g["tokens"][0] == orc.argmax(o) or orc.top2_margin(o) < 1e-3, (step, g["tokens"], orc.argmax(o))
        tol = LOGIT_ABS * max(1.0, float(np.abs(o).max()) / LOGIT_SCALE_REF)
        rel = float(np.linalg.norm((gl - o).astype(np.float64)) / np.linalg.norm(o.astype(np.float64)))
        assert float(np.abs(gl - o).max()) < tol and rel < LOGIT_REL_L2, (step, float(np.abs(gl - o).max()), rel)


def test_tensor_parallel_sampling_matches_oracle(orc):
    """Sampling (src/main.rs:192-305) on a 2-rank model: the vocabulary shards
    of the last step's logits are gathered and every rank samples the full
    distribution with the same draw; all ranks pick the oracle's token."""
    world = 2
    if n_gpus() < world:
        pytest.skip("needs %d GPUs" % world)
    cfg = dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000,
               max_seq=96, rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=1, scale_dtype=0)
    prompt, recent = [5, 17, 900, 3], [5, 17, 900, 3, 3]
    settings = [(1.2, 0.8, 0.9, 0.1), (1.0, 1.0, 1.0, 0.5), (1.3, 0.7, 0.95, 0.93)]
    got = run_tp(world, dict(cfg=cfg, seed=21, prompt=prompt, forced=[], kv=0, sample=settings, recent=recent))
    logits = np.asarray(got[0]["logits"], np.float32)        # rank shards in rank order: the full vocabulary
    samples = got[-1]["samples"]
    for i, (penalty, temperature, top_p, u) in enumerate(settings):
        toks = [samples[r][i] for r in range(world)]
        assert len(set(toks)) == 1, toks                       # every rank picks the same token
        t_orc, margin = orc.sample(logits, recent, penalty, temperature, top_p, u)
        assert toks[0] == t_orc or margin < 1e-6, (i, toks, t_orc, margin)
