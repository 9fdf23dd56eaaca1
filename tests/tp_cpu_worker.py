"""One gloo rank (CPU) of the tensor-parallel checks in tests/test_tp_cpu.py:
(1) llmrs_b200.connect_tensor_parallel hands every rank the others' handles in
rank order; (2) the partition the CUDA path uses -- query/KV heads, o_proj and
down_proj input columns, FFN rows, LM-head vocab rows, partial sums added in
rank order and then the residual -- restated with the CPU oracle's Backend
operations reproduces the unsharded oracle's logits and greedy tokens."""
import datetime
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def load_pkg():
    import importlib.util
    pkg = os.path.join(ROOT, "llm.rs_b200")
    spec = importlib.util.spec_from_file_location("llmrs_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llmrs_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


class FakeModel:
    """Stands in for llmrs_b200.Model: the handle exchange needs no GPU."""

    def __init__(self, rank):
        self.rank = rank
        self.got = None

    def tp_handle(self):
        return bytes([self.rank + 1]) * 64, 0

    def tp_connect(self, handles):
        self.got = handles


def main():
    import torch.distributed as dist
    from oracle import oracle as O

    spec = json.loads(sys.argv[1])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    O.set_threads(1)

    fm = FakeModel(rank)
    load_pkg().connect_tensor_parallel(fm)
    assert fm.got == [bytes([q + 1]) * 64 for q in range(world)], fm.got

    cfg, seed = spec["cfg"], spec["seed"]
    H, D, Hq, Hkv, F, V, S = (cfg[k] for k in ("hidden", "head_dim", "n_heads", "n_kv_heads", "ffn", "vocab",
                                               "max_seq"))
    hq, hkv, f, vl = Hq // world, Hkv // world, F // world, V // world
    nrep = Hq // Hkv
    om = O.Model(cfg)
    om.init_synthetic(seed)

    def q4(layer, which, n, k):
        codes, scales = om.tensor(layer, which)
        return codes.reshape(n, k // 2), scales.reshape(n, k // 32)

    def rows(w, r0, r1):
        return np.ascontiguousarray(w[0][r0:r1]), np.ascontiguousarray(w[1][r0:r1])

    def cols(w, c0, c1):
        return np.ascontiguousarray(w[0][:, c0 // 2:c1 // 2]), np.ascontiguousarray(w[1][:, c0 // 32:c1 // 32])

    def lin(x, w, n):
        return O.matmul_transposed_q4(x, w[0].ravel(), w[1].ravel(), n)[0]

    def all_reduce_then_residual(part, x):
        parts = [None] * world
        dist.all_gather_object(parts, part)
        s = parts[0].copy()
        for q in range(1, world):
            s = (s + parts[q]).astype(np.float32)
        return (s + x).astype(np.float32)

    layers = []
    for l in range(cfg["n_layers"]):
        wq = rows(q4(l, O.W_Q, Hq * D, H), rank * hq * D, (rank + 1) * hq * D)
        wk = rows(q4(l, O.W_K, Hkv * D, H), rank * hkv * D, (rank + 1) * hkv * D)
        wv = rows(q4(l, O.W_V, Hkv * D, H), rank * hkv * D, (rank + 1) * hkv * D)
        wo = cols(q4(l, O.W_O, H, Hq * D), rank * hq * D, (rank + 1) * hq * D)
        gu = q4(l, O.W_GATE_UP, 2 * F, H)
        wg = rows(gu, rank * f, (rank + 1) * f)
        wu = rows(gu, F + rank * f, F + (rank + 1) * f)
        wd = cols(q4(l, O.W_DOWN, H, F), rank * f, (rank + 1) * f)
        an = om.tensor(l, O.W_ATTN_NORM)[0]
        mn = om.tensor(l, O.W_MLP_NORM)[0]
        layers.append(dict(wq=wq, wk=wk, wv=wv, wo=wo, wg=wg, wu=wu, wd=wd, an=an, mn=mn,
                           kc=np.zeros((hkv, S, D), np.float32), vc=np.zeros((hkv, S, D), np.float32)))
    embed = om.tensor(0, O.W_EMBED)[0].reshape(V, H)
    fnorm = om.tensor(0, O.W_FINAL_NORM)[0]
    lm = rows(q4(0, O.W_LM_HEAD, V, H), rank * vl, (rank + 1) * vl)
    inv = np.float32(1.0) / np.sqrt(np.float32(D))
    eps = cfg["rms_eps"]

    def step(tok, pos):
        x = embed[tok].astype(np.float32)
        for Lw in layers:
            h = O.rms_norm(x, Lw["an"], eps)[0]
            q = lin(h, Lw["wq"], hq * D).reshape(hq, D)
            k = lin(h, Lw["wk"], hkv * D).reshape(hkv, D)
            v = lin(h, Lw["wv"], hkv * D).reshape(hkv, D)
            for g in range(hkv):
                Lw["kc"][g, pos] = O.rope_inplace(k[g], D, pos)
                Lw["vc"][g, pos] = v[g]
            ctx = np.zeros((hq, D), np.float32)
            for hh in range(hq):
                g = hh // nrep
                qh = O.rope_inplace(q[hh], D, pos)
                sc = O.matmul_slice(qh[None, :], Lw["kc"][g, :pos + 1], pos + 1, D)
                ctx[hh] = O.matmul_f32(O.softmax(O.scale(sc, inv)), Lw["vc"][g, :pos + 1])[0]
            x = all_reduce_then_residual(lin(ctx.ravel(), Lw["wo"], H), x)
            h2 = O.rms_norm(x, Lw["mn"], eps)[0]
            act = O.silu_mul(lin(h2, Lw["wg"], f), lin(h2, Lw["wu"], f))
            x = all_reduce_then_residual(lin(act, Lw["wd"], H), x)
        part = lin(O.rms_norm(x, fnorm, eps)[0], lm, vl)
        shards = [None] * world
        dist.all_gather_object(shards, part)
        return np.concatenate(shards)

    toks = spec["tokens"]
    out = [step(t, i).tolist() for i, t in enumerate(toks)]
    if rank == 0:
        print("TPCPU " + json.dumps(out))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
