"""One rank of a tensor-parallel decode run (launched by tests/test_gpu_tp.py
through torch.distributed.run): builds this rank's shard of a synthetic model (or loads it from a checkpoint),
connects to the other ranks over CUDA IPC, runs a prompt and teacher-forced
decode steps, and rank 0 prints every step's token and the full logits
(rank shards concatenated in rank order) as one JSON line."""
import datetime
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_pkg():
    import importlib.util
    pkg = os.path.join(ROOT, "llm.rs_b200")
    spec = importlib.util.spec_from_file_location("llmrs_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llmrs_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def main():
    import torch.distributed as dist

    spec = json.loads(sys.argv[1])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    L = load_pkg()
    ctx = L.Context(local)
    cfg = dict(spec["cfg"], tp_rank=rank, tp_size=world)
    m = L.Model(ctx, cfg)
    if spec.get("ckpt"):  # every rank reads the whole checkpoint and keeps its shard
        L.load_safetensors(m, spec["ckpt"])
    else:
        m.init_synthetic(spec["seed"])
    kv = spec.get("kv", 0)
    if kv:
        m.kv_fill_synthetic(spec["seed"], kv)
    L.connect_tensor_parallel(m)
    steps = []
    tok, lg = m.prefill(spec["prompt"], kv)
    steps.append((tok, lg))
    pos = kv + len(spec["prompt"])
    for t in spec["forced"]:
        tok, lg = m.decode_step(t, pos)
        steps.append((tok, lg))
        pos += 1
    samples = []
    for (penalty, temperature, top_p, u) in spec.get("sample", []):  # after the last step, same draw on every rank
        samples.append(L.tp_sample(m, spec["recent"], penalty, temperature, top_p, u))
    got = [None] * world
    dist.all_gather_object(got, [(int(t), l.astype(np.float32).tobytes()) for t, l in steps])
    sampled = [None] * world
    dist.all_gather_object(sampled, samples)
    if rank == 0:
        out = []
        for i in range(len(steps)):
            toks = [got[r][i][0] for r in range(world)]
            logits = np.concatenate([np.frombuffer(got[r][i][1], np.float32) for r in range(world)])
            out.append({"tokens": toks, "logits": logits.tolist()})
        if spec.get("sample"):
            out.append({"samples": sampled})
        print("TPRESULT " + json.dumps(out))
    dist.barrier()
    m.close()
    ctx.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
