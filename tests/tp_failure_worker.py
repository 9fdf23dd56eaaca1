"""One rank of tests/test_gpu_tp_failure.py (launched through
torch.distributed.run on 2 GPUs): a tensor-parallel model whose peers stop
answering.  Both ranks run two decode steps; then rank 1 sits out the third
(a host-side fault between steps: it never launches it, none of its kernels
is in flight), so rank 0's exchange waits run out after the short peer
timeout and its step fails with LLMRS_ETIMEDOUT.  The ranks learn of it on the
host (a gloo barrier), resynchronise (resync_tensor_parallel) and re-run the
second and third steps, which must give the tokens of the undisturbed run."""
import datetime
import json
import os
import sys
import time

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
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    L = load_pkg()
    ctx = L.Context(local)
    m = L.Model(ctx, dict(spec["cfg"], tp_rank=rank, tp_size=world))
    m.init_synthetic(spec["seed"])
    L.connect_tensor_parallel(m)
    m.set_peer_timeout(spec["timeout_ms"])
    t0 = spec["token"]
    ta, _ = m.decode_step(t0, 0, want_logits=False)
    tb, _ = m.decode_step(ta, 1, want_logits=False)
    tc_ref, _ = m.decode_step(tb, 2, want_logits=False)
    out = dict(rank=rank, tokens=[ta, tb, tc_ref], epoch_before=m.tp_epoch())
    # the fault: rank 1 does not launch the step at position 3
    if rank == 0:
        t = time.time()
        try:
            m.decode_step(tc_ref, 3, want_logits=False)
            out["fault"] = "completed"
        except L.LlmrsError as e:
            out["fault"] = e.code
        out["fault_seconds"] = round(time.time() - t, 3)
    out["epoch_after_fault"] = m.tp_epoch()
    dist.barrier()  # the ranks learn of the failed step on the host
    out["agreed"] = L.resync_tensor_parallel(m)
    # resume: the second and third steps again, on both ranks
    tb2, _ = m.decode_step(ta, 1, want_logits=False)
    tc2, _ = m.decode_step(tb2, 2, want_logits=False)
    out["resumed"] = [tb2, tc2]
    got = [None] * world
    dist.all_gather_object(got, out)
    if rank == 0:
        print("TPFAIL " + json.dumps(got))
    dist.barrier()
    m.close()
    ctx.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
