"""One gloo rank (CPU) of tests/test_tp_cpu.py's failure checks of the
tensor-parallel host protocol, with a stand-in for llmrs_b200.Model:

  skip    rank 1 sits out one decode step (a host-side fault: it never launches
          it), so its completed-step count is one behind rank 0's; then every
          rank calls llmrs_b200.resync_tensor_parallel, which must bring both to
          the larger count with exactly one tp_resync call each.
  vanish  rank 1 exits without joining the resync; rank 0's resync must end
          with an error within the process group's short timeout instead of
          waiting for good.
"""
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


class FakeModel:
    """Completed-step count and the resync call of llmrs_b200.Model, without a GPU."""

    def __init__(self, epoch):
        self.epoch = epoch
        self.resyncs = []

    def decode_step(self):
        self.epoch += 1

    def tp_epoch(self):
        return self.epoch

    def tp_resync(self, epoch):
        self.resyncs.append(epoch)
        self.epoch = epoch


def main():
    import torch.distributed as dist

    mode = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5 if mode == "vanish" else 60))
    L = load_pkg()
    m = FakeModel(7)
    for step in range(3):
        if mode == "skip" and rank == 1 and step == 1:
            continue  # rank 1 never launches this step
        m.decode_step()
    if mode == "skip":
        agreed = L.resync_tensor_parallel(m)
        res = [None] * world
        dist.all_gather_object(res, dict(rank=rank, agreed=agreed, epoch=m.epoch, resyncs=m.resyncs))
        if rank == 0:
            print("RESYNC " + json.dumps(res))
        dist.barrier()
        dist.destroy_process_group()
        return
    # vanish: rank 1 leaves before the resync (between steps, nothing in flight)
    if rank == 1:
        os._exit(0)
    t0 = time.time()
    try:
        L.resync_tensor_parallel(m)
        out = dict(error=None)
    except Exception as e:  # the peer never answers: the collective times out
        out = dict(error=type(e).__name__)
    out["seconds"] = round(time.time() - t0, 2)
    out["resyncs"] = m.resyncs
    print("VANISH " + json.dumps(out), flush=True)
    os._exit(0)


if __name__ == "__main__":
    main()
