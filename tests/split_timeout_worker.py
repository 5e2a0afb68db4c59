"""A sequence-split peer that stops answering, without any GPU fault (launched
under torchrun by test_gpu_split.py, one rank per GPU).

Both ranks connect with a 300 ms bound on the exchange wait and decode a
short prompt together. Then rank 1 skips one continuation request: rank 0's
attention combine waits for a record that never comes, gives up after the
bound, and the request returns Q35_ETIMEOUT with the session reset. Rank 1
has no kernel in flight meanwhile (it only waits on the host). Afterwards
both ranks start a fresh request together and must again agree bit for bit.
Rank 0 writes a JSON verdict.

  torchrun --nproc-per-node 2 split_timeout_worker.py OUT.json
"""
import datetime
import hashlib
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "enginesmith-qwen35-08b-long-decode-m5max-round005_b200"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

WAIT_MS = 300


def main():
    import torch
    import torch.distributed as dist
    import q35
    import inputs as I

    out_path = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    # host-side coordination only: no collective runs while a split kernel is in flight
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    model_dir = os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3")
    if rank == 0 and not os.path.exists(os.path.join(model_dir, "model.safetensors")):
        q35.write_synthetic_model(model_dir, 3)
    dist.barrier()
    prompt = [int(v) for v in I.Rng(92, 7).ints(100, 248320)]
    m = q35.Model.load(model_dir, local, capacity=256)
    q35.split_connect_dist(m, wait_ms=WAIT_MS)
    verdict = {"world": world, "wait_ms": WAIT_MS}

    first = m.generate(prompt, 2, True)  # both ranks together
    dist.barrier()
    if rank == 0:
        t0 = time.perf_counter()
        try:
            m.generate([], 3, False)  # rank 1 does not join this request
            verdict["timed_out"] = False
        except q35.Q35Error as e:
            verdict["timed_out"] = e.code == q35.ETIMEOUT
            verdict["message"] = str(e)
        verdict["seconds"] = time.perf_counter() - t0
        verdict["position_after"] = m.position
        try:
            m.generate([], 1, False)
            verdict["state_reset"] = False
        except q35.Q35Error as e:
            verdict["state_reset"] = "no continuation state" in str(e)
    dist.barrier()  # rank 1 waited on the host only; nothing of it was in flight
    again = m.generate(prompt, 2, True)  # both ranks again, fresh epoch
    digest = hashlib.sha256(m.last_logits()[0].tobytes()).hexdigest()
    all_d = [None] * world
    dist.all_gather_object(all_d, (again, digest))
    if rank == 0:
        verdict["recovered_same_tokens"] = all(a[0] == first for a in all_d)
        verdict["recovered_ranks_identical"] = all(a[1] == all_d[0][1] for a in all_d)
        with open(out_path, "w") as f:
            json.dump(verdict, f)
    dist.barrier()
    m.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
