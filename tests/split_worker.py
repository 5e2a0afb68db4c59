"""Sequence-split check, one rank per GPU (launched under torchrun by
test_gpu_split.py). Every rank decodes the same prompts with its share of
the K/V; rank 0 checks the ranks' logits agree bit for bit and compares with
the oracle's restatement of the split attention (oracle/q35_oracle.cpp,
attn_f32_split):
  (a) a short prompt decoded from scratch by both: same tokens, same logits;
  (b) a long prompt consumed on the GPUs, the ranks' state dumps gathered
      (each rank holds positions p % world == rank) and imported into the
      oracle, which continues teacher-forced: same logits each step;
  (c) the same long prompt on the tensor-core prompt route (every rank runs
      the whole prompt, then keeps its share of the K/V rows): the gathered
      rows equal a single-GPU tensor-route session's bit for bit, the ranks'
      replicated state agrees, and the oracle continues from the gathered
      state with the same logits.
It also records the distance to a single-GPU session (information only: the
split merges in another order, and this random-init model's nearly flat
logits amplify last-bit differences). Writes a JSON verdict.

  torchrun --nproc-per-node G split_worker.py SHORT_LEN SHORT_STEPS LONG_LEN LONG_STEPS OUT.json
"""
import datetime
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "enginesmith-qwen35-08b-long-decode-m5max-round005_b200"), HERE,
          os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def f32(bf16):
    return (bf16.astype(np.uint32) << 16).view(np.float32)


def main():
    import torch
    import torch.distributed as dist
    import q35
    import inputs as I

    n_short, s_short, n_long, s_long, out_path = (int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]),
                                                  int(sys.argv[4]), sys.argv[5])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=torch.device("cuda", local))
    model_dir = os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3")
    if rank == 0 and not os.path.exists(os.path.join(model_dir, "model.safetensors")):
        q35.write_synthetic_model(model_dir, 3)
    dist.barrier()
    cap = ((max(n_short + s_short, n_long + s_long) + 64) // 64 + 1) * 64
    p_short = [int(v) for v in I.Rng(90, 7).ints(n_short, 248320)]
    p_long = [int(v) for v in I.Rng(91, 7).ints(n_long, 248320)]

    m = q35.Model.load(model_dir, local, capacity=cap)
    q35.split_connect_dist(m)
    assert m.split_world == world
    verdict = {"world": world}
    if rank == 0:
        import q35_oracle as O
        O.set_threads(os.cpu_count() or 1)
        om = O.OracleModel(model_dir)
    dist.barrier()

    # (a) short prompt from scratch
    toks = m.generate(p_short, 1, True)
    logits = [m.last_logits()[0]]
    for _ in range(s_short):
        toks += m.generate([], 1, False)
        logits.append(m.last_logits()[0])
    digest = [hashlib.sha256(lg.tobytes()).hexdigest() for lg in logits]
    all_d = [None] * world
    dist.all_gather_object(all_d, digest)
    if rank == 0:
        verdict["ranks_identical_a"] = all(d == all_d[0] for d in all_d)
        s = O.OracleSession(om, cap)
        s.set_split(world)
        for t in p_short[:-1]:
            s.step(t, head=False)
        otoks, olog = [s.step(p_short[-1])], [s.logits()]
        for _ in range(s_short):
            otoks.append(s.step(otoks[-1]))
            olog.append(s.logits())
        verdict["tokens_equal_a"] = otoks == toks
        verdict["logits_equal_a"] = [bool(np.array_equal(a, b)) for a, b in zip(logits, olog)]
        # distance to a single-GPU session on the same tokens (teacher-forced)
        single = q35.Model.load(model_dir, local, capacity=cap)
        st = single.generate(p_short, 1, True)
        rels, agree = [], 0
        for i in range(s_short + 1):
            a, b = f32(logits[i]), f32(single.last_logits()[0])
            rels.append(float(np.linalg.norm(a - b) / np.linalg.norm(b)))
            agree += int(st[-1] == toks[i])
            if i < s_short:
                if st[-1] != toks[i]:
                    single.force_pending(toks[i])
                st += single.generate([], 1, False)
        verdict["vs_single_rel"] = [round(r, 5) for r in rels]
        verdict["vs_single_agree"] = agree
        single.close()
    dist.barrier()

    # (b) long prompt, state gathered into the oracle, teacher-forced steps
    first = m.generate(p_long, 1, True)
    kv, st, hi = m.dump_state()
    parts = [None] * world
    dist.all_gather_object(parts, (kv, hashlib.sha256(st.tobytes()).hexdigest(),
                                   hashlib.sha256(hi.tobytes()).hexdigest()))
    gpu_toks, gpu_log = [], []
    for _ in range(s_long):
        gpu_toks += m.generate([], 1, False)
        gpu_log.append(m.last_logits()[0])
    counts = [int(np.count_nonzero(np.any(p[0][0, 0, 0] != 0, axis=-1))) for p in parts]
    t_split = m.decode_timed(32)  # every rank, before rank 0 turns to the oracle
    dist.barrier()
    if rank == 0:
        verdict["us_split"] = 1e3 * t_split / 32
        verdict["replicated_state_b"] = all(p[1:] == parts[0][1:] for p in parts)
        full = np.zeros_like(parts[0][0])
        for p in parts:
            full += p[0]
        verdict["local_positions_b"] = counts
        verdict["position_b"] = n_long
        s = O.OracleSession(om, cap)
        s.set_split(world)
        s.import_state(n_long, full, st, hi)
        prev, eq = first[0], []
        for i in range(s_long):
            tok = s.step(prev)
            eq.append(bool(np.array_equal(s.logits(), gpu_log[i])) and tok == gpu_toks[i])
            prev = gpu_toks[i]
        verdict["logits_equal_b"] = eq
    dist.barrier()

    # (c) the long prompt on the tensor-core route
    mt = q35.Model.load(model_dir, local, capacity=cap, tensor_prompt=True)
    q35.split_connect_dist(mt)
    first_c = mt.generate(p_long, 1, True)
    kv_c, st_c, hi_c = mt.dump_state()
    parts = [None] * world
    dist.all_gather_object(parts, (kv_c, hashlib.sha256(st_c.tobytes()).hexdigest(),
                                   hashlib.sha256(hi_c.tobytes()).hexdigest()))
    gpu_toks, gpu_log = [], []
    for _ in range(s_long):
        gpu_toks += mt.generate([], 1, False)
        gpu_log.append(mt.last_logits()[0])
    digest = [hashlib.sha256(lg.tobytes()).hexdigest() for lg in gpu_log]
    all_d = [None] * world
    dist.all_gather_object(all_d, digest)
    dist.barrier()
    if rank == 0:
        verdict["ranks_identical_c"] = all(d == all_d[0] for d in all_d)
        verdict["replicated_state_c"] = all(p[1:] == parts[0][1:] for p in parts)
        full = np.zeros_like(parts[0][0])
        for p in parts:
            full += p[0]
        # rows the prompt route wrote (the last prompt token is the split decode step's)
        single = q35.Model.load(model_dir, local, capacity=cap, tensor_prompt=True)
        single.generate(p_long, 1, True)
        kv_s, _, _ = single.dump_state()
        single.close()
        verdict["rows_equal_single_c"] = bool(np.array_equal(full[..., :n_long - 1, :], kv_s[..., :n_long - 1, :]))
        s = O.OracleSession(om, cap)
        s.set_split(world)
        s.import_state(n_long, full, st_c, hi_c)
        prev, eq = first_c[0], []
        for i in range(s_long):
            tok = s.step(prev)
            eq.append(bool(np.array_equal(s.logits(), gpu_log[i])) and tok == gpu_toks[i])
            prev = gpu_toks[i]
        verdict["logits_equal_c"] = eq
    dist.barrier()
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump(verdict, f)
    mt.close()
    m.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
