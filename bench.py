"""Decode-throughput benchmark of the q35 B200 engine (BASELINE.json metric:
decode tok/s at long context, per GPU and aggregate, with the HBM roofline).

Workload: the seeded random-init model (hidden
1024, 24 layers [GDN x3, attention] x6, Q4 group-64), a prompt of `--context`
uniform random ids consumed by the engine, then greedy decode at batch 1. A
step is one decode token of one session; every GPU runs its own session
(independent sessions, weak scaling). Inputs are synthetic and seeded.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--context C] [--impl q35|reference] [--split]
                  [--prompt-route tensor|decode]

The prompt is consumed on the tensor cores by default (as the reference's
prefill: GEMM projections and flash attention over 2048-token chunks); its
wall time is reported in the "prefill" field, beside the decode metric.

--split (N > 1, config 5's second part): ONE session whose attention K/V is
sequence-split over the N GPUs (rank r keeps positions p % N == r, the ranks
exchange partial (m, l, o) over NVLink every attention layer); `value` is
that single stream's tok/s (strong scaling).

Rank 0 prints one JSON line. `value` is device-timed (CUDA events on the
session stream, max over ranks); `e2e` times the public q35_generate call
(continuation request, tokens returned to a host buffer).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "enginesmith-qwen35-08b-long-decode-m5max-round005_b200")
for p in (PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

# BASELINE.json's metric; the context the line was measured at is config.context
METRIC = "decode tok/s at 32K/64K/128K ctx per GPU & 8-GPU aggregate; % HBM roofline"
SYNTH_DIR = os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3")
# bytes streamed per decode token (weights incl. tied head, GDN state R+W,
# conv history + weights) plus 12,288 bytes of K/V per context token
BYTES_FIXED = 422_940_672 + 37_748_736 + 2_211_840
BYTES_PER_CTX = 12_288


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reduce_max(x: float, world: int, device) -> float:
    """Max of a per-rank scalar over all ranks (every rank gets the result)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_tok_s(world: int, steps: int, seconds_max: float) -> float:
    """Whole-job tokens per second: every rank decodes `steps` tokens of its own
    session; the job takes as long as the slowest rank."""
    return world * steps / seconds_max


def ensure_model(world, rank):
    import q35
    import torch.distributed as dist
    if rank == 0 and not os.path.exists(os.path.join(SYNTH_DIR, "model.safetensors")):
        q35.write_synthetic_model(SYNTH_DIR, 3)
    if world > 1:
        dist.barrier()
    return SYNTH_DIR


def cpu_baseline_oracle(model_dir, m, ntok, threads):
    """Oracle (scalar restatement of the reference kernels) decoding from the
    GPU session's own state; returns (tok/s, tokens, agreement)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import q35_oracle as O
    O.set_threads(threads)
    kv, st, hi = m.dump_state()
    pos = m.position
    om = O.OracleModel(model_dir)
    s = O.OracleSession(om, ((pos + ntok + 32) // 32) * 32)
    s.import_state(pos, kv, st, hi)
    del kv
    gpu = m.generate([], ntok, False)  # GPU tokens for the same steps (teacher forcing)
    prev = None
    t0 = time.perf_counter()
    agree = 0
    first = m._pending_for_bench
    prev = first
    for t in gpu:
        agree += int(s.step(prev, head=True) == t)
        prev = t
    dt = time.perf_counter() - t0
    return ntok / dt, ntok, agree


def run_reference(args, world, rank):
    """Reference arm: the reference's decode arithmetic on the host cores (the
    CPU restatement in oracle/, since the Metal/Rust reference cannot run here)."""
    if rank != 0:
        return 0
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import q35_oracle as O
    import inputs as I
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    import q35
    if not os.path.exists(os.path.join(SYNTH_DIR, "model.safetensors")):
        q35.write_synthetic_model(SYNTH_DIR, 3)
    om = O.OracleModel(SYNTH_DIR)
    ctx = args.context
    cap = ((ctx + args.steps + args.warmup + 32) // 32) * 32
    s = O.OracleSession(om, cap)
    # a seeded state of the workload's size: K/V for ctx positions, GDN state, history
    pool = I.f2bf(I.Rng(11).normal(1 << 20))
    reps = (6 * 2 * 2 * ctx * 256 + pool.size - 1) // pool.size
    kv = np.tile(pool, reps)[: 6 * 2 * 2 * ctx * 256].reshape(6, 2, 2, ctx, 256)
    st = I.Rng(12).normal(18 * 16 * 128 * 128, 0.05).reshape(18, 16, 128, 128)
    hi = I.f2bf(I.Rng(13).normal(18 * 3 * 6144)).reshape(18, 3, 6144)
    s.import_state(ctx, kv, st, hi)
    del kv
    tok = 1
    for _ in range(args.warmup):
        tok = s.step(tok, head=True)
    budget = float(os.environ.get("Q35_REF_BUDGET_S", "150"))
    n, t0 = 0, time.perf_counter()
    while n < args.steps:
        tok = s.step(tok, head=True)
        n += 1
        if time.perf_counter() - t0 > budget:
            break
    dt = time.perf_counter() - t0
    v = n / dt
    out = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": 1e3 * dt / n, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16/f32 (Q4 weights)", "data": "synthetic",
        "config": {"workload": f"config4: full model decode at {ctx} ctx, batch 1 (seeded synthetic state)",
                   "context": ctx, "global_batch": 1, "parallelism": "host threads"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{n} decode tokens at {ctx} context on {threads} host threads"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2048)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--context", type=int, default=65536)
    ap.add_argument("--impl", default="q35", choices=["q35", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--split", action="store_true")
    ap.add_argument("--prompt-route", default="tensor", choices=["tensor", "decode"],
                    help="prompt on the tensor cores (the reference's GEMM/flash-attention prefill) "
                         "or through the decode step's kernels")
    ap.add_argument("--batch-members", type=int, default=32,
                    help="also time this many sessions decoded together on the tensor cores (0: skip)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup()
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import datetime
    import numpy as np
    import torch
    import torch.distributed as dist
    import q35
    import inputs as I

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local))
    model_dir = ensure_model(world, rank)
    cap = ((args.context + args.warmup + 2 * args.steps + args.cpu_tokens + 64) // 32) * 32
    split = args.split and world > 1
    tensor_prompt = args.prompt_route == "tensor" and not split  # a split session takes the decode route
    m = q35.Model.load(model_dir, local, capacity=cap, tensor_prompt=tensor_prompt)
    if split:
        q35.split_connect_dist(m)  # one stream over all ranks: the same prompt everywhere
    streams = 1 if split else world
    prompt = [int(v) for v in I.Rng(3 + (0 if split else rank), 50).ints(args.context, 248320)]
    t0 = time.perf_counter()
    first = m.generate(prompt, 1, True)
    prefill_s = time.perf_counter() - t0
    m.decode_timed(args.warmup)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- timed region (device clock) ----
    m.attn_timing(reset=1)
    start_pos = m.position
    with ClockSampler(local) as clk:
        barrier()
        ms = m.decode_timed(args.steps)
        barrier()
    attn_us, attn_launches = m.attn_timing(reset=0)
    ms_max = reduce_max(ms, world, "cuda")
    value = aggregate_tok_s(streams, args.steps, ms_max / 1e3)

    # ---- end to end: the public generate call, host buffers ----
    barrier()
    t0 = time.perf_counter()
    toks = m.generate([], args.steps, False)
    e2e_s = time.perf_counter() - t0
    e2e = aggregate_tok_s(streams, args.steps, reduce_max(e2e_s, world, "cuda"))
    m._pending_for_bench = toks[-1]

    # ---- roofline of the dominant kernel (attention) ----
    peak, peak_kind = peaks()
    avg_len = start_pos + (args.steps + 1) / 2.0
    # K/V rows this rank's attention launches read (its share under a split)
    local_len = avg_len / world if split else avg_len
    attn_bytes = 2 * 2 * 256 * 2 * local_len + 4096 * 2 + 2 * 512 * 2 + 2048 * 2
    attn_avg_s = attn_us / max(attn_launches, 1) * 1e-6
    achieved = attn_bytes / attn_avg_s / 1e9 if attn_launches else None
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "attn_traffic.json")) as f:
            tr = json.load(f)
        traffic = tr["dram_bytes_per_ctx_token"] * local_len
    except Exception:
        pass
    step_bytes = BYTES_FIXED + BYTES_PER_CTX * (start_pos + args.steps / 2.0) / (world if split else 1)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, n, agree = cpu_baseline_oracle(model_dir, m, args.cpu_tokens, threads)
        cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n} decode tokens at {m.position - n} context from the GPU state "
                         f"(teacher-forced, {agree}/{n} argmax agree)"}

    # ---- batched sessions on the tensor cores (extra measurement, not `value`) ----
    batched = None
    nb = args.batch_members if not split else 0
    if nb > 0:
        members = [m] + [q35.Model.load(model_dir, local, capacity=cap) for _ in range(nb - 1)]
        for mb in members[1:]:
            mb.copy_from(m)
        bt = q35.Batch(members, tensor_cores=True)
        bt.decode_timed(4)
        barrier()
        bms = bt.decode_timed(16)
        barrier()
        bt.close()
        for mb in members[1:]:
            mb.close()
        bmax = reduce_max(bms, world, "cuda")
        batched = {"route": "tcgen05 GEMM projections and head (q35_batch_create_ex, Q35_BATCH_TENSOR_CORES)",
                   "members_per_gpu": nb, "context": m.position, "steps": 16,
                   "us_per_step": 1e3 * bmax / 16, "tok_s": aggregate_tok_s(world * nb, 16, bmax / 1e3),
                   "note": "members forked from this session's state (q35_session_copy); device-timed"}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if split else "weak", "vs_baseline": None,
            "dtype": "bf16 (Q4 weights, f32 state/accumulation)",
            "data": "synthetic (seeded random-init weights and prompt ids)",
            "config": {"workload": (f"config5 (sequence split): one session, {args.context}-token prompt, "
                                    f"attention K/V split over {world} GPUs" if split else
                                    f"config4: Qwen3.5-0.8B-class hybrid Q4 model, {args.context}-token "
                                    f"prompt then greedy decode, batch 1 per GPU"),
                       "model": "q35-0.8B-hybrid-q4 (random init, seed 3)", "context": args.context,
                       "global_batch": streams, "seq_len": args.context,
                       "parallelism": f"sequence split x{world}" if split else f"sessions x{world}",
                       "l2": "inputs larger than L2 (each step streams ~%.2f GB)" % (step_bytes / 1e9),
                       "prefill_s": round(prefill_s, 2)},
            "prefill": {"route": ("tensor cores: tcgen05 GEMM projections, causal flash attention, "
                                  "2048-token chunks" if tensor_prompt else "decode step kernels, 16-token chunks"),
                        "tokens": args.context, "seconds": prefill_s, "tok_s": args.context / prefill_s,
                        "note": "wall clock of q35_generate(prompt, 1) (the prompt, then its last token decoded)"},
            "gpu_launches": args.steps * (18 * 3 + 6 * 4 + 24 * 2 + 1),
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4},
            "roofline": {"bound": "hbm", "kernel": "k_attn (split GQA decode attention)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": (achieved / peak) if achieved else None,
                         "traffic": traffic, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": attn_bytes,
                         "avg_launch_us": attn_avg_s * 1e6, "launches": attn_launches},
            "step_roofline": {"bytes_per_token": step_bytes,
                              "achieved_gbs": step_bytes * (value / streams) / 1e9,
                              "frac": step_bytes * (value / streams) / 1e9 / peak},
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "batched": batched,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()  # no rank unmaps its exchange buffer while a peer still decodes
    m.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
