"""Decode-throughput benchmark of the q35 B200 engine (BASELINE.json metric:
decode tok/s at 32K/64K/128K context per GPU and 8-GPU aggregate, with the
HBM roofline).

Headline workload: the seeded random-init model
(hidden 1024, 24 layers [GDN x3, attention] x6, Q4 group-64), a prompt of
`--context` (65,536) uniform random ids consumed by the engine, then greedy
decode at batch 1. A step is one decode token of one session; every GPU runs
its own session (independent sessions, weak scaling, no collective on the data
path). Inputs are synthetic and seeded.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--context C]
                  [--impl q35|reference] [--split] [--prompt-route tensor|decode]

Besides `value` (device-timed decode tok/s at --context, max over ranks), the
JSON line carries:
  by_context  the same measurement at the other contexts of the metric (32K, 128K)
  config5     BASELINE config 5: 8 sessions at 131,072 context (prompt seeds
              3..10) split 8/N per GPU, each GPU decoding its share as one batch;
              aggregate tok/s (strong scaling over N)
  e2e         the drop-in `engine` executable timed as the harness times it: a
              continuation request generate([], K, reset=false) from writing the
              JSON line to reading the reply
  roofline    the kernel with the larger share of the step (the attention launches
              or the Q4 matvec launches; both in roofline_kernels): its bytes per
              launch over its device-clock launch time, from the faster of two
              32-step passes with the in-kernel timers on right after the timed
              region (the timed region itself runs with them off), against the
              measured HBM peak
  cpu_baseline the oracle decoding from this GPU session's own state
              (teacher-forced, with its argmax agreement), on the host cores
  prefill     the prompt's wall time (tensor-core route by default)

--split (N > 1, config 5's second part): ONE session whose attention K/V is
sequence-split over the N GPUs; `value` is that single stream's tok/s (strong
scaling).

`--impl reference` runs the reference's decode arithmetic on the host cores
(the CPU restatement in oracle/; the Rust/Metal reference cannot run here) on
rank 0; other ranks exit at once. That arm never loads the CUDA library.
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
ENGINE = os.path.join(PKG, "lib", "engine")
for p in (PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

# BASELINE.json's metric; the context the line was measured at is config.context
METRIC = "decode tok/s at 32K/64K/128K ctx per GPU & 8-GPU aggregate; % HBM roofline"
SYNTH_DIR = os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3")
MODEL_SEED = 3
# decode steps of the instrumented pass after each timed region (the kernels'
# device-clock timers on, for the roofline fields; not part of the timed region)
INSTRUMENTED_STEPS = 32
INSTRUMENTED_PASSES = 2
# bytes streamed per decode token (weights incl. tied head, GDN state R+W,
# conv history + weights) plus 12,288 bytes of K/V per context token
BYTES_FIXED = 422_940_672 + 37_748_736 + 2_211_840
BYTES_PER_CTX = 12_288
VOCAB = 248320
# the session capacity q35_open accepts is a positive multiple of this
# (include/q35.h, q35_opts.capacity; q35_check_opts validates it)
CAPACITY_ALIGN = 64
C5_CONTEXT = 131072
C5_SESSIONS = 8
C5_SEEDS = list(range(3, 3 + C5_SESSIONS))


def capacity_for(tokens: int) -> int:
    """Smallest session capacity q35_open accepts that holds `tokens` positions."""
    return max(CAPACITY_ALIGN, -(-int(tokens) // CAPACITY_ALIGN) * CAPACITY_ALIGN)


def parse_contexts(s: str) -> list[int]:
    return [int(x) for x in s.split(",") if x.strip()] if s else []


def plan(args, world: int) -> dict:
    """Host arithmetic of one run: the contexts measured, the token budget of
    every session the bench opens and the capacity they share (the config-5
    members are filled by copying a prefilled session, which needs equal
    capacities). A CPU test checks these against q35_check_opts for the
    driver's argument sets."""
    split = args.split and world > 1
    ctxs = [args.context] + [c for c in parse_contexts(args.contexts) if c != args.context]
    if split:
        ctxs = [args.context]
    c5 = (not split) and args.config5 and C5_SESSIONS % world == 0
    # the longest context a session reaches: prompt, first token, warm-up,
    # timed steps, the CPU sample's GPU tokens, a margin
    need = max(ctxs) + 1 + args.warmup + args.steps + INSTRUMENTED_PASSES * INSTRUMENTED_STEPS + args.cpu_tokens + 64
    if c5:
        need = max(need, C5_CONTEXT + 1 + args.warmup + args.steps + 64)
    return {"split": split, "contexts": ctxs, "config5": c5, "capacity": capacity_for(need),
            "engine_capacity": capacity_for(args.context + 1 + args.warmup + args.steps + 64),
            "c5_per_gpu": C5_SESSIONS // world if c5 else 0}


def prompt_ids(seed: int, n: int) -> list[int]:
    import inputs as I
    return [int(v) for v in I.Rng(seed, 50).ints(n, VOCAB)]


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples (every 20 ms) over the whole
    measurement; the summary keeps the samples taken inside the timed
    windows the caller marks, else the samples under load."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.windows = []
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def mark(self, t0: float, t1: float):
        self.windows.append((t0, t1))

    def stop(self):
        if self.proc is not None:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
            self.proc = None

    @staticmethod
    def _when(stamp: str):
        import datetime
        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.datetime.strptime(stamp.strip(), fmt).timestamp()
            except ValueError:
                pass
        return None

    def summary(self):
        rows = []
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10:
                continue
            try:
                rows.append((self._when(f[0]), float(f[2]), float(f[3]), float(f[5]) if f[5] else 0.0,
                             [n for n, v in zip(self.NAMES, f[6:10]) if v.lower().startswith("active")]))
            except ValueError:
                continue
        inside = [r for r in rows if r[0] is not None and
                  any(a - 0.03 <= r[0] <= b + 0.03 for a, b in self.windows)]
        sel, basis = inside, "inside the timed windows"
        if len(sel) < 3:
            sel, basis = [r for r in rows if r[3] >= 50.0], "samples with the GPU busy (>= 50%)"
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "basis": "none"}
        return {"sm_mhz": statistics.median(r[1] for r in sel), "sm_max_mhz": max(r[2] for r in sel),
                "reasons": sorted({n for r in sel for n in r[4]}), "samples": len(sel), "basis": basis}


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
    session(s); the job takes as long as the slowest rank."""
    return world * steps / seconds_max


def ensure_model(world, rank):
    import q35
    import torch.distributed as dist
    if rank == 0 and not os.path.exists(os.path.join(SYNTH_DIR, "model.safetensors")):
        q35.write_synthetic_model(SYNTH_DIR, MODEL_SEED)
    if world > 1:
        dist.barrier()
    return SYNTH_DIR


def cpu_baseline_oracle(model_dir, m, ntok, threads, budget_s):
    """Oracle (scalar restatement of the reference kernels) decoding from the
    GPU session's own state, fed the GPU's tokens (teacher forcing), for at
    most `ntok` tokens or `budget_s` seconds. Returns (tok/s, tokens, agree)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import q35_oracle as O
    O.set_threads(threads)
    kv, st, hi = m.dump_state()
    pos = m.position
    first = m.pending
    om = O.OracleModel(model_dir)
    s = O.OracleSession(om, capacity_for(pos + ntok + 64))
    s.import_state(pos, kv, st, hi)
    del kv
    gpu = m.generate([], ntok, False)  # the GPU's tokens for the same steps
    prev, agree, n = first, 0, 0
    t0 = time.perf_counter()
    for t in gpu:
        agree += int(s.step(prev, head=True) == t)
        prev = t
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return n / dt, n, agree


def run_reference(args, world, rank):
    """Reference arm: the reference's decode arithmetic on the host cores (the
    CPU restatement in oracle/, since the Metal/Rust reference cannot run
    here), on the headline workload's shapes from a seeded synthetic state.
    Loads only oracle/ (the synthetic-model writer is compiled into it)."""
    if rank != 0:
        return 0
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import q35_oracle as O
    import inputs as I
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    if not os.path.exists(os.path.join(SYNTH_DIR, "model.safetensors")):
        O.write_synthetic_model(SYNTH_DIR, MODEL_SEED)
    om = O.OracleModel(SYNTH_DIR)
    ctx = args.context
    s = O.OracleSession(om, capacity_for(ctx + args.steps + args.warmup + 64))
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
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16 storage, Q4 weights)", "data": "synthetic",
        "config": {"workload": f"config4: full model decode at {ctx} ctx, batch 1 (seeded synthetic state)",
                   "context": ctx, "global_batch": 1, "parallelism": "host threads"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{n} decode tokens at {ctx} context on {threads} host threads"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)
    return 0


class EngineProc:
    """The drop-in `engine` executable over its JSON-lines protocol."""

    def __init__(self, model_dir, device, capacity, prompt_route):
        cmd = [ENGINE, "--model", model_dir, "--device", str(device), "--capacity", str(capacity)]
        if prompt_route == "decode":
            cmd.append("--decode-prompt")
        self.p = subprocess.Popen(cmd, stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True,
                                  bufsize=1 << 20)
        self.id = 0

    def ask(self, op, **kw):
        self.id += 1
        req = dict(id=self.id, op=op, **kw)
        self.p.stdin.write(json.dumps(req, separators=(",", ":")) + "\n")
        self.p.stdin.flush()
        line = self.p.stdout.readline()
        if not line:
            raise RuntimeError(f"engine exited (rc {self.p.poll()})")
        r = json.loads(line)
        if not r.get("ok"):
            raise RuntimeError(f"engine error: {r}")
        return r

    def close(self):
        try:
            self.p.stdin.close()
            self.p.wait(timeout=120)
        except Exception:
            self.p.kill()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--context", type=int, default=65536, help="the headline context (config 4)")
    ap.add_argument("--contexts", default="32768,131072",
                    help="other contexts of the metric, measured the same way (comma list; empty: none)")
    ap.add_argument("--impl", default="q35", choices=["q35", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=64, help="GPU tokens replayed by the CPU baseline (at most)")
    ap.add_argument("--cpu-budget-s", type=float, default=15.0, help="time bound of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config5", dest="config5", action="store_false")
    ap.add_argument("--c5-route", default="both", choices=["exact", "tensor", "both"],
                    help="config-5 batches: the exact CUDA-core route, the tensor-core route, or both")
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--split", action="store_true")
    ap.add_argument("--prompt-route", default="tensor", choices=["tensor", "decode"],
                    help="prompt on the tensor cores (the reference's GEMM/flash-attention prefill) "
                         "or through the decode step's kernels")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup()
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import datetime
    import torch
    import torch.distributed as dist
    import q35

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local))
    pl = plan(args, world)
    model_dir = ensure_model(world, rank)
    cap = pl["capacity"]
    split = pl["split"]
    tensor_prompt = args.prompt_route == "tensor"  # a split rank runs the whole prompt, then keeps its share
    m = q35.Model.load(model_dir, local, capacity=cap, tensor_prompt=tensor_prompt)
    if split:
        q35.split_connect_dist(m)  # one stream over all ranks: the same prompt everywhere
    streams = 1 if split else world
    peak, peak_kind = peaks()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clk = ClockSampler(local).start()

    def measure(ctx, seed, timed_steps):
        """Prompt of ctx ids, warm-up, then `timed_steps` device-timed decode
        steps (barrier + synchronize on both sides, max over ranks)."""
        prompt = prompt_ids(seed, ctx)
        barrier()
        t0 = time.perf_counter()
        m.generate(prompt, 1, True)
        prefill_s = time.perf_counter() - t0
        m.decode_timed(args.warmup)
        m.attn_timing(reset=0)  # the kernels' device-clock timers stay off in the timed region
        m.launch_count(reset=True)
        start_pos = m.position
        barrier()
        w0 = time.time()
        ms = m.decode_timed(timed_steps)
        barrier()
        clk.mark(w0, time.time())
        launches = m.launch_count(reset=True)
        # instrumented passes right after it (same session and graphs): the
        # timers on, INSTRUMENTED_STEPS steps each, for the kernels' launch
        # times; of INSTRUMENTED_PASSES passes the one with the shorter step is
        # kept (a short pass can catch a transient slowdown of the box)
        best = None
        for _ in range(INSTRUMENTED_PASSES):
            m.attn_timing(reset=1)
            pass_ms = m.decode_timed(INSTRUMENTED_STEPS)
            q = m.qmv_timing()  # before attn_timing's reset clears it
            at = m.attn_timing(reset=0)
            if best is None or pass_ms < best[0]:
                best = (pass_ms, q, at)
        inst_ms, (qmv_us, qmv_launches, qmv_bytes), (attn_us, attn_launches) = best
        barrier()
        ms_max = reduce_max(ms, world, "cuda")
        tok_s = aggregate_tok_s(streams, timed_steps, ms_max / 1e3)
        # K/V rows the attention launches of the instrumented passes read (per rank)
        avg_len = start_pos + timed_steps + (INSTRUMENTED_PASSES * INSTRUMENTED_STEPS + 1) / 2.0
        local_len = avg_len / world if split else avg_len
        attn_bytes = 2 * 2 * 256 * 2 * local_len + 4096 * 2 + 2 * 512 * 2 + 2048 * 2
        attn_avg_s = attn_us / max(attn_launches, 1) * 1e-6
        step_bytes = BYTES_FIXED + BYTES_PER_CTX * (start_pos + timed_steps / 2.0) / (world if split else 1)
        return {"context": ctx, "tok_s": tok_s, "ms_max": ms_max, "ms_per_step": ms_max / timed_steps,
                "prefill_s": reduce_max(prefill_s, world, "cuda"), "launches": launches,
                "attn_bytes": attn_bytes, "attn_avg_s": attn_avg_s, "attn_launches": attn_launches,
                "local_len": local_len, "step_bytes": step_bytes,
                "qmv_us": qmv_us, "qmv_launches": qmv_launches, "qmv_bytes": qmv_bytes, "attn_us": attn_us,
                "inst_ms_per_step": inst_ms / INSTRUMENTED_STEPS,
                "step_frac": step_bytes * (tok_s / streams) / 1e9 / peak}

    # ---- headline: decode at --context (config 4) ----
    head = measure(args.context, MODEL_SEED + (0 if split else rank), args.steps)
    head_pos = m.position

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, n, agree = cpu_baseline_oracle(model_dir, m, args.cpu_tokens, threads, args.cpu_budget_s)
        cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n} decode tokens at {head_pos} context from the GPU session's own state "
                         f"(teacher-forced on the GPU's tokens: {agree}/{n} argmax agree)",
               "agree": agree, "tokens": n}
    barrier()

    # ---- the metric's other contexts (same session, reset per prompt) ----
    by_context = {str(head["context"]): round(head["tok_s"], 2)}
    extra = {}
    for ctx in pl["contexts"][1:]:
        r = measure(ctx, MODEL_SEED + 100 + rank, args.steps)
        by_context[str(ctx)] = round(r["tok_s"], 2)
        extra[str(ctx)] = {"tok_s": r["tok_s"], "ms_per_step": r["ms_per_step"], "prefill_s": r["prefill_s"],
                           "step_roofline_frac": r["step_frac"],
                           "attn_frac": (r["attn_bytes"] / r["attn_avg_s"] / 1e9 / peak) if r["attn_launches"] else None,
                           "qmv_frac": (r["qmv_bytes"] / (r["qmv_us"] * 1e-6) / 1e9 / peak) if r["qmv_launches"] else None}

    # ---- config 5: 8 sessions at 131,072 context over N GPUs, batched per GPU ----
    config5 = None
    if pl["config5"]:
        per = pl["c5_per_gpu"]
        seeds = C5_SEEDS[rank * per:(rank + 1) * per]
        members = [q35.Model.load(model_dir, local, capacity=cap) for _ in range(per)]
        c5_prefill = 0.0
        for mb, sd in zip(members, seeds):
            t0 = time.perf_counter()
            m.generate(prompt_ids(sd, C5_CONTEXT), 1, True)  # the main session prefills, the member copies
            c5_prefill += time.perf_counter() - t0
            mb.copy_from(m)
        snap = [q35.Model.load(model_dir, local, capacity=cap) for _ in range(per)] if args.c5_route == "both" else []
        for a, b in zip(snap, members):
            a.copy_from(b)  # both routes start from the same states
        routes = ["exact", "tensor"] if args.c5_route == "both" else [args.c5_route]
        config5 = {"sessions": C5_SESSIONS, "sessions_per_gpu": per, "context": C5_CONTEXT, "seeds": C5_SEEDS,
                   "steps": args.steps, "prefill_s_per_gpu": reduce_max(c5_prefill, world, "cuda")}
        for i, route in enumerate(routes):
            group = members if i == 0 else snap
            bt = q35.Batch(group, tensor_cores=(route == "tensor"))
            bt.decode_timed(args.warmup)
            bt.launch_count(reset=True)
            barrier()
            w0 = time.time()
            bms = bt.decode_timed(args.steps)
            barrier()
            clk.mark(w0, time.time())
            bl = bt.launch_count(reset=True)
            bt.close()
            bmax = reduce_max(bms, world, "cuda")
            c5_bytes = BYTES_FIXED + per * (37_748_736 + 2_211_840 +
                                            BYTES_PER_CTX * (C5_CONTEXT + args.warmup + args.steps / 2.0))
            config5[route] = {"tok_s": aggregate_tok_s(world * per, args.steps, bmax / 1e3),
                              "us_per_step": 1e3 * bmax / args.steps, "gpu_launches": bl,
                              "step_roofline_frac": c5_bytes * (args.steps / (bmax / 1e3)) / 1e9 / peak}
        best = max(routes, key=lambda r: config5[r]["tok_s"])
        config5["tok_s"] = config5[best]["tok_s"]
        config5["route"] = best
        for mb in members + snap:
            mb.close()
    clk.stop()

    # ---- end to end: the drop-in engine executable, timed as the harness does ----
    e2e = None
    if args.e2e and not split:
        eng = EngineProc(model_dir, local, pl["engine_capacity"], args.prompt_route)
        try:
            eng.ask("hello")
            prompt = prompt_ids(MODEL_SEED + 200 + rank, args.context)
            t0 = time.perf_counter()
            eng.ask("generate", prompt=prompt, max_tokens=1, reset=True)
            ttft = time.perf_counter() - t0
            eng.ask("generate", prompt=[], max_tokens=args.warmup, reset=False)
            barrier()
            t0 = time.perf_counter()
            r = eng.ask("generate", prompt=[], max_tokens=args.steps, reset=False)
            dt = time.perf_counter() - t0
            assert len(r["tokens"]) == args.steps
        finally:
            eng.close()
        dt_max = reduce_max(dt, world, "cuda")
        e2e = {"value": aggregate_tok_s(world, args.steps, dt_max), "unit": "tok/s",
               "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4,
               "how": ("engine executable (JSON lines over pipes): generate([], K, reset=false) timed from "
                       "writing the request to reading the reply, as the harness times a decode request; "
                       "a continuation carries no input (the pending token stays on the device) and each "
                       "token comes back as 4 bytes"),
               "prefill_request_s": reduce_max(ttft, world, "cuda"), "context": args.context}

    if rank == 0:
        achieved = head["attn_bytes"] / head["attn_avg_s"] / 1e9 if head["attn_launches"] else None
        traffic = None
        try:
            with open(os.path.join(ROOT, "profiles", "attn_traffic.json")) as f:
                traffic = json.load(f)["dram_bytes_per_ctx_token"] * head["local_len"]
        except Exception:
            pass
        inst_note = (f"device-clock launch times from the faster of {INSTRUMENTED_PASSES} {INSTRUMENTED_STEPS}-step "
                     f"instrumented passes right after the timed region ({head['inst_ms_per_step']:.4f} ms per "
                     f"step with the timers on, {head['ms_per_step']:.4f} without)")
        attn_roof = {"bound": "hbm", "kernel": "k_attn (split GQA decode attention, live device clock)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": (achieved / peak) if achieved else None,
                     "traffic": traffic, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": head["attn_bytes"],
                     "avg_launch_us": head["attn_avg_s"] * 1e6, "launches": head["attn_launches"],
                     "us_total": head["attn_us"], "measured": inst_note}
        qmv_roof = None
        if head["qmv_launches"]:
            qb = head["qmv_bytes"] / head["qmv_launches"]
            qs = head["qmv_us"] / head["qmv_launches"] * 1e-6
            qtraffic = None
            try:
                with open(os.path.join(ROOT, "profiles", "qmv_traffic.json")) as f:
                    qtraffic = json.load(f)["dram_bytes_per_algorithmic_byte"] * qb
            except Exception:
                pass
            qmv_roof = {"bound": "hbm", "kernel": "k_qmv (the decode step's Q4 matvec launches, live device clock)",
                        "achieved": qb / qs / 1e9, "peak": peak, "unit": "GB/s", "frac": qb / qs / 1e9 / peak,
                        "traffic": qtraffic, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": qb,
                        "avg_launch_us": qs * 1e6, "launches": head["qmv_launches"],
                        "us_total": head["qmv_us"], "measured": inst_note}
        # the headline roofline is the kernel with the larger share of the step
        roofline = attn_roof
        if qmv_roof and head["qmv_us"] > head["attn_us"]:
            roofline = qmv_roof
        out = {
            "metric": METRIC, "value": head["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
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
                       "capacity": cap,
                       "l2": "inputs larger than L2 (each step streams ~%.2f GB)" % (head["step_bytes"] / 1e9)},
            "by_context": by_context,
            "contexts": extra,
            "prefill": {"route": ("tensor cores: tcgen05 GEMM projections, causal flash attention, "
                                  "2048-token chunks" if tensor_prompt else "decode step kernels, 16-token chunks"),
                        "tokens": args.context, "seconds": head["prefill_s"],
                        "tok_s": args.context / head["prefill_s"],
                        "note": "wall clock of q35_generate(prompt, 1) (the prompt, then its last token decoded)"},
            "gpu_launches": head["launches"],
            "gpu_launches_note": "kernel nodes of the decode graphs replayed in the timed region (this rank)",
            "e2e": e2e,
            "roofline": roofline,
            "roofline_kernels": {"k_attn": attn_roof, "k_qmv": qmv_roof},
            "step_roofline": {"bytes_per_token": head["step_bytes"],
                              "achieved_gbs": head["step_bytes"] * (head["tok_s"] / streams) / 1e9,
                              "frac": head["step_frac"], "peak_kind": peak_kind},
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "config5": config5,
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
