"""Op-level benchmarks of the q35 kernels on the BASELINE.json configs 1-3.

  python -m q35.opbench --op qmv|gdn|attn|head|qgemm [--len N] [--iters K] [--copies R]
                        [--tokens T --rows N --k K]   (qgemm: the tensor-core Q4 GEMM)
  python -m q35.opbench --op pattn --len P0 --tokens T  (prompt-chunk flash attention of T
                        tokens at positions P0.., tensor FLOP/s of its two GEMMs)
  python -m q35.opbench --op prefill --len N            (an N-token prompt through the session
                        API on the tensor cores: wall-clock tok/s)
  python -m q35.opbench --op batch --len N --members B [--route exact|tensor|single]
                        (B sessions at context N decoded as one batch: one session
                        consumes a seeded N-token prompt (tensor cores), B - 1 copies
                        of it join,
                        4 warm-up steps, --iters timed steps; aggregate tok/s by
                        CUDA events on the batch stream)

Each call works on a fresh copy of its big operands (weights, recurrent
state, or K/V cache), rotating over enough copies that the working set is
larger than the 126 MB L2, so every call streams its bytes from HBM. The
timed calls are captured in one CUDA graph and replayed after warm-up; times
are CUDA events on the replay stream; the line printed is JSON with the
per-call time and the algorithmic bytes moved per call.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def main():
    import numpy as np
    import torch
    import q35
    import inputs as I

    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["qmv", "gdn", "attn", "head", "qgemm", "pattn", "prefill", "batch"],
                    required=True)
    ap.add_argument("--members", type=int, default=8)
    ap.add_argument("--route", choices=["exact", "tensor", "single"], default="tensor")
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--rows", type=int, default=7168)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--len", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--copies", type=int, default=0)
    args = ap.parse_args()
    dev = torch.device("cuda:0")
    def T(a):
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint16:
            a = a.view(np.int16)
        elif a.dtype == np.uint32:
            a = a.view(np.int32)
        return torch.from_numpy(a).to(dev)

    if args.op == "prefill":
        import time
        d = os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3")
        if not os.path.exists(os.path.join(d, "model.safetensors")):
            q35.write_synthetic_model(d, 3)
        m = q35.Model.load(d, 0, capacity=((args.len + 2048 + 63) // 64) * 64, tensor_prompt=True)
        rng = np.random.default_rng(1)
        m.generate([int(v) for v in rng.integers(0, q35.VOCAB, 2048)], 1, True)  # warm-up
        prompt = [int(v) for v in rng.integers(0, q35.VOCAB, args.len)]
        t0 = time.perf_counter()
        m.generate(prompt, 1, True)
        dt = time.perf_counter() - t0
        m.close()
        print(json.dumps({"op": "prefill", "len": args.len, "seconds": dt, "tok_s": args.len / dt,
                          "note": "wall clock of generate(prompt, 1): the prompt on the tensor cores, then "
                                  "its last token decoded"}))
        return
    if args.op == "batch":
        d = os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3")
        if not os.path.exists(os.path.join(d, "model.safetensors")):
            q35.write_synthetic_model(d, 3)
        n = 1 if args.route == "single" else args.members
        steps = args.iters
        cap = ((args.len + 1 + 4 + steps + 64 + 63) // 64) * 64
        ms = [q35.Model.load(d, 0, capacity=cap, tensor_prompt=True) for _ in range(n)]
        rng = np.random.default_rng(2)
        ms[0].generate([int(v) for v in rng.integers(0, q35.VOCAB, args.len)], 1, True)
        for m in ms[1:]:
            m.copy_from(ms[0])
        if args.route == "single":
            ms[0].decode_timed(4)
            t_ms = ms[0].decode_timed(steps)
        else:
            bt = q35.Batch(ms, tensor_cores=args.route == "tensor")
            bt.decode_timed(4)
            t_ms = bt.decode_timed(steps)
            bt.close()
        for m in ms:
            m.close()
        us = 1000.0 * t_ms / steps
        print(json.dumps({"op": "batch", "len": args.len, "route": args.route, "members": n, "steps": steps,
                          "us_per_step": us, "tok_s": n * steps / (t_ms / 1000.0)}))
        return
    if args.op == "qmv":
        w, s, b, x = I.config1(0)
        copies = args.copies or 256
        W = T(w).repeat(copies, 1).view(copies, *w.shape)
        S = T(s).repeat(copies, 1).view(copies, *s.shape)
        B = T(b).repeat(copies, 1).view(copies, *b.shape)
        X = T(x)
        y = torch.empty(3584, dtype=torch.uint16, device=dev)
        nbytes = w.nbytes + s.nbytes + b.nbytes + x.nbytes + 3584 * 2

        def call(i):
            q35.qmv_q4(W[i % copies], S[i % copies], B[i % copies], X, out=y)
    elif args.op == "gdn":
        d = I.config2(1)
        copies = args.copies or 64
        st = T(d["state"]).repeat(copies).view(copies, -1)
        hist = T(d["hist"])
        ws = q35.workspace("gdn")
        ins = {k: T(d[k]) for k in ("raw", "z", "a", "b", "conv_w", "a_log", "dt", "norm_w", "ow", "os", "ob", "res")}
        nbytes = 2 * d["state"].nbytes + d["conv_w"].nbytes + 2 * d["hist"].nbytes + d["ow"].nbytes + \
            d["os"].nbytes + d["ob"].nbytes + 2 * (6144 + 2048 + 32 + 1024 + 1024)

        def call(i):
            q35.gdn_step(ins["raw"], ins["z"], ins["a"], ins["b"], hist, ins["conv_w"], ins["a_log"], ins["dt"],
                         st[i % copies], ins["norm_w"], ins["ow"], ins["os"], ins["ob"], residual=ins["res"], ws=ws)
    elif args.op == "head":
        # tied-embedding head of the vocabulary: [248320][1024] Q4, final norm gain, x
        copies = args.copies or 2
        g = torch.Generator(device=dev).manual_seed(5)
        W = torch.randint(-2**31, 2**31 - 1, (copies, q35.VOCAB, 128), dtype=torch.int32, device=dev, generator=g)
        rs = I.Rng(5, 9)
        sc = T(np.full((q35.VOCAB, 16), I.f2bf(np.array([0.004], np.float32))[0], np.uint16))
        bi = T(I.f2bf(rs.normal(q35.VOCAB * 16, 0.03)).reshape(q35.VOCAB, 16))
        x = T(I.f2bf(rs.normal(1024)))
        gain = T(I.f2bf(1.0 + rs.normal(1024, 0.02)))
        ws = q35.workspace("head")
        nbytes = q35.VOCAB * (512 + 64) + q35.VOCAB * 2

        def call(i):
            q35.head_argmax(W[i % copies], sc, bi, x, gain, ws=ws)
    elif args.op == "qgemm":
        n, k, t = args.rows, args.k, args.tokens
        g = torch.Generator(device="cpu").manual_seed(5)
        w = torch.randint(-2**31, 2**31 - 1, (n, k // 8), generator=g, dtype=torch.int64).to(torch.int32)
        sc = (torch.rand((n, k // 64), generator=g) * 0.015 + 0.005).to(torch.bfloat16)
        per = n * k // 2 + 2 * n * (k // 64) * 2
        copies = args.copies or max(2, int(np.ceil(300e6 / per)))
        W = [w.to(dev) for _ in range(copies)]
        S = sc.to(dev).view(torch.int16)
        B = (-8.0 * sc.float()).to(torch.bfloat16).to(dev).view(torch.int16)
        X = torch.randn((t, k), generator=g).to(torch.bfloat16).to(dev).view(torch.int16)
        Y = torch.empty((t, n), dtype=torch.int16, device=dev)
        wsb = torch.empty(int(q35.lib().q35_op_qgemm_workspace_bytes(t, n, k)), dtype=torch.uint8, device=dev)
        nbytes = per + t * k * 2 + t * n * 2
        flops = 2.0 * n * k * t

        def call(i):
            q35.qgemm_q4(W[i % copies], S, B, X, out=Y, ws=wsb)
    elif args.op == "pattn":
        p0, t = args.len, args.tokens
        cap = ((p0 + t + 63) // 64) * 64
        r = I.Rng(7, 5)
        kc = np.zeros((2, cap, 256), np.uint16)
        vc = np.zeros((2, cap, 256), np.uint16)
        if p0:
            kc[:, :p0] = I.f2bf(r.normal(2 * p0 * 256)).reshape(2, p0, 256)
            vc[:, :p0] = I.f2bf(r.normal(2 * p0 * 256)).reshape(2, p0, 256)
        copies = args.copies or 1
        KC = [T(I.to_chain_major(kc)) for _ in range(copies)]
        VC = [T(I.to_chain_major(vc)) for _ in range(copies)]
        ins = {"q_raw": T(I.f2bf(r.normal(t * 4096)).reshape(t, 4096)),
               "k_raw": T(I.f2bf(r.normal(t * 512)).reshape(t, 512)),
               "v_raw": T(I.f2bf(r.normal(t * 512)).reshape(t, 512)),
               "q_gain": T(I.f2bf(1.0 + r.normal(256, 0.02))), "k_gain": T(I.f2bf(1.0 + r.normal(256, 0.02)))}
        ws, _ = q35._prompt_ws(t, cap, dev)
        gated = torch.empty((t, 2048), dtype=torch.int16, device=dev)
        keys = t * p0 + t * (t + 1) // 2  # (query token, key) pairs under the causal mask
        flops = 2.0 * 2 * 256 * 8 * keys  # S = Q K^T and O = P V for 8 query heads
        nbytes = 2 * 2 * (p0 + t) * 256 * 2 + t * (4096 + 2 * 512 + 2048) * 2

        def call(i):
            q35.prompt_attention(ins["q_raw"], ins["k_raw"], ins["v_raw"], ins["q_gain"], ins["k_gain"],
                                 KC[i % copies], VC[i % copies], cap, p0, ws=ws, out=gated)
    else:
        d = I.config3(2, args.len)
        per = d["kc"].nbytes * 2
        copies = args.copies or max(2, int(np.ceil(300e6 / per)))
        KC = [T(d["kc"]) for _ in range(copies)]
        VC = [T(d["vc"]) for _ in range(copies)]
        ins = {k: T(d[k]) for k in ("q_raw", "k_raw", "v_raw", "q_gain", "k_gain")}
        ws = q35.workspace("attn")
        nbytes = 2 * 2 * args.len * 256 * 2 + 4096 * 2 + 2048 * 2

        def call(i):
            q35.attn_decode(ins["q_raw"], ins["k_raw"], ins["v_raw"], ins["q_gain"], ins["k_gain"],
                            KC[i % copies], VC[i % copies], d["cap"], d["pos"], ws=ws)

    for i in range(10):
        call(i)
    torch.cuda.synchronize()
    # the timed calls are replayed from one CUDA graph, so host-side launch
    # cost does not show up as device time
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(args.iters):
            call(i)
    g.replay()
    torch.cuda.synchronize()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    e.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(e) * 1e3 / args.iters
    out = {"op": args.op, "len": args.len if args.op == "attn" else None, "us_per_call": us,
           "bytes_per_call": nbytes, "gbs": nbytes / us / 1e3, "copies": copies}
    if args.op == "qgemm":
        out.update({"tokens": args.tokens, "rows": args.rows, "k": args.k, "tflops": flops / us / 1e6})
    if args.op == "pattn":
        out.update({"len": args.len, "tokens": args.tokens, "flops_per_call": flops, "tflops": flops / us / 1e6})
    print(json.dumps(out))


if __name__ == "__main__":
    main()
