"""Golden vectors of the B200 tensor core's bf16 MMA accumulation, written on
a GPU through the engine's own GEMM (run on a B200:
python tests/golden/make_mma_golden.py [OUT_DIR]; writes tc_mma_steps.npz and
tc_mma_chains.npz into tests/golden/ by default).

tc_mma_steps.npz: weights that dequantise to exactly 1 (scale 0, bias 1), so
every product equals the activation x[t][k]. With K = 512, one 128-row tile
and 256 tokens, the GEMM's plan makes 8 K splits of one 64-wide block each
and stores their f32 partials in the caller's workspace (after a 16,640-byte
header) as part[(split * T + t) * rows + row]. Only k < 64 is nonzero, so
split 0's partial is the raw f32 result of four 16-wide MMA steps over
x[t][0:64]. Case kinds: 16 terms (one step), 32 (two), 64 (four), 16 with a
wider exponent spread.

tc_mma_chains.npz: random Q4 weights with scales and biases spread over 14
binades and activations over 13, so the products carry 16-bit mantissas of
widely different exponents. 74 row tiles and K = 4096 make the plan take 4 K
splits of 16 blocks (64 MMA steps); token t's activations are nonzero only in
the first 16, 32, 64 or all 1,024 elements of each split (1, 2, 4 or 64
steps). Each case stores both factors (bf16 bits: the dequantised weight
bf16(s q + b), rounded once, and the activation) of the steps that count and
the device's f32 partial.

The oracle's tc_step restatement is checked against both on the CPU
(tests/test_oracle.py).
"""
import os
import random
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "enginesmith-qwen35-08b-long-decode-m5max-round005_b200"))

T, N, K = 256, 128, 512
HDR = 4096 * 4 + 256
NK = {0: 16, 1: 32, 2: 64, 3: 16}


def cases(seed):
    rng = random.Random(seed)
    xs = np.zeros((T, 64), np.float32)
    nk = np.zeros(T, np.int32)
    for t in range(T):
        kind = t % 4
        e0 = rng.randrange(-4, 5)
        spread = 40 if kind == 3 else 26
        nk[t] = NK[kind]
        for k in range(NK[kind]):
            if rng.random() < 0.15:
                continue
            sign = -1.0 if rng.random() < 0.5 else 1.0
            xs[t, k] = sign * (1 + rng.randrange(128) / 128.0) * 2.0 ** (e0 - rng.randrange(0, spread))
    return xs, nk


def main():
    import torch
    import q35
    dev = torch.device("cuda:0")
    w = torch.zeros((N, K // 8), dtype=torch.int32, device=dev)
    sc = torch.zeros((N, K // 64), dtype=torch.int16, device=dev)
    bi = torch.full((N, K // 64), 0x3F80, dtype=torch.int16, device=dev)  # bf16 1.0
    ws = torch.zeros(int(q35.lib().q35_op_qgemm_workspace_bytes(T, N, K)), dtype=torch.uint8, device=dev)
    all_x, all_n, all_g = [], [], []
    for seed in range(4):
        xs, nk = cases(seed)
        full = np.zeros((T, K), np.float32)
        full[:, :64] = xs
        xb = (torch.from_numpy(full).view(torch.int32) >> 16).to(torch.int16).to(dev)
        q35.qgemm_q4(w, sc, bi, xb, ws=ws)
        torch.cuda.synchronize()
        part = ws[HDR:HDR + 8 * T * N * 4].view(torch.float32).view(8, T, N).cpu().numpy()
        assert np.all(part[:, :, :1] == part) and np.all(part[1:] == 0)
        all_x.append(xs)
        all_n.append(nk)
        all_g.append(part[0, :, 0].copy())
    out_dir = sys.argv[1] if len(sys.argv) > 1 else HERE
    np.savez_compressed(os.path.join(out_dir, "tc_mma_steps.npz"), x=np.concatenate(all_x),
                        nk=np.concatenate(all_n), gpu=np.concatenate(all_g))
    chains(out_dir)
    print("wrote", out_dir)


def f2bf(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf2f(h):
    return (np.ascontiguousarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def chain_inputs(seed, N=9472, K=4096, T=32):
    r = np.random.default_rng(1000 + seed)
    w = r.integers(0, 2**32, (N, K // 8), dtype=np.uint64).astype(np.uint32)
    sc = f2bf(r.standard_normal((N, K // 64)) * np.exp2(r.integers(-12, 2, (N, K // 64))))
    bi = f2bf(r.standard_normal((N, K // 64)) * np.exp2(r.integers(-12, 2, (N, K // 64))))
    x = r.standard_normal((T, K)) * np.exp2(r.integers(-10, 3, (T, K)))
    for t in range(T):  # tokens 0-7: 1 step per split, 8-15: 2, 16-23: 4, 24-31: 64
        x[t].reshape(4, 1024)[:, [1, 2, 4, 64][t // 8] * 16:] = 0
    return w, sc, bi, f2bf(x)


def dequant_row(w, sc, bi, r, K):
    """bf16(s q + b) of row r, one rounding (as the GEMM's packed bf16 fma)."""
    q = ((w[r][:, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(-1).astype(np.float64)
    v = np.repeat(bf2f(sc[r]).astype(np.float64), 64) * q + np.repeat(bf2f(bi[r]).astype(np.float64), 64)
    m, e = np.frexp(v)
    return f2bf(np.ldexp(np.rint(np.ldexp(m, 8)), e - 8).astype(np.float32))


def chains(out_dir, seeds=2, rows=16, long_cases=64):
    import torch
    import q35
    N, K, T = 9472, 4096, 32
    acc = {n: ([], [], []) for n in (1, 2, 4, 64)}
    for seed in range(seeds):
        w, sc, bi, x = chain_inputs(seed, N, K, T)
        W = torch.from_numpy(w.view(np.int32)).cuda()
        S = torch.from_numpy(sc.view(np.int16)).cuda()
        B = torch.from_numpy(bi.view(np.int16)).cuda()
        X = torch.from_numpy(x.view(np.int16)).cuda()
        ws = torch.zeros(int(q35.lib().q35_op_qgemm_workspace_bytes(T, N, K)), dtype=torch.uint8, device="cuda")
        q35.qgemm_q4(W, S, B, X, ws=ws)
        torch.cuda.synchronize()
        part = ws[HDR:HDR + 4 * T * N * 4].view(torch.float32).view(4, T, N)[:, :, :rows].cpu().numpy()
        for r in range(rows):
            wd = dequant_row(w, sc, bi, r, K)
            for t in range(T):
                n = [1, 2, 4, 64][t // 8]
                for sp in range(4):
                    a, b, g = acc[n]
                    if n == 64 and len(g) >= long_cases:
                        continue
                    a.append(wd[sp * 1024:sp * 1024 + 16 * n])
                    b.append(x[t, sp * 1024:sp * 1024 + 16 * n])
                    g.append(part[sp, t, r])
    out = {}
    for n, (a, b, g) in acc.items():
        out[f"a{n}"], out[f"b{n}"], out[f"gpu{n}"] = np.array(a), np.array(b), np.array(g, np.float32)
    np.savez_compressed(os.path.join(out_dir, "tc_mma_chains.npz"), **out)


if __name__ == "__main__":
    main()
