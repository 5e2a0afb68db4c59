"""Golden vectors of the B200 tensor core's bf16 MMA accumulation, written on
a GPU through the engine's own GEMM (run: python tests/golden/make_mma_golden.py [OUT.npz]
on a B200; writes tests/golden/tc_mma_steps.npz by default).

The GEMM (q35_op_qgemm_q4) is given weights that dequantise to exactly 1
(scale 0, bias 1), so every product equals the activation x[t][k]. With
K = 512, one 128-row tile and 256 tokens, its plan makes 8 K splits of one
64-wide block each and stores their f32 partials in the caller's workspace
(after a 16,640-byte header) as part[(split * T + t) * 128 + row]. Only
k < 64 is nonzero, so split 0's partial is the raw f32 result of four
16-wide MMA steps over x[t][0:64]. Case kinds: 16 terms (one step), 32 (two
steps), 64 (four steps), 16 with a wider exponent spread. The oracle's
tc_step restatement is checked against these on the CPU
(tests/test_oracle.py)."""
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
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "tc_mma_steps.npz")
    np.savez_compressed(out, x=np.concatenate(all_x), nk=np.concatenate(all_n), gpu=np.concatenate(all_g))
    print("wrote", out)


if __name__ == "__main__":
    main()
