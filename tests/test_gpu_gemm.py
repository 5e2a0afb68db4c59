"""Q4 GEMM on the tensor cores (tcgen05, the batched-session route) against a
float32 reference of the same operator: W dequantised as bf16(s q + b) (each
s q is exact, so the dequantised weights are identical), y = x W^T
accumulated in float32 (TF32 off), output rounded to bf16. The tensor core's
accumulation order differs from the reference's, so the bar is the north
star's tolerance (norm-wise relative error <= 1e-2), and per output at most
one bf16 ulp plus 1e-4 of the largest output (float32 accumulation order). Shapes cover every projection of the model,
the vocabulary head, token counts 1..256 (the MMA's N: padding) and above
(token tiles of 256, the last one partial, as a prompt chunk uses), K splits (K = 2048, 3584) and partial row tiles."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def make(n, k, t, seed):
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    codes = torch.randint(0, 2**31 - 1, (n, k // 8), generator=g, dtype=torch.int64)
    codes = (codes * 2 + torch.randint(0, 2, (n, k // 8), generator=g)).to(torch.int64) & 0xFFFFFFFF
    w = codes.to(torch.int64).to(torch.int32)  # same bits
    scales = (torch.rand((n, k // 64), generator=g) * 0.015 + 0.005).to(torch.bfloat16)
    biases = (-8.0 * scales.float()).to(torch.bfloat16)
    x = torch.randn((t, k), generator=g).to(torch.bfloat16)
    return w, scales, biases, x


def reference(w, scales, biases, x):
    import torch
    n, kw = w.shape
    sh = torch.arange(8, dtype=torch.int32) * 4
    q = ((w.unsqueeze(-1) >> sh) & 15).reshape(n, kw * 8).float()
    s = scales.float().repeat_interleave(64, dim=1)
    b = biases.float().repeat_interleave(64, dim=1)
    wd = (s * q + b).to(torch.bfloat16).float()
    return x.float().cuda() @ wd.cuda().T


@pytest.mark.parametrize("t,n,k", [
    (1, 3584, 1024), (8, 8224, 1024), (16, 1024, 3584), (17, 1024, 2048), (64, 7168, 1024),
    (100, 5120, 1024), (256, 4096, 1024), (48, 248320, 1024), (200, 1000, 2048),
    (300, 8224, 1024), (2048, 1024, 3584), (1000, 3584, 1024),
])
def test_qgemm_matches_f32(cuda, t, n, k):
    import torch
    import q35
    torch.backends.cuda.matmul.allow_tf32 = False
    w, s, b, x = make(n, k, t, seed=n + k + t)
    ref = reference(w, s, b, x)
    W, S, B, X = w.cuda(), s.cuda().view(torch.uint16), b.cuda().view(torch.uint16), x.cuda().view(torch.uint16)
    y = q35.qgemm_q4(W, S, B, X)
    torch.cuda.synchronize()
    yf = y.view(torch.bfloat16).float()
    err = float(torch.linalg.norm(yf - ref) / torch.linalg.norm(ref))
    assert err <= 1e-2, err
    # per output: the bf16 rounding (one ulp) plus float32 accumulation-order
    # error, which is absolute (~K eps |terms|) and shows near cancellation
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - 7)
    bound = ulp + 1e-4 * float(ref.abs().max())
    worst = float(((yf - ref).abs() / bound).max())
    assert worst <= 1.0, worst
    # residual form: bf16(res + bf16(W x)), residual aliasing the output
    res = torch.randn((t, n), device="cuda").to(torch.bfloat16)
    y2 = res.clone().view(torch.uint16)
    q35.qgemm_q4(W, S, B, X, residual=y2, out=y2)
    torch.cuda.synchronize()
    want = (res.float() + yf.to(torch.bfloat16).float()).to(torch.bfloat16)
    got = y2.view(torch.bfloat16)
    assert float((got.float() - want.float()).abs().max()) <= float(want.float().abs().max()) * 2**-7


def test_qgemm_rejects_bad_arguments(cuda):
    import torch
    import q35
    w, s, b, x = make(256, 1024, 4, 1)
    W, S, B, X = w.cuda(), s.cuda().view(torch.uint16), b.cuda().view(torch.uint16), x.cuda().view(torch.uint16)
    with pytest.raises(q35.Q35Error):
        q35.qgemm_q4(W, S, B, torch.zeros((4097, 1024), dtype=torch.uint16, device="cuda"))
    with pytest.raises(q35.Q35Error):
        q35.qgemm_q4(W[:, :4], S, B, X)  # k = 32, not a multiple of 512


@pytest.mark.parametrize("t,n,k", [
    (1, 3584, 1024), (8, 1024, 3584), (17, 1024, 2048), (64, 7168, 1024), (300, 1000, 2048), (5, 512, 4096),
])
def test_qgemm_bitexact_with_oracle_restatement(cuda, oracle_threads, t, n, k):
    """The GEMM equals the oracle's restatement of it bit for bit (weights
    bf16(s q + b) rounded once; per K split, 16-wide MMA steps with the
    tensor core's measured accumulation rule, tc_step; split partials summed
    in order; bf16 output, and the residual form)."""
    import torch
    import q35
    O = oracle_threads
    w, s, b, x = make(n, k, t, seed=7 * n + k + t)
    W, S, B, X = w.cuda(), s.cuda().view(torch.uint16), b.cuda().view(torch.uint16), x.cuda().view(torch.uint16)
    y = q35.qgemm_q4(W, S, B, X).cpu().numpy().view(np.uint16)
    torch.cuda.synchronize()
    wn = w.numpy().view(np.uint32)
    sn, bn, xn = (a.view(torch.int16).numpy().view(np.uint16) for a in (s, b, x))
    f = O.qgemm_tc(wn, sn, bn, xn)
    want = O.f2bf(f)
    bad = int(np.count_nonzero(y != want))
    assert bad == 0, f"{bad} of {y.size} outputs differ"
    res = torch.randn((t, n)).to(torch.bfloat16)
    y2 = res.clone().view(torch.uint16).cuda()
    q35.qgemm_q4(W, S, B, X, residual=y2, out=y2)
    rn = res.view(torch.int16).numpy().view(np.uint16)
    want2 = O.f2bf(O.bf2f(rn) + O.bf2f(want))
    assert np.array_equal(y2.cpu().numpy().view(np.uint16), want2)
