"""CPU checks of the oracle (no GPU): it is pinned against independent float64
restatements of each operator's mathematics, against the known-answer cases
of the reference's own audits, and against the committed golden fixtures."""
import os

import numpy as np
import pytest

import inputs as I

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def O(oracle_threads):
    return oracle_threads


def ulp_bf16(r):
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(r), 1e-30))) - 7)


def test_bf16_rounding(O):
    xs = np.array([1.0, 1.00390625, 1.005859375, 1.0078125, -2.5, 3.4e38, 1e-40, np.inf, -np.inf], np.float32)
    for x in xs:
        assert O.lib().orc_f2bf(float(x)) == I.f2bf(np.array([x]))[0]
    # ties to even: 1 + 2^-8 is exactly half-way between bf16 1.0 and 1.0078125
    assert I.bf2f(I.f2bf(np.array([1.00390625], np.float32)))[0] == 1.0
    assert I.bf2f(I.f2bf(np.array([1.01171875], np.float32)))[0] == np.float32(1.015625)


def test_fexp_accuracy(O):
    xs = np.concatenate([np.linspace(-103.9, 88.7, 20001), np.linspace(-1, 1, 2001),
                         I.Rng(1).normal(5000, 20.0)]).astype(np.float32)
    f = np.array([O.lib().orc_fexp(float(x)) for x in xs], np.float64)
    ref = np.exp(xs.astype(np.float64))
    ok = ref > 1.2e-38  # normal range
    rel = np.abs(f[ok] - ref[ok]) / ref[ok]
    assert rel.max() < 3 * 2.0 ** -24, rel.max()
    assert O.lib().orc_fexp(0.0) == 1.0
    assert O.lib().orc_fexp(float("-inf")) == 0.0
    assert O.lib().orc_fexp(-3.4e38) == 0.0


def test_sigmoid_softplus_steps(O):
    for x in I.Rng(2).normal(2000, 5.0):
        e = I.bf2f(I.f2bf(np.float32(np.exp(abs(np.float64(x))))))[0]
        d = I.bf2f(I.f2bf(np.float32(1.0) + e))[0]
        y = I.bf2f(I.f2bf(np.float32(1.0) / d))[0]
        want = I.bf2f(I.f2bf(np.float32(y if x < 0 else np.float32(1.0) - y)))[0]
        assert O.lib().orc_sigmoid_bf(float(x)) == want
    # softplus against the float64 function (BF16 steps: within 2 bf16 ulps)
    for x in I.Rng(3).normal(500, 4.0):
        v = O.lib().orc_softplus_bf(float(x))
        r = np.log1p(np.exp(-abs(float(x)))) + max(float(x), 0.0)
        assert abs(v - r) <= 2 * ulp_bf16(r) + 1e-6


def dequant(w, s, b):
    q = I.unpack_q4(w).astype(np.float64)
    n, k = q.shape
    sc = np.repeat(I.bf2f(s).astype(np.float64), 64, axis=1)
    bi = np.repeat(I.bf2f(b).astype(np.float64), 64, axis=1)
    return sc * q + bi


@pytest.mark.parametrize("n,k,seed", [(3584, 1024, 0), (1024, 2048, 10), (1024, 3584, 11), (16, 1024, 12)])
def test_qmv_matches_float64(O, n, k, seed):
    w, s, b, _ = I.config1(seed, n, k)
    x = I.f2bf(I.Rng(seed, 9).normal(k))
    x[:8] = I.f2bf(np.array([0, -0.0, 1, -1, 1e-5, -1e-5, 88, -88], np.float32))
    ref = dequant(w, s, b) @ I.bf2f(x).astype(np.float64)
    yf = O.qmv_q4_f32(w, s, b, x).astype(np.float64)
    assert np.max(np.abs(yf - ref)) <= 1e-5 * np.max(np.abs(ref))
    yb = O.qmv_q4(w, s, b, x)
    assert np.all(np.abs(I.bf2f(yb) - ref) <= ulp_bf16(ref) + 1e-6 * np.max(np.abs(ref)))


def test_embedding_known_answer(O):
    w, s, b, _ = I.config1(0)
    q = I.unpack_q4(w)
    for t in (0, 7, 3583):
        want = I.f2bf((I.bf2f(np.repeat(s[t], 64)) * q[t].astype(np.float32)) + I.bf2f(np.repeat(b[t], 64)))
        assert np.array_equal(O.embedding_q4(w, s, b, t), want)


def test_rms_norm_matches_float64(O):
    r = I.Rng(4)
    x = I.f2bf(r.normal(1024, 3.0))
    g = I.f2bf(1.0 + r.normal(1024, 0.02))
    xf = I.bf2f(x).astype(np.float64)
    ref = xf / np.sqrt(np.mean(xf * xf) + 1e-6) * I.bf2f(g)
    out = I.bf2f(O.rms_norm(x, g)).astype(np.float64)
    assert np.all(np.abs(out - ref) <= 2 * ulp_bf16(ref) + 1e-7)


def test_gdn_step_matches_float64(O):
    """Delta rule S = e^g S + beta k (v - S^T k)^T, o = S^T q."""
    d = I.config2(1)
    hist = d["hist"].copy()
    conv, g, beta = O.gdn_conv_prepare(d["raw"], d["a"], d["b"], hist, d["conv_w"], d["a_log"], d["dt"])
    # history shift
    assert np.array_equal(hist[:6144], d["hist"][6144:12288])
    assert np.array_equal(hist[12288:], d["raw"])
    # conv + SiLU against float64
    h = I.bf2f(d["hist"]).astype(np.float64).reshape(3, 6144)
    wv = I.bf2f(d["conv_w"]).astype(np.float64).reshape(6144, 4)
    acc = h[0] * wv[:, 0] + h[1] * wv[:, 1] + h[2] * wv[:, 2] + I.bf2f(d["raw"]) * wv[:, 3]
    silu = acc / (1 + np.exp(-acc))
    cf = I.bf2f(conv).astype(np.float64)
    assert np.all(np.abs(cf[4096:] - silu[4096:]) <= 4 * ulp_bf16(silu[4096:]) + 1e-6)
    # q, k are l2-normalised (q additionally scaled by 1/sqrt(128)^2 = 1/128, k by 1/sqrt(128))
    for blk, scale in ((0, 1 / 128), (1, 1 / np.sqrt(128))):
        for hh in range(16):
            v = silu[blk * 2048 + hh * 128: blk * 2048 + hh * 128 + 128]
            ref = v / np.sqrt(np.sum(v * v) + 1e-6) * np.sqrt(128) * scale
            got = cf[blk * 2048 + hh * 128: blk * 2048 + hh * 128 + 128]
            assert np.linalg.norm(got - ref) <= 2e-2 * np.linalg.norm(ref)
    # gates
    a = I.bf2f(d["a"]).astype(np.float64) + I.bf2f(d["dt"])
    g_ref = np.exp(-np.exp(d["a_log"].astype(np.float64)) * np.log1p(np.exp(a)))
    assert np.allclose(g, g_ref, rtol=2e-2)
    assert np.allclose(I.bf2f(beta), 1 / (1 + np.exp(-I.bf2f(d["b"]).astype(np.float64))), atol=8e-3)
    # recurrence against float64 from the same inputs
    st = d["state"].copy()
    y = O.gdn_recur(conv, g, beta, st)
    S = d["state"].astype(np.float64).reshape(16, 128, 128)
    Q = cf[:2048].reshape(16, 128)
    K = cf[2048:4096].reshape(16, 128)
    V = cf[4096:].reshape(16, 128)
    S = S * g.astype(np.float64)[:, None, None]
    mem = np.einsum("hvk,hk->hv", S, K)
    delta = (V - mem) * I.bf2f(beta).astype(np.float64)[:, None]
    S = S + delta[:, :, None] * K[:, None, :]
    o = np.einsum("hvk,hk->hv", S, Q)
    assert np.max(np.abs(st.reshape(16, 128, 128) - S)) <= 1e-5 * np.max(np.abs(S))
    assert np.linalg.norm(I.bf2f(y) - o.reshape(-1)) <= 1e-2 * np.linalg.norm(o)


def attention_f64(query, kc, vc, length):
    q = I.bf2f(query).astype(np.float64).reshape(8, 256) / 16
    out = np.zeros((8, 256))
    for h in range(8):
        k = I.bf2f(kc[h // 4, :length]).astype(np.float64)
        v = I.bf2f(vc[h // 4, :length]).astype(np.float64)
        s = k @ q[h]
        p = np.exp(s - s.max())
        out[h] = p @ v / p.sum()
    return out.reshape(-1)


@pytest.mark.parametrize("length", [1, 31, 1023, 1024, 1025, 4096])
def test_attention_matches_float64(O, length):
    c = I.config3(2, length)
    kc, vc = c["kc"].copy(), c["vc"].copy()
    q = O.attn_prepare(c["q_raw"], c["k_raw"], c["v_raw"], c["q_gain"], c["k_gain"], c["pos"], c["cap"], kc, vc)
    o = O.attn_decode_f32(q, kc, vc, length, c["cap"]).astype(np.float64)
    ref = attention_f64(q, kc, vc, length)
    # the reference route keeps bf16 partials from 1024 keys on
    tol = 2e-3 if length >= 1024 else 1e-5
    assert np.linalg.norm(o - ref) <= tol * np.linalg.norm(ref)


@pytest.mark.parametrize("n,k,seed", [(3584, 1024, 0), (1024, 2048, 4), (77, 3584, 9)])
def test_gemm_numerics_matvec(O, n, k, seed):
    """The tensor-core routes' matvec restatement (weights bf16(s q + b)
    rounded once; per 16-wide K step the tensor core's truncating
    accumulation, tc_step; K splits summed in order): against the exact dot
    product of the same weights in float64, within the accumulation's own
    error bound. Each step truncates its 17 aligned terms 2 bits below the
    f32 ulp of their largest and the sum once more, so its error is below
    17/4 + 1 ulps of the largest magnitude it sees, which the sum of
    |products| bounds; each split partial adds one rounding."""
    w, s, b, x = I.config1(seed, n, k)
    q = I.unpack_q4(w).astype(np.float64)
    sc = np.repeat(I.bf2f(s).astype(np.float64), 64, axis=1)
    bi = np.repeat(I.bf2f(b).astype(np.float64), 64, axis=1)
    m, e = np.frexp(sc * q + bi)  # exact in float64; one bf16 rounding, ties to even
    wd = np.ldexp(np.rint(np.ldexp(m, 8)), e - 8)
    xv = I.bf2f(x).astype(np.float64)
    ref = wd @ xv
    got = O.qmv_gemm_f32(w, s, b, x).astype(np.float64)
    mag = np.abs(wd) @ np.abs(xv)
    steps = k // 16
    bound = (steps * (17 / 4 + 1) + 8) * 2.0 ** -23 * mag
    assert np.all(np.abs(got - ref) <= bound), float(np.max(np.abs(got - ref) / bound))
    # and the tensor core's rule is not the exact sum rounded once: some rows differ from it
    assert np.any(got != ref.astype(np.float32))


def attention_flash_f64(query, kc, vc, length):
    """The tensor-core prompt route's attention: exact scores rounded to f32,
    weights bf16(2^((s - max) log2(e) / 16)), exact weighted sums."""
    q = I.bf2f(query).astype(np.float64).reshape(8, 256)
    out = np.zeros((8, 256))
    for h in range(8):
        k = I.bf2f(kc[h // 4, :length]).astype(np.float64)
        v = I.bf2f(vc[h // 4, :length]).astype(np.float64)
        s = (k @ q[h]).astype(np.float32)
        arg = ((s - s.max()).astype(np.float32) * np.float32(0.0901684400555602)).astype(np.float32)
        p = I.bf2f(I.f2bf(np.exp2(arg.astype(np.float64)).astype(np.float32))).astype(np.float64)
        out[h] = p @ v / p.sum()
    return out.reshape(-1)


@pytest.mark.parametrize("length", [1, 31, 64, 1025])
def test_flash_attention_restatement(O, length):
    """The oracle's restatement of the prompt route's attention follows its
    formula, and stays within the bf16 weights' error of exact attention."""
    c = I.config3(2, length)
    kc, vc = c["kc"].copy(), c["vc"].copy()
    q = O.attn_prepare(c["q_raw"], c["k_raw"], c["v_raw"], c["q_gain"], c["k_gain"], c["pos"], c["cap"], kc, vc)
    o = O.attn_flash_f32(q, kc, vc, length, c["cap"]).astype(np.float64)
    ref = attention_flash_f64(q, kc, vc, length)
    assert np.linalg.norm(o - ref) <= 1e-6 * np.linalg.norm(ref)
    exact = attention_f64(q, kc, vc, length)
    assert np.linalg.norm(o - exact) <= 1e-2 * np.linalg.norm(exact)


def test_rope_and_qk_norm(O):
    """Per-head RMSNorm, then RoPE on dims < 64 with pairs (i, i+32), theta 1e7."""
    c = I.config3(2, 100)
    kc, vc = c["kc"].copy(), c["vc"].copy()
    pos = c["pos"]
    q = O.attn_prepare(c["q_raw"], c["k_raw"], c["v_raw"], c["q_gain"], c["k_gain"], pos, c["cap"], kc, vc)
    x = I.bf2f(c["q_raw"]).astype(np.float64).reshape(8, 512)[:, :256]
    n = x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + 1e-6) * I.bf2f(c["q_gain"])
    inv = 1e7 ** (-np.arange(32) / 32)
    ang = pos * inv
    r = n.copy()
    r[:, :32] = n[:, :32] * np.cos(ang) - n[:, 32:64] * np.sin(ang)
    r[:, 32:64] = n[:, :32] * np.sin(ang) + n[:, 32:64] * np.cos(ang)
    got = I.bf2f(q).reshape(8, 256).astype(np.float64)
    # bf16 steps before the rotation: element error bounded by a few ulps of the pair's inputs
    scale = np.maximum(np.abs(n), np.abs(np.roll(n, 32, axis=1)))
    assert np.all(np.abs(got - r) <= 4 * ulp_bf16(scale) + 1e-6)
    assert np.linalg.norm(got - r) <= 5e-3 * np.linalg.norm(r)
    assert np.array_equal(vc[:, pos], c["v_raw"].reshape(2, 256))


def test_greedy_known_answers(O):
    # planted maxima: the lowest planted id wins
    lg = I.f2bf(I.Rng(9).normal(248320, 0.5))
    for planted in ([5, 100000], [248319], [0, 31, 32, 1023]):
        x = lg.copy()
        x[planted] = I.f2bf(np.array([9.0], np.float32))[0]
        t, lse = O.greedy(x)
        assert t == min(planted)
    # bf16 log-softmax ties: lse = bf16(log(248318 + e + e^1.015625)) = 12.4375, and
    # 1.015625 - 12.4375 rounds to the same bf16 as 1.0 - 12.4375, so the lower id wins
    x = np.zeros(248320, np.uint16)
    x[7] = I.f2bf(np.array([1.015625], np.float32))[0]
    x[3] = I.f2bf(np.array([1.0], np.float32))[0]
    t, lse = O.greedy(x)
    assert I.bf2f(np.array([lse], np.uint16))[0] == 12.4375
    assert t == 3
    # lse against float64
    ref = np.log(np.sum(np.exp(I.bf2f(lg).astype(np.float64))))
    _, lse = O.greedy(lg)
    assert abs(I.bf2f(np.array([lse], np.uint16))[0] - ref) <= ulp_bf16(ref)


def test_golden_config1(O):
    g = np.load(os.path.join(GOLD, "config1_qmv.npz"))
    w, s, b, x = I.config1(0)
    res = I.f2bf(I.Rng(5).normal(3584))
    assert np.array_equal(O.qmv_q4(w, s, b, x), g["y"])
    assert np.array_equal(O.qmv_q4(w, s, b, x, residual=res), g["y_res"])


def test_golden_config2(O):
    g = np.load(os.path.join(GOLD, "config2_gdn.npz"))
    d = I.config2(1)
    hist, state = d["hist"].copy(), d["state"].copy()
    out = O.gdn_step(d["raw"], d["z"], d["a"], d["b"], hist, d["conv_w"], d["a_log"], d["dt"], state,
                     d["norm_w"], d["ow"], d["os"], d["ob"], residual=d["res"])
    assert np.array_equal(out, g["out"]) and np.array_equal(hist, g["hist"])
    assert np.array_equal(state.reshape(16, 128, 128)[:, ::17, :], g["state_rows"])


@pytest.mark.parametrize("length", [1, 1024, 4096])
def test_golden_config3(O, length):
    g = np.load(os.path.join(GOLD, "config3_attn.npz"))
    c = I.config3(2, length)
    kc, vc = c["kc"].copy(), c["vc"].copy()
    q = O.attn_prepare(c["q_raw"], c["k_raw"], c["v_raw"], c["q_gain"], c["k_gain"], c["pos"], c["cap"], kc, vc)
    assert np.array_equal(O.attn_decode_gate(q, kc, vc, length, c["cap"], c["q_raw"]), g[f"gated_{length}"])
    assert np.array_equal(kc[:, c["pos"]], g[f"krow_{length}"])


def test_golden_tensor_routes(O):
    """The tensor-core routes' restatements reproduce their committed outputs."""
    g = np.load(os.path.join(GOLD, "tensor_routes.npz"))
    for n, k, seed in ((3584, 1024, 0), (1024, 3584, 11)):
        w, s, b, x = I.config1(seed, n, k)
        assert np.array_equal(O.qmv_gemm_f32(w, s, b, x), g[f"gemm_{n}x{k}"])
    for length in (1, 31, 1025, 4096):
        c = I.config3(2, length)
        kc, vc = c["kc"].copy(), c["vc"].copy()
        q = O.attn_prepare(c["q_raw"], c["k_raw"], c["v_raw"], c["q_gain"], c["k_gain"], c["pos"], c["cap"], kc, vc)
        assert np.array_equal(O.attn_flash_gate(q, kc, vc, length, c["cap"], c["q_raw"]), g[f"flash_{length}"])


def test_golden_greedy_audit(O):
    g = np.load(os.path.join(GOLD, "greedy_audit.npz"))
    seed = np.array([0x918BEACD729A], np.uint64)
    for si in range(64):
        lg = O.xorshift_logits(seed, si)
        t, l = O.greedy(lg)
        assert t == g["token"][si] and l == g["lse"][si]


def test_golden_model_tokens(O, synth_model_dir):
    g = np.load(os.path.join(GOLD, "config4_model.npz"))
    om = O.OracleModel(synth_model_dir)
    s = O.OracleSession(om, 256)
    toks = s.generate([int(v) for v in g["prompt"]], len(g["tokens"]))
    assert toks == [int(v) for v in g["tokens"]]


def test_tc_step_rule_cases(O):
    """The tensor core's MMA step as restated (oracle tc_step): terms aligned
    to the largest exponent and truncated to 2 bits below its f32 ulp, summed,
    the sum truncated to f32. Cases that separate it from the other rules
    (sequential round-to-nearest adds, one rounding of the exact sum)."""
    z = [0.0] * 13
    # 1 + 2^-24 + 2^-24: both small terms kept (grid 2^-25): 1 + 2^-23 (sequential adds give 1)
    assert O.tc_step(0.0, [1.0, 2.0 ** -24, 2.0 ** -24] + z) == 1.0 + 2.0 ** -23
    # 1 - 2^-30: the small term truncates to 0 -> 1 (truncating the exact sum gives 1 - 2^-24)
    assert O.tc_step(0.0, [1.0, -(2.0 ** -30), 0.0] + z) == 1.0
    # 1 + 3 * 2^-25 = 1 + 0.75 ulp: truncated -> 1 (rounding the exact sum gives 1 + 2^-23)
    assert O.tc_step(0.0, [1.0, 3 * 2.0 ** -25, 0.0] + z) == 1.0
    # the accumulator is aligned with the products
    assert O.tc_step(2.0 ** 24, [1.0] * 16) == 2.0 ** 24 + 16
    assert O.tc_step(-3.5, [3.5] + [0.0] * 15) == 0.0


def test_tc_step_against_device_golden(O):
    """tc_step over 1,024 sums measured on a B200 through the engine's GEMM
    (tests/golden/make_mma_golden.py): bit for bit."""
    path = os.path.join(GOLD, "tc_mma_steps.npz")
    if not os.path.exists(path):
        pytest.skip("tc_mma_steps.npz not generated yet (needs a GPU)")
    d = np.load(path)
    bad = 0
    for x, nk, g in zip(d["x"], d["nk"], d["gpu"]):
        acc = 0.0
        for s in range(0, int(nk), 16):
            acc = O.tc_step(acc, x[s:s + 16])
        bad += np.float32(acc).view(np.uint32) != np.float32(g).view(np.uint32)
    assert bad == 0, f"{bad} of {len(d['gpu'])} sums differ"


@pytest.mark.parametrize("length", [1, 31, 64, 1025])
def test_flash_tc_restatement_close_to_flash_formula(O, length):
    """The prompt route's exact restatement (attn_flash_tc_gate: the tensor
    core's truncating MMA accumulation, fexp weights, the kernels' key splits)
    stays within bf16 rounding of the flash formula with exact sums
    (attn_flash_gate)."""
    c = I.config3(2, length)
    kc, vc = c["kc"].copy(), c["vc"].copy()
    q = O.attn_prepare(c["q_raw"], c["k_raw"], c["v_raw"], c["q_gain"], c["k_gain"], c["pos"], c["cap"], kc, vc)
    a = I.bf2f(O.attn_flash_tc_gate(q, kc, vc, length - 1, c["cap"], 0, length, c["q_raw"])).astype(np.float64)
    b = I.bf2f(O.attn_flash_gate(q, kc, vc, length, c["cap"], c["q_raw"])).astype(np.float64)
    assert np.linalg.norm(a - b) <= 1e-2 * np.linalg.norm(b)


def test_tc_step_against_device_chains(O):
    """tc_step over chains of 1, 2, 4 and 64 MMA steps measured on a B200
    with products of widely different exponents (weights from Q4 scales and
    biases over 14 binades, activations over 13; tests/golden/make_mma_golden.py):
    bit for bit. These pin the alignment by the factors' exponent sum."""
    path = os.path.join(GOLD, "tc_mma_chains.npz")
    if not os.path.exists(path):
        pytest.skip("tc_mma_chains.npz not generated yet (needs a GPU)")
    d = np.load(path)
    for n in (1, 2, 4, 64):
        a, b, g = I.bf2f(d[f"a{n}"]), I.bf2f(d[f"b{n}"]), d[f"gpu{n}"]
        bad = 0
        for ai, bi, gi in zip(a, b, g):
            acc = 0.0
            for s in range(0, 16 * n, 16):
                acc = O.tc_step(acc, ai[s:s + 16], bi[s:s + 16])
            bad += np.float32(acc).view(np.uint32) != np.float32(gi).view(np.uint32)
        assert bad == 0, f"{n} steps: {bad} of {len(g)} differ"
