"""Batched sessions: sessions decoded together through one batched step
(weights streamed once per step for all members) emit, bit for bit, the
tokens, logits and device state each emits decoding alone. The reference
serves one stream per engine (engine.rs); this is the same greedy loop
(model.rs:228-307 per session) with its weight reads shared."""
import numpy as np
import pytest

import inputs as I

pytestmark = pytest.mark.gpu

CAP = 4096


@pytest.fixture(scope="module")
def sessions(cuda, synth_model_dir):
    import q35
    ms = [q35.Model.load(synth_model_dir, 0, capacity=CAP) for _ in range(8)]
    yield ms
    for m in ms:
        m.close()


def prompt(seed, n):
    return [int(v) for v in I.Rng(300 + seed, 5).ints(n, 248320)]


def alone(m, p, steps):
    """Prompt, then `steps` tokens decoded alone (one continuation call per
    entry of `steps`); returns tokens, last logits, lse and state."""
    toks = m.generate(p, 1, True)
    for k in steps:
        toks += m.generate([], k, False)
    lg, lse = m.last_logits()
    return toks, lg, lse, m.dump_state()


def check_member(m, ref, toks):
    rt, rlg, rlse, (rk, rs, rh) = ref
    assert toks == rt
    lg, lse = m.last_logits()
    assert np.array_equal(lg, rlg) and lse == rlse, "logits differ"
    k, s, h = m.dump_state()
    assert np.array_equal(k, rk), "KV cache differs"
    assert np.array_equal(s, rs), "GDN state differs"
    assert np.array_equal(h, rh), "conv history differs"


@pytest.mark.parametrize("lens,steps", [
    ([5], [3]),
    ([5, 40, 1100], [1, 8, 3]),
    ([1, 2, 17, 64, 65, 500, 1030, 2000], [9, 2]),
])
def test_batch_matches_alone(sessions, lens, steps):
    import q35
    n = len(lens)
    ms = sessions[:n]
    prompts = [prompt(i, L) for i, L in enumerate(lens)]
    refs = [alone(m, p, steps) for m, p in zip(ms, prompts)]
    firsts = [m.generate(p, 1, True) for m, p in zip(ms, prompts)]
    b = q35.Batch(ms)
    try:
        outs = [list(f) for f in firsts]
        for k in steps:
            rows = b.decode(k)
            for t in range(n):
                outs[t] += rows[t]
    finally:
        b.close()
    for t in range(n):
        check_member(ms[t], refs[t], outs[t])
        assert ms[t].position == lens[t] - 1 + 1 + sum(steps)


def test_member_continues_alone_after_batch(sessions):
    import q35
    ms = sessions[:2]
    prompts = [prompt(20, 33), prompt(21, 7)]
    refs = [alone(m, p, [4, 6]) for m, p in zip(ms, prompts)]
    outs = [m.generate(p, 1, True) for m, p in zip(ms, prompts)]
    b = q35.Batch(ms)
    try:
        rows = b.decode(4)
    finally:
        b.close()
    for t in range(2):
        outs[t] += rows[t] + ms[t].generate([], 6, False)
        check_member(ms[t], refs[t], outs[t])


def test_batch_timed_advances_like_decode(sessions):
    import q35
    ms = sessions[:3]
    prompts = [prompt(30 + i, 10 + i) for i in range(3)]
    refs = [alone(m, p, [12, 2]) for m, p in zip(ms, prompts)]
    outs = [m.generate(p, 1, True) for m, p in zip(ms, prompts)]
    b = q35.Batch(ms)
    try:
        ms_time = b.decode_timed(12)
        assert ms_time > 0
        rows = b.decode(2)
    finally:
        b.close()
    for t in range(3):
        rt = refs[t][0]
        assert rows[t] == rt[-2:]
        lg, lse = ms[t].last_logits()
        assert np.array_equal(lg, refs[t][1]) and lse == refs[t][2]


def test_batch_argument_errors(sessions, synth_model_dir):
    import q35
    with pytest.raises(q35.Q35Error):
        q35.Batch([])
    with pytest.raises(q35.Q35Error):
        q35.Batch([sessions[0], sessions[0]])
    fresh = q35.Model.load(synth_model_dir, 0, capacity=CAP)
    try:
        b = q35.Batch([sessions[0], fresh])  # fresh: no continuation state
        try:
            sessions[0].generate(prompt(40, 3), 1, True)
            with pytest.raises(q35.Q35Error, match="no continuation state"):
                b.decode(1)
        finally:
            b.close()
    finally:
        fresh.close()
    m = sessions[1]
    m.generate(prompt(41, CAP - 3), 1, True)  # position CAP - 3
    b = q35.Batch([m])
    try:
        with pytest.raises(q35.Q35Error, match="capacity"):
            b.decode(4)
        assert len(b.decode(3)[0]) == 3
    finally:
        b.close()


def test_session_copy_continues_identically(sessions):
    import q35
    src, dst = sessions[0], sessions[1]
    p = prompt(50, 1500)
    src.generate(p, 2, True)
    dst.generate(prompt(51, 9), 1, True)  # unrelated state, overwritten
    dst.copy_from(src)
    assert dst.position == src.position
    assert np.array_equal(dst.last_logits()[0], src.last_logits()[0])
    b = q35.Batch([src, dst])
    try:
        rows = b.decode(10)
    finally:
        b.close()
    assert rows[0] == rows[1]
    ks, ss, hs = src.dump_state()
    kd, sd, hd = dst.dump_state()
    assert np.array_equal(ks, kd) and np.array_equal(ss, sd) and np.array_equal(hs, hd)


def test_tensor_batch_columns_independent_and_close(sessions, oracle_threads, synth_model_dir):
    """Tensor-core route: members that are copies of one session emit the same
    tokens and logits (each GEMM column and per-token step is independent of
    the others); different members decode their own streams; and one step
    from a session's state equals the oracle's restatement of this route bit
    for bit (OracleSession.set_gemm with the batch's 5 tokens per GEMM launch:
    weights bf16(s q + b) rounded once, the tensor core's measured MMA
    accumulation per 16-wide K step, the launches' K splits summed in order)
    and picks the same token."""
    import q35
    O = oracle_threads

    def f32(x):
        return (x.astype(np.uint32) << 16).view(np.float32)

    src = sessions[0]
    pending = src.generate(prompt(60, 40), 1, True)[0]
    kv, st, hi = src.dump_state()
    pos = src.position
    for m in sessions[1:4]:
        m.copy_from(src)
    sessions[4].generate(prompt(61, 33), 1, True)
    b = q35.Batch(sessions[:5], tensor_cores=True)
    try:
        rows = b.decode(1)
        logits = [sessions[t].last_logits()[0] for t in range(5)]
        more = b.decode(5)
    finally:
        b.close()
    assert rows[0] == rows[1] == rows[2] == rows[3]
    assert more[0] == more[1] == more[2] == more[3]
    assert all(np.array_equal(logits[0], logits[t]) for t in range(1, 4))
    assert sessions[4].position == 33 + 6
    # the oracle, from the same state, with the tensor route's numerics
    om = O.OracleModel(synth_model_dir)
    s = O.OracleSession(om, ((pos + 64) // 32) * 32)
    s.import_state(pos, kv, st, hi)
    s.set_gemm(True)
    s.set_gemm_tokens(5)
    tok = s.step(pending)
    ref = f32(s.logits())
    got = f32(logits[0])
    rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    print(f"tensor route vs oracle restatement: logits rel err {rel:.2e}, "
          f"{int(np.count_nonzero(logits[0] != s.logits()))} of {ref.size} differ")
    assert np.array_equal(logits[0], s.logits()), rel
    assert tok == rows[0][0]


def test_tensor_batch_limits(sessions):
    import q35
    with pytest.raises(q35.Q35Error, match="1..8"):
        q35.Batch(sessions[:8] + [sessions[0]])  # 9 members, exact route
