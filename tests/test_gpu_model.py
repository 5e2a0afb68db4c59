"""Full decode path (session API, CUDA-graph token loop) against the oracle
and the protocol invariants of Model::generate (model.rs:97-122,
docs/protocol.md:40-47) on the seeded random-init model of config 4."""
import numpy as np
import pytest

import inputs as I

pytestmark = pytest.mark.gpu

CAP = 8192


@pytest.fixture(scope="module")
def model(cuda, synth_model_dir):
    import q35
    m = q35.Model.load(synth_model_dir, 0, capacity=CAP)
    yield m
    m.close()


@pytest.fixture(scope="module")
def oracle_model(oracle_threads, synth_model_dir):
    return oracle_threads.OracleModel(synth_model_dir)


def teacher_forced(oracle_threads, oracle_model, prompt, tokens, cap=CAP):
    """Feed the GPU's tokens to the oracle; count steps whose argmax agrees."""
    O = oracle_threads
    s = O.OracleSession(oracle_model, cap)
    for t in prompt[:-1]:
        s.step(int(t), head=False)
    agree, prev = 0, int(prompt[-1])
    for t in tokens:
        agree += int(s.step(prev, head=True) == t)
        prev = int(t)
    return agree, s


def test_greedy_agreement_257(model, oracle_threads, oracle_model):
    prompt = [int(v) for v in I.Rng(3, 40).ints(8, 248320)]
    toks = model.generate(prompt, 257, True)
    assert len(toks) == 257 and all(0 <= t < 248320 for t in toks)
    agree, s = teacher_forced(oracle_threads, oracle_model, prompt, toks)
    assert agree >= 0.99 * 257, f"greedy agreement {agree}/257"
    lg, lse = model.last_logits()
    lo = s.logits()
    g, r = I.bf2f(lg).astype(np.float64), I.bf2f(lo).astype(np.float64)
    rel = np.linalg.norm(g - r) / np.linalg.norm(r)
    assert rel <= 1e-2, f"logits relative error {rel}"


@pytest.mark.parametrize("n", [1, 2, 5, 17])
def test_split_equals_monolithic(model, n):
    prompt = [int(v) for v in I.Rng(5, n).ints(3 + n, 248320)]
    mono = model.generate(prompt, n, True)
    first = model.generate(prompt, 1, True)
    rest = model.generate([], n - 1, False) if n > 1 else []
    assert first + rest == mono
    assert model.position == len(prompt) - 1 + n


def test_continuation_chain(model):
    prompt = [11, 22, 33, 44]
    mono = model.generate(prompt, 12, True)
    parts = model.generate(prompt, 4, True)
    for k in (4, 1, 3):
        parts += model.generate([], k, False)
    assert parts == mono


def test_reset_isolation(model):
    a = [int(v) for v in I.Rng(6).ints(40, 248320)]
    b = [int(v) for v in I.Rng(7).ints(9, 248320)]
    fresh = model.generate(b, 6, True)
    model.generate(a, 20, True)
    assert model.generate(b, 6, True) == fresh


def test_validation_errors_keep_state(model):
    import q35
    prompt = [1, 2, 3]
    ref = model.generate(prompt, 6, True)
    model.generate(prompt, 3, True)
    pos = model.position
    cases = [
        ([], 4, True, "reset needs nonempty prompt"),
        ([5], 4, False, "continuation prompt must be empty"),
        ([248320], 1, True, "token outside vocabulary"),
        ([1], 0, True, "invalid output length"),
        (list(range(CAP)), 2, True, "context capacity exceeded"),
        ([], CAP, False, "context capacity exceeded"),
    ]
    for p, n, r, msg in cases:
        with pytest.raises(q35.Q35Error) as e:
            model.generate(p, n, r)
        assert e.value.code == q35.EINVAL and msg in str(e.value)
        assert model.position == pos
    assert model.generate([], 3, False) == ref[3:]


def test_no_continuation_state(cuda, synth_model_dir):
    import q35
    m = q35.Model.load(synth_model_dir, 0, capacity=64)
    with pytest.raises(q35.Q35Error) as e:
        m.generate([], 1, False)
    assert "no continuation state" in str(e.value)
    # capacity edge: prompt + count - 1 == capacity is allowed
    toks = m.generate(list(range(1, 61)), 5, True)
    assert len(toks) == 5 and m.position == 64
    m.close()


def test_cancel(cuda, synth_model_dir):
    import q35
    m = q35.Model.load(synth_model_dir, 0, capacity=1024)
    m.cancel()
    with pytest.raises(q35.Q35Error) as e:
        m.generate([1, 2, 3], 4, True)
    assert e.value.code == q35.ECANCEL and "input disconnected" in str(e.value)
    m.close()


def test_teacher_forced_long_context(model, oracle_threads, oracle_model):
    """Decode from a GPU-prefilled 4,096-token state; the oracle replays from
    the dumped state (KV caches, GDN state, conv history) with the GPU's tokens."""
    prompt = [int(v) for v in I.Rng(8).ints(4096, 248320)]
    first = model.generate(prompt, 1, True)
    kv, st, hi = model.dump_state()
    pos = model.position
    toks = model.generate([], 64, False)
    O = oracle_threads
    s = O.OracleSession(oracle_model, CAP)
    s.import_state(pos, kv, st, hi)
    agree, prev = 0, first[0]
    for t in toks:
        agree += int(s.step(prev, head=True) == t)
        prev = t
    assert agree >= 63, f"teacher-forced agreement {agree}/64"
