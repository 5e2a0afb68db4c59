"""Full-model decode parity at the long contexts of BASELINE configs 4 and 5
(65,536 and 131,072 tokens), teacher-forced as the harness judges a stream
(docs/protocol.md, "Correctness": a differing stream is replayed through the
reference with the candidate's tokens forced, and a step whose token is not
the reference's top choice is a mismatch).

The GPU consumes the prompt minus its last token on the tensor-core route
(the bench's and the engine's default), then the pending token is forced to
the prompt's last id, so the next request consumes exactly the prompt. The
GPU state at that point (K/V of every attention layer, GDN state, conv
history) is dumped and imported into the oracle, which then replays the
decode with the GPU's tokens fed back: its argmax must agree on >= 99 % of
the steps (257 steps at 64K, 64 at 128K) and the last step's logits must be
within 1e-2 relative error. The CPU prefill itself is
infeasible at these lengths; the prompt route's own parity is checked
layer by layer in test_gpu_prompt_tensor.py."""
import numpy as np
import pytest

import inputs as I

pytestmark = pytest.mark.gpu


def _capacity(tokens):
    return -(-tokens // 64) * 64


@pytest.mark.parametrize("context,steps,seed", [(65536, 257, 3), (131072, 64, 4)])
def test_teacher_forced_decode_at_long_context(cuda, synth_model_dir, oracle_threads, context, steps, seed):
    import q35
    O = oracle_threads
    prompt = [int(v) for v in I.Rng(seed, 50).ints(context, 248320)]
    cap = _capacity(context + steps + 64)
    m = q35.Model.load(synth_model_dir, 0, capacity=cap, tensor_prompt=True)
    try:
        m.generate(prompt[:-1], 1, True)
        m.force_pending(prompt[-1])
        assert m.position == context - 1
        kv, st, hi = m.dump_state()
        gpu = m.generate([], steps, False)
        g_logits, _ = m.last_logits()
    finally:
        m.close()
    om = O.OracleModel(synth_model_dir)
    s = O.OracleSession(om, cap)
    s.import_state(context - 1, kv, st, hi)
    del kv
    agree, prev = 0, prompt[-1]
    for t in gpu:
        agree += int(s.step(prev, head=True) == t)
        prev = t
    g = O.bf2f(g_logits).astype(np.float64)
    r = O.bf2f(s.logits()).astype(np.float64)
    rel = float(np.linalg.norm(g - r) / np.linalg.norm(r))
    print(f"context {context}: {agree}/{steps} teacher-forced argmax agree, last logits rel err {rel:.2e}")
    assert agree >= int(np.ceil(0.99 * steps)), f"agreement {agree}/{steps}"
    assert rel <= 1e-2, rel
