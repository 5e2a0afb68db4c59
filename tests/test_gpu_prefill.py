"""Prompt chunks: consuming a prompt 16 tokens per launch leaves the same
device state, bit for bit, as consuming it one token per step, and the same
tokens follow (the reference consumes prompts through the rows = 1 matvec /
recurrence path, model.rs:100-110). Lengths straddle chunk edges and the
1,024-key switch between the two attention routes."""
import numpy as np
import pytest

import inputs as I

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair(cuda, synth_model_dir):
    import q35
    a = q35.Model.load(synth_model_dir, 0, capacity=4096)
    b = q35.Model.load(synth_model_dir, 0, capacity=4096, token_by_token_prompt=True)
    yield a, b
    a.close()
    b.close()


@pytest.mark.parametrize("n", [1, 2, 16, 17, 18, 49, 1030, 2100])
def test_chunked_prompt_matches_token_by_token(pair, n):
    a, b = pair
    prompt = [int(v) for v in I.Rng(70 + n, 3).ints(n, 248320)]
    ta = a.generate(prompt, 4, True)
    tb = b.generate(prompt, 4, True)
    assert ta == tb
    la, lsa = a.last_logits()
    lb, lsb = b.last_logits()
    assert np.array_equal(la, lb) and lsa == lsb
    ka, sa, ha = a.dump_state()
    kb, sb, hb = b.dump_state()
    assert np.array_equal(ka, kb), "KV cache differs"
    assert np.array_equal(sa, sb), "GDN state differs"
    assert np.array_equal(ha, hb), "conv history differs"
