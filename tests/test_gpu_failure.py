"""Failure detection without a GPU fault.

(1) The bounded mbarrier wait every kernel uses gives up on a barrier that
nothing completes, reports the site code, and leaves the context usable.
(2) An expired device wait recorded in a session (host-side injection, as a
kernel whose wait ran out would record it) makes the next request fail with
Q35_ETIMEOUT and reset the session (source/src/model.rs:166-178); the session
then serves a fresh request exactly as a new one would."""
import numpy as np
import pytest

import inputs as I

pytestmark = pytest.mark.gpu

K_ERR_PROBE_WAIT = 6


def test_bounded_wait_gives_up(cuda, oracle_threads):
    import q35
    import torch
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = q35.diag_bounded_wait(1000, err)
    assert rc == q35.ETIMEOUT
    assert int(err.item()) == K_ERR_PROBE_WAIT
    # the context still works: a matvec right after is bit-exact
    w, s, b, x = I.config1(21)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(
        {np.uint16: np.int16, np.uint32: np.int32}[a.dtype.type])).cuda()
    y = q35.qmv_q4(T(w), T(s), T(b), T(x)).cpu().numpy().view(np.uint16)
    assert np.array_equal(y, oracle_threads.qmv_q4(w, s, b, x))


def test_expired_wait_resets_session(cuda, synth_model_dir):
    import q35
    m = q35.Model.load(synth_model_dir, 0, capacity=256)
    try:
        prompt = [3, 1415, 9265, 35]
        first = m.generate(prompt, 3, True)
        m.inject_device_error(2)
        with pytest.raises(q35.Q35Error) as ei:
            m.generate([], 2, False)
        assert ei.value.code == q35.ETIMEOUT and "device wait expired (site 2)" in str(ei.value)
        assert m.position == 0
        with pytest.raises(q35.Q35Error) as ei:
            m.generate([], 1, False)
        assert ei.value.code == q35.EINVAL and "no continuation state" in str(ei.value)
        again = m.generate(prompt, 3, True)
        assert again == first
    finally:
        m.close()


def test_probe_rejects_bad_arguments(cuda):
    import q35
    import torch
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert q35.diag_bounded_wait(0, err) == q35.EINVAL
