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


def test_op_status_reports_recorded_waits(cuda):
    """q35_op_status reads the bounded-wait word an asynchronous op leaves in
    its workspace: Q35_OK after a clean call; Q35_ETIMEOUT with the site code
    once a site is recorded there (host-side injection, as an expired wait
    would record it); the op's next call clears it."""
    import ctypes
    import q35
    import torch
    lib = q35.lib()
    lib.q35_op_status.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32),
                                  ctypes.c_void_p]
    lib.q35_op_status.restype = ctypes.c_int
    site = ctypes.c_uint32(99)
    st = torch.cuda.current_stream().cuda_stream
    rng = I.Rng(41)
    cap = 128
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()
    q_raw, k_raw, v_raw = (T(I.f2bf(rng.normal(n))) for n in (4096, 512, 512))
    qg, kg = T(I.f2bf(1 + 0.1 * rng.normal(256))), T(I.f2bf(1 + 0.1 * rng.normal(256)))
    kc = torch.zeros(2 * cap * 256, dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    ws = q35.workspace("attn")
    q35.attn_decode(q_raw, k_raw, v_raw, qg, kg, kc, vc, cap, 0, ws=ws)
    assert lib.q35_op_status(ws.data_ptr(), 0, ctypes.byref(site), st) == q35.OK and site.value == 0
    ws.view(torch.int32)[3] = 2  # Ctl::err sits after three 32-bit words
    assert lib.q35_op_status(ws.data_ptr(), 0, ctypes.byref(site), st) == q35.ETIMEOUT and site.value == 2
    q35.attn_decode(q_raw, k_raw, v_raw, qg, kg, kc, vc, cap, 1, ws=ws)
    assert lib.q35_op_status(ws.data_ptr(), 0, ctypes.byref(site), st) == q35.OK
    # the GEMM's word: after its tile counters
    w, s, b, _ = I.config1(42)
    x = T(I.f2bf(rng.normal(8 * 1024)))
    Tw = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(
        {np.uint16: np.int16, np.uint32: np.int32}[a.dtype.type])).cuda()
    gws = torch.empty(int(lib.q35_op_qgemm_workspace_bytes(8, 3584, 1024)), dtype=torch.uint8, device="cuda")
    q35.qgemm_q4(Tw(w), Tw(s), Tw(b), x.view(8, 1024), ws=gws)
    assert lib.q35_op_status(gws.data_ptr(), 1, ctypes.byref(site), st) == q35.OK
    gws.view(torch.int32)[4096] = 8
    assert lib.q35_op_status(gws.data_ptr(), 1, ctypes.byref(site), st) == q35.ETIMEOUT and site.value == 8
    q35.qgemm_q4(Tw(w), Tw(s), Tw(b), x.view(8, 1024), ws=gws)
    assert lib.q35_op_status(gws.data_ptr(), 1, None, st) == q35.OK
    assert lib.q35_op_status(ws.data_ptr(), 7, None, st) == q35.EINVAL
