"""The allocation-free attention entry point (q35_op_attn_decode_noalloc)
against the workspace entry point (q35_op_attn_decode), through the C ABI.

Two calls in a row share the library's static scratch: a 1,500-key call on
the split route (64 chains from 1,024 keys on, f32 partials) leaves its
partials behind, then a 700-key call on the short route (32 chains below
1,024 keys, f32 partials) must not see them. Each call's
gated output and K/V append must equal the workspace entry point's bit for
bit (the tolerance every attention test here uses), on identical copies of
the inputs. Collected last so it also runs after every other test's kernels.
"""
import ctypes

import numpy as np
import pytest

import inputs as I

pytestmark = pytest.mark.gpu


def _noalloc_fn():
    import q35
    fn = q35.lib().q35_op_attn_decode_noalloc
    P = ctypes.c_void_p
    fn.restype = ctypes.c_int
    fn.argtypes = [P] * 7 + [ctypes.c_uint32, ctypes.c_uint32, P, ctypes.c_char_p, ctypes.c_size_t, P]
    return fn


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _call_noalloc(fn, ins, kc, vc, cap, pos):
    import torch
    gated = torch.empty(2048, dtype=torch.uint16, device="cuda")
    err = ctypes.create_string_buffer(256)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = fn(*[p(ins[k]) for k in ("q_raw", "k_raw", "v_raw", "q_gain", "k_gain")], p(kc), p(vc),
            cap, pos, p(gated), err, len(err), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, f"noalloc entry point failed ({rc}): {err.value.decode()}"
    return gated


@pytest.mark.parametrize("lengths", [(1500, 700)])
def test_noalloc_matches_workspace_entry(cuda, lengths):
    import q35
    import torch
    fn = _noalloc_fn()
    ws = q35.workspace("attn")
    for seed, length in enumerate(lengths, start=5):
        d = I.config3(seed, length)
        cap, pos = d["cap"], d["pos"]
        ins = {k: _dev(d[k]) for k in ("q_raw", "k_raw", "v_raw", "q_gain", "k_gain")}
        kc, vc = I.to_chain_major(d["kc"]), I.to_chain_major(d["vc"])
        kc_a, vc_a, kc_b, vc_b = _dev(kc), _dev(vc), _dev(kc), _dev(vc)
        ref = q35.attn_decode(*[ins[k] for k in ("q_raw", "k_raw", "v_raw", "q_gain", "k_gain")],
                              kc_a, vc_a, cap, pos, ws=ws)
        got = _call_noalloc(fn, ins, kc_b, vc_b, cap, pos)
        torch.cuda.synchronize()
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        assert np.array_equal(g, r), f"len {length}: {np.sum(g != r)} of 2048 gated outputs differ"
        assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b), f"len {length}: K/V append differs"


def test_noalloc_rejects_bad_sizes(cuda):
    fn = _noalloc_fn()
    import torch
    t = torch.zeros(4096, dtype=torch.uint16, device="cuda")
    p = ctypes.c_void_p(t.data_ptr())
    err = ctypes.create_string_buffer(256)
    assert fn(p, p, p, p, p, p, p, 96, 0, p, err, len(err), None) == -1
    assert b"multiple of 64" in err.value
    assert fn(p, p, p, p, p, p, p, 64, 64, p, err, len(err), None) == -1
    assert b"below capacity" in err.value
