"""ctypes bindings of the q35 CPU oracle (libq35oracle.so).

TEST INFRASTRUCTURE ONLY: the scalar-f32 restatement of the reference's
decode arithmetic used as the checker for the CUDA path. Only tests/, the
smoke check and bench.py's CPU-baseline leg may import this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_char_p, c_float, c_int, c_uint16, c_uint32, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libq35oracle.so")
VOCAB = 248320


ROOT = os.path.dirname(HERE)
SYNTH_SRC = os.path.join(ROOT, "enginesmith-qwen35-08b-long-decode-m5max-round005_b200", "csrc", "q35_synth.cpp")


def build() -> None:
    """Compile the oracle (and the synthetic-model writer it carries) with
    g++ (no GPU needed)."""
    srcs = [os.path.join(HERE, "q35_oracle.cpp"), SYNTH_SRC]
    if os.path.exists(LIB_PATH) and all(os.path.getmtime(LIB_PATH) >= os.path.getmtime(s) for s in srcs
                                        if os.path.exists(s)):
        return
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-ffp-contract=off",
                           "-pthread", "-I", os.path.join(ROOT, "include"), "-o", LIB_PATH, *srcs])


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        P = c_void_p
        sig = {
            "orc_set_threads": (None, [c_int]),
            "q35_write_synthetic_model": (c_int, [c_char_p, ctypes.c_uint64, c_char_p, ctypes.c_size_t]),
            "orc_get_threads": (c_int, []),
            "orc_f2bf": (c_uint16, [c_float]),
            "orc_bf2f": (c_float, [c_uint16]),
            "orc_sigmoid_bf": (c_float, [c_float]),
            "orc_softplus_bf": (c_float, [c_float]),
            "orc_fexp": (c_float, [c_float]),
            "orc_embedding_q4": (None, [P, P, P, c_uint32, c_int, P]),
            "orc_qmv_q4": (None, [P, P, P, P, P, c_int, c_int, P]),
            "orc_qmv_q4_f32": (None, [P, P, P, P, c_int, c_int, P]),
            "orc_rms_norm": (None, [P, P, c_int, c_float, P]),
            "orc_swiglu": (None, [P, P, c_int, P]),
            "orc_gdn_conv_prepare": (None, [P] * 10),
            "orc_gdn_recur": (None, [P] * 5),
            "orc_gdn_norm_gate": (None, [P] * 4),
            "orc_gdn_step": (None, [P] * 15),
            "orc_attn_prepare": (None, [P, P, P, P, P, c_uint32, c_uint32, P, P, P]),
            "orc_attn_decode_gate": (None, [P, P, P, c_uint32, c_uint32, P, P]),
            "orc_attn_decode_f32": (None, [P, P, P, c_uint32, c_uint32, P]),
            "orc_head": (c_uint32, [P, P, P, P, c_int, c_int, P, P]),
            "orc_greedy": (c_uint32, [P, c_int, P]),
            "orc_greedy_with_lse": (c_uint32, [P, c_int, c_uint16]),
            "orc_xorshift_logits": (None, [P, c_int, c_int, P]),
            "orc_model_load": (P, [c_char_p, c_char_p, c_int]),
            "orc_model_free": (None, [P]),
            "orc_session_new": (P, [P, c_uint32]),
            "orc_session_free": (None, [P]),
            "orc_session_reset": (None, [P]),
            "orc_session_position": (c_uint32, [P]),
            "orc_session_step": (c_uint32, [P, c_uint32, c_int]),
            "orc_session_set_split": (None, [P, c_int]),
            "orc_session_set_gemm": (None, [P, c_int]),
            "orc_session_set_gemm_tokens": (None, [P, c_int]),
            "orc_session_set_chunk": (None, [P, c_uint32, c_uint32]),
            "orc_attn_flash_tc_gate": (None, [P, P, P, c_uint32, c_uint32, c_uint32, c_uint32, P, P]),
            "orc_qgemm_tc": (None, [P, P, P, P, c_int, c_int, c_int, c_int, P]),
            "tc_step": (c_float, [c_float, P, P]),
            "orc_session_set_flash": (None, [P, c_int]),
            "orc_session_logits": (None, [P, P]),
            "orc_session_lse": (c_uint16, [P]),
            "orc_session_final_hidden": (None, [P, P]),
            "orc_session_import": (None, [P, c_uint32, c_uint32, P, P, P, P]),
            "orc_session_export": (None, [P, P, P, P]),
            "orc_attn_flash_f32": (None, [P, P, P, c_uint32, c_uint32, P]),
            "orc_attn_flash_gate": (None, [P, P, P, c_uint32, c_uint32, P, P]),
            "orc_qmv_gemm_f32": (None, [P, P, P, P, c_int, c_int, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else c_void_p(a.ctypes.data)


def write_synthetic_model(path: str, seed: int) -> None:
    """The seeded random-init model (config.json + model.safetensors in the
    MLX layout), byte for byte what the CUDA library's writer produces: the
    same C++ source is compiled into this library."""
    err = ctypes.create_string_buffer(1024)
    rc = lib().q35_write_synthetic_model(path.encode(), seed, err, len(err))
    if rc != 0:
        raise RuntimeError(f"synthetic model: {err.value.decode()}")


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


# ---- bf16 helpers (numpy) ----
def f2bf(x: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 bit patterns, round-to-nearest-even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf2f(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- ops ----
def embedding_q4(w, s, b, token: int) -> np.ndarray:
    k = w.shape[1] * 8
    out = np.zeros(k, np.uint16)
    lib().orc_embedding_q4(_p(w), _p(s), _p(b), token, k, _p(out))
    return out


def qmv_q4(w, s, b, x, residual=None) -> np.ndarray:
    n, kw = w.shape
    y = np.zeros(n, np.uint16)
    lib().orc_qmv_q4(_p(w), _p(s), _p(b), _p(x), _p(residual), n, kw * 8, _p(y))
    return y


def qmv_q4_f32(w, s, b, x) -> np.ndarray:
    n, kw = w.shape
    y = np.zeros(n, np.float32)
    lib().orc_qmv_q4_f32(_p(w), _p(s), _p(b), _p(x), n, kw * 8, _p(y))
    return y


def qmv_gemm_f32(w, s, b, x) -> np.ndarray:
    """The tensor-core routes' matvec: weights bf16(s q + b), exact dot products, f32 out."""
    n, k = w.shape[0], w.shape[1] * 8
    y = np.zeros(n, np.float32)
    lib().orc_qmv_gemm_f32(_p(w), _p(s), _p(b), _p(x), n, k, _p(y))
    return y


def qgemm_tc(w, s, b, x, tiles: int = 0) -> np.ndarray:
    """The engine's tensor-core GEMM (q35_op_qgemm_q4) restated: x [T][K]
    bf16 -> y [T][N] f32 before the bf16 output rounding."""
    T, K = x.shape
    N = w.shape[0]
    y = np.zeros((T, N), np.float32)
    lib().orc_qgemm_tc(_p(w), _p(s), _p(b), _p(np.ascontiguousarray(x)), T, N, K, tiles, _p(y))
    return y


def tc_step(acc: float, a, b=None) -> float:
    """One 16-wide MMA step of the tensor core (f32 accumulator): acc + sum
    a[i] b[i] (b defaults to ones, i.e. the products given as a)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ones(16, np.float32) if b is None else np.ascontiguousarray(b, np.float32)
    assert a.size == 16 and b.size == 16
    return float(lib().tc_step(acc, _p(a), _p(b)))


def rms_norm(x, gain, eps=1e-6) -> np.ndarray:
    out = np.zeros_like(x)
    lib().orc_rms_norm(_p(x), _p(gain), x.size, eps, _p(out))
    return out


def swiglu(gate, up) -> np.ndarray:
    out = np.zeros_like(gate)
    lib().orc_swiglu(_p(gate), _p(up), gate.size, _p(out))
    return out


def gdn_conv_prepare(raw, a_raw, b_raw, history, conv_w, a_log, dt_bias):
    """Returns (conv[6144] u16, g[16] f32, beta[16] u16); history updated in place."""
    conv = np.zeros(6144, np.uint16)
    g = np.zeros(16, np.float32)
    beta = np.zeros(16, np.uint16)
    lib().orc_gdn_conv_prepare(_p(raw), _p(a_raw), _p(b_raw), _p(history), _p(conv_w), _p(a_log),
                               _p(dt_bias), _p(conv), _p(g), _p(beta))
    return conv, g, beta


def gdn_recur(conv, g, beta, state) -> np.ndarray:
    y = np.zeros(2048, np.uint16)
    lib().orc_gdn_recur(_p(conv), _p(g), _p(beta), _p(state), _p(y))
    return y


def gdn_norm_gate(y, z, w) -> np.ndarray:
    out = np.zeros(2048, np.uint16)
    lib().orc_gdn_norm_gate(_p(y), _p(z), _p(w), _p(out))
    return out


def gdn_step(raw, z, a_raw, b_raw, history, conv_w, a_log, dt_bias, state, norm_w, ow, os_, ob,
             residual=None) -> np.ndarray:
    out = np.zeros(1024, np.uint16)
    lib().orc_gdn_step(*[_p(t) for t in (raw, z, a_raw, b_raw, history, conv_w, a_log, dt_bias, state,
                                         norm_w, ow, os_, ob, residual, out)])
    return out


def attn_prepare(q_raw, k_raw, v_raw, q_gain, k_gain, pos: int, capacity: int, kcache, vcache):
    query = np.zeros(2048, np.uint16)
    lib().orc_attn_prepare(_p(q_raw), _p(k_raw), _p(v_raw), _p(q_gain), _p(k_gain), pos, capacity,
                           _p(query), _p(kcache), _p(vcache))
    return query


def attn_decode_gate(query, kcache, vcache, length: int, capacity: int, q_raw) -> np.ndarray:
    gated = np.zeros(2048, np.uint16)
    lib().orc_attn_decode_gate(_p(query), _p(kcache), _p(vcache), length, capacity, _p(q_raw), _p(gated))
    return gated


def attn_decode_f32(query, kcache, vcache, length: int, capacity: int) -> np.ndarray:
    o = np.zeros(2048, np.float32)
    lib().orc_attn_decode_f32(_p(query), _p(kcache), _p(vcache), length, capacity, _p(o))
    return o


def attn_flash_f32(query, kcache, vcache, length: int, capacity: int) -> np.ndarray:
    """The tensor-core prompt route's attention output (f32 [8*256])."""
    out = np.zeros(2048, np.float32)
    lib().orc_attn_flash_f32(_p(query), _p(kcache), _p(vcache), length, capacity, _p(out))
    return out


def attn_flash_tc_gate(query, kcache, vcache, pos: int, capacity: int, p0c: int, tokens: int, q_raw) -> np.ndarray:
    """The prompt route's gated attention for the token at `pos` of the
    chunk (p0c, tokens), exactly as the tensor-core kernels compute it."""
    out = np.zeros(2048, np.uint16)
    lib().orc_attn_flash_tc_gate(_p(np.ascontiguousarray(query)), _p(kcache), _p(vcache), pos, capacity, p0c,
                                 tokens, _p(np.ascontiguousarray(q_raw)), _p(out))
    return out


def attn_flash_gate(query, kcache, vcache, length: int, capacity: int, q_raw) -> np.ndarray:
    """The prompt route's attention with the output gate (bf16 [8*256])."""
    gated = np.zeros(2048, np.uint16)
    lib().orc_attn_flash_gate(_p(query), _p(kcache), _p(vcache), length, capacity, _p(q_raw), _p(gated))
    return gated


def head(w, s, b, x):
    """Returns (token, logits u16[N], lse u16)."""
    n, kw = w.shape
    logits = np.zeros(n, np.uint16)
    lse = np.zeros(1, np.uint16)
    t = lib().orc_head(_p(w), _p(s), _p(b), _p(x), n, kw * 8, _p(logits), _p(lse))
    return int(t), logits, int(lse[0])


def greedy(logits):
    lse = np.zeros(1, np.uint16)
    t = lib().orc_greedy(_p(logits), logits.size, _p(lse))
    return int(t), int(lse[0])


def greedy_with_lse(logits, lse: int) -> int:
    return int(lib().orc_greedy_with_lse(_p(logits), logits.size, lse))


def xorshift_logits(seed: np.ndarray, si: int, n: int = VOCAB) -> np.ndarray:
    """Logits of greedy-audit case si; `seed` (uint64[1]) advances in place."""
    out = np.zeros(n, np.uint16)
    lib().orc_xorshift_logits(_p(seed), si, n, _p(out))
    return out


# ---- model ----
class OracleModel:
    def __init__(self, model_dir: str):
        err = ctypes.create_string_buffer(1024)
        self.m = lib().orc_model_load(model_dir.encode(), err, len(err))
        if not self.m:
            raise RuntimeError(err.value.decode())

    def __del__(self):
        if getattr(self, "m", None):
            lib().orc_model_free(self.m)
            self.m = None


class OracleSession:
    def __init__(self, model: OracleModel, capacity: int):
        self.model = model
        self.capacity = capacity
        self.s = lib().orc_session_new(model.m, capacity)

    def __del__(self):
        if getattr(self, "s", None):
            lib().orc_session_free(self.s)
            self.s = None

    def reset(self):
        lib().orc_session_reset(self.s)

    @property
    def position(self) -> int:
        return int(lib().orc_session_position(self.s))

    def set_split(self, world: int) -> None:
        """Attention of later steps as the engine's sequence split over
        `world` ranks (1 = the reference's single-device attention)."""
        lib().orc_session_set_split(self.s, world)

    def set_gemm(self, on: bool) -> None:
        """Projections and head of later steps with the engine's tensor-core
        route's numerics (bf16-dequantised weights, exact dot products)."""
        lib().orc_session_set_gemm(self.s, 1 if on else 0)

    def set_gemm_tokens(self, tokens: int) -> None:
        """Tokens per GEMM launch of the engine route restated by set_gemm
        (the batch's member count, or the prompt chunk's token count)."""
        lib().orc_session_set_gemm_tokens(self.s, tokens)

    def set_chunk(self, p0: int, tokens: int) -> None:
        """The prompt chunk (first position, token count) of the next steps:
        the GEMM token count, and the exact flash restatement in flash mode."""
        lib().orc_session_set_chunk(self.s, p0, tokens)

    def set_flash(self, on: bool) -> None:
        """Attention of later steps with the engine's tensor-core prompt
        route's numerics (flash attention: bf16 weights, exact sums)."""
        lib().orc_session_set_flash(self.s, 1 if on else 0)

    def step(self, token: int, head: bool = True) -> int:
        return int(lib().orc_session_step(self.s, token, 1 if head else 0))

    def logits(self) -> np.ndarray:
        out = np.zeros(VOCAB, np.uint16)
        lib().orc_session_logits(self.s, _p(out))
        return out

    def lse(self) -> int:
        return int(lib().orc_session_lse(self.s))

    def generate(self, prompt, count: int):
        """Reference semantics of Model::generate(prompt, count, reset=true)."""
        self.reset()
        for t in prompt[:-1]:
            self.step(int(t), head=False)
        out = []
        tok = int(prompt[-1])
        for _ in range(count):
            tok = self.step(tok, head=True)
            out.append(tok)
        return out

    def export_state(self):
        """(kv [6,2,2,pos,256] u16, state [18,16,128,128] f32, hist [18,3,6144] u16)."""
        pos = self.position
        kv = np.zeros((6, 2, 2, pos, 256), np.uint16)
        st = np.zeros((18, 16, 128, 128), np.float32)
        hi = np.zeros((18, 3, 6144), np.uint16)
        lib().orc_session_export(self.s, _p(kv), _p(st), _p(hi))
        return kv, st, hi

    def import_state(self, pos: int, kv: np.ndarray, state: np.ndarray, hist: np.ndarray):
        """kv [6,2,2,pos,256] u16 (layer, K|V, head, pos, d); state [18,...]; hist [18,...]."""
        kv = np.ascontiguousarray(kv)
        ks = [np.ascontiguousarray(kv[a, 0]) for a in range(6)]
        vs = [np.ascontiguousarray(kv[a, 1]) for a in range(6)]
        st = [np.ascontiguousarray(state[g]) for g in range(18)]
        hi = [np.ascontiguousarray(hist[g]) for g in range(18)]
        KP = (c_void_p * 6)(*[k.ctypes.data for k in ks])
        VP = (c_void_p * 6)(*[v.ctypes.data for v in vs])
        SP = (c_void_p * 18)(*[s.ctypes.data for s in st])
        HP = (c_void_p * 18)(*[h.ctypes.data for h in hi])
        self._keep = (ks, vs, st, hi)
        lib().orc_session_import(self.s, pos, pos, KP, VP, SP, HP)
