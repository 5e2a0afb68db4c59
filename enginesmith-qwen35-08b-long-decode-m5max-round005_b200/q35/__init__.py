"""Python host over the q35 C ABI (``lib/libq35cuda.so``).

Mirrors the reference host's model interface (source/src/model.rs):
``Model.load(path)`` (model.rs:37), ``Model.generate(prompt, count, reset)``
(model.rs:97-122) raising on the same validation failures, and
``Model.cancel()`` for the ``cancelled`` flag (model.rs:33). The op-level
wrappers take torch CUDA tensors (torch is only used for device memory and
streams) and call the CUDA kernels through the C ABI. There is no CPU
fallback: importing this module without the built library raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_size_t, c_uint16, c_uint32, c_uint64, c_void_p

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libq35cuda.so")
ENGINE_PATH = os.path.join(PKG_DIR, "lib", "engine")
HEADER_PATH = os.path.join(os.path.dirname(PKG_DIR), "include", "q35.h")

VOCAB = 248320
HIDDEN = 1024
DEFAULT_CAPACITY = 262144
SPLIT_HANDLE_BYTES = 64
BATCH_TENSOR_CORES = 1

OK, EINVAL, ECUDA, ECANCEL, EIO, ENOMEM, ETIMEOUT, ENCCL = 0, -1, -2, -3, -4, -5, -6, -7
FLAG_TOKEN_BY_TOKEN_PROMPT = 1
FLAG_TENSOR_PROMPT = 2


class Q35Error(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class _Opts(ctypes.Structure):
    _fields_ = [("capacity", c_uint32), ("decode_batch", c_uint32),
                ("prefill_batch", c_uint32), ("flags", c_uint32), ("prompt_chunk", c_uint32)]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"q35 CUDA library not built: {LIB_PATH} (run `make` at the repo root)")
    lib = ctypes.CDLL(LIB_PATH)
    P = c_void_p
    sig = {
        "q35_open": (c_int, [c_char_p, c_int, POINTER(_Opts), POINTER(c_void_p), c_char_p, c_size_t]),
        "q35_generate": (c_int, [P, POINTER(c_uint32), c_size_t, c_size_t, c_int, POINTER(c_uint32)]),
        "q35_cancel": (None, [P]),
        "q35_last_error": (c_char_p, [P]),
        "q35_close": (None, [P]),
        "q35_position": (c_uint32, [P]),
        "q35_capacity": (c_uint32, [P]),
        "q35_pending": (c_int, [P, POINTER(c_uint32)]),
        "q35_check_opts": (c_int, [POINTER(_Opts), c_char_p, c_size_t]),
        "q35_launch_count": (c_int, [P, c_int, POINTER(c_uint64)]),
        "q35_batch_launch_count": (c_int, [P, c_int, POINTER(c_uint64)]),
        "q35_dump_state": (c_int, [P, P, P, P]),
        "q35_last_logits": (c_int, [P, P, P]),
        "q35_decode_timed": (c_int, [P, c_size_t, POINTER(c_float)]),
        "q35_attn_timing": (c_int, [P, c_int, POINTER(ctypes.c_double), POINTER(c_uint32)]),
        "q35_qmv_timing": (c_int, [P, POINTER(ctypes.c_double), POINTER(c_uint32), POINTER(ctypes.c_double)]),
        "q35_op_qmv_q4": (c_int, [P, P, P, P, P, P, c_int, c_int, P]),
        "q35_op_embedding_q4": (c_int, [P, P, P, c_uint32, c_int, P, P]),
        "q35_op_qgemm_workspace_bytes": (c_size_t, [c_uint32, c_uint32, c_uint32]),
        "q35_op_qgemm_q4": (c_int, [P, P, P, P, c_uint32, c_uint32, c_uint32, P, P, P, c_size_t, P]),
        "q35_op_rms_norm": (c_int, [P, P, P, P]),
        "q35_op_gdn_workspace_bytes": (c_size_t, []),
        "q35_op_gdn_step": (c_int, [P] * 17),
        "q35_op_attn_workspace_bytes": (c_size_t, []),
        "q35_op_attn_decode": (c_int, [P, P, P, P, P, P, P, c_uint32, c_uint32, P, P, P]),
        "q35_op_prompt_workspace_bytes": (c_size_t, [c_uint32, c_uint32]),
        "q35_op_prompt_gdn": (c_int, [P, P, P, P, P, P, P, P, P, c_uint32, P, P, c_size_t, P]),
        "q35_op_prompt_attention": (c_int, [P, P, P, P, P, P, P, c_uint32, c_uint32, c_uint32, P, P, c_size_t, P]),
        "q35_op_head_workspace_bytes": (c_size_t, []),
        "q35_op_head_argmax": (c_int, [P, P, P, P, P, P, P, P, P, P]),
        "q35_op_greedy": (c_int, [P, P, P, P, P]),
        "q35_write_synthetic_model": (c_int, [c_char_p, c_uint64, c_char_p, c_size_t]),
        "q35_version": (c_char_p, []),
        "q35_diag_bounded_wait": (c_int, [c_uint32, P, P]),
        "q35_diag_inject_device_error": (c_int, [P, c_uint32]),
        "q35_session_copy": (c_int, [P, P]),
        "q35_force_pending": (c_int, [P, c_uint32]),
        "q35_split_prepare": (c_int, [P, c_int, c_int, P]),
        "q35_split_connect": (c_int, [P, P]),
        "q35_split_world": (c_int, [P]),
        "q35_split_set_wait": (c_int, [P, c_uint32]),
        "q35_batch_create": (c_int, [POINTER(c_void_p), c_int, POINTER(c_void_p), c_char_p, c_size_t]),
        "q35_batch_create_ex": (c_int, [POINTER(c_void_p), c_int, c_uint32, POINTER(c_void_p), c_char_p, c_size_t]),
        "q35_batch_decode": (c_int, [P, c_size_t, POINTER(c_uint32)]),
        "q35_batch_decode_timed": (c_int, [P, c_size_t, POINTER(c_float)]),
        "q35_batch_last_error": (c_char_p, [P]),
        "q35_batch_destroy": (None, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def check_opts(capacity: int = 0, decode_batch: int = 0, prefill_batch: int = 0, flags: int = 0,
               prompt_chunk: int = 0) -> None:
    """Raise Q35Error when q35_open would reject these session options
    (host arithmetic only; no device needed)."""
    opts = _Opts(capacity, decode_batch, prefill_batch, flags, prompt_chunk)
    err = ctypes.create_string_buffer(512)
    rc = lib().q35_check_opts(ctypes.byref(opts), err, len(err))
    if rc != OK:
        raise Q35Error(rc, err.value.decode())


def write_synthetic_model(path: str, seed: int) -> None:
    """Seeded random-init model in the MLX layout (config.json + model.safetensors)."""
    err = ctypes.create_string_buffer(1024)
    rc = lib().q35_write_synthetic_model(path.encode(), seed, err, len(err))
    if rc != OK:
        raise Q35Error(rc, err.value.decode())


# ---------------------------------------------------------------------------
# session API (Model)
# ---------------------------------------------------------------------------
class Model:
    """One decode session on one GPU (Model in source/src/model.rs)."""

    def __init__(self, handle, capacity: int):
        self._h = handle
        self.capacity = capacity

    @classmethod
    def load(cls, path: str, device: int = 0, capacity: int = 0, decode_batch: int = 0,
             prefill_batch: int = 0, token_by_token_prompt: bool = False, tensor_prompt: bool = False,
             prompt_chunk: int = 0) -> "Model":
        """tensor_prompt: prompts on the tensor cores (Q35_FLAG_TENSOR_PROMPT) in
        chunks of prompt_chunk tokens (0 = 2048)."""
        flags = (FLAG_TOKEN_BY_TOKEN_PROMPT if token_by_token_prompt else 0) | (FLAG_TENSOR_PROMPT if tensor_prompt else 0)
        opts = _Opts(capacity, decode_batch, prefill_batch, flags, prompt_chunk)
        h = c_void_p()
        err = ctypes.create_string_buffer(2048)
        rc = lib().q35_open(path.encode(), device, ctypes.byref(opts), ctypes.byref(h), err, len(err))
        if rc != OK:
            raise Q35Error(rc, err.value.decode())
        return cls(h, capacity or DEFAULT_CAPACITY)

    def _check(self, rc: int) -> None:
        if rc != OK:
            raise Q35Error(rc, lib().q35_last_error(self._h).decode())

    def generate(self, prompt, count: int, reset: bool) -> list[int]:
        n = len(prompt)
        arr = (c_uint32 * max(n, 1))(*prompt)
        out = (c_uint32 * max(count, 1))()
        self._check(lib().q35_generate(self._h, arr, n, count, 1 if reset else 0, out))
        return list(out[:count])

    def cancel(self) -> None:
        lib().q35_cancel(self._h)

    @property
    def position(self) -> int:
        return int(lib().q35_position(self._h))

    @property
    def pending(self) -> int:
        """The token the next continuation consumes first (last emitted id)."""
        t = c_uint32()
        self._check(lib().q35_pending(self._h, ctypes.byref(t)))
        return int(t.value)

    def launch_count(self, reset: bool = False) -> int:
        """Kernel launches of the decode graphs replayed since the last reset."""
        n = c_uint64()
        self._check(lib().q35_launch_count(self._h, 1 if reset else 0, ctypes.byref(n)))
        return int(n.value)

    def decode_timed(self, steps: int) -> float:
        ms = c_float()
        self._check(lib().q35_decode_timed(self._h, steps, ctypes.byref(ms)))
        return float(ms.value)

    def attn_timing(self, reset: int = -1):
        """(total_us, launches) of the attention launches since the last reset;
        reset=1 clears and enables the device timer, 0 clears and disables."""
        us = ctypes.c_double()
        n = c_uint32()
        self._check(lib().q35_attn_timing(self._h, reset, ctypes.byref(us), ctypes.byref(n)))
        return float(us.value), int(n.value)

    def qmv_timing(self):
        """(total_us, launches, weight_bytes) of the matvec launches since the
        last attn_timing reset (the same device-clock switch)."""
        us, nb = ctypes.c_double(), ctypes.c_double()
        n = c_uint32()
        self._check(lib().q35_qmv_timing(self._h, ctypes.byref(us), ctypes.byref(n), ctypes.byref(nb)))
        return float(us.value), int(n.value), float(nb.value)

    def dump_state(self):
        """Return (kv [6,2,2,pos,256] u16, state [18,16,128,128] f32, hist [18,3,6144] u16)."""
        import numpy as np
        pos = self.position
        kv = np.zeros((6, 2, 2, pos, 256), np.uint16)
        st = np.zeros((18, 16, 128, 128), np.float32)
        hi = np.zeros((18, 3, 6144), np.uint16)
        self._check(lib().q35_dump_state(self._h, kv.ctypes.data, st.ctypes.data, hi.ctypes.data))
        return kv, st, hi

    def last_logits(self):
        import numpy as np
        lg = np.zeros(VOCAB, np.uint16)
        lse = np.zeros(1, np.uint16)
        self._check(lib().q35_last_logits(self._h, lg.ctypes.data, lse.ctypes.data))
        return lg, int(lse[0])

    def split_prepare(self, rank: int, world: int) -> bytes:
        """First half of the sequence-split set-up: this rank's exchange-buffer
        handle (SPLIT_HANDLE_BYTES bytes) for the other ranks."""
        h = ctypes.create_string_buffer(SPLIT_HANDLE_BYTES)
        self._check(lib().q35_split_prepare(self._h, rank, world, h))
        return h.raw

    def split_connect(self, handles: list) -> None:
        """Second half: every rank's handle in rank order."""
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        self._check(lib().q35_split_connect(self._h, buf))

    def split_set_wait(self, ms: int) -> None:
        """Bound of the exchange wait for the peers' records (before connecting)."""
        self._check(lib().q35_split_set_wait(self._h, ms))

    @property
    def split_world(self) -> int:
        return int(lib().q35_split_world(self._h))

    def force_pending(self, token: int) -> None:
        """Teacher forcing: the next continuation consumes `token` instead of
        the last emitted id."""
        self._check(lib().q35_force_pending(self._h, token))

    def copy_from(self, other: "Model") -> None:
        """Take `other`'s whole decode state (same device, model and capacity)."""
        self._check(lib().q35_session_copy(self._h, other._h))

    def inject_device_error(self, site: int) -> None:
        """Host-side fault injection: record an expired device wait (site code)."""
        self._check(lib().q35_diag_inject_device_error(self._h, site))

    def close(self) -> None:
        if self._h:
            lib().q35_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def split_connect_dist(model, group=None, wait_ms: int = 0) -> None:
    """Sequence-split set-up over torch.distributed, one process per GPU: each
    rank prepares its exchange buffer, the handles are all-gathered in rank
    order (any backend; the handles are plain bytes) and each rank connects.
    Every rank of `group` must call this with its own session."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    if wait_ms:
        model.split_set_wait(wait_ms)
    mine = model.split_prepare(rank, world)
    handles = [None] * world
    dist.all_gather_object(handles, mine, group=group)
    if any(not isinstance(h, (bytes, bytearray)) or len(h) != SPLIT_HANDLE_BYTES for h in handles):
        raise Q35Error(EINVAL, "split: malformed exchange handle")
    model.split_connect([bytes(h) for h in handles])


class Batch:
    """Sessions of one device and one model decoded together: each step reads
    the weights once for all members. Exact route (default, up to 8 members):
    each member emits the tokens it would emit alone. tensor_cores=True (up to
    64 members): projections and head as tcgen05 GEMMs, equal to the exact
    route within tolerance. Members must hold a continuation state (a generate
    call succeeded on them). Keep the member Models alive while the batch is."""

    def __init__(self, models: list["Model"], tensor_cores: bool = False):
        n = len(models)
        arr = (c_void_p * max(n, 1))(*[m._h.value if isinstance(m._h, c_void_p) else m._h for m in models])
        h = c_void_p()
        err = ctypes.create_string_buffer(1024)
        rc = lib().q35_batch_create_ex(arr, n, BATCH_TENSOR_CORES if tensor_cores else 0, ctypes.byref(h), err,
                                       len(err))
        if rc != OK:
            raise Q35Error(rc, err.value.decode())
        self._h = h
        self._models = list(models)
        self.n = n

    def _check(self, rc: int) -> None:
        if rc != OK:
            raise Q35Error(rc, lib().q35_batch_last_error(self._h).decode())

    def decode(self, steps: int) -> list[list[int]]:
        """`steps` greedy tokens per member; row t belongs to models[t]."""
        out = (c_uint32 * (self.n * steps))()
        self._check(lib().q35_batch_decode(self._h, steps, out))
        return [list(out[t * steps:(t + 1) * steps]) for t in range(self.n)]

    def decode_timed(self, steps: int) -> float:
        ms = c_float()
        self._check(lib().q35_batch_decode_timed(self._h, steps, ctypes.byref(ms)))
        return float(ms.value)

    def launch_count(self, reset: bool = False) -> int:
        """Kernel launches of the batch's decode graphs since the last reset."""
        n = c_uint64()
        self._check(lib().q35_batch_launch_count(self._h, 1 if reset else 0, ctypes.byref(n)))
        return int(n.value)

    def close(self) -> None:
        if self._h:
            lib().q35_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# op API (torch CUDA tensors; nothing allocated by the library)
# ---------------------------------------------------------------------------
def _ptr(t):
    return None if t is None else c_void_p(t.data_ptr())


def _stream():
    import torch
    return c_void_p(torch.cuda.current_stream().cuda_stream)


def _op(rc: int, what: str) -> None:
    if rc != OK:
        raise Q35Error(rc, f"{what} failed ({rc})")


def qmv_q4(w, scales, biases, x, residual=None, out=None):
    """y[N] = bf16(W x) (+ residual) — linear.metal qmv_q4 / qmv_add_q4."""
    import torch
    n, kw = w.shape
    y = out if out is not None else torch.empty(n, dtype=torch.uint16, device=w.device)
    _op(lib().q35_op_qmv_q4(_ptr(w), _ptr(scales), _ptr(biases), _ptr(x), _ptr(residual), _ptr(y),
                            n, kw * 8, _stream()), "qmv_q4")
    return y


def qgemm_q4(w, scales, biases, x, residual=None, out=None, ws=None):
    """y[T][N] = bf16(x W^T) (+ residual) on the tensor cores (tcgen05), W the
    Q4 matrix dequantised as bf16(s q + b); x [T][K] bf16 with T <= 4096."""
    import torch
    n, kw = w.shape
    t = x.shape[0]
    y = out if out is not None else torch.empty((t, n), dtype=torch.uint16, device=w.device)
    need = int(lib().q35_op_qgemm_workspace_bytes(t, n, kw * 8))
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=w.device)
    _op(lib().q35_op_qgemm_q4(_ptr(w), _ptr(scales), _ptr(biases), _ptr(x), t, n, kw * 8, _ptr(residual),
                              _ptr(y), _ptr(ws), ws.numel(), _stream()), "qgemm_q4")
    return y


def embedding_q4(w, scales, biases, token: int):
    import torch
    k = w.shape[1] * 8
    out = torch.empty(k, dtype=torch.uint16, device=w.device)
    _op(lib().q35_op_embedding_q4(_ptr(w), _ptr(scales), _ptr(biases), token, k, _ptr(out), _stream()),
        "embedding_q4")
    return out


def rms_norm(x, gain):
    import torch
    out = torch.empty_like(x)
    _op(lib().q35_op_rms_norm(_ptr(x), _ptr(gain), _ptr(out), _stream()), "rms_norm")
    return out


def workspace(kind: str, device="cuda"):
    import torch
    n = {"gdn": lib().q35_op_gdn_workspace_bytes, "attn": lib().q35_op_attn_workspace_bytes,
         "head": lib().q35_op_head_workspace_bytes}[kind]()
    return torch.empty(n, dtype=torch.uint8, device=device)


def gdn_step(raw_qkv, z, a_raw, b_raw, history, conv_w, a_log, dt_bias, state, norm_w, ow, os_, ob,
             residual=None, ws=None):
    import torch
    out = torch.empty(1024, dtype=torch.uint16, device=raw_qkv.device)
    ws = ws if ws is not None else workspace("gdn", raw_qkv.device)
    _op(lib().q35_op_gdn_step(*[_ptr(t) for t in (raw_qkv, z, a_raw, b_raw, history, conv_w, a_log,
                                                  dt_bias, state, norm_w, ow, os_, ob, residual, out,
                                                  ws)], _stream()), "gdn_step")
    return out


def attn_decode(q_raw, k_raw, v_raw, q_gain, k_gain, kcache, vcache, capacity: int, pos: int, ws=None):
    import torch
    gated = torch.empty(2048, dtype=torch.uint16, device=q_raw.device)
    ws = ws if ws is not None else workspace("attn", q_raw.device)
    _op(lib().q35_op_attn_decode(_ptr(q_raw), _ptr(k_raw), _ptr(v_raw), _ptr(q_gain), _ptr(k_gain),
                                 _ptr(kcache), _ptr(vcache), capacity, pos, _ptr(gated), _ptr(ws),
                                 _stream()), "attn_decode")
    return gated


def _prompt_ws(tokens: int, capacity: int, device):
    import torch
    n = lib().q35_op_prompt_workspace_bytes(tokens, capacity)
    if n == 0:
        raise Q35Error(EINVAL, "prompt op: invalid shape")
    return torch.empty(n, dtype=torch.uint8, device=device), n


def prompt_gdn(raw_qkv, z, ab, history, conv_w, a_log, dt_bias, state, norm_w):
    """One GDN layer's prompt-chunk steps over T tokens (q35_op_prompt_gdn):
    raw_qkv [T][6144], z [T][2048], ab [T][32]; history and state updated in
    place; returns gated [T][2048] (bf16 bits)."""
    import torch
    t = raw_qkv.shape[0]
    gated = torch.empty((t, 2048), dtype=torch.uint16, device=raw_qkv.device)
    ws, n = _prompt_ws(t, 0, raw_qkv.device)
    _op(lib().q35_op_prompt_gdn(_ptr(raw_qkv), _ptr(z), _ptr(ab), _ptr(history), _ptr(conv_w), _ptr(a_log),
                                _ptr(dt_bias), _ptr(state), _ptr(norm_w), t, _ptr(gated), _ptr(ws), n,
                                _stream()), "prompt_gdn")
    return gated


def prompt_attention(q_raw, k_raw, v_raw, q_gain, k_gain, kcache, vcache, capacity: int, p0: int, ws=None,
                     out=None):
    """One attention layer's prompt-chunk steps for tokens at p0 .. p0 + T - 1
    (q35_op_prompt_attention): appends their K/V to the chain-layout caches and
    returns gated [T][2048] (bf16 bits). ws: a workspace of
    q35_op_prompt_workspace_bytes(T, capacity) bytes (allocated if None)."""
    import torch
    t = q_raw.shape[0]
    gated = out if out is not None else torch.empty((t, 2048), dtype=torch.uint16, device=q_raw.device)
    if ws is None:
        ws, n = _prompt_ws(t, capacity, q_raw.device)
    else:
        n = ws.numel() * ws.element_size()
    _op(lib().q35_op_prompt_attention(_ptr(q_raw), _ptr(k_raw), _ptr(v_raw), _ptr(q_gain), _ptr(k_gain),
                                      _ptr(kcache), _ptr(vcache), capacity, p0, t, _ptr(gated), _ptr(ws), n,
                                      _stream()), "prompt_attention")
    return gated


def head_argmax(w, scales, biases, x, gain=None, ws=None):
    import torch
    dev = w.device
    logits = torch.empty(VOCAB, dtype=torch.uint16, device=dev)
    token = torch.zeros(1, dtype=torch.int32, device=dev)
    lse = torch.zeros(1, dtype=torch.uint16, device=dev)
    ws = ws if ws is not None else workspace("head", dev)
    _op(lib().q35_op_head_argmax(_ptr(w), _ptr(scales), _ptr(biases), _ptr(x), _ptr(gain),
                                 _ptr(logits), _ptr(token), _ptr(lse), _ptr(ws), _stream()),
        "head_argmax")
    return logits, token, lse


def diag_bounded_wait(polls: int, err_word) -> int:
    """Run the kernels' bounded wait on a barrier nothing completes; returns the
    status code (Q35_ETIMEOUT when the wait gave up) and leaves the site code
    in err_word (a 1-element int32 CUDA tensor)."""
    return lib().q35_diag_bounded_wait(polls, _ptr(err_word), _stream())


def greedy(logits, ws=None):
    """Greedy selection on given bf16 logits [248320] (linear.metal greedy_bf16)."""
    import torch
    dev = logits.device
    token = torch.zeros(1, dtype=torch.int32, device=dev)
    lse = torch.zeros(1, dtype=torch.uint16, device=dev)
    ws = ws if ws is not None else workspace("head", dev)
    _op(lib().q35_op_greedy(_ptr(logits), _ptr(token), _ptr(lse), _ptr(ws), _stream()), "greedy")
    return token, lse
