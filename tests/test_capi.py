"""The C-ABI boundary without a GPU: the library loads and exports every
function include/q35.h declares; the synthetic-model writer produces the
694-tensor MLX layout; the engine executable rejects bad arguments."""
import json
import os
import re
import struct
import subprocess

import pytest

import q35


def declared_functions():
    src = open(q35.HEADER_PATH).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(q35_\w+)\s*\(", src)))


def test_header_symbols_exported():
    lib = q35.lib()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert b"sm_100a" in lib.q35_version()


def test_synthetic_model_layout(synth_model_dir):
    path = os.path.join(synth_model_dir, "model.safetensors")
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
    names = [k for k in hdr if k != "__metadata__"]
    assert len(names) == 694
    assert all(k.startswith("language_model.model.") for k in names)
    e = hdr["language_model.model.embed_tokens.weight"]
    assert e["dtype"] == "U32" and e["shape"] == [248320, 128]
    assert hdr["language_model.model.layers.3.self_attn.q_proj.scales"]["shape"] == [4096, 16]
    assert hdr["language_model.model.layers.0.linear_attn.A_log"]["dtype"] == "F32"
    cfg = json.load(open(os.path.join(synth_model_dir, "config.json")))
    tc = cfg["text_config"]
    assert (tc["hidden_size"], tc["num_hidden_layers"], tc["vocab_size"]) == (1024, 24, 248320)


def test_synthetic_model_deterministic(tmp_path, synth_model_dir):
    # the writer is a pure function of the seed
    import hashlib
    d = str(tmp_path / "m")
    q35.write_synthetic_model(d, 3)
    h = lambda p: hashlib.sha256(open(p, "rb").read()).hexdigest()
    assert h(os.path.join(d, "model.safetensors")) == h(os.path.join(synth_model_dir, "model.safetensors"))


def test_engine_argument_errors():
    assert os.path.exists(q35.ENGINE_PATH)
    r = subprocess.run([q35.ENGINE_PATH], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "--model MODEL_DIR required" in r.stderr
    r = subprocess.run([q35.ENGINE_PATH, "--bogus"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "unknown argument --bogus" in r.stderr
    r = subprocess.run([q35.ENGINE_PATH, "--model", "/nonexistent"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 1 and r.stderr.startswith("engine: ")


def test_open_reports_errors_without_crashing():
    import ctypes
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(512)
    opts = q35._Opts(96, 0, 0, 0)  # capacity not a multiple of 64
    rc = q35.lib().q35_open(b"/nonexistent", 0, ctypes.byref(opts), ctypes.byref(h), err, len(err))
    assert rc == q35.EINVAL and b"multiple of 64" in err.value and not h.value


def test_open_rejects_bad_prompt_chunk():
    import ctypes
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(512)
    for bad in (16, 48, 4096):
        opts = q35._Opts(4096, 0, 0, q35.FLAG_TENSOR_PROMPT, bad)
        rc = q35.lib().q35_open(b"/nonexistent", 0, ctypes.byref(opts), ctypes.byref(h), err, len(err))
        assert rc == q35.EINVAL and b"prompt_chunk" in err.value and not h.value


def test_op_workspace_queries():
    """The ops' workspace sizes are host arithmetic: 0 marks an invalid shape."""
    lib = q35.lib()
    pw = lib.q35_op_prompt_workspace_bytes
    assert pw(0, 0) == 0 and pw(2049, 4096) == 0 and pw(1, 100) == 0
    sizes = [pw(t, 4096) for t in (1, 32, 33, 2048)]
    assert all(s > 0 for s in sizes) and sizes == sorted(sizes)
    assert pw(2048, 262144) > pw(2048, 4096)  # more key splits for a larger cache
    qw = lib.q35_op_qgemm_workspace_bytes
    assert qw(0, 1024, 1024) == 0 and qw(4097, 1024, 1024) == 0 and qw(8, 1024, 1000) == 0
    assert qw(1, 1024, 1024) > 0 and qw(4096, 1024, 3584) > 0


def test_prompt_ops_reject_bad_arguments():
    """The prompt-chunk ops validate their arguments before touching a device."""
    import ctypes
    lib = q35.lib()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    gdn = lib.q35_op_prompt_gdn
    # a null input, zero tokens, too many tokens, a workspace below the query
    assert gdn(None, p, p, p, p, p, p, p, p, 4, p, p, 1 << 30, None) == q35.EINVAL
    assert gdn(p, p, p, p, p, p, p, p, p, 0, p, p, 1 << 30, None) == q35.EINVAL
    assert gdn(p, p, p, p, p, p, p, p, p, 2049, p, p, 1 << 30, None) == q35.EINVAL
    assert gdn(p, p, p, p, p, p, p, p, p, 4, p, p, 16, None) == q35.EINVAL
    att = lib.q35_op_prompt_attention
    # capacity not a multiple of 64, the tokens past the capacity, a small workspace
    assert att(p, p, p, p, p, p, p, 100, 0, 4, p, p, 1 << 30, None) == q35.EINVAL
    assert att(p, p, p, p, p, p, p, 128, 126, 4, p, p, 1 << 30, None) == q35.EINVAL
    assert att(p, p, p, p, p, p, p, 128, 0, 4, p, p, 16, None) == q35.EINVAL
