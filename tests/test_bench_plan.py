"""bench.py's host arithmetic on CPU: for the argument sets the round-end
driver uses (`--steps 20 --warmup 5` at 1, 2, 4 and 8 GPUs) and for the
defaults, every session capacity the bench opens passes the library's own
option check (q35_check_opts, the validation q35_open runs) and holds the
tokens the run will consume; the reference arm never loads the CUDA library."""
import argparse
import hashlib
import os
import subprocess
import sys

import pytest

import q35

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _args(**kw):
    a = argparse.Namespace(steps=256, warmup=8, context=65536, contexts="32768,131072", split=False,
                           config5=True, cpu_tokens=64)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


ARGSETS = [
    dict(steps=20, warmup=5),             # the driver's BENCH/SCALE command
    dict(),                               # bench.py defaults
    dict(steps=2048, warmup=16),
    dict(steps=1, warmup=3),
    dict(steps=7, warmup=5, context=32768, contexts=""),
    dict(steps=20, warmup=5, context=131072, contexts=""),
    dict(steps=33, warmup=3, context=1000, contexts="1023,4097"),
]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("kw", ARGSETS)
def test_capacities_accepted_and_sufficient(kw, world):
    a = _args(**kw)
    pl = bench.plan(a, world)
    for cap in (pl["capacity"], pl["engine_capacity"]):
        assert cap % 64 == 0
        q35.check_opts(capacity=cap, flags=q35.FLAG_TENSOR_PROMPT)  # raises when q35_open would refuse
    longest = max(pl["contexts"]) + 1 + a.warmup + a.steps + bench.INSTRUMENTED_PASSES * bench.INSTRUMENTED_STEPS + a.cpu_tokens
    assert pl["capacity"] >= longest
    if pl["config5"]:
        assert pl["capacity"] >= bench.C5_CONTEXT + 1 + a.warmup + a.steps
        assert pl["c5_per_gpu"] * world == bench.C5_SESSIONS
    assert pl["engine_capacity"] >= a.context + 1 + a.warmup + a.steps


def test_split_plan_measures_one_context():
    pl = bench.plan(_args(split=True, steps=20, warmup=5), 2)
    assert pl["split"] and pl["contexts"] == [65536] and not pl["config5"]
    q35.check_opts(capacity=pl["capacity"])


def test_capacity_for_matches_the_library_rule():
    for n in (1, 63, 64, 65, 65632, 65536 + 20 + 5 + 64, 131072 + 2048):
        cap = bench.capacity_for(n)
        assert cap >= n and cap - n < 64
        q35.check_opts(capacity=cap)
    with pytest.raises(q35.Q35Error, match="multiple of 64"):
        q35.check_opts(capacity=65632)  # the rounding that voided a whole driver run


def test_check_opts_messages():
    with pytest.raises(q35.Q35Error, match="prompt_chunk"):
        q35.check_opts(capacity=4096, prompt_chunk=48)
    q35.check_opts()  # defaults are valid


def test_reference_arm_loads_only_the_oracle(tmp_path):
    """`bench.py --impl reference` (tiny context) prints its JSON line, and
    neither imports the q35 package nor maps libq35cuda.so."""
    code = r"""
import json, runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3", "--context", "64"]
try:
    runpy.run_path("bench.py", run_name="__main__")
except SystemExit as e:
    assert not e.code, e.code
maps = open("/proc/self/maps").read()
print(json.dumps({"q35_imported": "q35" in sys.modules, "cuda_lib_mapped": "libq35cuda" in maps,
                  "oracle_mapped": "libq35oracle" in maps}))
"""
    env = dict(os.environ, Q35_SYNTH_DIR=os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3"))
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    import json
    line, probe = json.loads(lines[0]), json.loads(lines[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert probe == {"q35_imported": False, "cuda_lib_mapped": False, "oracle_mapped": True}


def test_oracle_writer_matches_library_writer(tmp_path, synth_model_dir):
    """The oracle library's copy of the synthetic-model writer (used by the
    reference arm) writes the same bytes as the CUDA library's."""
    import q35_oracle
    d = str(tmp_path / "m")
    q35_oracle.write_synthetic_model(d, 3)
    h = lambda p: hashlib.sha256(open(p, "rb").read()).hexdigest()
    for name in ("model.safetensors", "config.json"):
        assert h(os.path.join(d, name)) == h(os.path.join(synth_model_dir, name))
