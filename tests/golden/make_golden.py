"""Regenerate the golden fixtures under tests/golden/ from the CPU oracle.

Inputs are the seeded synthetic configs of BASELINE.json (tests/inputs.py);
only outputs (and a few intermediate states) are stored, so the fixtures stay
small. The GPU parity tests compare the CUDA path against these files and
against the live oracle; the CPU tests check that the oracle still reproduces
them bit for bit.

    python tests/golden/make_golden.py          (every fixture)
    python tests/golden/make_golden.py tensor   (tensor_routes.npz only)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "enginesmith-qwen35-08b-long-decode-m5max-round005_b200"))

import inputs as I  # noqa: E402
import q35_oracle as O  # noqa: E402


def tensor_routes():
    """The tensor-core routes' restatements: the GEMM-numerics matvec (config 1
    shapes, f32 before the output rounding) and the prompt route's flash
    attention with the gate (config 3, at a few lengths)."""
    outs = {}
    for n, k, seed in ((3584, 1024, 0), (1024, 3584, 11)):
        w, s, b, x = I.config1(seed, n, k)
        outs[f"gemm_{n}x{k}"] = O.qmv_gemm_f32(w, s, b, x)
    for length in (1, 31, 1025, 4096):
        c = I.config3(2, length)
        kc, vc = c["kc"].copy(), c["vc"].copy()
        q = O.attn_prepare(c["q_raw"], c["k_raw"], c["v_raw"], c["q_gain"], c["k_gain"], c["pos"], c["cap"], kc, vc)
        outs[f"flash_{length}"] = O.attn_flash_gate(q, kc, vc, length, c["cap"], c["q_raw"])
    np.savez_compressed(os.path.join(HERE, "tensor_routes.npz"), **outs)


def main():
    O.set_threads(os.cpu_count() or 1)
    if sys.argv[1:] == ["tensor"]:
        tensor_routes()
        return
    tensor_routes()
    # config 1: Q4 matvec 3584 x 1024, seed 0 (and the residual form)
    w, s, b, x = I.config1(0)
    res = I.f2bf(I.Rng(5).normal(3584))
    np.savez_compressed(os.path.join(HERE, "config1_qmv.npz"), y=O.qmv_q4(w, s, b, x),
                        y_res=O.qmv_q4(w, s, b, x, residual=res),
                        emb=np.stack([O.embedding_q4(w, s, b, t) for t in (0, 1, 1000, 3583)]))
    # config 2: one GDN step, seed 1
    d = I.config2(1)
    hist, state = d["hist"].copy(), d["state"].copy()
    out = O.gdn_step(d["raw"], d["z"], d["a"], d["b"], hist, d["conv_w"], d["a_log"], d["dt"], state,
                     d["norm_w"], d["ow"], d["os"], d["ob"], residual=d["res"])
    conv, g, beta = O.gdn_conv_prepare(d["raw"], d["a"], d["b"], d["hist"].copy(), d["conv_w"], d["a_log"], d["dt"])
    np.savez_compressed(os.path.join(HERE, "config2_gdn.npz"), out=out, hist=hist, conv=conv, g=g, beta=beta,
                        state_rows=state.reshape(16, 128, 128)[:, ::17, :].copy(),
                        state_sum=np.float64(state.astype(np.float64).sum()))
    # config 3: gated GQA decode, seed 2, at the reference's route boundaries and 32K
    outs = {}
    for length in (1, 31, 1023, 1024, 1025, 4096, 32768):
        c = I.config3(2, length)
        kc, vc = c["kc"].copy(), c["vc"].copy()
        q = O.attn_prepare(c["q_raw"], c["k_raw"], c["v_raw"], c["q_gain"], c["k_gain"], c["pos"], c["cap"], kc, vc)
        outs[f"gated_{length}"] = O.attn_decode_gate(q, kc, vc, length, c["cap"], c["q_raw"])
        outs[f"krow_{length}"] = kc[:, c["pos"]].copy()
    np.savez_compressed(os.path.join(HERE, "config3_attn.npz"), **outs)
    # greedy audit cases (examples/greedy_audit.rs:27-40)
    seed = np.array([0x918BEACD729A], np.uint64)
    toks, lses = [], []
    for si in range(64):
        lg = O.xorshift_logits(seed, si)
        t, l = O.greedy(lg)
        toks.append(t)
        lses.append(l)
    np.savez_compressed(os.path.join(HERE, "greedy_audit.npz"), token=np.array(toks, np.uint32),
                        lse=np.array(lses, np.uint16))
    # config 4 model (seed 3), short prompt: 12 greedy tokens
    model_dir = os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3")
    if not os.path.exists(os.path.join(model_dir, "model.safetensors")):
        import q35
        q35.write_synthetic_model(model_dir, 3)
    om = O.OracleModel(model_dir)
    ss = O.OracleSession(om, 256)
    prompt = [int(v) for v in I.Rng(3, 40).ints(8, 248320)]
    toks = ss.generate(prompt, 12)
    np.savez_compressed(os.path.join(HERE, "config4_model.npz"), prompt=np.array(prompt, np.uint32),
                        tokens=np.array(toks, np.uint32), lse=np.uint16(ss.lse()),
                        logits_head=ss.logits()[:4096].copy())
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
