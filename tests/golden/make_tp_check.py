"""Generate tests/golden/tp_check_7b_2l.json, the fixture bench.py checks its tensor-parallel
engines against before timing (the `tp_parity` object of the bench line).

    python tests/golden/make_tp_check.py

The model is the benchmark's 7B Llama shape (d 4096, 32 heads x 128, FFN 11008, vocab 32000,
fp16 weights from the seeded generator) cut to 2 layers; 8 ids from the seeded id stream are fed
teacher-forced at positions 0..7. For every step the CPU oracle (oracle/vsl_oracle.c, the
restatement of the reference's decode math) gives the argmax id, the top-8 logits and the logits
at 64 fixed vocabulary indices. The benchmark compares its engine's logits at those indices
(max-abs <= 2e-2) and its argmax ids (identical) without running the oracle itself.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "vulkan-symbiote-loader_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402
from vsl import synth  # noqa: E402

SPEC = dict(n_layers=2, d_model=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000,
            rope_theta=10000.0, rms_eps=1e-5, wdtype=1, seed=8, sigma=0.02, n_steps=8, max_seq=64)


def main():
    s = SPEC
    m = O.Model.synthetic(n_layers=s["n_layers"], d=s["d_model"], n_heads=s["n_heads"], n_kv=s["n_kv_heads"],
                          ffn=s["ffn"], vocab=s["vocab"], rope_theta=s["rope_theta"], eps=s["rms_eps"],
                          wdtype=s["wdtype"], kvdtype=O.F16, max_seq=s["max_seq"], max_batch=1, seed=s["seed"],
                          sigma=s["sigma"])
    ids = synth.synth_ids(s["seed"], 2, s["n_steps"], s["vocab"]).tolist()
    probe = np.linspace(0, s["vocab"] - 1, 64).astype(int).tolist()
    steps = []
    for p, t in enumerate(ids):
        oid, lg = m.step([t], [p])
        lg = lg[0].astype(np.float64)
        top = np.argsort(-lg, kind="stable")[:8]
        steps.append(dict(argmax=int(oid[0]), top8=[[int(i), float(lg[i])] for i in top],
                          probe=[float(lg[i]) for i in probe],
                          margin=float(lg[top[0]] - lg[top[1]])))
    m.close()
    out = dict(SPEC, ids=ids, probe_index=probe, steps=steps, source="oracle/vsl_oracle.c (fp32 math, fp16 KV)")
    with open(os.path.join(HERE, "tp_check_7b_2l.json"), "w") as f:
        json.dump(out, f, indent=0)
    print("wrote tp_check_7b_2l.json; smallest top-1 margin", min(st["margin"] for st in steps))


if __name__ == "__main__":
    main()
