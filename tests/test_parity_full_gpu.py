"""Parity at the configurations the benchmark runs.

* 7B Llama shape, fp16, all 32 layers, exactly the benchmark's model (seed 1, sigma 0.02): a
  64-token prompt through the prompt pass (vsl_engine_prefill) against the oracle fed the same
  prompt token by token, then 32 teacher-forced decode steps through vsl_engine_step_host.
* 8B Llama-3 shape, bf16, GQA 32/8, batch 16 with 8192 prefilled fp16 KV positions per sequence
  (the benchmark's cache length and batch; 2 of the 32 layers), teacher-forced decode steps on the
  tcgen05 projection and attention routes the benchmark takes.

Bars (fp16/bf16): logits max-abs <= 2e-2 and top-1 agreement on >= 99% of
compared steps; the oracle is the CPU restatement of the reference's decode math
(oracle/vsl_oracle.c), following VulkanSymbioteEngine::generate's loop
(vk_symbiote/src/VulkanSymbioteEngine.cpp:678-765).
"""
import numpy as np
import pytest

import oracle as O
import vsl
from vsl import synth

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2
CFG_7B = dict(n_layers=32, d_model=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000,
              rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.F16)
CFG_8B = dict(n_layers=2, d_model=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
              rope_theta=500000.0, rms_eps=1e-5, wdtype=vsl.BF16)


def _oracle(cfg, seed, max_seq, batch=1):
    return O.Model.synthetic(n_layers=cfg["n_layers"], d=cfg["d_model"], n_heads=cfg["n_heads"],
                             n_kv=cfg["n_kv_heads"], ffn=cfg["ffn"], vocab=cfg["vocab"], rope_theta=cfg["rope_theta"],
                             eps=cfg["rms_eps"], wdtype=cfg["wdtype"], kvdtype=O.F16, max_seq=max_seq,
                             max_batch=batch, seed=seed, sigma=0.02)


def test_7b_fp16_full_depth_prompt_and_decode():
    seed, n_prompt, n_steps, max_seq = 1, 64, 32, 256
    prompt = synth.synth_ids(seed, 0, n_prompt, CFG_7B["vocab"])
    forced = synth.synth_ids(seed, 1, n_steps, CFG_7B["vocab"])
    orc = _oracle(CFG_7B, seed, max_seq)
    with vsl.Engine.synthetic(CFG_7B, seed=seed, sigma=0.02, max_seq=max_seq) as e:
        nxt, lg = e.prefill(prompt, want_logits=True)
        for p, t in enumerate(prompt):
            oid, olg = orc.step([t], [p], want_logits=p == n_prompt - 1)
        diffs, agree = [float(np.abs(lg - olg[0]).max())], [nxt == int(oid[0])]
        for s in range(n_steps):
            gid, glg = e.step_host(np.array([forced[s]], np.int32), want_logits=True)
            oid, olg = orc.step([forced[s]], [n_prompt + s])
            diffs.append(float(np.abs(glg - olg).max()))
            agree.append(int(gid[0]) == int(oid[0]))
        assert e.device_status() == 0
    orc.close()
    assert max(diffs) <= LOGIT_TOL, diffs
    assert np.mean(agree) >= 0.99, agree


def test_8b_bf16_batch16_8192_prefilled_positions():
    seed, batch, prefill, n_steps = 41, 16, 8192, 3
    max_seq = prefill + 64
    ids = synth.synth_ids(seed, 1, n_steps * batch, CFG_8B["vocab"]).reshape(n_steps, batch)
    orc = _oracle(CFG_8B, seed, max_seq, batch)
    orc.fill_kv_synthetic(7, 1.0, prefill, batch)
    worst, agree = 0.0, []
    with vsl.Engine.synthetic(CFG_8B, seed=seed, sigma=0.02, max_batch=batch, max_seq=max_seq) as e:
        e.fill_kv_synthetic(7, 1.0, prefill, batch)
        for s in range(n_steps):
            gid, glg = e.step_host(ids[s], want_logits=True)
            oid, olg = orc.step(ids[s], np.full(batch, prefill + s, np.int32))
            worst = max(worst, float(np.abs(glg - olg).max()))
            agree.extend((gid == oid).tolist())
        assert e.device_status() == 0
        assert e.positions(batch).tolist() == [prefill + n_steps] * batch
    orc.close()
    assert worst <= LOGIT_TOL, worst
    assert np.mean(agree) >= 0.99, np.mean(agree)
