"""Weight residency under an HBM budget (NomadPackManager plan, pack streaming).

CPU: the plan itself through the C ABI. GPU: an engine whose budget keeps only some layers in
HBM streams the others from pinned host memory through two slots every step; its outputs must
be bit-identical to the fully resident engine's (same kernels, same weights), with and without
CUDA-graph capture, and match the CPU oracle.
"""
import numpy as np
import pytest

import vsl
from vsl import synth

GB = 1e9


def test_plan_no_budget_or_fits():
    assert vsl.pack_plan(100, 32, 1000, 0.0) == (32, 0)
    assert vsl.pack_plan(10**9, 32, 10**9, 40.0) == (32, 0)


def test_plan_partial():
    layer, fixed = 2 * 10**9, 10 * 10**9
    # budget = fixed + two slots + 5 layers
    r, s = vsl.pack_plan(layer, 32, fixed, (fixed + 2 * layer + 5 * layer + layer // 2) / GB)
    assert (r, s) == (5, 27)


def test_plan_infeasible():
    with pytest.raises(vsl.VslError) as e:
        vsl.pack_plan(4 * 10**9, 80, 60 * 10**9, 64.0)
    assert e.value.code == -8


def test_plan_70b_shape_under_64gb():
    # 70B Llama shape fp16: one layer = (q+k+v+o + gate/up/down) weights + two norms
    d, hd, nh, nkv, ff = 8192, 128, 64, 8, 28672
    layer = ((nh + 2 * nkv) * hd * d + d * nh * hd + 3 * ff * d) * 2 + 2 * d * 4
    emb = 2 * 128256 * d * 2
    kv = 2 * 80 * 2304 * nkv * hd * 2  # 2048-token prompt + 128 decode steps, fp16, batch 1
    r, s = vsl.pack_plan(layer, 80, emb + kv + (1 << 30), 64.0)
    assert r + s == 80 and s > 0 and r > 0
    assert emb + kv + (1 << 30) + (r + 2) * layer <= 64 * GB


def _layer_bytes(cfg, es):
    A = 256
    up = lambda v: (v + A - 1) // A * A
    d, hd = cfg["d_model"], cfg["head_dim"]
    qkv = (cfg["n_heads"] + 2 * cfg["n_kv_heads"]) * hd
    return (up(qkv * d * es) + up(d * cfg["n_heads"] * hd * es) + up(2 * cfg["ffn"] * d * es) +
            up(d * cfg["ffn"] * es) + 2 * up(d * 4))


@pytest.mark.gpu
@pytest.mark.parametrize("use_graph", [1, 0])
def test_streamed_engine_matches_resident(use_graph):
    cfg = dict(n_layers=6, d_model=1024, n_heads=8, n_kv_heads=4, head_dim=128, ffn=2816, vocab=6000,
               rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.F16)
    prompt = synth.synth_ids(5, 0, 12, cfg["vocab"])
    with vsl.Engine.synthetic(cfg, seed=5, max_seq=128, use_graph=use_graph) as e:
        m = e.memory_stats()
        w, kv, other = m["weights"], m["kv"], m["other"]
        assert e.residency()["streamed_layers"] == 0
        ref_ids = e.generate(prompt, 24)
        _, ref_lg = e.step_host([ref_ids[-1]], want_logits=True)
    layer = _layer_bytes(cfg, 2)
    budget = (w + kv + other - 2.5 * layer) / GB  # room for 1.5 layers besides the two slots
    with vsl.Engine.synthetic(cfg, seed=5, max_seq=128, use_graph=use_graph, vram_budget_gb=budget) as e:
        res = e.residency()
        assert res["streamed_layers"] >= 3 and res["resident_layers"] >= 1
        assert res["resident_layers"] + res["streamed_layers"] == cfg["n_layers"]
        assert e.memory_stats()["weights"] < w
        ids = e.generate(prompt, 24)
        _, lg = e.step_host([ids[-1]], want_logits=True)
        assert e.device_status() == 0
    assert ids == ref_ids
    assert np.array_equal(lg, ref_lg)


@pytest.mark.gpu
def test_streamed_engine_matches_oracle():
    import oracle as O
    cfg = dict(n_layers=4, d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1376, vocab=3000,
               rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.BF16)
    with vsl.Engine.synthetic(cfg, seed=6, max_seq=96) as e:
        m = e.memory_stats()
        w, kv, other = m["weights"], m["kv"], m["other"]
    layer = _layer_bytes(cfg, 2)
    with vsl.Engine.synthetic(cfg, seed=6, max_seq=96, vram_budget_gb=(w + kv + other - 1.5 * layer) / GB) as e:
        assert e.residency()["streamed_layers"] >= 2
        orc = O.Model.synthetic(n_layers=4, d=512, n_heads=8, n_kv=2, ffn=1376, vocab=3000, rope_theta=10000.0,
                                eps=1e-5, wdtype=O.BF16, kvdtype=O.F16, max_seq=96, max_batch=1, seed=6)
        ids = synth.synth_ids(6, 1, 20, cfg["vocab"])
        worst, agree = 0.0, 0
        for p, t in enumerate(ids):
            gid, glg = e.step_host([t], want_logits=True)
            oid, olg = orc.step([t], [p])
            worst = max(worst, float(np.abs(glg - olg).max()))
            agree += int(gid[0] == oid[0])
        assert worst <= 2e-2 and agree >= 19
        assert e.device_status() == 0


@pytest.mark.gpu
def test_engine_refuses_budget_below_fixed_part():
    cfg = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=8, head_dim=64, ffn=1376, vocab=3000,
               rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.F16)
    with pytest.raises(vsl.VslError) as e:
        vsl.Engine.synthetic(cfg, seed=1, max_seq=64, vram_budget_gb=0.001)
    assert e.value.code == -8
