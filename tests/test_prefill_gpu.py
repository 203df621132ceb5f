"""Prompt pass (vsl_engine_prefill) parity: a prompt processed in chunks of up to 64 rows must
leave the engine exactly where the token-by-token loop leaves it.

Bars: fp32 -> the golden greedy ids and logits within 1e-4 of the oracle; fp16/bf16 -> logits
of the last prompt token and of the decode steps after it within 2e-2 of the oracle, top-1
agreement >= 99%. The oracle processes the prompt one token at a time (its only mode), so
these tests also show that chunked causal attention over per-row positions equals the
sequential loop."""
import numpy as np
import pytest

import oracle as O
import vsl
from vsl import synth

pytestmark = pytest.mark.gpu

LOGIT_TOL_F16 = 2e-2


def _oracle(cfg, seed, max_seq, max_batch=1):
    return O.Model.synthetic(n_layers=cfg["n_layers"], d=cfg["d_model"], n_heads=cfg["n_heads"],
                             n_kv=cfg["n_kv_heads"], ffn=cfg["ffn"], vocab=cfg["vocab"], rope_theta=cfg["rope_theta"],
                             eps=cfg["rms_eps"], wdtype=cfg["wdtype"],
                             kvdtype=O.F16 if cfg["wdtype"] != O.F32 else O.F32, max_seq=max_seq,
                             max_batch=max_batch, seed=seed)


def _oracle_prompt(orc, prompt):
    """Token-by-token prompt on the oracle; logits of the last prompt token."""
    lg = None
    for p, t in enumerate(prompt):
        _, lg = orc.step([t], [p])
    return lg[0]


def test_tiny_fp32_prefill_then_decode_matches_golden(golden, fixture_gguf):
    g = golden("tiny_fp32")
    with vsl.Engine.from_gguf(fixture_gguf("tiny_fp32"), max_seq=128) as e:
        nxt, _ = e.prefill(g["prompt"])
        assert nxt == g["ids"][0]
        assert e.positions(1)[0] == len(g["prompt"])
        e.run(g["n_new"] - 1)
        assert [nxt] + e.read_tokens(g["n_new"] - 1).reshape(-1).tolist() == g["ids"]
        assert e.device_status() == 0


def test_tiny_fp32_prefill_logits_match_oracle(golden, fixture_gguf):
    g = golden("tiny_fp32")
    path = fixture_gguf("tiny_fp32")
    orc = O.Model.from_gguf(path, kvdtype=O.F32, max_seq=128)
    olg = _oracle_prompt(orc, g["prompt"])
    with vsl.Engine.from_gguf(path, max_seq=128) as e:
        nxt, lg = e.prefill(g["prompt"], want_logits=True)
        assert nxt == int(np.argmax(olg))
        assert float(np.abs(lg - olg).max()) < 1e-4
        # a second prefill continues the same sequence (prompt given in two parts)
        e.reset()
        half = len(g["prompt"]) // 2
        e.prefill(g["prompt"][:half])
        nxt2, lg2 = e.prefill(g["prompt"][half:], want_logits=True)
        assert nxt2 == nxt and float(np.abs(lg2 - olg).max()) < 1e-4


@pytest.mark.parametrize("wdtype,n_prompt,max_seq,hd", [(vsl.F16, 100, 256, 128), (vsl.BF16, 64, 256, 128),
                                                        (vsl.BF16, 200, 2048, 128), (vsl.F16, 300, 512, 128),
                                                        (vsl.BF16, 90, 256, 64), (vsl.F16, 150, 256, 64)])
def test_half_prefill_chunks_match_oracle(wdtype, n_prompt, max_seq, hd):
    """Prompts in chunks of up to 128 rows (300 tokens = 128 + 128 + 44) on the tcgen05
    projections; head_dim 128 takes the tensor-core prompt attention (one query block per head),
    head_dim 64 the split-K kernel, whose split counters must stay valid when the last chunk has
    fewer rows than the first. Then 6 teacher-forced decode steps."""
    cfg = dict(n_layers=2, d_model=1024, n_heads=1024 // hd, n_kv_heads=256 // hd, head_dim=hd, ffn=2816,
               vocab=6000, rope_theta=10000.0, rms_eps=1e-5, wdtype=wdtype)
    seed = 41
    prompt = synth.synth_ids(seed, 5, n_prompt, cfg["vocab"]).tolist()
    follow = synth.synth_ids(seed, 6, 6, cfg["vocab"]).tolist()
    orc = _oracle(cfg, seed, max_seq)
    with vsl.Engine.synthetic(cfg, seed=seed, max_batch=1, max_seq=max_seq) as e:
        nxt, lg = e.prefill(prompt, want_logits=True)
        olg = _oracle_prompt(orc, prompt)
        worst = float(np.abs(lg - olg).max())
        agree = [nxt == int(np.argmax(olg))]
        for k, t in enumerate(follow):
            gid, glg = e.step_host([t], want_logits=True)
            oid, olg = orc.step([t], [n_prompt + k])
            worst = max(worst, float(np.abs(glg - olg).max()))
            agree.append(int(gid[0]) == int(oid[0]))
        assert e.device_status() == 0
    assert worst <= LOGIT_TOL_F16, worst
    assert np.mean(agree) >= 0.99, agree


def test_ragged_prompts_then_batched_decode():
    """Three sequences prefilled separately (70, 5 and 1 tokens), then decoded as one batch."""
    cfg = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=4, head_dim=64, ffn=1376, vocab=4096,
               rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.F16)
    seed = 43
    lens = [70, 5, 1]
    prompts = [synth.synth_ids(seed, 10 + b, n, cfg["vocab"]).tolist() for b, n in enumerate(lens)]
    orcs = [_oracle(cfg, seed, 128) for _ in lens]
    worst, agree = 0.0, []
    with vsl.Engine.synthetic(cfg, seed=seed, max_batch=3, max_seq=128) as e:
        for b, p in enumerate(prompts):
            nxt, lg = e.prefill(p, seq=b, want_logits=True)
            olg = _oracle_prompt(orcs[b], p)
            worst = max(worst, float(np.abs(lg - olg).max()))
            agree.append(nxt == int(np.argmax(olg)))
        assert e.positions(3).tolist() == lens
        ids = synth.synth_ids(seed, 20, 4 * 3, cfg["vocab"]).reshape(4, 3)
        for s in range(4):
            gid, glg = e.step_host(ids[s], want_logits=True)
            for b in range(3):
                oid, olg = orcs[b].step([ids[s, b]], [lens[b] + s])
                worst = max(worst, float(np.abs(glg[b] - olg[0]).max()))
                agree.append(int(gid[b]) == int(oid[0]))
        assert e.device_status() == 0
    assert worst <= LOGIT_TOL_F16, worst
    assert np.mean(agree) >= 0.99, agree


def test_prefill_bounds():
    cfg = dict(n_layers=1, d_model=256, n_heads=4, n_kv_heads=4, head_dim=64, ffn=512, vocab=1000,
               rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.F32)
    with vsl.Engine.synthetic(cfg, seed=1, max_batch=2, max_seq=32) as e:
        with pytest.raises(vsl.VslError):
            e.prefill(list(range(33)))
        with pytest.raises(vsl.VslError):
            e.prefill([1, 2, 3], seq=2)
        with pytest.raises(vsl.VslError):
            e.prefill([], seq=0)
        e.prefill(list(range(30)), seq=1)
        with pytest.raises(vsl.VslError):  # 30 + 3 > 32
            e.prefill([1, 2, 3], seq=1)
        assert e.positions(2).tolist() == [0, 30]
        assert e.device_status() == 0
