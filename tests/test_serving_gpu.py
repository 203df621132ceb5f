"""Batched serving: vsl_engine_generate_batch (one prompt pass per sequence, then batched decode
steps) and continuous batching through vsl_engine_reset_seq + vsl_engine_prefill into a freed
slot while the other sequences keep decoding. fp32 models: identical greedy ids to generating
each prompt alone (the exact-id bar)."""
import numpy as np
import pytest

import vsl
from vsl import synth

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=4, head_dim=64, ffn=1376, vocab=4096,
           rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.F32)


def _prompts(n, seed=3):
    lens = [9, 70, 1, 33, 5, 130][:n]
    return [synth.synth_ids(seed, 30 + b, L, CFG["vocab"]).tolist() for b, L in enumerate(lens)]


def test_generate_batch_matches_single():
    prompts = _prompts(6)
    with vsl.Engine.synthetic(CFG, seed=5, max_batch=1, max_seq=256) as e:
        alone = [e.generate(p, 40) for p in prompts]
    with vsl.Engine.synthetic(CFG, seed=5, max_batch=6, max_seq=256) as e:
        both = e.generate_batch(prompts, 40)
        assert e.device_status() == 0
    assert both == alone


def test_generate_batch_stop_ids_per_sequence():
    prompts = _prompts(4)
    with vsl.Engine.synthetic(CFG, seed=6, max_batch=4, max_seq=256) as e:
        full = e.generate_batch(prompts, 30)
        stop = full[1][7]  # ends sequence 1 after 8 ids (and any other sequence that emits it)
        cut = e.generate_batch(prompts, 30, stop_ids=[stop])
        for f, c in zip(full, cut):
            assert c == (f[:f.index(stop) + 1] if stop in f else f)
        with pytest.raises(vsl.VslError):  # 130-token prompt + 200 new > max_seq 256
            e.generate_batch(_prompts(6)[5:], 200)


def test_continuous_batching_refills_a_slot():
    """Slot 1 finishes and is refilled with a new prompt while slots 0 and 2 keep decoding;
    every sequence produces the ids it produces alone."""
    p = _prompts(4)
    with vsl.Engine.synthetic(CFG, seed=7, max_batch=1, max_seq=256) as e:
        ref = {i: e.generate(p[i], 24) for i in range(4)}
    with vsl.Engine.synthetic(CFG, seed=7, max_batch=3, max_seq=256) as e:
        first = [e.prefill(p[b], seq=b)[0] for b in range(3)]
        e.run(7, batch=3)
        log = e.read_tokens(7, batch=3)
        got = {b: [first[b]] + log[:, b].tolist() for b in range(3)}
        assert got[1] == ref[1][:8]
        # admit request 3 into slot 1
        e.reset_seq(1)
        nxt, _ = e.prefill(p[3], seq=1)
        e.run(16, batch=3)
        log = e.read_tokens(7 + 16, batch=3)
        for b in (0, 2):
            assert got[b] + log[7:, b].tolist() == ref[b][:24]
        assert [nxt] + log[7:, 1].tolist() == ref[3][:17]
        assert e.positions(3).tolist() == [len(p[0]) + 23, len(p[3]) + 16, len(p[2]) + 23]
        assert e.device_status() == 0
