"""CPU oracle pins: known answers derived from the reference source, the float64 NumPy
restatement's golden fixtures, and bit-exactness of the seeded generator across NumPy/C."""
import math

import numpy as np
import pytest

import oracle as O
from vsl import synth


def test_synth_numpy_matches_c_all_dtypes():
    for tid in (1, 2, 256 + 16 * 3 + 7, 0x40000001):
        a = synth.synth_f32(5, tid, 50000, 0.02, start=123)
        b = O.synth_fill(5, tid, 50000, 0.02, O.F32, start=123)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    a16 = synth.synth_tensor(9, 300, (4000,), synth.GGML_F16).view(np.uint16)
    assert np.array_equal(a16, O.synth_fill(9, 300, 4000, 0.02, O.F16))
    abf = synth.synth_tensor(9, 300, (4000,), synth.GGML_BF16)
    assert np.array_equal(abf, O.synth_fill(9, 300, 4000, 0.02, O.BF16))
    assert np.array_equal(synth.synth_ids(0, 0, 64, 32000), O.synth_ids(0, 0, 64, 32000))


def test_synth_distribution():
    v = synth.synth_f32(0, 1, 1 << 20, 0.02)
    assert abs(v.mean()) < 1e-4 and abs(v.std() - 0.02) < 2e-4
    ids = synth.synth_ids(0, 0, 1 << 16, 32000)
    assert ids.min() >= 0 and ids.max() < 32000


def test_half_to_float_exhaustive():
    # convert_fp16_to_fp32 (GGUFLoader.cpp:1225-1262) is the exact IEEE conversion
    L = O.lib()
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([L.orc_h2f(int(x)) for x in h], np.float32)
    same = (ref.view(np.uint32) == got.view(np.uint32)) | (np.isnan(ref) & np.isnan(got))
    assert same.all()


def test_float_to_half_round_nearest_even():
    L = O.lib()
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(4000).astype(np.float32) * s for s in (1e-7, 1e-5, 1e-2, 1, 1e3, 6e4)])
    edge = np.array([65504, 65519.996, 65520, 2.0 ** -24, 2.0 ** -25, 1.5 * 2.0 ** -25, 0.0, -0.0, np.inf, -np.inf,
                     1 + 2.0 ** -11, 1 + 3 * 2.0 ** -11], np.float32)
    xs = np.concatenate([xs, edge])
    with np.errstate(over="ignore"):
        ref = xs.astype(np.float16).view(np.uint16)
    got = np.array([L.orc_f2h(float(x)) for x in xs], np.uint16)
    assert np.array_equal(ref, got)


def test_bf16_round_nearest_even():
    L = O.lib()
    rng = np.random.default_rng(1)
    xs = rng.standard_normal(5000).astype(np.float32)
    ref = synth.f32_to_bf16_bits(xs)
    got = np.array([L.orc_f2bf(float(x)) for x in xs], np.uint16)
    assert np.array_equal(ref, got)


def test_argmax_first_maximum():
    # greedy_sampling (VulkanSymbioteEngine.cpp:1794-1804) keeps the first index on ties
    v = np.array([0.5, 2.0, -1.0, 2.0, 2.0], np.float32)
    assert O.argmax(v) == 1
    assert O.argmax(np.full(7, -3.0, np.float32)) == 0


def test_rope_table_known_answer():
    # Utils.cpp:101-110: freq = theta^(-i/hd) for even i, angle = pos * freq
    hd, theta = 8, 10000.0
    c, s = O.rope_table(5, hd, theta)
    for p in range(5):
        for j in range(hd // 2):
            ang = p * theta ** (-(2 * j) / hd)
            assert c[p, j] == pytest.approx(math.cos(ang), abs=1e-7)
            assert s[p, j] == pytest.approx(math.sin(ang), abs=1e-7)
    v = np.arange(1, 9, dtype=np.float32)
    r = O.rope_apply(v, 1, hd, c[3], s[3])
    for j in range(hd // 2):
        a, b = v[2 * j], v[2 * j + 1]
        assert r[2 * j] == pytest.approx(a * c[3, j] - b * s[3, j], rel=1e-6)
        assert r[2 * j + 1] == pytest.approx(a * s[3, j] + b * c[3, j], rel=1e-6)


def test_rmsnorm_known_answer():
    # rms_norm.comp:30-34: x / sqrt(sum(x^2)/d + eps) * w
    x = np.array([[1, 2, 3, 4]], np.float32)
    w = np.array([1, 0.5, 2, 1], np.float32)
    y = O.rmsnorm(x, w, 1e-5)
    den = math.sqrt(30 / 4 + 1e-5)
    assert np.allclose(y, x / den * w, rtol=1e-6)


def test_swiglu_known_answer():
    g = np.array([0.0, 1.0, -2.0], np.float32)
    u = np.array([3.0, 2.0, 1.0], np.float32)
    a = O.swiglu(g, u)
    ref = g / (1 + np.exp(-g)) * u
    assert np.allclose(a, ref, rtol=1e-6)


@pytest.mark.parametrize("dtype", [O.F32, O.F16, O.BF16])
def test_gemv_vs_float64(dtype):
    rng = np.random.default_rng(2)
    N, K, B = 37, 136, 3
    w32 = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    if dtype == O.F16:
        W = w32.astype(np.float16)
        wf = W.astype(np.float64)
        W = W.view(np.uint16)
    elif dtype == O.BF16:
        W = synth.f32_to_bf16_bits(w32).reshape(N, K)
        wf = synth.bf16_bits_to_f32(W).astype(np.float64)
    else:
        W, wf = w32, w32.astype(np.float64)
    x = rng.standard_normal((B, K)).astype(np.float32)
    y = O.gemv(W, dtype, x)
    assert np.allclose(y, x.astype(np.float64) @ wf.T, rtol=1e-5, atol=1e-5)


def test_attention_vs_float64_gqa():
    rng = np.random.default_rng(3)
    nh, nkv, hd, max_seq, L = 8, 2, 64, 40, 33
    q = rng.standard_normal(nh * hd).astype(np.float32)
    K = rng.standard_normal((nkv, max_seq, hd)).astype(np.float32)
    V = rng.standard_normal((nkv, max_seq, hd)).astype(np.float32)
    o = O.attention(q, K, V, O.F32, nh, nkv, hd, max_seq, L)
    for h in range(nh):
        g = h * nkv // nh
        s = K[g, :L].astype(np.float64) @ q[h * hd:(h + 1) * hd] / math.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        assert np.allclose(o[h * hd:(h + 1) * hd], p @ V[g, :L], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("name", ["tiny_fp32", "gqa_fp16"])
def test_oracle_matches_golden(name, golden, fixture_gguf):
    g = golden(name)
    m = O.Model.from_gguf(fixture_gguf(name), kvdtype=O.F16 if g["kv_dtype"] == "f16" else O.F32,
                          max_seq=g["prompt"].__len__() + g["n_new"] + 1)
    ids, logits = m.greedy(g["prompt"], g["n_new"], want_logits=True)
    assert ids == g["ids"]
    err = max(abs(float(logits[i][j]) - v) for i, row in enumerate(g["top5"]) for j, v in row)
    assert err < (1e-4 if g["dtype"] == 0 else 2e-4)


def test_oracle_synthetic_equals_gguf(golden, fixture_gguf):
    g = golden("gqa_fp16")
    s = g["shape"]
    a = O.Model.from_gguf(fixture_gguf("gqa_fp16"), kvdtype=O.F16, max_seq=64)
    b = O.Model.synthetic(n_layers=s["n_layers"], d=s["d_model"], n_heads=s["n_heads"], n_kv=s["n_kv_heads"],
                          ffn=s["ffn"], vocab=s["vocab"], rope_theta=s["rope_theta"], wdtype=O.F16, kvdtype=O.F16,
                          max_seq=64, seed=g["seed"])
    ia, la = a.greedy(g["prompt"][:8], 6, want_logits=True)
    ib, lb = b.greedy(g["prompt"][:8], 6, want_logits=True)
    assert ia == ib
    assert all(np.array_equal(x, y) for x, y in zip(la, lb))


def test_oracle_batch_rows_independent():
    kw = dict(n_layers=2, d=128, n_heads=4, n_kv=2, ffn=344, vocab=500, wdtype=O.BF16, kvdtype=O.F16, max_seq=32,
              max_batch=3, seed=11)
    m = O.Model.synthetic(**kw)
    m.fill_kv_synthetic(4, 1.0, 10, 3)
    _, lg = m.step(np.array([5, 17, 499], np.int32), np.array([10, 10, 10], np.int32))
    m1 = O.Model.synthetic(**kw)
    m1.fill_kv_synthetic(4, 1.0, 10, 3)
    _, l1 = m1.step(np.array([5], np.int32), np.array([10], np.int32))
    assert np.array_equal(l1[0], lg[0])
    assert not np.array_equal(lg[0], lg[1])


def test_tp_check_fixture_is_the_oracles():
    """tests/golden/tp_check_7b_2l.json (what bench.py checks tensor-parallel engines against)
    holds the oracle's ids and logits of its model."""
    import json
    import os
    with open(os.path.join(os.path.dirname(__file__), "golden", "tp_check_7b_2l.json")) as f:
        g = json.load(f)
    m = O.Model.synthetic(n_layers=g["n_layers"], d=g["d_model"], n_heads=g["n_heads"], n_kv=g["n_kv_heads"],
                          ffn=g["ffn"], vocab=g["vocab"], rope_theta=g["rope_theta"], eps=g["rms_eps"],
                          wdtype=g["wdtype"], kvdtype=O.F16, max_seq=g["max_seq"], max_batch=1, seed=g["seed"],
                          sigma=g["sigma"])
    assert g["ids"] == O.synth_ids(g["seed"], 2, g["n_steps"], g["vocab"]).tolist()
    for p, (t, st) in enumerate(zip(g["ids"], g["steps"])):
        oid, lg = m.step([t], [p])
        assert int(oid[0]) == st["argmax"]
        assert np.abs(lg[0][g["probe_index"]] - np.asarray(st["probe"])).max() == 0.0
        assert all(lg[0][i] == v for i, v in st["top8"])
    m.close()
