"""Block-quantized weights (Q8_0 / Q4_0 / Q4_1) on the B200: the quantized GEMV against a torch fp32
reference of the same dequantized weights (every epilogue and row count), and the engine
against the goldens (GGUF fixtures, greedy ids) and the oracle (seeded 7B/8B-shaped models,
teacher-forced logits within 2e-2, top-1 agreement >= 99%)."""
import numpy as np
import pytest

import oracle as O
import vsl
from vsl import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

LOGIT_TOL = 2e-2


def _qweights(dtype, N, K, seed=1, tid=300):
    blocks = synth.synth_q_blocks(seed, tid, N, K, dtype)
    deq = synth.dequant_q_blocks(blocks, dtype, K)
    packed = vsl.repack_gguf_rows(dtype, blocks, N, K)
    return torch.from_numpy(packed).cuda(), torch.from_numpy(deq).cuda()


@pytest.mark.parametrize("dtype", [vsl.Q8_0, vsl.Q4_0, vsl.Q4_1])
@pytest.mark.parametrize("N,K", [(4096, 4096), (333, 1376), (1024, 11008)])
@pytest.mark.parametrize("B", [1, 2, 4, 6])
def test_gemv_quantized_store(dtype, N, K, B):
    W, Wd = _qweights(dtype, N, K)
    x = torch.randn(B, K, device="cuda")
    y = torch.zeros(B, N, device="cuda")
    vsl.gemv(dtype, W, N, K, x, B, y)
    torch.cuda.synchronize()
    ref = (x.double() @ Wd.double().T).float()
    err = (y - ref).abs().max().item()
    assert err <= 1e-4 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("dtype", [vsl.Q8_0, vsl.Q4_0, vsl.Q4_1])
def test_device_synthesis_equals_repacked_numpy_blocks(dtype):
    """The engine's seeded quantized weights (generated on the device) are, byte for byte, the
    NumPy GGUF blocks of the same seed repacked into the device row layout."""
    rows, cols, seed, tid = 37, 1376, 9, synth.tid_layer(0, synth.K_DOWN)
    want = vsl.repack_gguf_rows(dtype, synth.synth_q_blocks(seed, tid, rows, cols, dtype), rows, cols)
    dev = torch.zeros(want.size, dtype=torch.uint8, device="cuda")
    vsl.synth_fill_q(dev, dtype, seed, tid, rows, cols)
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy().reshape(want.shape), want)


@pytest.mark.parametrize("dtype", [vsl.Q8_0, vsl.Q4_0, vsl.Q4_1])
def test_gemv_quantized_epilogues(dtype):
    N, K, B = 2 * 704, 512, 3  # interleaved gate/up rows for SwiGLU
    W, Wd = _qweights(dtype, N, K, tid=301)
    x = torch.randn(B, K, device="cuda")
    nw = torch.rand(K, device="cuda") + 0.5
    xn = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-5) * nw
    acc = (xn.double() @ Wd.double().T).float()
    # residual add with fused RMSNorm of x
    y0 = torch.randn(B, N, device="cuda")
    y = y0.clone()
    vsl.gemv(dtype, W, N, K, x, B, y, vsl.EPI_ADD, nw, 1e-5)
    torch.cuda.synchronize()
    assert (y - (y0 + acc)).abs().max().item() < 1e-4
    # SwiGLU over (gate_i, up_i) row pairs
    a = torch.zeros(B, N // 2, device="cuda")
    vsl.gemv(dtype, W, N, K, x, B, a, vsl.EPI_SWIGLU, nw, 1e-5)
    torch.cuda.synchronize()
    g, u = acc[:, 0::2], acc[:, 1::2]
    assert (a - torch.nn.functional.silu(g) * u).abs().max().item() < 1e-4


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q41"])
def test_quantized_gguf_greedy_matches_golden(golden, fixture_gguf, name):
    g = golden(name)
    with vsl.Engine.from_gguf(fixture_gguf(name), max_seq=128) as e:
        assert e.config["wdtype"] == g["dtype"]
        assert e.generate(g["prompt"], g["n_new"]) == g["ids"]
        # token-by-token host path agrees with the top-5 of the golden
        e.reset()
        seq = g["prompt"] + g["ids"][:-1]
        worst = 0.0
        for p, tok in enumerate(seq):
            _, lg = e.step_host([tok], want_logits=True)
            k = p - (len(g["prompt"]) - 1)
            if k >= 0:
                for j, v in g["top5"][k]:
                    worst = max(worst, abs(float(lg[0, j]) - v))
        assert worst < 1e-3
        assert e.device_status() == 0


@pytest.mark.parametrize("name", ["tiny_q4", "tiny_q41"])
def test_legacy_q4_nibble_order_matches_oracle(fixture_gguf, golden, name):
    """legacy_q4 = 1 reads the file the way the reference's loader does (different weights)."""
    g = golden(name)
    path = fixture_gguf(name)
    orc = O.Model.from_gguf(path, kvdtype=O.F16, max_seq=128, legacy_q4=1)
    want, _ = orc.greedy(g["prompt"], 16)
    with vsl.Engine.from_gguf(path, max_seq=128, legacy_q4=1) as e:
        assert e.generate(g["prompt"], 16) == want
    assert want != g["ids"][:16]


def _teacher_forced(cfg, seed, n_steps, batch=1):
    max_seq = n_steps + 64
    e = vsl.Engine.synthetic(cfg, seed=seed, max_batch=batch, max_seq=max_seq)
    orc = O.Model.synthetic(n_layers=cfg["n_layers"], d=cfg["d_model"], n_heads=cfg["n_heads"],
                            n_kv=cfg["n_kv_heads"], ffn=cfg["ffn"], vocab=cfg["vocab"], rope_theta=cfg["rope_theta"],
                            eps=cfg["rms_eps"], wdtype=cfg["wdtype"], kvdtype=O.F16, max_seq=max_seq,
                            max_batch=batch, seed=seed)
    ids = synth.synth_ids(seed, 1, n_steps * batch, cfg["vocab"]).reshape(n_steps, batch)
    worst, agree = 0.0, []
    for s in range(n_steps):
        gid, glg = e.step_host(ids[s], want_logits=True)
        oid, olg = orc.step(ids[s], np.full(batch, s, np.int32))
        worst = max(worst, float(np.abs(glg - olg).max()))
        agree.append(float(np.mean(gid == oid)))
    assert e.device_status() == 0
    e.close()
    return worst, float(np.mean(agree))


@pytest.mark.parametrize("dtype", [vsl.Q8_0, vsl.Q4_0, vsl.Q4_1])
def test_7b_shape_quantized_reduced_depth(dtype):
    cfg = dict(n_layers=2, d_model=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000,
               rope_theta=10000.0, rms_eps=1e-5, wdtype=dtype)
    worst, agree = _teacher_forced(cfg, seed=51, n_steps=8)
    assert worst <= LOGIT_TOL and agree >= 0.99, (worst, agree)


def test_quantized_gqa_batch6_prefill():
    """batch 6 (GEMV launches of 4 + 2 rows) and a 70-token prompt pass on Q8_0 weights."""
    cfg = dict(n_layers=2, d_model=1024, n_heads=8, n_kv_heads=2, head_dim=128, ffn=2816, vocab=6000,
               rope_theta=500000.0, rms_eps=1e-5, wdtype=vsl.Q8_0)
    worst, agree = _teacher_forced(cfg, seed=52, n_steps=5, batch=6)
    assert worst <= LOGIT_TOL and agree >= 0.99, (worst, agree)
    prompt = synth.synth_ids(53, 0, 70, cfg["vocab"]).tolist()
    orc = O.Model.synthetic(n_layers=2, d=1024, n_heads=8, n_kv=2, ffn=2816, vocab=6000, rope_theta=500000.0,
                            eps=1e-5, wdtype=vsl.Q8_0, kvdtype=O.F16, max_seq=128, max_batch=1, seed=52)
    for p, t in enumerate(prompt):
        _, olg = orc.step([t], [p])
    with vsl.Engine.synthetic(cfg, seed=52, max_batch=1, max_seq=128) as e:
        nxt, lg = e.prefill(prompt, want_logits=True)
        assert float(np.abs(lg - olg[0]).max()) <= LOGIT_TOL
        assert nxt == int(np.argmax(olg[0]))
