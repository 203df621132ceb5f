"""Short-cache decode attention (vsl_flash_decode_short: one CTA per sequence and KV group, a
round of 256 positions, 128 with fp32 KV, processed at once) against the oracle's per-row
attention: MHA and GQA, head_dim 64 and 128, fp16 and fp32 caches over permuted pages, ragged
lengths from 1 to several rounds, cache tails filled with NaN bit patterns (never read), the
sparse mask, and bit-identical repeats. The engine takes this kernel for decode steps while
max_seq <= 1024 (attn_route 0) or always (attn_route 3).
"""
import numpy as np
import pytest

import oracle as O
import vsl

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

PAGE = 64


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run(hd, kvdt, nh, nkv, lens, max_len, seed, sparse=None):
    rng = np.random.default_rng(seed)
    B = len(lens)
    max_pages = max_len // PAGE
    n_pages = B * max_pages + 3
    perm = rng.permutation(n_pages)[:B * max_pages].reshape(B, max_pages).astype(np.int32)
    Kd = rng.standard_normal((B, nkv, max_len, hd)).astype(np.float32)
    Vd = rng.standard_normal((B, nkv, max_len, hd)).astype(np.float32)
    if kvdt == vsl.F16:
        Kd, Vd = Kd.astype(np.float16), Vd.astype(np.float16)
    nan = np.float16(np.nan) if kvdt == vsl.F16 else np.float32(np.nan)
    Kp = np.full((n_pages, nkv, PAGE, hd), nan, Kd.dtype)
    Vp = np.full((n_pages, nkv, PAGE, hd), nan, Vd.dtype)
    for b in range(B):
        for t in range(lens[b]):  # only the positions each sequence has written
            Kp[perm[b, t // PAGE], :, t % PAGE] = Kd[b, :, t]
            Vp[perm[b, t // PAGE], :, t % PAGE] = Vd[b, :, t]
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    pos = np.array([l - 1 for l in lens], np.int32)
    kc = dev(Kp.view(np.uint16) if kvdt == vsl.F16 else Kp)
    vc = dev(Vp.view(np.uint16) if kvdt == vsl.F16 else Vp)
    out = torch.full((B, nh * hd), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = []
    for _ in range(2):
        vsl.flash_decode_short(dev(q), kc, vc, kvdt, dev(perm), max_pages, PAGE, dev(pos), B, nh, nkv, hd, max_len,
                               out, sparse=sparse, status=status)
        torch.cuda.synchronize()
        got.append(out.cpu().numpy().copy())
    assert status.item() == 0
    assert np.array_equal(got[0], got[1])
    for b in range(B):
        kk = Kd[b].view(np.uint16) if kvdt == vsl.F16 else Kd[b]
        vv = Vd[b].view(np.uint16) if kvdt == vsl.F16 else Vd[b]
        first = O.sparse_first(*sparse, int(pos[b])) if sparse else 0
        ref = O.attention(q[b], kk, vv, O.F16 if kvdt == vsl.F16 else O.F32, nh, nkv, hd, max_len, lens[b],
                          first=first)
        assert np.allclose(got[0][b], ref, rtol=2e-4, atol=2e-5), (b, lens[b])
    return got[0]


@pytest.mark.parametrize("hd,kvdt", [(128, vsl.F16), (64, vsl.F16), (128, vsl.F32), (64, vsl.F32)])
@pytest.mark.parametrize("nh,nkv", [(4, 4), (8, 2), (8, 1)])
def test_short_attention_matches_oracle(hd, kvdt, nh, nkv):
    # 1 position, one chunk, a chunk boundary, a full round, across rounds (fp32 rounds are 128)
    run(hd, kvdt, nh, nkv, [1, 64, 65, 256, 257, 700], max_len=768, seed=hd + nh + nkv + kvdt)


def test_short_attention_sparse_mask():
    mask = (100, 40, 4, 128)
    lens = [50, 101, 130, 300, 521, 700]  # dense, just past the switch, across blocks and rounds
    got = run(128, vsl.F16, 8, 2, lens, max_len=768, seed=7, sparse=mask)
    dense = run(128, vsl.F16, 8, 2, lens, max_len=768, seed=7)
    assert np.array_equal(got[0], dense[0])  # below the switch: the same kernel path, the same bits
    assert not np.allclose(got[-1], dense[-1], atol=1e-3)


def test_engine_short_route_matches_split_k():
    """The engine's decode steps with the short-cache kernel (attn_route 3) and the split-K kernel
    (attn_route 1) give the same greedy ids and logits within fp32 reassociation."""
    from vsl import synth
    cfg = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1376, vocab=4096,
               rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.F16)
    prompt = synth.synth_ids(5, 0, 90, cfg["vocab"]).tolist()
    ids = synth.synth_ids(5, 1, 12, cfg["vocab"]).tolist()
    res = []
    for route in (3, 1):
        with vsl.Engine.synthetic(cfg, seed=5, max_seq=384, attn_route=route) as e:
            e.prefill(prompt)
            lg = [e.step_host(np.array([t], np.int32), want_logits=True)[1] for t in ids]
            assert e.device_status() == 0
            res.append(np.stack(lg))
    assert np.abs(res[0] - res[1]).max() < 1e-3
    assert (res[0].argmax(-1) == res[1].argmax(-1)).all()
