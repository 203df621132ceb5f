"""Long-context sparse attention on the GPU against the oracle's restatement of the reference's
mask (vk_symbiote/shaders/sparse_attention.comp:77-131, switched at VulkanSymbioteEngine.cpp:788):
the split-K kernel (vsl_flash_decode_sparse) with small window parameters that put the window's
start inside, at and across split and page boundaries; the tcgen05 kernel
(vsl_flash_decode_tc_sparse) at the reference's defaults past 8192 positions; and the engine with
sparse_min_len set, teacher-forced against the oracle model with the same mask.
"""
import numpy as np
import pytest

import oracle as O
import vsl
from vsl import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def scatter_pages(dense, page_table, page, n_pages):
    B, nkv, L, hd = dense.shape
    out = np.zeros((n_pages, nkv, page, hd), dense.dtype)
    for b in range(B):
        for t in range(L):
            out[page_table[b, t // page], :, t % page] = dense[b, :, t]
    return out


@pytest.mark.parametrize("hd,kvdt", [(64, vsl.F32), (128, vsl.F16)])
def test_split_k_sparse_matches_oracle(hd, kvdt):
    rng = np.random.default_rng(hd)
    nh, nkv, page, max_len = 8, 2, 64, 704
    mask = (100, 40, 4, 128)  # min_len, window, global tokens, block
    lens = [50, 101, 130, 257, 300, 521, 700]  # dense, just past the switch, across blocks and splits
    B = len(lens)
    max_pages = max_len // page
    n_pages = B * max_pages
    perm = rng.permutation(n_pages).reshape(B, max_pages).astype(np.int32)
    Kd = rng.standard_normal((B, nkv, max_len, hd)).astype(np.float32)
    Vd = rng.standard_normal((B, nkv, max_len, hd)).astype(np.float32)
    if kvdt == vsl.F16:
        Kd, Vd = Kd.astype(np.float16), Vd.astype(np.float16)
    kc = dev(scatter_pages(Kd, perm, page, n_pages).view(np.uint16) if kvdt == vsl.F16 else scatter_pages(Kd, perm, page, n_pages))
    vc = dev(scatter_pages(Vd, perm, page, n_pages).view(np.uint16) if kvdt == vsl.F16 else scatter_pages(Vd, perm, page, n_pages))
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    pos = np.array([l - 1 for l in lens], np.int32)
    firsts = [O.sparse_first(*mask, p) for p in pos]
    assert firsts[0] == 0 and firsts[1] > 0  # both sides of the switch are covered
    for split in (64, 128, 256):
        n = vsl.flash_decode_workspace_size(B, nh, nkv, hd, max_len, split)
        ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
        out = torch.full((B, nh * hd), float("nan"), device="cuda")
        for rep in range(2):  # counters left at zero for the next call
            vsl.flash_decode(dev(q), kc, vc, kvdt, dev(perm), max_pages, page, dev(pos), B, nh, nkv, hd, max_len,
                             split, out, ws, n, sparse=mask)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            for b in range(B):
                kk = Kd[b].view(np.uint16) if kvdt == vsl.F16 else Kd[b]
                vv = Vd[b].view(np.uint16) if kvdt == vsl.F16 else Vd[b]
                ref = O.attention(q[b], kk, vv, O.F16 if kvdt == vsl.F16 else O.F32, nh, nkv, hd, max_len, lens[b],
                                  first=firsts[b])
                assert np.allclose(got[b], ref, rtol=2e-4, atol=2e-5), (b, split, rep)
    # a dense call on the same data differs from the sparse one past the switch
    n = vsl.flash_decode_workspace_size(B, nh, nkv, hd, max_len, 256)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    dense = torch.zeros((B, nh * hd), device="cuda")
    vsl.flash_decode(dev(q), kc, vc, kvdt, dev(perm), max_pages, page, dev(pos), B, nh, nkv, hd, max_len, 256, dense,
                     ws, n)
    torch.cuda.synchronize()
    assert not torch.allclose(dense[-1], out[-1], atol=1e-3)
    assert torch.equal(dense[0], out[0])  # below the switch: the same kernel path, the same bits


def test_tc_sparse_matches_oracle_past_8192():
    rng = np.random.default_rng(11)
    nh, nkv, page = 32, 8, 64
    mask = (8192, 512, 16, 1024)
    lens = [8192, 8193, 9216, 9217, 10000, 1500]
    B = len(lens)
    max_len = 10048
    max_pages = max_len // page
    n_pages = B * max_pages
    perm = rng.permutation(n_pages).reshape(B, max_pages).astype(np.int32)
    Kd = rng.standard_normal((B, nkv, max_len, 128)).astype(np.float16)
    Vd = rng.standard_normal((B, nkv, max_len, 128)).astype(np.float16)
    kc = dev(scatter_pages(Kd, perm, page, n_pages).view(np.uint16))
    vc = dev(scatter_pages(Vd, perm, page, n_pages).view(np.uint16))
    q = rng.standard_normal((B, nh * 128)).astype(np.float32)
    pos = np.array([l - 1 for l in lens], np.int32)
    n = vsl.flash_decode_tc_workspace_size(B, nkv)
    ws = torch.zeros(n // 4 + 64, dtype=torch.int32, device="cuda")
    out = torch.full((B, nh * 128), float("nan"), device="cuda")
    for rep in range(2):
        vsl.flash_decode_tc(dev(q), kc, vc, n_pages, dev(perm), max_pages, page, dev(pos), B, nh, nkv, 128, max_len,
                            out, ws, n, sparse=mask)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for b in range(B):
            first = O.sparse_first(*mask, int(pos[b]))
            ref = O.attention(q[b], Kd[b].view(np.uint16), Vd[b].view(np.uint16), O.F16, nh, nkv, 128, max_len,
                              lens[b], first=first)
            assert np.allclose(got[b], ref, rtol=5e-4, atol=2e-4), (b, rep, first)


def test_engine_sparse_attention_teacher_forced():
    cfg = dict(n_layers=2, d_model=1024, n_heads=8, n_kv_heads=2, head_dim=128, ffn=2816, vocab=4096,
               rope_theta=500000.0, rms_eps=1e-5, wdtype=vsl.BF16)
    batch, prefill, n_steps, seed = 3, 8190, 5, 13  # steps cross the switch at 8192 positions
    max_seq = 8320
    e = vsl.Engine.synthetic(cfg, seed=seed, max_batch=batch, max_seq=max_seq, sparse_min_len=8192)
    orc = O.Model.synthetic(n_layers=2, d=1024, n_heads=8, n_kv=2, ffn=2816, vocab=4096, rope_theta=500000.0,
                            wdtype=O.BF16, kvdtype=O.F16, max_seq=max_seq, max_batch=batch, seed=seed)
    orc.set_sparse(8192, 512, 16, 1024)
    e.fill_kv_synthetic(5, 1.0, prefill, batch)
    orc.fill_kv_synthetic(5, 1.0, prefill, batch)
    ids = synth.synth_ids(seed, 1, n_steps * batch, cfg["vocab"]).reshape(n_steps, batch)
    worst, agree = 0.0, []
    for s in range(n_steps):
        gid, glg = e.step_host(ids[s], want_logits=True)
        oid, olg = orc.step(ids[s], np.full(batch, prefill + s, np.int32))
        worst = max(worst, float(np.abs(glg - olg).max()))
        agree.extend((gid == oid).tolist())
    assert e.device_status() == 0
    e.close()
    orc.close()
    assert worst <= 2e-2, worst
    assert np.mean(agree) >= 0.99
