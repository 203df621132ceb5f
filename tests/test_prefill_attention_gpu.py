"""Prompt attention on the tensor cores (vsl_flash_prefill, query blocks of 128 rows) against the
oracle's per-row attention (the reference's attention.comp run once per prompt token): causal
rows of one sequence over a paged fp16 cache with permuted pages, MHA and GQA, chunks that start
at, inside and past 128-position boundaries, more than 128 rows (two query blocks), the sparse
mask, and NaN bit patterns in the cache past the sequence end (which must not reach the output).
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


def run_case(nh, nkv, p0, P, max_len, seed, sparse=None, reps=2):
    rng = np.random.default_rng(seed)
    hd = 128
    L = p0 + P
    max_pages = max_len // PAGE
    n_pages = max_pages + 3  # a pool larger than the sequence's pages
    page_row = rng.permutation(n_pages)[:max_pages].astype(np.int32)
    Kd = rng.standard_normal((nkv, max_len, hd)).astype(np.float16)
    Vd = rng.standard_normal((nkv, max_len, hd)).astype(np.float16)
    nan16 = np.uint16(0x7E00)
    kpool = np.full((n_pages, nkv, PAGE, hd), nan16, np.uint16)  # unwritten cache reads as NaN
    vpool = np.full((n_pages, nkv, PAGE, hd), nan16, np.uint16)
    for t in range(L):
        kpool[page_row[t // PAGE], :, t % PAGE] = Kd[:, t].view(np.uint16)
        vpool[page_row[t // PAGE], :, t % PAGE] = Vd[:, t].view(np.uint16)
    q = rng.standard_normal((P, nh, hd)).astype(np.float32)
    pos = (p0 + np.arange(P)).astype(np.int32)
    out = torch.full((P, nh, hd), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kc, vc = dev(kpool), dev(vpool)
    results = []
    for _ in range(reps):
        vsl.flash_prefill(dev(q), kc, vc, n_pages, dev(page_row), max_pages, PAGE, dev(pos), P, nh, nkv, hd, max_len,
                          out, sparse=sparse, status=status)
        torch.cuda.synchronize()
        results.append(out.cpu().numpy().copy())
    assert status.item() == 0
    for r in results[1:]:
        assert np.array_equal(r, results[0])  # deterministic
    got = results[0]
    Kn = np.nan_to_num(Kd.astype(np.float32)).astype(np.float16)
    Vn = np.nan_to_num(Vd.astype(np.float32)).astype(np.float16)
    for r in range(P):
        first = O.sparse_first(*sparse, int(pos[r])) if sparse else 0
        ref = O.attention(q[r].reshape(-1), Kn.view(np.uint16), Vn.view(np.uint16), O.F16, nh, nkv, hd, max_len,
                          int(pos[r]) + 1, first=first)
        assert np.allclose(got[r].reshape(-1), ref, rtol=5e-4, atol=2e-4), (r, p0, P)
    return got


@pytest.mark.parametrize("nh,nkv", [(4, 4), (8, 2)])
@pytest.mark.parametrize("p0,P", [(0, 128), (0, 1), (0, 37), (64, 64), (200, 128), (383, 130)])
def test_prefill_attention_matches_oracle(nh, nkv, p0, P):
    run_case(nh, nkv, p0, P, max_len=640, seed=p0 * 7 + P + nh)


def test_prefill_attention_sparse_mask():
    mask = (100, 40, 4, 128)  # switch at 100 positions, window 40, 4 global tokens, 128-position blocks
    got = run_case(8, 2, 90, 128, max_len=320, seed=3, sparse=mask)
    assert O.sparse_first(*mask, 90) == 0 and O.sparse_first(*mask, 217) > 0  # both sides of the switch
    dense = run_case(8, 2, 90, 128, max_len=320, seed=3, reps=1)
    assert np.array_equal(dense[:10], got[:10])  # rows below the switch: the same bits
    assert not np.allclose(dense[-1], got[-1], atol=1e-3)


def test_prefill_attention_arguments_checked():
    q = torch.zeros(4, 2, 128, device="cuda")
    kc = torch.zeros(4, 2, PAGE, 128, dtype=torch.int16, device="cuda")
    pr = torch.zeros(4, dtype=torch.int32, device="cuda")
    pos = torch.arange(4, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    with pytest.raises(vsl.VslError) as e:
        vsl.flash_prefill(q, kc, kc, 4, pr, 4, PAGE, pos, 4, 2, 2, 64, 256, out)  # head_dim 64
    assert e.value.code == -9
    with pytest.raises(vsl.VslError) as e:
        vsl.flash_prefill(q, kc, kc, 4, pr, 4, 32, pos, 4, 2, 2, 128, 128, out)  # page of 32 positions
    assert e.value.code == -9
    with pytest.raises(vsl.VslError) as e:
        vsl.flash_prefill(q, kc, kc, 4, pr, 4, PAGE, pos, 4, 2, 2, 128, 512, out)  # max_len past the pages
    assert e.value.code == -1
