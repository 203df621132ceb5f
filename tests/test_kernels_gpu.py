"""Per-kernel parity of the sm_100a kernels (called through the C ABI) against the CPU oracle.

Tolerances: projections accumulate in fp32 in a different order than the oracle, so each
output may differ by a few fp32 ulps of the sum of |w*x| terms; the bound used is
2e-6 * sum|w||x| + 1e-6. Index and bookkeeping outputs (argmax ids, KV placement, seeded
tensors) must be bit-exact.
"""
import math

import numpy as np
import pytest

import oracle as O
import vsl
from vsl import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream():
    return torch.cuda.current_stream().cuda_stream


def make_w(rng, N, K, dtype, scale=0.05):
    w32 = (rng.standard_normal((N, K)) * scale).astype(np.float32)
    if dtype == vsl.F16:
        h = w32.astype(np.float16)
        return h.view(np.uint16), h.astype(np.float32)
    if dtype == vsl.BF16:
        b = synth.f32_to_bf16_bits(w32).reshape(N, K)
        return b, synth.bf16_bits_to_f32(b).reshape(N, K)
    return w32, w32


def bound(wf, x):
    return 2e-6 * (np.abs(x).astype(np.float64) @ np.abs(wf).T.astype(np.float64)) + 1e-6


@pytest.mark.parametrize("dtype", [vsl.F32, vsl.F16, vsl.BF16])
@pytest.mark.parametrize("N,K", [(1, 8), (3, 136), (130, 1376), (1000, 512), (257, 4096)])
@pytest.mark.parametrize("B", [1, 3, 6])
def test_gemv_store(dtype, N, K, B):
    if dtype == vsl.F32 and K == 8:
        K = 4
    rng = np.random.default_rng(N * 7 + K + B)
    W, wf = make_w(rng, N, K, dtype)
    x = rng.standard_normal((B, K)).astype(np.float32)
    y = torch.full((B, N), float("nan"), device="cuda")
    vsl.gemv(dtype, dev(W), N, K, dev(x), B, y, vsl.EPI_STORE, stream=stream())
    torch.cuda.synchronize()
    ref = O.gemv(W, {vsl.F32: O.F32, vsl.F16: O.F16, vsl.BF16: O.BF16}[dtype], x)
    assert np.all(np.abs(y.cpu().numpy() - ref) <= bound(wf, x))


@pytest.mark.parametrize("dtype", [vsl.F16, vsl.BF16])
def test_gemv_norm_add_swiglu(dtype):
    rng = np.random.default_rng(5)
    N, K, B = 688, 1024, 3
    W, wf = make_w(rng, N, K, dtype)
    odt = O.F16 if dtype == vsl.F16 else O.BF16
    x = rng.standard_normal((B, K)).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    xn = O.rmsnorm(x, nw, 1e-5)
    # fused RMSNorm + residual add
    y0 = rng.standard_normal((B, N)).astype(np.float32)
    y = dev(y0)
    vsl.gemv(dtype, dev(W), N, K, dev(x), B, y, vsl.EPI_ADD, dev(nw), 1e-5, stream=stream())
    torch.cuda.synchronize()
    ref = y0 + O.gemv(W, odt, xn)
    assert np.all(np.abs(y.cpu().numpy() - ref) <= bound(wf, xn) + 1e-6 * np.abs(y0))
    # SwiGLU over interleaved rows (gate_i, up_i)
    a = torch.zeros((B, N // 2), device="cuda")
    vsl.gemv(dtype, dev(W), N, K, dev(x), B, a, vsl.EPI_SWIGLU, dev(nw), 1e-5, stream=stream())
    torch.cuda.synchronize()
    gu = O.gemv(W, odt, xn)
    ref = O.swiglu(gu[:, 0::2], gu[:, 1::2])
    assert np.allclose(a.cpu().numpy(), ref, rtol=1e-4, atol=1e-5)


def test_gemv_rejects_bad_arguments():
    W = torch.zeros((4, 12), dtype=torch.float16, device="cuda")  # 24-byte rows: not 16-byte aligned
    x = torch.zeros((1, 12), device="cuda")
    y = torch.zeros((1, 4), device="cuda")
    with pytest.raises(vsl.VslError) as e:
        vsl.gemv(vsl.F16, W, 4, 12, x, 1, y)
    assert e.value.code == -1
    with pytest.raises(vsl.VslError):
        vsl.gemv(7, W, 4, 12, x, 1, y)


def scatter_pages(cache_dense, page_table, page_size, n_pages):
    """cache_dense [B][n_kv][len][hd] -> paged [n_pages][n_kv][page][hd] using page_table [B][max_pages]."""
    B, nkv, L, hd = cache_dense.shape
    out = np.zeros((n_pages, nkv, page_size, hd), cache_dense.dtype)
    for b in range(B):
        for t in range(L):
            out[page_table[b, t // page_size], :, t % page_size] = cache_dense[b, :, t]
    return out


@pytest.mark.parametrize("hd,kvdt", [(64, vsl.F32), (128, vsl.F16), (64, vsl.F16)])
@pytest.mark.parametrize("nh,nkv", [(4, 4), (8, 2), (8, 1)])
def test_flash_decode_paged_gqa(hd, kvdt, nh, nkv):
    rng = np.random.default_rng(hd + nh + nkv)
    B, page, max_len = 3, 64, 320
    lens = [1, 64, 300]
    max_pages = max_len // page
    n_pages = B * max_pages + 2
    perm = rng.permutation(n_pages)[:B * max_pages].reshape(B, max_pages).astype(np.int32)
    Kd = rng.standard_normal((B, nkv, max_len, hd)).astype(np.float32)
    Vd = rng.standard_normal((B, nkv, max_len, hd)).astype(np.float32)
    if kvdt == vsl.F16:
        Kd, Vd = Kd.astype(np.float16), Vd.astype(np.float16)
    Kp, Vp = scatter_pages(Kd, perm, page, n_pages), scatter_pages(Vd, perm, page, n_pages)
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    pos = np.array([l - 1 for l in lens], np.int32)
    for split in (64, 128):
        ws_bytes = vsl.flash_decode_workspace_size(B, nh, nkv, hd, max_len, split)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
        out = torch.full((B, nh * hd), float("nan"), device="cuda")
        kc = dev(Kp.view(np.uint16) if kvdt == vsl.F16 else Kp)
        vc = dev(Vp.view(np.uint16) if kvdt == vsl.F16 else Vp)
        for rep in range(2):  # the split counters must be left at zero for the next call
            vsl.flash_decode(dev(q), kc, vc, kvdt, dev(perm), max_pages, page, dev(pos), B, nh, nkv, hd, max_len,
                             split, out, ws, ws_bytes, stream=stream())
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            for b in range(B):
                kk = Kd[b].view(np.uint16) if kvdt == vsl.F16 else Kd[b]
                vv = Vd[b].view(np.uint16) if kvdt == vsl.F16 else Vd[b]
                ref = O.attention(q[b], kk, vv, O.F16 if kvdt == vsl.F16 else O.F32, nh, nkv, hd, max_len, lens[b])
                assert np.allclose(got[b], ref, rtol=2e-4, atol=2e-5), (b, split, rep)


@pytest.mark.parametrize("dtype,kvdt", [(vsl.F32, vsl.F32), (vsl.F16, vsl.F16), (vsl.BF16, vsl.F16)])
def test_qkv_rope_kv_append(dtype, kvdt):
    rng = np.random.default_rng(9)
    nh, nkv, hd, K, B = 8, 2, 64, 512, 2
    N = (nh + 2 * nkv) * hd
    W, wf = make_w(rng, N, K, dtype)
    odt = {vsl.F32: O.F32, vsl.F16: O.F16, vsl.BF16: O.BF16}[dtype]
    x = rng.standard_normal((B, K)).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    page, max_pages = 64, 4
    n_pages = B * max_pages
    pt = np.arange(n_pages, dtype=np.int32)[::-1].copy().reshape(B, max_pages)
    pos = np.array([5, 130], np.int32)
    cos, sin = O.rope_table(page * max_pages, hd, 10000.0)
    q = torch.zeros((B, nh * hd), device="cuda")
    tdt = torch.float32 if kvdt == vsl.F32 else torch.float16
    kc = torch.zeros((n_pages, nkv, page, hd), dtype=tdt, device="cuda")
    vc = torch.zeros_like(kc)
    vsl.qkv_rope_append(dtype, dev(W), nh, nkv, hd, K, dev(x), dev(nw), 1e-5, B, dev(pos), dev(cos), dev(sin), q, kc,
                        vc, kvdt, dev(pt), max_pages, page, stream=stream())
    torch.cuda.synchronize()
    xn = O.rmsnorm(x, nw, 1e-5)
    y = O.gemv(W, odt, xn)
    tol = bound(wf, xn)
    qd, kvd = nh * hd, nkv * hd
    for b in range(B):
        p = pos[b]
        qr = O.rope_apply(y[b, :qd], nh, hd, cos[p], sin[p])
        kr = O.rope_apply(y[b, qd:qd + kvd], nkv, hd, cos[p], sin[p])
        vr = y[b, qd + kvd:]
        assert np.all(np.abs(q[b].cpu().numpy() - qr) <= tol[b, :qd] * 2 + 1e-6)
        page_id = pt[b, p // page]
        kg = kc[page_id, :, p % page].float().cpu().numpy().reshape(-1)
        vg = vc[page_id, :, p % page].float().cpu().numpy().reshape(-1)
        if kvdt == vsl.F16:
            kr, vr = kr.astype(np.float16).astype(np.float32), vr.astype(np.float16).astype(np.float32)
            assert np.allclose(kg, kr, rtol=2e-3, atol=1e-4) and np.allclose(vg, vr, rtol=2e-3, atol=1e-4)
        else:
            assert np.all(np.abs(kg - kr) <= tol[b, qd:qd + kvd] * 2 + 1e-6)
            assert np.all(np.abs(vg - vr) <= tol[b, qd + kvd:] + 1e-6)
        # nothing else in the caches was touched
        mask = torch.ones_like(kc, dtype=torch.bool)
        mask[page_id, :, p % page] = False
    written = (kc != 0).sum().item()
    assert written == B * nkv * hd


def test_lm_head_argmax_ties_and_offset():
    rng = np.random.default_rng(11)
    V, K, B = 1000, 256, 3
    W, wf = make_w(rng, V, K, vsl.F16)
    W[700] = W[300]  # identical rows: equal logits, the lower index must win
    W[901] = W[300]
    x = rng.standard_normal((B, K)).astype(np.float32)
    x[1] = wf[300] * 40  # make row 300 (and its copies) the maximum for sequence 1
    nw = np.ones(K, np.float32)
    logits = torch.zeros((B, V), device="cuda")
    slots = torch.zeros(B, dtype=torch.int64, device="cuda")
    vsl.lm_head_sample(vsl.F16, dev(W), V, K, dev(x), dev(nw), 1e-5, B, logits, slots, vocab_offset=5000,
                       stream=stream())
    torch.cuda.synchronize()
    lg = logits.cpu().numpy()
    ref = O.gemv(W, O.F16, O.rmsnorm(x, nw, 1e-5))
    assert np.all(np.abs(lg - ref) <= 1e-4 * np.abs(ref) + 1e-5)
    s = slots.cpu().numpy().view(np.uint64)
    idx = 0xFFFFFFFF - (s & np.uint64(0xFFFFFFFF)).astype(np.int64)
    for b in range(B):
        assert idx[b] == 5000 + O.argmax(lg[b])
    assert idx[1] == 5300


def test_argmax_kernel_first_max():
    v = np.full((2, 5000), -1.0, np.float32)
    v[0, [17, 4000]] = 3.0
    v[1, 4999] = 0.5
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    vsl.argmax(dev(v), 2, 5000, out, stream=stream())
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [17, 4999]


@pytest.mark.parametrize("dtype", [vsl.F32, vsl.F16, vsl.BF16])
def test_synth_fill_bit_exact(dtype):
    n, start = 100003, 77
    tdt = {vsl.F32: torch.float32, vsl.F16: torch.float16, vsl.BF16: torch.bfloat16}[dtype]
    out = torch.zeros(n, dtype=tdt, device="cuda")
    vsl.synth_fill(out, dtype, 42, 256 + 16 * 5 + 6, start, n, 0.02, stream=stream())
    torch.cuda.synchronize()
    ref = O.synth_fill(42, 256 + 16 * 5 + 6, n, 0.02, {vsl.F32: O.F32, vsl.F16: O.F16, vsl.BF16: O.BF16}[dtype],
                       start=start)
    got = out.cpu()
    got = got.view(torch.int32).numpy().view(np.uint32) if dtype == vsl.F32 else got.view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, ref.view(np.uint32) if dtype == vsl.F32 else ref)


def test_embed_gather_clamps_ids():
    rng = np.random.default_rng(12)
    V, d = 50, 72
    E, ef = make_w(rng, V, d, vsl.BF16)
    ids = np.array([0, 49, 50, 1000], np.int32)
    x = torch.zeros((4, d), device="cuda")
    vsl.embed_gather(vsl.BF16, dev(E), V, d, dev(ids), 4, x, stream=stream())
    torch.cuda.synchronize()
    got = x.cpu().numpy()
    for b, i in enumerate(ids):
        assert np.array_equal(got[b], ef[min(i, V - 1)])


def test_rmsnorm_kernel():
    rng = np.random.default_rng(13)
    x = rng.standard_normal((3, 4096)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(4096)).astype(np.float32)
    y = torch.zeros((3, 4096), device="cuda")
    vsl.rmsnorm(dev(x), dev(w), 3, 4096, 1e-5, y, stream=stream())
    torch.cuda.synchronize()
    assert np.allclose(y.cpu().numpy(), O.rmsnorm(x, w, 1e-5), rtol=1e-5, atol=1e-6)
