"""Batched projections on the tcgen05 tensor cores (vsl_skinny_gemm_tc) against an fp64
reference of the same math (fp32 activations, 16-bit weights upcast exactly).

The activations enter the tensor cores as hi + lo 16-bit pairs, so the result differs from
the fp32-activation product by the dropped remainder (|x - hi - lo| <= 2^-22 |x| for fp16,
2^-16 |x| for bf16) plus fp32 accumulation rounding: bound = rel * sum|w||x| + 1e-6 with
rel = 4e-6 (fp16) / 4e-5 (bf16).
"""
import numpy as np
import pytest

import vsl
from vsl import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

REL = {vsl.F16: 4e-6, vsl.BF16: 4e-5}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_w(rng, N, K, dtype, scale=0.05):
    w32 = (rng.standard_normal((N, K)) * scale).astype(np.float32)
    if dtype == vsl.F16:
        h = w32.astype(np.float16)
        return h.view(np.uint16), h.astype(np.float32)
    b = synth.f32_to_bf16_bits(w32).reshape(N, K)
    return b, synth.bf16_bits_to_f32(b).reshape(N, K)


_keep = []


def workspace(N, K, B):
    """Zeroed device workspace, 1 KB aligned (returned as a raw pointer; the tensor is kept)."""
    n = vsl.skinny_gemm_tc_workspace_size(N, K, B)
    t = torch.zeros(n // 4 + 512, dtype=torch.int32, device="cuda")
    _keep.append(t)
    return (t.data_ptr() + 1023) // 1024 * 1024, n


def run(dtype, N, K, B, epi, norm=False, seed=0):
    rng = np.random.default_rng(seed)
    wbits, wf = make_w(rng, N, K, dtype)
    x = rng.standard_normal((B, K)).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32) if norm else None
    xr = x.astype(np.float64)
    if norm:
        xr = np.stack([(x[b] / np.sqrt(np.mean(x[b].astype(np.float64) ** 2) + 1e-5)) * nw for b in range(B)])
    acc = xr @ wf.T.astype(np.float64)
    tol = REL[dtype] * (np.abs(xr) @ np.abs(wf).T.astype(np.float64)) + 1e-6
    if epi == vsl.EPI_SWIGLU:
        g, u = acc[:, 0::2], acc[:, 1::2]
        ref = g / (1.0 + np.exp(-g)) * u
        y0 = np.zeros((B, N // 2), np.float32)
        tol = (tol[:, 0::2] + tol[:, 1::2]) * (1.0 + np.abs(u) + np.abs(g))
    elif epi == vsl.EPI_ADD:
        y0 = rng.standard_normal((B, N)).astype(np.float32)
        ref = y0.astype(np.float64) + acc
    else:
        y0 = np.zeros((B, N), np.float32)
        ref = acc
    W, X, Y = dev(wbits), dev(x), dev(y0)
    NW = dev(nw) if norm else None
    ws, nbytes = workspace(N, K, B)
    vsl.skinny_gemm_tc(dtype, W, N, K, X, B, Y, epi, NW, 1e-5, ws, nbytes)
    torch.cuda.synchronize()
    out = Y.cpu().numpy().astype(np.float64)
    err = np.abs(out - ref)
    assert np.all(err <= tol), (float(err.max()), float((err / tol).max()))
    # the kernel leaves its arrival counters at zero: a second call gives identical results
    Y2 = dev(y0)
    vsl.skinny_gemm_tc(dtype, W, N, K, X, B, Y2, epi, NW, 1e-5, ws, nbytes)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)
    return out


@pytest.mark.parametrize("dtype", [vsl.F16, vsl.BF16])
@pytest.mark.parametrize("N,K", [(128, 64), (4096, 4096), (11008, 4096), (4096, 11008), (333, 1376)])
@pytest.mark.parametrize("B", [5, 8, 16, 64, 100, 128])
def test_tc_store(dtype, N, K, B):
    run(dtype, N, K, B, vsl.EPI_STORE)


@pytest.mark.parametrize("B", [6, 17, 40])
def test_tc_add_and_norm(B):
    run(vsl.F16, 1000, 4096, B, vsl.EPI_ADD, seed=3)
    run(vsl.BF16, 2048, 2048, B, vsl.EPI_STORE, norm=True, seed=4)


@pytest.mark.parametrize("dtype", [vsl.F16, vsl.BF16])
def test_tc_swiglu(dtype):
    run(dtype, 2 * 1376, 1024, 12, vsl.EPI_SWIGLU, norm=True, seed=5)


def test_tc_matches_gemv_chunks():
    """Same projection through the GEMV (4-row chunks) and the tensor cores."""
    rng = np.random.default_rng(9)
    N, K, B = 4096, 4096, 16
    wbits, _ = make_w(rng, N, K, vsl.BF16)
    x = rng.standard_normal((B, K)).astype(np.float32)
    W, X = dev(wbits), dev(x)
    Y1 = torch.zeros(B, N, device="cuda")
    Y2 = torch.zeros(B, N, device="cuda")
    vsl.gemv(vsl.BF16, W, N, K, X, B, Y1)
    ws, nbytes = workspace(N, K, B)
    vsl.skinny_gemm_tc(vsl.BF16, W, N, K, X, B, Y2, vsl.EPI_STORE, None, 0.0, ws, nbytes)
    torch.cuda.synchronize()
    scale = (X.abs().double() @ W.view(torch.bfloat16).abs().double().T).float()
    assert torch.all((Y1 - Y2).abs() <= 8e-5 * scale + 1e-6)


def test_tc_shared_workspace_across_shapes():
    """One workspace (sized for the largest N and K) serves projections of different shapes in
    turn, as in a decode step; each keeps matching its fp64 reference."""
    rng = np.random.default_rng(11)
    shapes = [(6144, 1024), (1024, 4096), (8192, 1024), (1024, 2816)]
    B = 16
    n = vsl.skinny_gemm_tc_workspace_size(max(s[0] for s in shapes), max(s[1] for s in shapes), B)
    t = torch.zeros(n // 4 + 512, dtype=torch.int32, device="cuda")
    ws = (t.data_ptr() + 1023) // 1024 * 1024
    for rep in range(3):
        for N, K in shapes:
            wbits, wf = make_w(rng, N, K, vsl.F16)
            x = rng.standard_normal((B, K)).astype(np.float32)
            Y = torch.zeros(B, N, device="cuda")
            vsl.skinny_gemm_tc(vsl.F16, dev(wbits), N, K, dev(x), B, Y, vsl.EPI_STORE, None, 0.0, ws, n)
            torch.cuda.synchronize()
            ref = x.astype(np.float64) @ wf.T.astype(np.float64)
            tol = REL[vsl.F16] * (np.abs(x).astype(np.float64) @ np.abs(wf).T.astype(np.float64)) + 1e-6
            assert np.all(np.abs(Y.cpu().numpy() - ref) <= tol), (rep, N, K)


def test_tc_rejects_bad_shapes():
    ws, nbytes = workspace(4096, 4096, 8)
    W = torch.zeros(4096 * 4096, dtype=torch.float16, device="cuda")
    X = torch.zeros(8 * 4096, device="cuda")
    Y = torch.zeros(8 * 4096, device="cuda")
    with pytest.raises(vsl.VslError):
        vsl.skinny_gemm_tc(vsl.F16, W, 4096, 4096, X, 129, Y, vsl.EPI_STORE, None, 0.0, ws, nbytes)
    with pytest.raises(vsl.VslError):
        vsl.skinny_gemm_tc(vsl.F32, W, 4096, 4096, X, 8, Y, vsl.EPI_STORE, None, 0.0, ws, nbytes)
    with pytest.raises(vsl.VslError):
        vsl.skinny_gemm_tc(vsl.F16, W, 4096, 4096, X, 8, Y, vsl.EPI_STORE, None, 0.0, ws, 1024)
