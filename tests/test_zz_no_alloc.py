"""The allocation-free attention entry point, vsl_flash_decode_noalloc.

It serves callers that must not have the library allocate device memory (hosts that own
every device byte through their own pool, or loops that cannot take an allocation's
synchronisation): its split-K scratch lives in a fixed device array inside libvsl.so.
This test calls it through the C ABI twice in a row and checks each result against the
allocating entry point, vsl_flash_decode, with a caller-owned workspace, at the same
tolerance the other attention tests use. The shape uses 11 splits per sequence, so the
partial results and split counters really live in the scratch, and the second call starts
from whatever the first one left there. It also checks the size limit.
"""
import ctypes as C

import numpy as np
import pytest

import vsl

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

RTOL, ATOL = 2e-4, 2e-5


def _noalloc():
    fn = vsl.lib().vsl_flash_decode_noalloc
    vp, i32 = C.c_void_p, C.c_int
    fn.restype = i32
    fn.argtypes = [vp, vp, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, i32, vp, vp]
    return fn


def _paged(rng, B, nkv, hd, max_len, page):
    max_pages = max_len // page
    n_pages = B * max_pages + 3
    table = rng.permutation(n_pages)[:B * max_pages].reshape(B, max_pages).astype(np.int32)
    K = np.zeros((n_pages, nkv, page, hd), np.float16)
    V = np.zeros_like(K)
    dense_k = rng.standard_normal((B, nkv, max_len, hd)).astype(np.float16)
    dense_v = rng.standard_normal((B, nkv, max_len, hd)).astype(np.float16)
    for b in range(B):
        for t in range(max_len):
            K[table[b, t // page], :, t % page] = dense_k[b, :, t]
            V[table[b, t // page], :, t % page] = dense_v[b, :, t]
    return table, max_pages, K, V


def test_noalloc_matches_allocating_entry_point_twice():
    rng = np.random.default_rng(2024)
    B, nh, nkv, hd, page, max_len, split = 3, 8, 2, 128, 64, 704, 64  # 11 splits per sequence
    table, max_pages, K, V = _paged(rng, B, nkv, hd, max_len, page)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    kc, vc, pt = dev(K.view(np.uint16)), dev(V.view(np.uint16)), dev(table)
    pos = dev(np.array([700, 64, 390], np.int32))
    st = torch.cuda.current_stream().cuda_stream
    fn = _noalloc()
    ws_bytes = vsl.flash_decode_workspace_size(B, nh, nkv, hd, max_len, split)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    for call in range(2):
        q = dev(rng.standard_normal((B, nh * hd)).astype(np.float32))
        ref = torch.full((B, nh * hd), float("nan"), device="cuda")
        vsl.flash_decode(q, kc, vc, vsl.F16, pt, max_pages, page, pos, B, nh, nkv, hd, max_len, split, ref, ws,
                         ws_bytes, stream=st)
        out = torch.full((B, nh * hd), float("nan"), device="cuda")
        rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), vsl.F16, pt.data_ptr(), max_pages, page, pos.data_ptr(),
                B, nh, nkv, hd, max_len, split, out.data_ptr(), st)
        assert rc == 0, vsl.lib().vsl_last_error_string()
        torch.cuda.synchronize()
        o, r = out.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(o).all(), call
        assert np.allclose(o, r, rtol=RTOL, atol=ATOL), (call, float(np.abs(o - r).max()))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    fn = _noalloc()
    # 64 sequences x 64 heads x 128 splits of 128-wide heads need far more than 4 MiB
    rc = fn(16, 16, 16, vsl.F16, 16, 128, 64, 16, 64, 64, 8, 128, 8192, 64, 16, None)
    assert rc == -9
    assert b"static scratch" in vsl.lib().vsl_last_error_string()
