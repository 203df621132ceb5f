"""The long-context sparse attention mask, without a GPU: the oracle's window start
(orc_sparse_first) against a literal transcription of the reference shader's index arithmetic,
and the oracle's masked attention against float64 NumPy.

Reference: vk_symbiote/shaders/sparse_attention.comp:77-131 (get_attention_window and the block
clamp of compute_ring_attention), dispatched when use_sparse_attention && seq_len > 8192
(vk_symbiote/src/VulkanSymbioteEngine.cpp:788); defaults window 512, 16 global tokens, block 1024
(vk_symbiote/include/vk_symbiote/Common.h:71-74). A decode query at position pos sees a sequence
of pos + 1 tokens with the cache in use.
"""
import numpy as np
import pytest

import oracle as O


def shader_window(pos, seq_len, window, global_tokens, block):
    """The shader's arithmetic, statement by statement (use_cache and use_sparse true)."""
    # get_attention_window
    global_end = global_tokens
    window_start = pos - window if pos > window else 0
    window_end = min(pos + window + 1, seq_len)
    if pos < global_end:
        start, end = 0, seq_len
    else:
        start, end = min(global_end, window_start), window_end
    # compute_ring_attention
    current_block = pos // block
    block_start = current_block * block
    block_end = min(block_start + block, seq_len)
    attend_start = max(start, block_start - window if block_start > window else 0)
    attend_end = min(end, block_end)
    return attend_start, attend_end


@pytest.mark.parametrize("min_len,window,global_tokens,block", [(8192, 512, 16, 1024), (100, 40, 4, 128),
                                                                (64, 64, 16, 64), (1, 7, 3, 10)])
def test_window_start_matches_the_shader(min_len, window, global_tokens, block):
    rng = np.random.default_rng(min_len)
    positions = list(range(0, 3 * block + 2 * window + 40)) + rng.integers(0, 40000, 400).tolist()
    for pos in positions:
        got = O.sparse_first(min_len, window, global_tokens, block, pos)
        if pos + 1 <= min_len:
            assert got == 0  # dense below the switch (seq_len > min_len)
            continue
        s, e = shader_window(pos, pos + 1, window, global_tokens, block)
        assert e == pos + 1 and got == s, (pos, got, s, e)
    assert O.sparse_first(0, window, global_tokens, block, 50000) == 0  # min_len 0: dense


def test_default_window_shape():
    # past the switch: one contiguous range from 512 before the query's 1024-block to the query
    for pos in (8192, 9000, 9215, 9216, 20000, 131071):
        assert O.sparse_first(8192, 512, 16, 1024, pos) == (pos // 1024) * 1024 - 512
    assert O.sparse_first(8192, 512, 16, 1024, 8191) == 0


def test_masked_attention_matches_float64():
    rng = np.random.default_rng(3)
    n_heads, n_kv, hd, max_seq, length = 8, 2, 64, 300, 257
    K = rng.standard_normal((n_kv, max_seq, hd)).astype(np.float32)
    V = rng.standard_normal((n_kv, max_seq, hd)).astype(np.float32)
    q = rng.standard_normal(n_heads * hd).astype(np.float32)
    for first in (0, 1, 63, 64, 200, 256):
        got = O.attention(q, K, V, O.F32, n_heads, n_kv, hd, max_seq, length, first=first)
        for h in range(n_heads):
            g = h * n_kv // n_heads
            s = (K[g, first:length].astype(np.float64) @ q[h * hd:(h + 1) * hd]) / np.sqrt(hd)
            p = np.exp(s - s.max())
            p /= p.sum()
            ref = p @ V[g, first:length].astype(np.float64)
            assert np.allclose(got[h * hd:(h + 1) * hd], ref, rtol=1e-4, atol=1e-5), (first, h)


def test_oracle_model_sparse_switch():
    """Below min_len the sparse model equals the dense one bit for bit; past it, it differs."""
    kw = dict(n_layers=1, d=256, n_heads=4, n_kv=2, ffn=512, vocab=500, wdtype=O.F32, kvdtype=O.F32, max_seq=160,
              seed=4)
    dense, sparse = O.Model.synthetic(**kw), O.Model.synthetic(**kw)
    sparse.set_sparse(min_len=100, window=40, global_tokens=4, block=64)
    dense.fill_kv_synthetic(9, 1.0, 120, 1)
    sparse.fill_kv_synthetic(9, 1.0, 120, 1)
    _, a = dense.step([7], [98])
    _, b = sparse.step([7], [98])
    assert np.array_equal(a, b)  # 99 positions: dense
    _, a = dense.step([7], [130])
    _, b = sparse.step([7], [130])
    assert not np.array_equal(a, b)
    dense.close()
    sparse.close()
