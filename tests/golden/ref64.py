"""Independent float64 NumPy restatement of the Llama decode step.

Second witness for the CPU oracle (test infrastructure only). It follows the same reference
conventions as the oracle -- embedding clamp (embedding_lookup.comp:32), RMSNorm
x / sqrt(mean(x^2)+eps) * w (rms_norm.comp:24-34), adjacent-pair RoPE with
f = theta^(-2i/hd) (Utils.cpp:101-110), GQA group h*kv/heads (attention.comp:92), scaled
max-subtracted softmax (attention.comp:116-189), silu(g)*u (feed_forward.comp:21,49-61),
first-max argmax (VulkanSymbioteEngine.cpp:1794-1804) -- but evaluates everything in
float64 with NumPy's own reductions, so it shares no arithmetic code with the oracle.
"""
from __future__ import annotations

import numpy as np


class Ref64:
    def __init__(self, shape, tensors: dict[str, np.ndarray], max_seq: int = 512, kv_round=None):
        """tensors: name -> float64 array [rows, cols] (GGUF row-major) or [n] for norms.
        kv_round: optional callable applied to K/V before caching (e.g. fp16 rounding)."""
        self.s = shape
        self.t = tensors
        self.max_seq = max_seq
        self.kv_round = kv_round
        hd = shape.head_dim
        self.K = np.zeros((shape.n_layers, shape.n_kv_heads, max_seq, hd))
        self.V = np.zeros_like(self.K)
        half = hd // 2
        i = np.arange(half, dtype=np.float64)
        freq = np.power(float(np.float32(shape.rope_theta)), -(2.0 * i) / hd)
        ang = np.arange(max_seq, dtype=np.float64)[:, None] * freq[None, :]
        self.cos, self.sin = np.cos(ang), np.sin(ang)

    def _norm(self, x, w):
        return x / np.sqrt(np.mean(x * x) + float(np.float32(self.s.rms_eps))) * w

    def _rope(self, v, pos):
        hd = self.s.head_dim
        v = v.reshape(-1, hd // 2, 2)
        a, b = v[..., 0].copy(), v[..., 1].copy()
        c, s = self.cos[pos], self.sin[pos]
        v[..., 0] = a * c - b * s
        v[..., 1] = a * s + b * c
        return v.reshape(-1)

    def step(self, tok: int, pos: int) -> np.ndarray:
        s, t = self.s, self.t
        hd = s.head_dim
        x = t["token_embd.weight"][min(tok, s.vocab - 1)].copy()
        for l in range(s.n_layers):
            p = f"blk.{l}."
            n = self._norm(x, t[p + "attn_norm.weight"])
            q = t[p + "attn_q.weight"] @ n
            k = t[p + "attn_k.weight"] @ n
            v = t[p + "attn_v.weight"] @ n
            q, k = self._rope(q, pos), self._rope(k, pos)
            k, v = k.reshape(s.n_kv_heads, hd), v.reshape(s.n_kv_heads, hd)
            if self.kv_round is not None:
                k, v = self.kv_round(k), self.kv_round(v)
            self.K[l, :, pos], self.V[l, :, pos] = k, v
            o = np.empty(s.n_heads * hd)
            for h in range(s.n_heads):
                g = h * s.n_kv_heads // s.n_heads
                sc = self.K[l, g, :pos + 1] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
                pr = np.exp(sc - sc.max())
                pr /= pr.sum()
                o[h * hd:(h + 1) * hd] = pr @ self.V[l, g, :pos + 1]
            x = x + t[p + "attn_output.weight"] @ o
            m = self._norm(x, t[p + "ffn_norm.weight"])
            gt = t[p + "ffn_gate.weight"] @ m
            up = t[p + "ffn_up.weight"] @ m
            a = gt / (1.0 + np.exp(-gt)) * up
            x = x + t[p + "ffn_down.weight"] @ a
        x = self._norm(x, t["output_norm.weight"])
        return t["output.weight"] @ x

    def greedy(self, prompt, n_new):
        pos = 0
        lg = None
        for tok in prompt:
            lg = self.step(int(tok), pos)
            pos += 1
        ids, logits = [], []
        for i in range(n_new):
            nxt = int(np.argmax(lg))  # NumPy argmax returns the first maximum
            ids.append(nxt)
            logits.append(lg)
            if i + 1 < n_new:
                lg = self.step(nxt, pos)
                pos += 1
        return ids, logits


def load_tensors_f64(path: str) -> dict[str, np.ndarray]:
    """Read every F32/F16/BF16/Q8_0/Q4_0/Q4_1 tensor of a GGUF as float64 (rows = ne[1], cols = ne[0])."""
    import os
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "..", "vulkan-symbiote-loader_b200"))
    from vsl import gguf, synth
    _meta, infos = gguf.read_gguf(path)
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, (gt, ne, off) in infos.items():
        n = int(np.prod(ne))
        if gt == synth.GGML_F32:
            a = np.frombuffer(mm, dtype=np.float32, count=n, offset=off).astype(np.float64)
        elif gt == synth.GGML_F16:
            a = np.frombuffer(mm, dtype=np.float16, count=n, offset=off).astype(np.float64)
        elif gt == synth.GGML_BF16:
            a = synth.bf16_bits_to_f32(np.frombuffer(mm, dtype=np.uint16, count=n, offset=off)).astype(np.float64)
        elif gt in synth.Q_STD:  # Q8_0 / Q4_0 / Q4_1 blocks, dequantized as the reference loader does
            nbytes = n // 32 * synth.Q_BLOCK_BYTES[gt]
            a = synth.dequant_q_blocks(np.frombuffer(mm, dtype=np.uint8, count=nbytes, offset=off), gt,
                                       int(ne[0])).astype(np.float64).reshape(-1)
        else:
            continue
        out[name] = a.reshape(list(reversed(ne))) if len(ne) > 1 else a
    return out
