"""Seeded synthetic tensors and token ids.

One definition, three implementations that agree bit for bit: this NumPy module (used to
write GGUF fixtures), the device initialiser in csrc/kernels/misc.cu (used to fill HBM
directly for models too large to ship as files) and the CPU oracle.

Element i of tensor `tid` under `seed`:
    base = splitmix64(seed ^ (tid * 0xD1B54A32D192ED03))
    h    = splitmix64(base + i)
    s    = sum of the four 16-bit lanes of h - 131070          (exact integer)
    w    = float32(s) * float32(sqrt(3) * sigma / 65536)      (one IEEE fp32 multiply)
then rounded to the tensor dtype (round-to-nearest-even). The sum of four uniform lanes is
the Irwin-Hall(4) distribution: mean 0, standard deviation `sigma`, close to normal.

Tensor ids: token_embd 1, output 2; per layer l and kind k (attn_norm 0, q 1, k 2, v 3,
output 4, ffn_norm 5, gate 6, up 7, down 8): 256 + 16 l + k; KV prefill 0x40000000 + 2 l +
(0 for K, 1 for V); prompt stream s: 0xFFFF0000 + s. Norm weights are 1.0.

Block-quantized tensors (GGUF Q8_0 / Q4_0 / Q4_1, blocks of 32 along a row of `cols`) are
defined in quantized form: element gi = r * cols + c has quant h(gi) % 255 - 127 (Q8_0), nibble
1 + h(gi) % 15 with value nibble - 8 (Q4_0; both symmetric around zero) or nibble h(gi) % 16
(Q4_1); block gb = r * (cols / 32) + c / 32 has the fp16 scale d = round(m * k),
m = 49152 + (h'(gb) & 0x7fff) with h' the stream of tensor id (tid ^ 0x5CA1E5) and
k = float32(sigma / std(quant) / 65536); value = quant * d in fp32, and for Q4_1 the block's fp16
minimum is round(-7.5 * d) and value = nibble * d + minimum (fp32 multiply, then fp32 add).
"""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1
GOLDEN = np.uint64(0x9E3779B97F4A7C15)
MUL1 = np.uint64(0xBF58476D1CE4E5B9)
MUL2 = np.uint64(0x94D049BB133111EB)
TID_MUL = 0xD1B54A32D192ED03
SQRT3 = 1.7320508075688772

TID_TOK_EMBD, TID_OUTPUT, TID_OUTPUT_NORM = 1, 2, 3
K_ATTN_NORM, K_Q, K_K, K_V, K_O, K_FFN_NORM, K_GATE, K_UP, K_DOWN = range(9)

GGML_F32, GGML_F16, GGML_BF16 = 0, 1, 30
GGML_Q4_0, GGML_Q4_1, GGML_Q8_0 = 2, 3, 8
# std of U{-127..127}, U{-7..7}, U{0..15}
Q_STD = {GGML_Q8_0: 73.6115932, GGML_Q4_0: 4.3204938, GGML_Q4_1: 4.6097722}
Q_BLOCK_BYTES = {GGML_Q8_0: 34, GGML_Q4_0: 18, GGML_Q4_1: 20}


def tid_layer(layer: int, kind: int) -> int:
    return 256 + 16 * layer + kind


def tid_kv(layer: int, is_v: int) -> int:
    return 0x40000000 + 2 * layer + is_v


def _smix_scalar(z: int) -> int:
    z = (z + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def _smix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z + GOLDEN
        z = (z ^ (z >> np.uint64(30))) * MUL1
        z = (z ^ (z >> np.uint64(27))) * MUL2
        return z ^ (z >> np.uint64(31))


def tensor_base(seed: int, tid: int) -> int:
    return _smix_scalar((seed ^ ((tid * TID_MUL) & M64)) & M64)


def scale(sigma: float) -> np.float32:
    return np.float32(SQRT3 * sigma / 65536.0)


def synth_f32(seed: int, tid: int, n: int, sigma: float = 0.02, start: int = 0,
              chunk: int = 1 << 22) -> np.ndarray:
    """fp32 values of elements [start, start+n) of tensor `tid`."""
    out = np.empty(n, dtype=np.float32)
    base = np.uint64(tensor_base(seed, tid))
    c = scale(sigma)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        idx = np.arange(start + s, start + e, dtype=np.uint64)
        with np.errstate(over="ignore"):
            h = _smix(idx + base)
        mask = np.uint64(0xFFFF)
        lanes = ((h & mask).astype(np.int64) + ((h >> np.uint64(16)) & mask).astype(np.int64)
                 + ((h >> np.uint64(32)) & mask).astype(np.int64) + (h >> np.uint64(48)).astype(np.int64)
                 - 131070)
        out[s:e] = lanes.astype(np.float32) * c
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (b & np.uint64(0x7FFFFFFF)) > np.uint64(0x7F800000)
    r = (b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    r = np.where(nan, (b >> np.uint64(16)) | np.uint64(0x40), r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def synth_tensor(seed: int, tid: int, shape: tuple[int, ...], dtype: int, sigma: float = 0.02) -> np.ndarray:
    """Tensor in its storage form: float32, float16, or uint16 bf16 bits."""
    n = int(np.prod(shape))
    v = synth_f32(seed, tid, n, sigma)
    if dtype == GGML_F16:
        v = v.astype(np.float16)  # NumPy's fp32->fp16 cast is round-to-nearest-even
    elif dtype == GGML_BF16:
        v = f32_to_bf16_bits(v)
    elif dtype != GGML_F32:
        raise ValueError(f"unsupported dtype {dtype}")
    return v.reshape(shape)


def synth_q_blocks(seed: int, tid: int, rows: int, cols: int, dtype: int, sigma: float = 0.02) -> np.ndarray:
    """GGUF block bytes [rows][cols / 32 * block bytes] of a seeded Q8_0 / Q4_0 / Q4_1 tensor
    (ggml layout: fp16 scale, for Q4_1 an fp16 minimum, then 32 int8 quants or 16 bytes holding
    elements i (low nibble) and i + 16 (high nibble))."""
    assert cols % 32 == 0 and dtype in Q_STD
    nb = cols // 32
    base = np.uint64(tensor_base(seed, tid))
    sbase = np.uint64(tensor_base(seed, tid ^ 0x5CA1E5))
    with np.errstate(over="ignore"):
        h = _smix(np.arange(rows * cols, dtype=np.uint64) + base).reshape(rows, nb, 32)
        hs = _smix(np.arange(rows * nb, dtype=np.uint64) + sbase).reshape(rows, nb)
    m = (np.uint64(49152) + (hs & np.uint64(0x7FFF))).astype(np.float32)
    d16 = (m * np.float32(sigma / Q_STD[dtype] / 65536.0)).astype(np.float16)
    bb = Q_BLOCK_BYTES[dtype]
    blk = np.empty((rows, nb, bb), np.uint8)
    blk[..., :2] = d16.view(np.uint8).reshape(rows, nb, 2)
    if dtype == GGML_Q8_0:
        blk[..., 2:] = ((h % np.uint64(255)).astype(np.int16) - 127).astype(np.int8).view(np.uint8)
    elif dtype == GGML_Q4_1:
        m16 = (d16.astype(np.float32) * np.float32(-7.5)).astype(np.float16)
        blk[..., 2:4] = m16.view(np.uint8).reshape(rows, nb, 2)
        n = (h % np.uint64(16)).astype(np.uint8)
        blk[..., 4:] = n[..., :16] | (n[..., 16:] << np.uint8(4))
    else:
        n = (np.uint64(1) + h % np.uint64(15)).astype(np.uint8)
        blk[..., 2:] = n[..., :16] | (n[..., 16:] << np.uint8(4))
    return blk.reshape(rows, nb * bb)


def dequant_q_blocks(blocks: np.ndarray, dtype: int, cols: int, legacy_q4: bool = False) -> np.ndarray:
    """fp32 values [rows][cols] of GGUF Q8_0 / Q4_0 / Q4_1 rows: quant * fp16 scale, one fp32
    multiply (Q4_1: then + fp16 minimum, one fp32 add; the reference's dequantize_tensor).
    legacy_q4 reads Q4_x byte i as elements 2i (low nibble) and 2i + 1 (high), the reference
    loader's order; otherwise ggml's i and i + 16."""
    bb = Q_BLOCK_BYTES[dtype]
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, cols // 32, bb)
    d = b[..., :2].copy().view(np.float16).astype(np.float32)  # [rows][nb][1]
    if dtype == GGML_Q8_0:
        q = b[..., 2:].view(np.int8).astype(np.float32)
        return (q * d).reshape(-1, cols)
    hb = 4 if dtype == GGML_Q4_1 else 2
    zp = 0 if dtype == GGML_Q4_1 else 8
    lo = (b[..., hb:] & 15).astype(np.int16) - zp
    hi = (b[..., hb:] >> 4).astype(np.int16) - zp
    q = (np.stack([lo, hi], -1).reshape(lo.shape[:-1] + (32,)) if legacy_q4
         else np.concatenate([lo, hi], -1)).astype(np.float32)
    v = (q * d).astype(np.float32)
    if dtype == GGML_Q4_1:
        v = v + b[..., 2:4].copy().view(np.float16).astype(np.float32)
    return v.reshape(-1, cols)


def synth_ids(seed: int, stream: int, n: int, vocab: int) -> np.ndarray:
    """Prompt ids uniform in [0, vocab): splitmix64 draw modulo vocab."""
    base = np.uint64(tensor_base(seed, 0xFFFF0000 + stream))
    idx = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = _smix(idx + base)
    return (h % np.uint64(vocab)).astype(np.int32)
