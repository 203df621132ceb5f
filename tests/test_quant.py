"""Block-quantized weights (GGUF Q8_0 / Q4_0 / Q4_1) without a GPU: the oracle's dequantisation
against an independent NumPy restatement of the reference loader (GGUFLoader.cpp:1150-1207) and hand-
computed known answers, the seeded quantized tensors in NumPy vs C, the C-ABI repack into the
device row layout, GGUF parsing, and the oracle's greedy ids against the float64 goldens."""
import numpy as np
import pytest

import oracle as O
import vsl
from vsl import gguf, synth


def _random_blocks(rng, dtype, rows, cols):
    nb = cols // 32
    bb = synth.Q_BLOCK_BYTES[dtype]
    b = rng.integers(0, 256, size=(rows, nb, bb), dtype=np.uint8)
    d = (rng.standard_normal((rows, nb)) * 0.01).astype(np.float16)  # finite scales
    b[..., :2] = d.view(np.uint8).reshape(rows, nb, 2)
    if dtype == synth.GGML_Q4_1:  # finite minimums
        m = (rng.standard_normal((rows, nb)) * 0.05).astype(np.float16)
        b[..., 2:4] = m.view(np.uint8).reshape(rows, nb, 2)
    return b.reshape(rows, nb * bb)


@pytest.mark.parametrize("dtype", [O.Q8_0, O.Q4_0, O.Q4_1])
@pytest.mark.parametrize("legacy", [0, 1])
def test_oracle_dequant_matches_numpy_restatement(dtype, legacy):
    if dtype == O.Q8_0 and legacy:
        pytest.skip("the nibble order concerns Q4_0 / Q4_1 only")
    rng = np.random.default_rng(7)
    blocks = _random_blocks(rng, dtype, 5, 96)
    ref = synth.dequant_q_blocks(blocks, dtype, 96, legacy_q4=bool(legacy)).reshape(-1)
    got = O.dequant_blocks(dtype, blocks, 5 * 96, legacy)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_known_answers():
    # Q8_0: d = 0.5 (fp16 0x3800), quants -3, 0, 127, -127, then zeros
    b8 = np.zeros(34, np.uint8)
    b8[0], b8[1] = 0x00, 0x38
    b8[2:6] = np.array([-3, 0, 127, -127], np.int8).view(np.uint8)
    v = O.dequant_blocks(O.Q8_0, b8, 32)
    assert v[:4].tolist() == [-1.5, 0.0, 63.5, -63.5] and not v[4:].any()
    # Q4_0: d = 2.0 (fp16 0x4000), byte 0 = 0xF1 (low 1, high 15), other bytes 0x88 (zeros)
    b4 = np.full(18, 0x88, np.uint8)
    b4[0], b4[1], b4[2] = 0x00, 0x40, 0xF1
    ggml = O.dequant_blocks(O.Q4_0, b4, 32, 0)  # element 0 = (1-8)*2, element 16 = (15-8)*2
    assert ggml[0] == -14.0 and ggml[16] == 14.0 and np.count_nonzero(ggml) == 2
    legacy = O.dequant_blocks(O.Q4_0, b4, 32, 1)  # reference loader order: elements 0 and 1
    assert legacy[0] == -14.0 and legacy[1] == 14.0 and np.count_nonzero(legacy) == 2
    # Q4_1: d = 2.0, m = -1.0 (fp16 0xBC00), byte 0 = 0xF1 (low 1, high 15), other nibbles 0
    b41 = np.zeros(20, np.uint8)
    b41[0], b41[1], b41[2], b41[3], b41[4] = 0x00, 0x40, 0x00, 0xBC, 0xF1
    ggml = O.dequant_blocks(O.Q4_1, b41, 32, 0)  # element 0 = 1*2 - 1, element 16 = 15*2 - 1
    assert ggml[0] == 1.0 and ggml[16] == 29.0 and (np.delete(ggml, [0, 16]) == -1.0).all()
    legacy = O.dequant_blocks(O.Q4_1, b41, 32, 1)
    assert legacy[0] == 1.0 and legacy[1] == 29.0 and (legacy[2:] == -1.0).all()


def test_dequant_negative_subnormal_scale_keeps_its_sign():
    """Block scales are IEEE fp16, read with their sign also when subnormal. The reference loader's
    dequantisation helper returns +mantissa * 2^-24 for every subnormal half, dropping the sign
    (vk_symbiote/src/GGUFLoader.cpp:1136-1137), so a block whose scale is a negative subnormal would
    come out negated there; the engine and this oracle follow the format (the two agree on every
    scale that is normal, zero or positive)."""
    b8 = np.zeros(34, np.uint8)
    b8[0], b8[1] = 0x03, 0x80  # fp16 0x8003 = -3 * 2^-24
    b8[2:5] = np.array([2, -5, 127], np.int8).view(np.uint8)
    v = O.dequant_blocks(O.Q8_0, b8, 32)
    d = -3.0 * 2.0 ** -24
    assert v[:3].tolist() == [2 * d, -5 * d, 127 * d] and not v[3:].any()
    reference_reading = 3.0 * 2.0 ** -24  # what GGUFLoader.cpp:1137 would use as the scale
    assert v[0] == -2 * reference_reading
    # Q4_0 with a negative subnormal scale: element 0 = (1 - 8) * d > 0
    b4 = np.full(18, 0x88, np.uint8)
    b4[0], b4[1], b4[2] = 0x01, 0x80, 0x81  # fp16 0x8001 = -2^-24; byte 0: low nibble 1, high 8
    v4 = O.dequant_blocks(O.Q4_0, b4, 32, 0)
    assert v4[0] == 7.0 * 2.0 ** -24 and np.count_nonzero(v4) == 1


@pytest.mark.parametrize("dtype", [O.Q8_0, O.Q4_0, O.Q4_1])
def test_seeded_quantized_tensor_numpy_equals_c(dtype):
    rows, cols, seed, tid = 7, 160, 11, synth.tid_layer(1, synth.K_GATE)
    blocks = synth.synth_q_blocks(seed, tid, rows, cols, dtype)
    ref = synth.dequant_q_blocks(blocks, dtype, cols)
    got = O.synthq_dequant(seed, tid, rows, cols, dtype)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert abs(float(ref.std()) - 0.02) < 0.004 and abs(float(ref.mean())) < 0.003


@pytest.mark.parametrize("dtype", [vsl.Q8_0, vsl.Q4_0, vsl.Q4_1])
@pytest.mark.parametrize("legacy", [False, True])
def test_repack_into_device_layout(dtype, legacy):
    rng = np.random.default_rng(3)
    rows, cols = 6, 4 * 32 + 64
    blocks = _random_blocks(rng, dtype, rows, cols)
    n_scale_parts = 2 if dtype == vsl.Q4_1 else 1  # Q4_1: scales, then minimums
    assert vsl.weight_row_bytes(dtype, cols) == ((cols if dtype == vsl.Q8_0 else cols // 2)
                                                 + n_scale_parts * 16 * -(-cols // 256))
    # a row-and-column slice (tensor-parallel shard): rows 1..4, columns 64..191
    out = vsl.repack_gguf_rows(dtype, blocks, rows, cols, legacy, row0=1, nrows=4, col0=64, ncols=128)
    want = synth.dequant_q_blocks(blocks, dtype, cols, legacy_q4=legacy)[1:5, 64:192]
    qb = 128 if dtype == vsl.Q8_0 else 64
    d = out[:, qb:qb + 8].copy().view(np.float16).astype(np.float32)  # 4 scales per row
    if dtype == vsl.Q8_0:
        q = out[:, :qb].view(np.int8).astype(np.float32).reshape(4, 4, 32)
    else:  # device order: byte i of a block = element i (low) | element i + 16 (high)
        zp = 0 if dtype == vsl.Q4_1 else 8
        raw = out[:, :qb].reshape(4, 4, 16)
        q = np.concatenate([(raw & 15).astype(np.float32) - zp, (raw >> 4).astype(np.float32) - zp], -1)
    got = (q * d[..., None]).astype(np.float32)
    if dtype == vsl.Q4_1:  # the minimums follow the 16 bytes of scales
        m = out[:, qb + 16:qb + 24].copy().view(np.float16).astype(np.float32)
        got = got + m[..., None]
        assert not out[:, qb + 8:qb + 16].any() and not out[:, qb + 24:].any()  # paddings are zero
    else:
        assert not out[:, qb + 8:].any()  # scale padding is zero
    assert np.array_equal(got.reshape(4, 128), want)


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4", "tiny_q41"])
def test_oracle_quantized_greedy_matches_float64_golden(golden, fixture_gguf, name):
    g = golden(name)
    path = fixture_gguf(name)
    cfg = vsl.gguf_model_config(path)
    assert cfg["wdtype"] == g["dtype"]
    m = O.Model.from_gguf(path, kvdtype=O.F16, max_seq=128)
    ids, _ = m.greedy(g["prompt"], g["n_new"])
    assert ids == g["ids"]
