"""GGUF writer/reader round trip and the C++ GGUFLoader (through the C ABI), no GPU needed."""
import os
import struct

import numpy as np
import pytest

import vsl
from vsl import gguf, synth


@pytest.fixture(scope="module")
def small_gguf(tmp_path_factory):
    shape = gguf.LlamaShape(2, 256, 4, 2, 688, 1000, rope_theta=500000.0, rms_eps=1e-6, context_length=2048)
    path = str(tmp_path_factory.mktemp("g") / "small.gguf")
    gguf.write_synthetic_llama(path, shape, synth.GGML_BF16, seed=5)
    return path, shape


def test_python_roundtrip(small_gguf):
    path, shape = small_gguf
    meta, infos = gguf.read_gguf(path)
    assert meta["llama.embedding_length"] == 256 and meta["general.alignment"] == 32
    gt, ne, off = infos["blk.1.ffn_down.weight"]
    assert gt == synth.GGML_BF16 and ne == [688, 256] and off % 32 == 0
    raw = np.fromfile(path, dtype=np.uint16, count=256 * 688, offset=off)
    assert np.array_equal(raw, synth.synth_tensor(5, synth.tid_layer(1, synth.K_DOWN), (256 * 688,), synth.GGML_BF16))


def test_cpp_loader_model_config(small_gguf):
    path, shape = small_gguf
    c = vsl.gguf_model_config(path)
    assert (c["n_layers"], c["d_model"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["ffn"], c["vocab"]) == \
        (2, 256, 4, 2, 64, 688, 1000)
    assert c["rope_theta"] == 500000.0 and c["rms_eps"] == pytest.approx(1e-6) and c["wdtype"] == vsl.BF16


def test_cpp_loader_tensor_offsets_match_python(small_gguf):
    path, _ = small_gguf
    _, infos = gguf.read_gguf(path)
    for name in ("token_embd.weight", "output_norm.weight", "blk.0.attn_q.weight", "blk.1.ffn_down.weight"):
        t, ne, off = vsl.gguf_tensor_info(path, name)
        assert (t, ne, off) == (infos[name][0], infos[name][1], infos[name][2]), name
    with pytest.raises(vsl.VslError):
        vsl.gguf_tensor_info(path, "blk.9.attn_q.weight")


def test_cpp_loader_rejects_bad_files(tmp_path, small_gguf):
    path, _ = small_gguf
    with pytest.raises(vsl.VslError) as e:
        vsl.gguf_model_config(str(tmp_path / "missing.gguf"))
    assert e.value.code == -6
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + b"\0" * 64)
    with pytest.raises(vsl.VslError) as e:
        vsl.gguf_model_config(str(bad))
    assert e.value.code == -7
    data = open(path, "rb").read()
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(data[: len(data) // 2])  # tensor data cut off
    with pytest.raises(vsl.VslError) as e:
        vsl.gguf_model_config(str(trunc))
    assert e.value.code == -7
    hdr = tmp_path / "hdr.gguf"
    hdr.write_bytes(data[:40])  # metadata cut off
    with pytest.raises(vsl.VslError) as e:
        vsl.gguf_model_config(str(hdr))
    assert e.value.code == -7
    ver = tmp_path / "ver.gguf"
    ver.write_bytes(b"GGUF" + struct.pack("<I", 9) + data[8:])
    with pytest.raises(vsl.VslError):
        vsl.gguf_model_config(str(ver))


def test_vocab_size_fallbacks(tmp_path):
    # no llama.vocab_size: the token array length, then token_embd rows (GGUFLoader.cpp:705-710)
    shape = gguf.LlamaShape(1, 64, 2, 2, 128, 77)
    meta = [m for m in gguf.llama_metadata(shape) if m[0] != "llama.vocab_size"]
    t = [("token_embd.weight", np.zeros((77, 64), np.float16), synth.GGML_F16)]
    p = str(tmp_path / "v.gguf")
    gguf.write_gguf(p, meta, t)
    assert vsl.gguf_model_config(p)["vocab"] == 77
    meta2 = meta + [("tokenizer.ggml.tokens", gguf.T_ARR, (gguf.T_STR, [f"t{i}" for i in range(90)]))]
    p2 = str(tmp_path / "v2.gguf")
    gguf.write_gguf(p2, meta2, t)
    assert vsl.gguf_model_config(p2)["vocab"] == 90
