"""The host C++ code that parses untrusted input (GGUFLoader, Tokenizer, ConfigManager), built
with AddressSanitizer and UndefinedBehaviorSanitizer and fuzzed with damaged GGUF files, random
text and random ids (tests/cpp/host_fuzz.cpp); and the loader's threaded reads and tensor cache
built with ThreadSanitizer (tests/cpp/loader_threads.cpp). No GPU and no CUDA code are involved."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from vsl import gguf, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "vulkan-symbiote-loader_b200", "csrc", "host")
SOURCES = ["gguf_loader.cpp", "tokenizer.cpp", "tokenizer_bpe.cpp", "config_manager.cpp", "quant_repack.cpp",
           "nomad_pack.cpp", "status.cpp"]


@pytest.fixture(scope="module")
def fuzz_bin(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("g++ not available")
    out = str(tmp_path_factory.mktemp("asan") / "host_fuzz")
    cmd = ["g++", "-std=c++17", "-g", "-O1", "-fsanitize=address,undefined", "-fno-sanitize-recover=undefined",
           "-fno-omit-frame-pointer", "-I" + os.path.join(ROOT, "include"), "-I" + HOST, "-I/usr/local/cuda/include",
           os.path.join(ROOT, "tests", "cpp", "host_fuzz.cpp")] + [os.path.join(HOST, s) for s in SOURCES] + \
          ["-o", out, "-lpthread"]
    subprocess.run(cmd, check=True, capture_output=True, timeout=600)
    return out


@pytest.fixture(scope="module")
def model_gguf(tmp_path_factory):
    shape = gguf.LlamaShape(1, 64, 2, 2, 128, 40)
    toks = [f"t{i}" for i in range(40)]
    meta = gguf.llama_metadata(shape) + [
        ("tokenizer.ggml.model", gguf.T_STR, "gpt2"), ("tokenizer.ggml.pre", gguf.T_STR, "llama-bpe"),
        ("tokenizer.ggml.tokens", gguf.T_ARR, (gguf.T_STR, toks)),
        ("tokenizer.ggml.token_type", gguf.T_ARR, (gguf.T_I32, [1] * 40)),
        ("tokenizer.ggml.merges", gguf.T_ARR, (gguf.T_STR, ["t 1", "t 2", "t1 0"])),
        ("tokenizer.ggml.scores", gguf.T_ARR, (gguf.T_F32, [0.0] * 40))]
    q = lambda dt, tid: (synth.synth_q_blocks(1, tid, 64, 64, dt), dt, (64, 64))  # noqa: E731
    tensors = [("token_embd.weight", np.zeros((40, 64), np.float16), synth.GGML_F16),
               ("output_norm.weight", np.ones(64, np.float32), synth.GGML_F32),
               ("blk.0.attn_q.weight", *q(synth.GGML_Q8_0, 2)),
               ("blk.0.attn_k.weight", *q(synth.GGML_Q4_0, 3)),
               ("blk.0.attn_v.weight", *q(synth.GGML_Q4_1, 4)),
               ("blk.0.attn_output.weight", np.zeros((64, 64), np.uint16), synth.GGML_BF16)]
    path = str(tmp_path_factory.mktemp("m") / "model.gguf")
    gguf.write_gguf(path, meta, tensors)
    sp = str(tmp_path_factory.mktemp("m") / "spm.gguf")  # a SentencePiece vocabulary as well
    # malformed byte pieces ("<0x-F>" once indexed the byte table at -15) are ordinary pieces
    pieces = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)] + ["▁t", "t1", "▁", "<0x-F>", "<0x+F>",
                                                                                "<0xG1>"]
    gguf.write_gguf(sp, gguf.llama_metadata(shape) + [
        ("tokenizer.ggml.model", gguf.T_STR, "llama"),
        ("tokenizer.ggml.tokens", gguf.T_ARR, (gguf.T_STR, pieces)),
        ("tokenizer.ggml.scores", gguf.T_ARR, (gguf.T_F32, [0.0] * len(pieces))),
        ("tokenizer.ggml.token_type", gguf.T_ARR, (gguf.T_I32, [2, 3, 3] + [6] * 256 + [1] * 6))],
        tensors[:2])
    return [path, sp]


@pytest.mark.parametrize("which,seed", [(0, 1), (0, 2), (1, 3)])
def test_host_parsers_under_sanitizers(fuzz_bin, model_gguf, tmp_path, which, seed):
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([fuzz_bin, model_gguf[which], str(tmp_path), str(seed), "1500"], capture_output=True,
                       text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "runtime error" not in r.stderr, r.stderr[-3000:]
    words = r.stdout.split()
    assert words[0] == "ok" and int(words[1]) == 1500 and int(words[2]) > 300  # most damaged files are refused


def test_loader_threads_under_thread_sanitizer(model_gguf, tmp_path):
    if not shutil.which("g++"):
        pytest.skip("g++ not available")
    out = str(tmp_path / "loader_threads")
    subprocess.run(["g++", "-std=c++17", "-g", "-O1", "-fsanitize=thread", "-I" + os.path.join(ROOT, "include"),
                    "-I" + HOST, "-I/usr/local/cuda/include", os.path.join(ROOT, "tests", "cpp", "loader_threads.cpp"),
                    os.path.join(HOST, "gguf_loader.cpp"), os.path.join(HOST, "status.cpp"), "-o", out, "-lpthread"],
                   check=True, capture_output=True, timeout=600)
    r = subprocess.run([out, model_gguf[0]], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, TSAN_OPTIONS="halt_on_error=1"))
    assert r.returncode == 0 and "ThreadSanitizer" not in r.stderr, r.stderr[-3000:]
    assert r.stdout.split() == ["ok", "6"]
