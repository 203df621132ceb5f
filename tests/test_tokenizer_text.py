"""Text of generated tokens after a prompt (Tokenizer::decode_continuation, used by
VulkanSymbioteEngine::generate and generate_text_batch), through tests/cpp/tokenizer_text.cpp
built with ASan + UBSan. No GPU needed."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "vulkan-symbiote-loader_b200", "csrc", "host")


def test_continuation_text(tmp_path):
    if not shutil.which("g++"):
        pytest.skip("g++ not available")
    exe = str(tmp_path / "tokenizer_text")
    subprocess.run(["g++", "-std=c++17", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=undefined",
                    "-I" + os.path.join(ROOT, "include"), "-I" + HOST,
                    os.path.join(ROOT, "tests", "cpp", "tokenizer_text.cpp")] +
                   [os.path.join(HOST, s) for s in ("tokenizer.cpp", "tokenizer_bpe.cpp", "gguf_loader.cpp",
                                                    "status.cpp")] + ["-o", exe, "-lpthread"],
                   check=True, capture_output=True, timeout=600)
    r = subprocess.run([exe], capture_output=True, text=True, errors="replace", timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.strip().splitlines()
    assert len(lines) == 7 and all(ln.endswith(" ok") for ln in lines), r.stdout
