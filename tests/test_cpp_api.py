"""The drop-in C++ API (include/vk_symbiote/*.h) compiled and linked against libvsl.so like
a caller of the reference would: config parsing and flags, the GGUF loader, the byte-level
tokenizer contract, and (GPU) VulkanSymbioteEngine generation against the golden ids."""
import json
import os
import subprocess

import pytest

import vsl

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def api_bin(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("cpp") / "api_check")
    lib = os.path.dirname(vsl.LIB_PATH)
    env = dict(os.environ)
    env.pop("CXX", None)
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "api_check.cpp"), "-L", lib, "-lvsl",
                    f"-Wl,-rpath,{lib}", "-L/usr/local/cuda/lib64", "-lcudart", "-o", out],
                   check=True, env=env)
    return out


@pytest.fixture(scope="module")
def config_file(tmp_path_factory):
    p = tmp_path_factory.mktemp("cfg") / "vsl.toml"
    p.write_text("# comment\n[memory]\nvram_budget_gb = 48.5\nprefetch_lookahead = 5  # trailing\n"
                 "[performance]\nuse_fp16_math = false\n[custom]\nname = \"symbiote\"\n")
    return str(p)


def run(api_bin, *args):
    r = subprocess.run([api_bin, *args], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout)


def test_config_loader_tokenizer(api_bin, config_file, fixture_gguf):
    out = run(api_bin, fixture_gguf("gqa_fp16"), config_file)
    assert out["file_ok"] == 1 and out["vram_explicit"] == 1
    assert out["vram_gb"] == pytest.approx(48.5) and out["lookahead"] == 5 and out["fp16"] == 0
    assert out["ram_gb"] == pytest.approx(12.5) and out["tp"] == 1 and out["model_path_ok"] == 1
    assert out["custom"] == "symbiote"
    assert out["loaded"] == 1
    assert (out["layers"], out["hidden"], out["heads"], out["kv_heads"], out["ffn"], out["vocab"], out["head_dim"]) \
        == (2, 384, 6, 2, 1040, 3000, 64)
    assert out["q_rows"] == 384 and out["norm0"] == 1.0 and out["tensors"] == 3 + 9 * 2
    # byte-level contract of the reference tokenizer: whitespace dropped, decode joins with spaces
    assert out["encode"] == [ord(c) for c in "hithere"]
    assert out["decode"] == "h i h"


@pytest.mark.gpu
def test_engine_generate_matches_golden(api_bin, config_file, golden, fixture_gguf):
    g = golden("gqa_fp16")
    out = run(api_bin, fixture_gguf("gqa_fp16"), config_file, "--gpu", ",".join(map(str, g["prompt"])),
              str(g["n_new"]))
    assert out["ids"] == g["ids"]
    assert out["generate_prefix_ok"] == 1 and 4 < out["generate_len"] <= 4 + 8
    assert out["bench_tok_s"] > 0 and out["kv_bytes"] > 0 and out["vram_used"] > out["kv_bytes"]
    assert out["tok_s_metric"] > 0 and out["gbps"] > 0
    assert out["overflow_throws"] == 1
    assert out["batch_equal"] == 1  # generate_text_batch (batched decode) == per-prompt generate
