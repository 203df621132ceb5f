import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "vulkan-symbiote-loader_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        with open(os.path.join(ROOT, "tests", "golden", name + ".json")) as f:
            return json.load(f)
    return load


@pytest.fixture(scope="session")
def fixture_gguf(tmp_path_factory, golden):
    """Path of the seeded GGUF behind a golden fixture (regenerated bit-exactly)."""
    from vsl import gguf
    cache = {}

    def make(name):
        if name not in cache:
            g = golden(name)
            s = g["shape"]
            shape = gguf.LlamaShape(s["n_layers"], s["d_model"], s["n_heads"], s["n_kv_heads"], s["ffn"],
                                    s["vocab"], rope_theta=s["rope_theta"], rms_eps=s["rms_eps"])
            path = str(tmp_path_factory.mktemp("gguf") / (name + ".gguf"))
            gguf.write_synthetic_llama(path, shape, g["dtype"], g["seed"], g["sigma"])
            cache[name] = path
        return cache[name]
    return make
