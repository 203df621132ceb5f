"""ConfigManager::save_to_file then load_from_file gives back every value it wrote, floats
included (tests/cpp/config_roundtrip.cpp, built here with ASan + UBSan; no GPU)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "vulkan-symbiote-loader_b200", "csrc", "host")


def test_config_save_load_round_trip(tmp_path):
    if not shutil.which("g++"):
        pytest.skip("g++ not available")
    exe = str(tmp_path / "config_roundtrip")
    subprocess.run(["g++", "-std=c++17", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=undefined",
                    "-I" + os.path.join(ROOT, "include"), "-I" + HOST,
                    os.path.join(ROOT, "tests", "cpp", "config_roundtrip.cpp"), os.path.join(HOST, "config_manager.cpp"),
                    os.path.join(HOST, "status.cpp"), "-o", exe], check=True, capture_output=True, timeout=600)
    r = subprocess.run([exe, str(tmp_path / "saved.toml")], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == "ok", r.stdout
