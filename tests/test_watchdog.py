"""Bounded host wait of tensor-parallel engines (csrc/host/watchdog.h): a stream whose NCCL work
waits on a rank that never arrives ends in VSL_ERR_TIMEOUT with the communicator aborted once, an
asynchronous NCCL error ends in VSL_ERR_NCCL, a failed stream in VSL_ERR_CUDA. Driven with fakes
of the stream, communicator and clock in tests/cpp/watchdog_check.cpp, built with ASan + UBSan;
no GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "vulkan-symbiote-loader_b200", "csrc", "host")


def test_watched_wait(tmp_path):
    if not shutil.which("g++"):
        pytest.skip("g++ not available")
    exe = str(tmp_path / "watchdog_check")
    subprocess.run(["g++", "-std=c++17", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=undefined",
                    "-I" + os.path.join(ROOT, "include"), "-I" + HOST,
                    os.path.join(ROOT, "tests", "cpp", "watchdog_check.cpp"), "-o", exe],
                   check=True, capture_output=True, timeout=300)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    lines = r.stdout.strip().splitlines()
    assert r.returncode == 0 and len(lines) == 6 and all(ln.endswith(" ok") for ln in lines), r.stdout + r.stderr
