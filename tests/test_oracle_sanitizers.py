"""The CPU oracle under AddressSanitizer and UndefinedBehaviorSanitizer, no GPU needed: the C
restatement is rebuilt with both sanitizers and, in a child process with their runtimes
preloaded, reproduces a float64 golden (GGUF load, greedy decode), the quantized
dequantisation of every block type, and a seeded GQA model's batched steps. A memory error or
undefined behaviour in the code that every parity test trusts fails here."""
import os
import shutil
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import json, os, sys
    root, lib = sys.argv[1], sys.argv[2]
    for p in (os.path.join(root, "vulkan-symbiote-loader_b200"), os.path.join(root, "oracle"),
              os.path.join(root, "tests", "golden")):
        sys.path.insert(0, p)
    import numpy as np
    import oracle as O
    O.LIB_PATH = lib
    assert O.lib()._name == lib  # the sanitizer build is the one in use
    from vsl import gguf, synth
    g = json.load(open(os.path.join(root, "tests", "golden", "tiny_q41.json")))
    s = g["shape"]
    path = os.path.join(sys.argv[3], "q41.gguf")
    gguf.write_synthetic_llama(path, gguf.LlamaShape(s["n_layers"], s["d_model"], s["n_heads"], s["n_kv_heads"],
                                                     s["ffn"], s["vocab"], rope_theta=s["rope_theta"],
                                                     rms_eps=s["rms_eps"]), g["dtype"], g["seed"], g["sigma"])
    m = O.Model.from_gguf(path, kvdtype=O.F16, max_seq=128)
    ids, _ = m.greedy(g["prompt"], 8)
    assert ids == g["ids"][:8], (ids, g["ids"][:8])
    m.close()
    rng = np.random.default_rng(1)
    for dt in (O.Q8_0, O.Q4_0, O.Q4_1):
        blocks = synth.synth_q_blocks(2, 3, 5, 96, dt)
        for legacy in (0, 1):
            v = O.dequant_blocks(dt, blocks, 5 * 96, legacy)
            assert np.isfinite(v).all()
    m = O.Model.synthetic(n_layers=2, d=256, n_heads=4, n_kv=2, ffn=688, vocab=500, wdtype=O.F16, kvdtype=O.F16,
                          max_seq=64, max_batch=3, seed=4)
    for p in range(6):
        _, lg = m.step(np.array([7, 8, 9], np.int32), np.array([p, p + 1, p + 2], np.int32))
        assert np.isfinite(lg).all()
    m.close()
    print("ok")
""")


def test_oracle_under_address_and_ub_sanitizers(tmp_path):
    gcc = shutil.which("gcc")
    if not gcc:
        pytest.skip("gcc not available")
    rt = [subprocess.run([gcc, f"-print-file-name={n}"], capture_output=True, text=True).stdout.strip()
          for n in ("libasan.so", "libubsan.so")]
    if not all(os.path.isabs(p) and os.path.exists(p) for p in rt):
        pytest.skip("sanitizer runtimes not installed")
    lib = str(tmp_path / "liboracle_san.so")
    subprocess.run([gcc, "-O1", "-g", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-std=c11",
                    "-fsanitize=address,undefined", "-fno-sanitize-recover=undefined", "-fno-omit-frame-pointer",
                    "-shared", "-o", lib, os.path.join(ROOT, "oracle", "vsl_oracle.c"), "-lm"],
                   check=True, capture_output=True, timeout=600)
    env = dict(os.environ, LD_PRELOAD=" ".join(rt), ASAN_OPTIONS="detect_leaks=0:verify_asan_link_order=0",
               UBSAN_OPTIONS="print_stacktrace=1", OMP_NUM_THREADS="4")
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT, lib, str(tmp_path)], capture_output=True, text=True,
                       timeout=900, env=env)
    assert r.returncode == 0 and "runtime error" not in r.stderr, r.stderr[-3000:]
    assert r.stdout.strip().splitlines()[-1] == "ok"
