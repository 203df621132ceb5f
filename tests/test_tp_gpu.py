"""Tensor parallelism on 2 GPUs (NCCL): TP=2 logits and greedy ids against a single-GPU
engine on the same seeded model, fp32 (tight) and bf16 GQA with batch 3 and a prefilled
cache (logit tolerance 2e-2). Skipped when fewer than 2 GPUs are visible."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_tp2_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "tp_worker.py"), str(out)]
    log_dir = tmp_path / "logs"
    cmd[7:7] = ["--log-dir", str(log_dir), "--redirects", "3", "--tee", "3"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if r.returncode != 0:
        logs = "".join(f"\n--- {p}\n" + p.read_text()[-4000:] for p in sorted(log_dir.rglob("*.log")))
        raise AssertionError(f"tp worker failed ({r.returncode}):{logs}\n{r.stderr[-2000:]}")
    res = json.loads(out.read_text())
    assert res["fp32_gqa"]["status"] == 0 and res["fp32_gqa"]["ids_equal"] and res["fp32_gqa"]["gen_equal"]
    assert res["fp32_gqa"]["max_abs"] < 1e-4
    assert res["bf16_8b_like"]["status"] == 0 and res["bf16_8b_like"]["max_abs"] < 2e-2
