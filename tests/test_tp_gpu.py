"""Tensor parallelism on 2 GPUs: TP=2 logits and greedy ids against a single-GPU engine on the
same seeded model, fp32 (tight) and bf16 GQA with batch 3 and a prefilled cache (logit
tolerance 2e-2), with the peer-memory all-reduce kernel (which must reproduce bit for bit) and
with NCCL, and the chunked prompt pass (prefill). Skipped when fewer than 2 GPUs are visible."""
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
    for tag in ("p2p", "nccl"):  # peer-memory all-reduce kernel, NCCL
        f = res[f"fp32_gqa_{tag}"]
        assert f["status"] == 0 and f["ids_equal"] and f["gen_equal"] and f["max_abs"] < 1e-4, (tag, f)
        assert f["pf_next_equal"] and f["pf_max_abs"] < 1e-4, (tag, f)  # prompt pass (prefill)
        b = res[f"bf16_8b_like_{tag}"]
        assert b["status"] == 0 and b["max_abs"] < 2e-2 and b["pf_max_abs"] < 2e-2, (tag, b)
    assert res["fp32_gqa_p2p_repeat_equal"] and res["bf16_8b_like_p2p_repeat_equal"]
