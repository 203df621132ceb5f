"""A tensor-parallel rank that stops taking part between steps (2 GPUs; skipped with fewer):
the other rank's peer exchange gives up after its one-second bound, step_host returns
VSL_ERR_TIMEOUT, the rest of the step does not wait again, and the engine then refuses work with
VSL_ERR_STATE. The missing rank stays alive (its buffers stay mapped) and waits on the host; no GPU
is faulted or hung. NVLS is off (NCCL_NVLS_ENABLE=0); the engine's own exchange uses plain peer
stores and loads."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_missing_rank_times_out_and_fails_the_engine(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "fail.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    log_dir = tmp_path / "logs"
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           "--log-dir", str(log_dir), "--redirects", "3", "--tee", "3",
           os.path.join(ROOT, "tests", "tp_failure_worker.py"), str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if r.returncode != 0:
        logs = "".join(f"\n--- {p}\n" + p.read_text()[-4000:] for p in sorted(log_dir.rglob("*.log")))
        raise AssertionError(f"worker failed ({r.returncode}):{logs}\n{r.stderr[-2000:]}")
    res = json.loads(out.read_text())
    assert res["status_together"] == 0
    assert res["alone"] == -4, res          # VSL_ERR_TIMEOUT from the expired peer wait
    assert 0.9 < res["alone_seconds"] < 10, res  # one bound, not one per exchange of the step
    assert res["after"] == -10, res         # VSL_ERR_STATE: the engine must be recreated
    assert res["status_after"] == -4, res
