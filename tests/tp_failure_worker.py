"""Worker of tests/test_tp_failure_gpu.py (run under torch.distributed.run, 2 ranks): a rank that
stops taking part between steps. Both ranks build a tensor-parallel engine (peer-memory
all-reduce) and decode one step together; then rank 1 stays alive but waits on the host, and rank
0 decodes alone. Rank 0's first exchange gives up after its bound (VSL_ERR_TIMEOUT in the device
status, returned by step_host), the rest of its step skips the exchanges, and the engine refuses
further work (VSL_ERR_STATE). Rank 1's memory stays mapped throughout; the failure is made on the
host (a rank that does not call), and no kernel waits without a bound."""
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "vulkan-symbiote-loader_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import vsl  # noqa: E402
from vsl import dist as vdist  # noqa: E402


def main():
    ws, rank, local = vdist.env()
    d = vdist.init(ws, timeout_s=300)
    torch.cuda.set_device(local)
    cfg = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=4, head_dim=64, ffn=1376, vocab=4096,
               rope_theta=1e4, rms_eps=1e-5, wdtype=vsl.F16)
    nid = vdist.nccl_id(d)
    e = vsl.Engine.synthetic(cfg, seed=3, device=local, max_seq=64, tp_rank=rank, tp_size=ws, nccl_id=nid,
                             use_p2p=1, nccl_timeout_ms=60000)
    ids0, _ = e.step_host(np.array([5], np.int32))
    res = {"step_together": int(ids0[0]), "status_together": e.device_status()}
    d.barrier()
    if rank == 0:
        t0 = time.perf_counter()
        try:
            e.step_host(np.array([7], np.int32))
            res["alone"] = "ok"
        except vsl.VslError as err:
            res["alone"] = err.code
        res["alone_seconds"] = time.perf_counter() - t0
        try:
            e.step_host(np.array([7], np.int32))
            res["after"] = "ok"
        except vsl.VslError as err:
            res["after"] = err.code
        res["status_after"] = e.device_status()
    d.barrier()  # rank 1 waited here on the host while rank 0 decoded alone
    e.close()
    if rank == 0:
        with open(sys.argv[1], "w") as f:
            json.dump(res, f)
    d.barrier()
    d.destroy_process_group()


if __name__ == "__main__":
    main()
