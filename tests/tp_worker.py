"""Tensor-parallel parity worker (run by tests/test_tp_gpu.py under torch.distributed.run):
every rank runs the TP engine; rank 0 also runs a single-GPU engine on the same seeded
model and writes the comparison to the JSON path given as argv[1]."""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "vulkan-symbiote-loader_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import vsl  # noqa: E402
from vsl import dist as vdist  # noqa: E402
from vsl import synth  # noqa: E402


def run(engine, cfg, steps, batch):
    ids = synth.synth_ids(7, 3, steps * batch, cfg["vocab"]).reshape(steps, batch)
    logits, out = [], []
    for s in range(steps):
        o, lg = engine.step_host(ids[s], want_logits=True)
        logits.append(lg)
        out.append(o)
    return np.stack(logits), np.stack(out)


def main():
    ws, rank, local = vdist.env()
    d = vdist.init(ws, timeout_s=120)
    torch.cuda.set_device(local)
    cases = {
        "fp32_gqa": dict(cfg=dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=4, head_dim=64, ffn=1376,
                                  vocab=4096, rope_theta=1e4, rms_eps=1e-5, wdtype=vsl.F32), batch=1, prefill=0),
        "bf16_8b_like": dict(cfg=dict(n_layers=2, d_model=1024, n_heads=16, n_kv_heads=4, head_dim=64, ffn=2816,
                                      vocab=8192, rope_theta=5e5, rms_eps=1e-5, wdtype=vsl.BF16), batch=3,
                             prefill=130),
    }
    result = {}
    prompt = synth.synth_ids(7, 9, 90, 4096).tolist()  # two prefill chunks (64 + 26 rows)
    for name, c in cases.items():
        kw = dict(device=local, max_batch=c["batch"], max_seq=256)
        runs = {}
        # the peer-memory all-reduce kernel (twice: bit for bit) and NCCL
        for tag, p2p in (("p2p", 1), ("p2p_again", 1), ("nccl", 0)):
            nid = vdist.nccl_id(d)  # a unique id forms exactly one communicator: one per engine
            e = vsl.Engine.synthetic(c["cfg"], seed=11, tp_rank=rank, tp_size=ws, nccl_id=nid, use_p2p=p2p, **kw)
            if c["prefill"]:
                e.fill_kv_synthetic(3, 1.0, c["prefill"], c["batch"])
            lg_tp, ids_tp = run(e, c["cfg"], 6, c["batch"])
            gen_tp = e.generate([5, 9, 13, 200], 24) if c["batch"] == 1 else None
            e.reset()
            pf_tp = e.prefill(prompt, seq=c["batch"] - 1, want_logits=True)
            runs[tag] = (lg_tp, ids_tp, gen_tp, e.device_status(), pf_tp)
            e.close()
            d.barrier()
        if rank == 0:
            e1 = vsl.Engine.synthetic(c["cfg"], seed=11, **kw)
            if c["prefill"]:
                e1.fill_kv_synthetic(3, 1.0, c["prefill"], c["batch"])
            lg_1, ids_1 = run(e1, c["cfg"], 6, c["batch"])
            gen_1 = e1.generate([5, 9, 13, 200], 24) if c["batch"] == 1 else None
            e1.reset()
            pf_1 = e1.prefill(prompt, seq=c["batch"] - 1, want_logits=True)
            e1.close()
            for tag in ("p2p", "nccl"):
                lg_tp, ids_tp, gen_tp, status, pf_tp = runs[tag]
                result[f"{name}_{tag}"] = dict(max_abs=float(np.abs(lg_tp - lg_1).max()),
                                               ids_equal=bool((ids_tp == ids_1).all()), gen_equal=gen_tp == gen_1,
                                               status=status, pf_max_abs=float(np.abs(pf_tp[1] - pf_1[1]).max()),
                                               pf_next_equal=pf_tp[0] == pf_1[0])
            result[f"{name}_p2p_repeat_equal"] = bool(np.array_equal(runs["p2p"][0], runs["p2p_again"][0]))
        d.barrier()
    if rank == 0:
        with open(sys.argv[1], "w") as f:
            json.dump(result, f)
    d.barrier()
    d.destroy_process_group()


if __name__ == "__main__":
    main()
