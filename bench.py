#!/usr/bin/env python3
"""Decode benchmark: 7B-shape fp16 batch-1 decode tok/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token of the 7B Llama shape (32 layers, d 4096, 32 heads x 128, FFN
11008, vocab 32000, fp16 weights, fp16 KV) at batch 1, after a 128-token prompt. With N > 1
(launched under torchrun) the model is split tensor-parallel over N GPUs (strong scaling:
the same model and batch, time per token shrinks). Weights are random-init from the seeded
generator, filled directly in HBM (identical to the GGUF the fixture writer would produce);
they total 13.5 GB, far above the 126 MB L2, so every step streams them from HBM.

Printed (rank 0, one JSON line): whole-job tok/s from CUDA events on the engine's stream
(max over ranks), the end-to-end tok/s through the host API (pinned host id in, host id
out, every step), the HBM roofline of the dominant kernel (the fused RMSNorm + gate/up +
SwiGLU projection, timed live with CUDA events on its own launches), the CPU oracle timed
on this host's cores, and the SM clocks sampled during the timed region.
`--impl reference` times the CPU restatement of the reference's decode path (oracle/) on
the same workload with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
# The decode path's tensor-parallel sums are the engine's own peer-memory exchange; NCCL only carries
# set-up and prompt-pass sums, so its NVLink multicast (NVLS) buffers are not needed.
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
sys.path.insert(0, os.path.join(ROOT, "vulkan-symbiote-loader_b200"))

CONFIG_7B = dict(n_layers=32, d_model=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000,
                 rope_theta=10000.0, rms_eps=1e-5, wdtype=1)
CONFIG_8B = dict(n_layers=32, d_model=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
                 rope_theta=500000.0, rms_eps=1e-5, wdtype=30)  # GGUF type 30 = bf16
PREFILL_8B, BATCH_8B = 8192, 16
CONFIG_70B = dict(n_layers=80, d_model=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=128256,
                  rope_theta=10000.0, rms_eps=1e-5, wdtype=1)
PREFILL_70B, BUDGET_70B = 2048, 64.0
PROMPT = 128
SEED = 1
SIGMA = 0.02


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=0, help="override depth (profiling captures only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--workload", default="7b", choices=["7b", "7b-q8", "7b-q4", "7b-q41", "8b", "70b", "70b-stream"],
                    help="7b: the headline (BASELINE configs[1]); 7b-q8 / 7b-q4 / 7b-q41: the same model with GGUF "
                         "Q8_0 / Q4_0 / Q4_1 block-quantized weights; 8b: BASELINE configs[3], batch 16 over "
                         "8192 prefilled KV positions each (bf16, GQA, tensor-core projections); 70b: BASELINE "
                         "configs[4] at batch 1 after a 2048-token prompt pass, tensor-parallel over --gpus "
                         "(run it under torchrun with 8 GPUs for the TP 8 figure); 70b-stream: BASELINE configs[4] "
                         "on one GPU under a 64 GB HBM cap (layers streamed from host)")
    ap.add_argument("--profile-case", choices=["tc_gemm", "attention_tc", "gemv_q8", "gemv_q4", "gemv_q41", "prefill",
                                               "decode_layers", "p2p"],
                    help="run one kernel case 3 times (for ncu captures): tc_gemm = 32000 x 4096 fp16 at "
                         "batch 16; attention_tc = 16 x 8192-position fp16 KV, 32/8 heads; gemv_q8 / gemv_q4 / gemv_q41 = "
                         "7B gate/up (22016 x 4096, RMSNorm + SwiGLU) with Q8_0 / Q4_0 / Q4_1 weights at batch 1; prefill = "
                         "three 128-token prompt passes on the 7B shape (--layers, default 4); decode_layers = "
                         "three graph-replayed decode steps of the 7B shape at --layers (default 4) layers after a "
                         "128-token prompt (every per-layer kernel in the engine's context); p2p = the peer-memory "
                         "all-reduce of a 16 KB residual between two receive buffers on one GPU, the second rank's "
                         "words placed by the host (two launches)")
    ap.add_argument("--profile-shape", default="32000,4096,16",
                    help="N,K,B of the tc_gemm profile case (weights N x K, batch B)")
    ap.add_argument("--sweep", action="store_true",
                    help="projection sweep (BASELINE configs[2]): one JSON line per shape and batch")
    ap.add_argument("--sweep-shapes", default="",
                    help="projection shapes NxK,NxK,... for --sweep (default: the 7B decode shapes and lm_head)")
    ap.add_argument("--sweep-batches", default="1,4,16,64", help="activation rows for --sweep")
    ap.add_argument("--split-len", type=int, default=0,
                    help="split-K attention positions per CTA (engine option split_len; 0 = automatic)")
    ap.add_argument("--attn-route", type=int, default=0, choices=[0, 1, 2, 3],
                    help="decode attention kernel (engine option attn_route): 0 automatic, 1 split-K, 2 tcgen05")
    ap.add_argument("--attn-prefetch", type=int, default=0, choices=[0, 1],
                    help="split-K attention requests the output projection into L2 (engine option attn_prefetch)")
    ap.add_argument("--p2p-chunk", type=int, default=0,
                    help="bytes per CTA of the peer-memory all-reduce (engine option p2p_chunk_bytes; 0 = automatic)")
    ap.add_argument("--timeline-prefill", action="store_true",
                    help="per-CTA timeline of one 128-token prompt pass of the 7B workload (trace build): time per "
                         "kernel role; not a benchmark number")
    ap.add_argument("--timeline", action="store_true",
                    help="per-CTA timeline of --steps decode steps of the 7B workload with the trace build "
                         "(lib/libvsl_trace.so, `make -C vulkan-symbiote-loader_b200 trace`): one JSON line per "
                         "rank with the time per kernel role; not a benchmark number")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """Polls SM clock, power and clock-event reasons through NVML while running."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int, period: float = 0.02):
        self.idx, self.period = device_index, period
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_baseline(cfg, seconds: float, threads: int | None = None):
    """Oracle decode steps of the same model on the host cores (bounded sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np

    import oracle as O
    from vsl import synth
    L = O.lib()
    if threads:
        L.orc_set_num_threads(threads)
    t0 = time.perf_counter()
    m = O.Model.synthetic(n_layers=cfg["n_layers"], d=cfg["d_model"], n_heads=cfg["n_heads"], n_kv=cfg["n_kv_heads"],
                          ffn=cfg["ffn"], vocab=cfg["vocab"], rope_theta=cfg["rope_theta"], eps=cfg["rms_eps"],
                          wdtype=cfg["wdtype"], kvdtype=O.F16, max_seq=PROMPT + 256, max_batch=1, seed=SEED,
                          sigma=SIGMA)
    m.fill_kv_synthetic(SEED + 100, 1.0, PROMPT, 1)  # stands in for the prompt's keys/values
    setup = time.perf_counter() - t0
    ids = synth.synth_ids(SEED, 0, 256, cfg["vocab"])
    n, t_total = 0, 0.0
    m.step(ids[:1], np.array([PROMPT], np.int32), want_logits=False)  # warm-up (page-in)
    while t_total < seconds and n < 255:
        t1 = time.perf_counter()
        m.step(ids[n + 1:n + 2], np.array([PROMPT + 1 + n], np.int32), want_logits=False)
        t_total += time.perf_counter() - t1
        n += 1
    cores = int(L.orc_num_threads())
    m.close()
    return {"value": n / t_total, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} decode tokens of the full {cfg['n_layers']}-layer model at positions "
                      f"{PROMPT + 1}..{PROMPT + n}, fp16 weights upcast exactly, fp32 math, {cores} OpenMP threads "
                      f"(setup {setup:.1f}s excluded)"}


def config_7b(args, ws, qname=None):
    """The `config` object of the 7B lines (our arm and the reference arm print the same one)."""
    return {"workload": f"7B Llama shape {qname or 'fp16'} (BASELINE configs[1]"
                        f"{' with block-quantized weights' if qname else ''}), batch 1, "
                        "128-token prompt (prefill), "
                        f"decode positions {PROMPT + args.warmup}..{PROMPT + args.warmup + args.steps - 1}",
            "model": "llama-7b-shape" + (f"-{args.layers}L" if args.layers else ""),
            "global_batch": 1, "seq_len": PROMPT + args.warmup + args.steps,
            "parallelism": f"tp{ws}" if ws > 1 else "single",
            "l2": "inputs larger than L2 (13.5 GB of weights streamed per step)"}


TP_CHECK = os.path.join(ROOT, "tests", "golden", "tp_check_7b_2l.json")


def tp_parity(np, vsl, vdist, dist, rank, ws, local):
    """Before the timed region: the engine under the timed run's tensor parallelism, on the
    benchmark's 7B shape cut to 2 layers, fed 8 ids teacher-forced, against the committed oracle
    fixture of that model (tests/golden/tp_check_7b_2l.json: argmax ids, top-8 and 64 probe
    logits per step) and, on rank 0 of a multi-GPU run, against a single-GPU engine of the same
    model (all logits). Bars: ids identical, logits within 2e-2."""
    with open(TP_CHECK) as f:
        g = json.load(f)
    cfg = {k: g[k] for k in ("n_layers", "d_model", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab",
                             "rope_theta", "rms_eps", "wdtype")}
    probe = np.asarray(g["probe_index"])

    def run(**kw):
        e = vsl.Engine.synthetic(cfg, seed=g["seed"], sigma=g["sigma"], device=local, max_seq=g["max_seq"], **kw)
        lgs, ids = [], []
        for t in g["ids"]:
            o, lg = e.step_host(np.array([t], np.int32), want_logits=True)
            lgs.append(lg[0])
            ids.append(int(o[0]))
        status = e.device_status()
        e.close()
        return np.stack(lgs), ids, status

    nid = vdist.nccl_id(dist)
    lg, ids, status = run(tp_rank=rank, tp_size=ws, nccl_id=nid)
    if dist:
        dist.barrier()
    if rank != 0:
        return None
    worst = 0.0
    for k, st in enumerate(g["steps"]):
        for i, v in st["top8"]:
            worst = max(worst, abs(float(lg[k, i]) - v))
        worst = max(worst, float(np.abs(lg[k, probe] - np.asarray(st["probe"])).max()))
    want = [st["argmax"] for st in g["steps"]]
    out = {"tp": ws, "layers": cfg["n_layers"], "steps": len(ids), "tol": 0.02,
           "vs_oracle_fixture": {"max_abs": round(worst, 6), "ids_equal": ids == want},
           "device_status": status}
    ok = status == 0 and worst <= 0.02 and ids == want
    if ws > 1:
        lg1, ids1, st1 = run()
        d1 = float(np.abs(lg - lg1).max())
        out["vs_single_gpu"] = {"max_abs": round(d1, 6), "ids_equal": ids == ids1}
        ok = ok and st1 == 0 and d1 <= 0.02 and ids == ids1
    out["ok"] = bool(ok)
    return out


def run_reference(args):
    from vsl import dist as vdist
    ws, rank, _ = vdist.env()
    if rank != 0:
        return 0
    cfg = dict(CONFIG_7B)
    if args.layers:
        cfg["n_layers"] = args.layers
    threads = os.cpu_count()
    # a bounded sample: each step is one decode token; total CPU time kept to about 2 minutes
    sec = min(120.0, max(10.0, 0.5 * (args.steps + args.warmup)))
    cb = cpu_baseline(cfg, sec, threads)
    cb["value"] = round(cb["value"], 4)  # the line's value
    line = {"metric": "decode tok/s (7B fp16, bs1)", "value": cb["value"], "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000.0 / cb["value"], 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded random-init weights)",
            "config": config_7b(args, args.gpus),
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": round(cb["value"], 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def profiled_traffic():
    """DRAM read+write bytes per launch of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "gemv_decode_7b_fp16_bs1.md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("| traffic per launch"):
                    return int(float(line.split("|")[2].split()[0]) * 1e6)
    except (OSError, ValueError, IndexError):
        pass
    return None


def dominant_kernel_roofline(torch, vsl, cfg, tp, hbm_peak, peak_kind):
    """Time the fused RMSNorm + gate/up + SwiGLU projection (the largest per-step byte share)
    on 7B-shape weights, rotating 8 copies (far above L2) with CUDA events."""
    d, F = cfg["d_model"], cfg["ffn"] // tp
    N, K = 2 * F, d
    copies = 8
    dt = cfg.get("wdtype", vsl.F16)
    quant = dt in (vsl.Q8_0, vsl.Q4_0, vsl.Q4_1)
    rb = vsl.weight_row_bytes(dt, K)
    W = torch.empty((copies, N, rb), dtype=torch.uint8, device="cuda")
    for c in range(copies):
        if quant:
            vsl.synth_fill_q(W[c], dt, 99, 1000 + c, N, K, 0.02)
        else:
            vsl.synth_fill(W[c], vsl.F16, 99, 1000 + c, 0, N * K, 0.02)
    x = torch.randn((1, K), device="cuda")
    nw = torch.ones(K, device="cuda")
    y = torch.empty((1, F), device="cuda")
    s = torch.cuda.Stream()
    st = s.cuda_stream
    with torch.cuda.stream(s):
        for i in range(3 * copies):
            vsl.gemv(dt, W[i % copies], N, K, x, 1, y, vsl.EPI_SWIGLU, nw, 1e-5, stream=st)
        reps = 20 * copies
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(reps):
            vsl.gemv(dt, W[i % copies], N, K, x, 1, y, vsl.EPI_SWIGLU, nw, 1e-5, stream=st)
        e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    bytes_per_launch = N * rb + K * 4 * 2 + F * 4  # weights (with block scales) + x + norm weights + output
    achieved = bytes_per_launch / (ms * 1e-3) / 1e9
    del W
    torch.cuda.empty_cache()
    if quant:
        qn = {vsl.Q8_0: "Q8_0", vsl.Q4_0: "Q4_0", vsl.Q4_1: "Q4_1"}[dt]
        return {"bound": "hbm", "kernel": f"vsl_gemv_q_kernel<{qn},1,EK_SWIGLU,NORM> "
                                          "(gate/up + SwiGLU, fused RMSNorm)",
                "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind, "bytes_per_launch": bytes_per_launch,
                "us_per_launch": round(ms * 1e3, 3), "traffic": None}
    return {"bound": "hbm", "kernel": "vsl_gemv_kernel<__half,1,EK_SWIGLU,NORM> (gate/up + SwiGLU, fused RMSNorm)",
            "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
            "peak_kind": peak_kind, "bytes_per_launch": bytes_per_launch, "us_per_launch": round(ms * 1e3, 3),
            "traffic": profiled_traffic() if tp == 1 else None,
            "traffic_source": "profiles/gemv_decode_7b_fp16_bs1.md (ncu, engine launch: includes the 16.8 MB "
                              "L2 prefetch of the next projection)"}


def run_ours(args):
    import numpy as np
    import torch

    import vsl
    from vsl import dist as vdist
    from vsl import synth
    ws, rank, local = vdist.env()
    dist = vdist.init(ws)
    torch.cuda.set_device(local)
    if args.workload == "70b-stream":
        return run_stream70(args)
    big = args.workload == "8b"
    w70 = args.workload == "70b"
    cfg = dict(CONFIG_8B if big else CONFIG_70B if w70 else CONFIG_7B)
    qname = {"7b-q8": "Q8_0", "7b-q4": "Q4_0", "7b-q41": "Q4_1"}.get(args.workload)
    if qname:
        cfg["wdtype"] = {"Q8_0": vsl.Q8_0, "Q4_0": vsl.Q4_0, "Q4_1": vsl.Q4_1}[qname]
    if args.layers:
        cfg["n_layers"] = args.layers
    B = BATCH_8B if big else 1
    start = PREFILL_8B if big else PREFILL_70B if w70 else PROMPT
    max_seq = start + args.warmup + 3 * args.steps + 8
    max_seq = (max_seq + 63) // 64 * 64
    parity = tp_parity(np, vsl, vdist, dist, rank, ws, local) if not (big or w70 or qname) else None
    nccl_id = vdist.nccl_id(dist)
    t0 = time.perf_counter()
    eng = vsl.Engine.synthetic(cfg, seed=SEED, sigma=SIGMA, device=local, max_batch=B, max_seq=max_seq,
                               tp_rank=rank, tp_size=ws, nccl_id=nccl_id, split_len=args.split_len,
                               p2p_chunk_bytes=args.p2p_chunk, attn_route=args.attn_route,
                               attn_prefetch=args.attn_prefetch)
    load_s = time.perf_counter() - t0
    if big:
        # 8192 positions of seeded N(0, 1) keys/values per sequence written straight into the
        # paged cache (no prefill pass), then greedy decode from one seeded id per sequence
        eng.fill_kv_synthetic(SEED + 100, 1.0, PREFILL_8B, B)
        eng.set_forced(synth.synth_ids(SEED, 0, B, cfg["vocab"]).reshape(1, B))
        eng.run(1, batch=B)
    elif w70:
        # the 2048-token prompt through the prompt pass once (time to first token, host call to
        # sampled id, max over ranks), after an untimed short prompt that allocates the pass's
        # buffers
        prompt = synth.synth_ids(SEED, 0, PREFILL_70B, cfg["vocab"])
        eng.prefill(prompt[:128])
        eng.reset()
        if dist:
            dist.barrier()
        t_p = time.perf_counter()
        eng.prefill(prompt)
        ttft_s = vdist.max_over_ranks(dist, time.perf_counter() - t_p)
    else:
        # prompt positions 0..127 through the prompt pass (one chunk of 128 rows); time to first
        # token through the host API (ids in, first sampled id out), the median of 3 after one
        # untimed call, each from an empty cache
        prompt = synth.synth_ids(SEED, 0, PROMPT, cfg["vocab"])
        ttft = []
        for i in range(4):
            eng.reset()
            if dist:
                dist.barrier()
            t_p = time.perf_counter()
            eng.prefill(prompt)
            ttft.append(time.perf_counter() - t_p)
        ttft_s = vdist.max_over_ranks(dist, sorted(ttft[1:])[1])
    eng.run(args.warmup, batch=B)
    stream = eng.stream
    s = torch.cuda.ExternalStream(stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kernels, bytes_start = eng.step_stats(B)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(s)
        eng.run(args.steps, batch=B)
        e1.record(s)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    ms = vdist.max_over_ranks(dist, ms)
    # per-step device times of the same graph replays, one event pair per step (the median is
    # insensitive to the ranks' launch skew at the first exchange of the window above)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev[0].record(s)
    for i in range(args.steps):
        eng.run(1, batch=B)
        ev[i + 1].record(s)
    torch.cuda.synchronize()
    step_ms = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps))
    step_ms_p50 = vdist.max_over_ranks(dist, step_ms[len(step_ms) // 2])
    _, bytes_end = eng.step_stats(B)
    status = eng.device_status()
    # end to end through the host API: pinned host ids in, sampled ids back, every step
    n_log = (1 if big else 0) + args.warmup + 2 * args.steps
    nxt = np.asarray(eng.read_tokens(n_log, batch=B)[-1], np.int32).reshape(B)
    for _ in range(2):
        nxt, _ = eng.step_host(nxt)
    if dist:
        dist.barrier()
    n_e2e = args.steps
    t1 = time.perf_counter()
    for _ in range(n_e2e):
        nxt, _ = eng.step_host(nxt)
    e2e_s = time.perf_counter() - t1
    e2e_s = vdist.max_over_ranks(dist, e2e_s)
    if status != 0 or eng.device_status() != 0:
        raise SystemExit(f"device status {status}")
    hbm_peak, peak_kind = peaks()
    roof = None if big or w70 else dominant_kernel_roofline(torch, vsl, cfg, ws, hbm_peak, peak_kind)
    eng.close()
    tok_s = args.steps * B / (ms / 1e3)
    step_bytes = 0.5 * (bytes_start + bytes_end)  # per GPU; KV grows by one position per step
    step_gbs = step_bytes / (ms / 1e3 / args.steps) / 1e9
    cb = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and not big and not w70 and not qname:
        cb = cpu_baseline(cfg, args.cpu_seconds)
    if rank == 0 and big:
        step_roof = {"bound": "hbm", "kernel": "whole decode step (weights + 16 x 8192-position KV)",
                     "achieved": round(step_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(step_gbs / hbm_peak, 4), "peak_kind": peak_kind,
                     "bytes_per_step_per_gpu": round(step_bytes), "traffic": None}
        line = {
            "metric": "decode tok/s (8B bf16 GQA, bs16, 8192-position KV)", "value": round(tok_s, 3),
            "unit": "tok/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "step_ms_p50": round(step_ms_p50, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights and KV in HBM)",
            "config": {"workload": "8B Llama-3 shape bf16 (BASELINE configs[3]), 16 sequences x 8192 prefilled "
                                   "fp16 KV positions, greedy decode",
                       "model": "llama-3-8b-shape" + (f"-{cfg['n_layers']}L" if args.layers else ""),
                       "global_batch": B, "seq_len": start + args.warmup + args.steps,
                       "parallelism": f"tp{ws}" if ws > 1 else "single",
                       "l2": "inputs larger than L2 (15 GB weights + 17 GB KV per step)"},
            "e2e": {"value": round(n_e2e * B / e2e_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                    "d2h_bytes_per_step": 4 * (B + 1), "api": "vsl_engine_step_host",
                    "d2h": "sampled ids + device status word"},
            "roofline": step_roof,
            "gpu_launches": kernels * args.steps, "kernels_per_step": kernels,
            "clocks": clk.summary(), "load_seconds": round(load_s, 2),
        }
        print(json.dumps(line), flush=True)
    elif rank == 0 and w70:
        line = {
            "metric": "decode tok/s (70B fp16, bs1)", "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "step_ms_p50": round(step_ms_p50, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random-init weights filled in HBM)",
            "config": {"workload": "70B Llama shape fp16 (BASELINE configs[4]), batch 1, 2048-token prompt (prefill), "
                                   f"decode positions {PREFILL_70B + args.warmup}..{PREFILL_70B + args.warmup + args.steps - 1}",
                       "model": "llama-70b-shape" + (f"-{cfg['n_layers']}L" if args.layers else ""),
                       "global_batch": 1, "seq_len": PREFILL_70B + args.warmup + args.steps,
                       "parallelism": f"tp{ws}" if ws > 1 else "single",
                       "l2": "inputs larger than L2 (140 GB of weights over the ranks per step)"},
            "e2e": {"value": round(n_e2e / e2e_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 8,
                    "api": "vsl_engine_step_host", "d2h": "sampled id + device status word"},
            "roofline": {"bound": "hbm", "kernel": "whole decode step (this rank's weights + KV)",
                         "achieved": round(step_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(step_gbs / hbm_peak, 4), "peak_kind": peak_kind,
                         "bytes_per_step_per_gpu": round(step_bytes), "traffic": None},
            "gpu_launches": kernels * args.steps, "kernels_per_step": kernels,
            "clocks": clk.summary(), "load_seconds": round(load_s, 2),
            "prefill": {"prompt_tokens": PREFILL_70B, "ttft_ms": round(ttft_s * 1e3, 3),
                        "tok_s": round(PREFILL_70B / ttft_s, 1), "api": "vsl_engine_prefill",
                        "timing": "host wall clock, one call, max over ranks"},
        }
        print(json.dumps(line), flush=True)
    elif rank == 0:
        line = {
            "metric": f"decode tok/s (7B {qname or 'fp16'}, bs1)", "value": round(tok_s, 3), "unit": "tok/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "step_ms_p50": round(step_ms_p50, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": qname.lower() + " weights, f32 math" if qname else "f16",
            "data": "synthetic (seeded random-init weights filled in HBM)",
            "config": config_7b(args, ws, qname),
            "e2e": {"value": round(n_e2e / e2e_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 8,
                    "api": "vsl_engine_step_host", "d2h": "sampled id + device status word"},
            "roofline": roof,
            "step_roofline": {"bytes_per_step_per_gpu": round(step_bytes), "achieved": round(step_gbs, 1),
                              "peak": hbm_peak, "unit": "GB/s", "frac": round(step_gbs / hbm_peak, 4),
                              "tok_s_at_peak": round(hbm_peak * 1e9 / step_bytes, 1)},
            "gpu_launches": kernels * args.steps, "kernels_per_step": kernels,
            "clocks": clk.summary(), "load_seconds": round(load_s, 2),
            "prefill": {"prompt_tokens": PROMPT, "ttft_ms": round(ttft_s * 1e3, 3),
                        "tok_s": round(PROMPT / ttft_s, 1), "api": "vsl_engine_prefill",
                        "timing": "host wall clock, median of 3 warm calls, max over ranks"},
        }
        if cb:
            line["cpu_baseline"] = cb
        if parity is not None:
            line["tp_parity"] = parity
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def host_link_gbs(torch):
    """Pinned host -> device copy bandwidth (1 GiB, best of 3), the bound of streamed layers."""
    n = 1 << 30
    h = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(n, dtype=torch.uint8, device="cuda")
    best = 0.0
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        d.copy_(h, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        best = max(best, n / (e0.elapsed_time(e1) * 1e-3) / 1e9)
    del h, d
    return best


def run_stream70(args):
    """70B fp16 at batch 1 on one GPU with the HBM budget capped at 64 GB: the layers that do
    not fit are held in pinned host memory and copied into two HBM slots every token, so the
    step is bound by the host link. The 2048-token prompt's keys/values are written straight
    into the cache (seeded N(0, 1)); decode then runs greedily."""
    import numpy as np
    import torch

    import vsl
    from vsl import synth
    torch.cuda.set_device(0)
    link = host_link_gbs(torch)
    cfg = dict(CONFIG_70B)
    max_seq = (PREFILL_70B + args.warmup + args.steps + 8 + 63) // 64 * 64
    t0 = time.perf_counter()
    eng = vsl.Engine.synthetic(cfg, seed=SEED, sigma=SIGMA, max_batch=1, max_seq=max_seq, vram_budget_gb=BUDGET_70B)
    load_s = time.perf_counter() - t0
    res = eng.residency()
    mem = eng.memory_stats()
    eng.fill_kv_synthetic(SEED + 100, 1.0, PREFILL_70B, 1)
    eng.set_forced(synth.synth_ids(SEED, 0, 1, cfg["vocab"]).reshape(1, 1))
    eng.run(1)
    eng.run(args.warmup)
    s = torch.cuda.ExternalStream(eng.stream)
    torch.cuda.synchronize()
    kernels, bytes_start = eng.step_stats(1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record(s)
        eng.run(args.steps)
        e1.record(s)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    nxt = np.asarray(eng.read_tokens(1 + args.warmup + args.steps)[-1], np.int32).reshape(1)
    t1 = time.perf_counter()
    for _ in range(args.steps):
        nxt, _ = eng.step_host(nxt)
    e2e_s = time.perf_counter() - t1
    if eng.device_status() != 0:
        raise SystemExit(f"device status {eng.device_status()}")
    eng.close()
    step_s = ms / 1e3 / args.steps
    streamed = res["streamed_bytes_per_step"]
    line = {
        "metric": "decode tok/s (70B fp16, bs1, 1 GPU under a 64 GB HBM cap)", "value": round(args.steps / (ms / 1e3), 4),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 2), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded random-init weights; streamed layers in pinned host memory)",
        "config": {"workload": "70B Llama shape fp16 (BASELINE configs[4]) at batch 1, 2048 prefilled KV positions, "
                               f"vram_budget_gb {BUDGET_70B}: {res['resident_layers']} layers resident, "
                               f"{res['streamed_layers']} streamed per token",
                   "model": "llama-70b-shape", "global_batch": 1, "seq_len": PREFILL_70B + args.warmup + args.steps,
                   "parallelism": "single", "l2": "inputs larger than L2"},
        "e2e": {"value": round(args.steps / e2e_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 8, "api": "vsl_engine_step_host", "d2h": "sampled id + device status word"},
        "roofline": {"bound": "host link", "kernel": "streamed layer copies (pinned host -> HBM slot)",
                     "achieved": round(streamed / step_s / 1e9, 1), "peak": round(link, 1), "unit": "GB/s",
                     "frac": round(streamed / step_s / 1e9 / link, 4), "peak_kind": "measured pinned H2D copy (1 GiB)",
                     "streamed_bytes_per_step": streamed, "traffic": None},
        "residency": res, "hbm_bytes": mem, "gpu_launches": kernels * args.steps, "kernels_per_step": kernels,
        "clocks": clk.summary(), "load_seconds": round(load_s, 1),
    }
    print(json.dumps(line), flush=True)
    return 0


SWEEP_SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]


def run_sweep(args):
    """y = x W^T with fp16 W [N][K] N(0, 0.02) and fp16-valued x [B][K] N(0, 1) (held as fp32 activations),
    fp32 accumulation. Rotates copies of W so that each pass reads more than the 126 MB L2."""
    import torch

    import vsl
    hbm_peak, peak_kind = peaks()
    shapes = [tuple(int(v) for v in t.split("x")) for t in args.sweep_shapes.split(",")] if args.sweep_shapes \
        else SWEEP_SHAPES
    batches = [int(v) for v in args.sweep_batches.split(",")]
    for N, K in shapes:
        copies = max(2, -(-400_000_000 // (N * K * 2)))
        W = torch.empty((copies, N, K), dtype=torch.float16, device="cuda")
        for c in range(copies):
            vsl.synth_fill(W[c], vsl.F16, 1, 5000 + c, 0, N * K, 0.02)
        for B in batches:
            x = torch.randn((B, K), device="cuda").half().float()
            y = torch.empty((B, N), device="cuda")
            tc = B >= 5  # the engine's route: GEMV up to 4 rows, tcgen05 tensor cores above
            if tc:
                nws = vsl.skinny_gemm_tc_workspace_size(N, K, B)
                wst = torch.zeros(nws // 4 + 512, dtype=torch.int32, device="cuda")
                wsp = (wst.data_ptr() + 1023) // 1024 * 1024
            s = torch.cuda.Stream()

            def call(i):
                if tc:
                    vsl.skinny_gemm_tc(vsl.F16, W[i % copies], N, K, x, B, y, vsl.EPI_STORE, None, 0.0, wsp, nws,
                                       s.cuda_stream)
                else:
                    vsl.gemv(vsl.F16, W[i % copies], N, K, x, B, y, stream=s.cuda_stream)
            # captured in a CUDA graph (as in the engine), so host launch cost is not timed
            reps = max(20, 4 * copies)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                for i in range(2 * copies):
                    call(i)
                s.synchronize()
                with torch.cuda.graph(g, stream=s):
                    for i in range(reps):
                        call(i)
            g.replay()
            torch.cuda.synchronize()
            cur = torch.cuda.current_stream()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            g.replay()
            e1.record(cur)
            torch.cuda.synchronize()
            del g
            us = e0.elapsed_time(e1) * 1e3 / reps
            algo = 2 * N * K + 2 * B * K + 2 * B * N
            gbs = algo / (us * 1e-6) / 1e9
            print(json.dumps({"sweep": "projection", "N": N, "K": K, "B": B, "us": round(us, 3),
                              "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 4), "peak": hbm_peak,
                              "peak_kind": peak_kind, "TFLOP/s": round(2 * B * N * K / (us * 1e-6) / 1e12, 2),
                              "path": "tcgen05" if tc else "gemv",
                              "launches_per_call": 2 if tc else -(-B // 4)}), flush=True)
        del W
        torch.cuda.empty_cache()
    return 0


def run_profile_case(args):
    """A single kernel case, launched three times, sized for an ncu capture (about 1-2 GB)."""
    import torch

    import vsl
    if args.profile_case == "decode_layers":
        from vsl import synth
        cfg = dict(CONFIG_7B)
        cfg["n_layers"] = args.layers or 4
        with vsl.Engine.synthetic(cfg, seed=SEED, sigma=SIGMA, max_batch=1, max_seq=512) as e:
            e.prefill(synth.synth_ids(SEED, 0, PROMPT, cfg["vocab"]))
            e.run(3)
            if e.device_status() != 0:
                raise SystemExit("device status")
    elif args.profile_case == "p2p":
        import numpy as np
        n, cap = 4096, 4096 * 4
        size = vsl.p2p_buffer_size(2, cap)
        bufs = [torch.zeros(size // 8, dtype=torch.int64, device="cuda") for _ in range(2)]
        slot = size // 4  # [2 parities][2 ranks] slots
        epochs = torch.zeros(64, dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        data = torch.randn(n, device="cuda")
        peer = np.random.default_rng(0).standard_normal(n).astype(np.float32).view(np.uint32)
        for epoch in (1, 2):  # the second rank's words of both calls: (piece, epoch tag) pairs
            w = peer.astype(np.uint64) | (np.uint64((epoch & 0x7FFFFFFF) | 0x80000000) << np.uint64(32))
            off = ((epoch & 1) * 2 + 1) * slot // 8
            bufs[0][off:off + n].copy_(torch.from_numpy(w.view(np.int64)).cuda())
        torch.cuda.synchronize()
        for _ in range(2):
            vsl.p2p_allreduce(bufs, 0, cap, data, n, 0, epochs, status)
        torch.cuda.synchronize()
        if status.item() != 0:
            raise SystemExit("p2p status")
    elif args.profile_case == "prefill":
        from vsl import synth
        cfg = dict(CONFIG_7B)
        cfg["n_layers"] = args.layers or 4
        with vsl.Engine.synthetic(cfg, seed=SEED, sigma=SIGMA, max_batch=1, max_seq=512) as e:
            prompt = synth.synth_ids(SEED, 0, PROMPT, cfg["vocab"])
            for _ in range(3):
                e.reset()
                e.prefill(prompt)
            if e.device_status() != 0:
                raise SystemExit("device status")
    elif args.profile_case in ("gemv_q8", "gemv_q4", "gemv_q41"):
        dt = {"gemv_q8": vsl.Q8_0, "gemv_q4": vsl.Q4_0, "gemv_q41": vsl.Q4_1}[args.profile_case]
        N, K = 2 * CONFIG_7B["ffn"], CONFIG_7B["d_model"]
        rb = vsl.weight_row_bytes(dt, K)
        Ws = [torch.empty(N, rb, dtype=torch.uint8, device="cuda") for _ in range(4)]  # > L2 in total
        for i, w in enumerate(Ws):
            vsl.synth_fill_q(w, dt, 7, 500 + i, N, K)
        x = torch.randn(1, K, device="cuda")
        nw = torch.ones(K, device="cuda")
        y = torch.zeros(1, N // 2, device="cuda")
        for i in range(3):
            vsl.gemv(dt, Ws[i % 4], N, K, x, 1, y, vsl.EPI_SWIGLU, nw, 1e-5)
    elif args.profile_case == "tc_gemm":
        N, K, B = (int(v) for v in args.profile_shape.split(","))
        # enough weight copies that every launch reads its weights from HBM (more than L2)
        Ws = [torch.randn(N, K, device="cuda").mul_(0.02).half() for _ in range(max(2, -(-300_000_000 // (N * K * 2))))]
        x = torch.randn(B, K, device="cuda")
        y = torch.zeros(B, N, device="cuda")
        n = vsl.skinny_gemm_tc_workspace_size(N, K, B)
        wst = torch.zeros(n // 4 + 512, dtype=torch.int32, device="cuda")
        ws = (wst.data_ptr() + 1023) // 1024 * 1024
        for i in range(3):
            vsl.skinny_gemm_tc(vsl.F16, Ws[i % len(Ws)], N, K, x, B, y, vsl.EPI_STORE, None, 0.0, ws, n)
    else:
        B, nh, nkv, L, page = 16, 32, 8, 8192, 64
        mp = L // page
        k = torch.randn(B * mp, nkv, page, 128, device="cuda").half()
        v = torch.randn(B * mp, nkv, page, 128, device="cuda").half()
        pt = torch.arange(B * mp, dtype=torch.int32, device="cuda").reshape(B, mp)
        pos = torch.full((B,), L - 1, dtype=torch.int32, device="cuda")
        q = torch.randn(B, nh, 128, device="cuda")
        out = torch.zeros(B, nh, 128, device="cuda")
        n = vsl.flash_decode_tc_workspace_size(B, nkv)
        w = torch.zeros(n // 4 + 64, dtype=torch.int32, device="cuda")
        for _ in range(3):
            vsl.flash_decode_tc(q, k, v, B * mp, pt, mp, page, pos, B, nh, nkv, 128, L, out, w, n)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": args.profile_case, "launches": 3}))
    return 0


ROLE_ORDER = ("qkv", "attention", "o", "allreduce", "gate_up", "down", "lm_head", "argmax_exchange", "other")


def run_timeline_prefill(args):
    """Where a prompt pass's time goes (trace build, one GPU): every CTA of the traced kernels
    stamps %globaltimer at entry, release from griddepcontrol.wait and exit. Per kernel role
    (activation split, QKV, attention, O, gate/up, down, lm_head) the line gives the launches per
    pass and, averaged over them, the span (end of the previous launch's last CTA to end of this
    launch's last CTA) and the median CTA duration after release, in microseconds."""
    os.environ["VSL_LIBRARY"] = "trace"
    import numpy as np
    import torch

    import vsl
    from vsl import synth
    assert vsl.LIB_PATH.endswith("libvsl_trace.so"), vsl.LIB_PATH
    cfg = dict(CONFIG_7B)
    if args.layers:
        cfg["n_layers"] = args.layers
    prompt = synth.synth_ids(SEED, 0, PROMPT, cfg["vocab"])
    with vsl.Engine.synthetic(cfg, seed=SEED, sigma=SIGMA, max_seq=512) as eng:
        for _ in range(3):
            eng.reset()
            eng.prefill(prompt)
        eng.reset()
        torch.cuda.synchronize()
        vsl.trace_records(reset=True)
        t0 = time.perf_counter()
        eng.prefill(prompt)
        host_ms = (time.perf_counter() - t0) * 1e3
        recs = vsl.trace_records(reset=True)
        if eng.device_status() != 0:
            raise SystemExit(f"device status {eng.device_status()}")
    # phase stamps of the prompt attention (tags 2201-2206): [t0, t1] of a phase per CTA
    ph = recs[(recs["tag"] > 2200) & (recs["tag"] < 2300)]
    epi = recs[(recs["tag"] >= 2090) & (recs["tag"] < 2100)]  # GEMM epilogue of a CTA's first segment
    recs = recs[((recs["tag"] <= 2200) | (recs["tag"] >= 2300)) & ((recs["tag"] < 2090) | (recs["tag"] >= 2100))]
    main = {(int(r["id"]), int(r["blk"])): int(r["t1"]) for r in recs[recs["tag"] == 2200]}
    phase_names = {2201: "stage_q", 2202: "scores_to_p_ready", 2203: "p_ready_to_pv_done", 2204: "softmax_warps_total",
                   2205: "mma_waits_q", 2206: "mma_waits_k_issues_s", 2207: "scores_load_and_row_max"}
    phases = {}
    for tag, name in phase_names.items():
        r = ph[ph["tag"] == tag]
        if len(r):
            rel = [int(x["t0"]) - main.get((int(x["id"]), int(x["blk"])), int(x["t0"])) for x in r]
            phases[name] = {"us_p50": round(float(np.median((r["t1"] - r["t0"]).astype(np.int64))) / 1e3, 2),
                            "starts_after_release_us_p50": round(float(np.median(rel)) / 1e3, 2)}
    epilogue = {}
    for ek, name in ((3, "qkv"), (2, "gate_up"), (1, "o_or_down")):
        r = epi[epi["tag"] == 2090 + ek]
        if len(r):
            epilogue[name] = round(float(np.median((r["t1"] - r["t0"]).astype(np.int64))) / 1e3, 2)
    launches = sorted((recs[recs["id"] == lid] for lid in np.unique(recs["id"])), key=lambda r: int(r["t1"].min()))
    roles, prev_end, after_attn = {}, None, False
    for r in launches:
        tag = int(r["tag"].max())
        if tag == 2100:
            role = "split"
        elif tag == 2200 or 900 <= tag < 1000:
            role, after_attn = "attention", True
        else:
            ek = (tag - 2000) // 10 if tag >= 2000 else tag // 100
            role = {3: "qkv", 2: "gate_up", 4: "lm_head"}.get(ek)
            if role is None:
                role = "o" if after_attn else "down"
                after_attn = False
        a = roles.setdefault(role, {"launches": 0, "span": 0.0, "cta_us": 0.0})
        a["launches"] += 1
        t2max = int(r["t2"].max())
        if prev_end is not None:
            a["span"] += (t2max - prev_end) / 1e3
        a["cta_us"] += float(np.median(r["t2"] - r["t1"])) / 1e3
        prev_end = t2max
    span_us = (max(int(r["t2"].max()) for r in launches) - min(int(r["t0"].min()) for r in launches)) / 1e3
    out = {k: {"launches": v["launches"], "span_us": round(v["span"] / v["launches"], 2),
               "cta_us_p50": round(v["cta_us"] / v["launches"], 2)} for k, v in roles.items()}
    print(json.dumps({"timeline": f"prompt pass, 7B fp16, {PROMPT} tokens", "layers": cfg["n_layers"],
                      "traced_span_us": round(span_us, 1), "host_ms": round(host_ms, 3), "roles": out,
                      "attention_phases": phases, "gemm_epilogue_us_p50": epilogue,
                      "library": "lib/libvsl_trace.so (trace build; timings perturbed slightly by the stamps)"}))
    return 0


def run_timeline(args):
    """Where a decode step's time goes: every CTA of every kernel stamps %globaltimer at entry, at
    its release from griddepcontrol.wait and at exit (trace build). Per kernel role (QKV, attention,
    O, all-reduce, gate/up, down, lm_head) the line gives, averaged over the layers and steps:
    span (end of the previous launch's last CTA to end of this launch's last CTA), release (end of
    the previous launch to the first CTA's release), ramp (first to last release), tail (median
    CTA end to last CTA end) and the median CTA duration after its release, in microseconds, plus
    the launch's weight bytes over its span."""
    os.environ["VSL_LIBRARY"] = "trace"
    import numpy as np
    import torch

    import vsl
    from vsl import dist as vdist
    from vsl import synth
    assert vsl.LIB_PATH.endswith("libvsl_trace.so"), vsl.LIB_PATH
    ws, rank, local = vdist.env()
    dist = vdist.init(ws)
    torch.cuda.set_device(local)
    w70 = args.workload == "70b"  # the 70B shape after a 2048-token prompt (--layers for a reduced depth)
    cfg = dict(CONFIG_70B if w70 else CONFIG_7B)
    if args.layers:
        cfg["n_layers"] = args.layers
    prompt_len = PREFILL_70B if w70 else PROMPT
    max_seq = (prompt_len + args.warmup + args.steps + 8 + 63) // 64 * 64
    nid = vdist.nccl_id(dist)
    eng = vsl.Engine.synthetic(cfg, seed=SEED, sigma=SIGMA, device=local, max_seq=max_seq, tp_rank=rank, tp_size=ws,
                               nccl_id=nid, split_len=args.split_len, p2p_chunk_bytes=args.p2p_chunk,
                               attn_route=args.attn_route, attn_prefetch=args.attn_prefetch)
    eng.prefill(synth.synth_ids(SEED, 0, prompt_len, cfg["vocab"]))
    eng.run(args.warmup)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    vsl.trace_records(reset=True)
    eng.run(args.steps)
    torch.cuda.synchronize()
    recs = vsl.trace_records(reset=True)
    if eng.device_status() != 0:
        raise SystemExit(f"device status {eng.device_status()}")
    eng.close()
    d, hd, F = cfg["d_model"], cfg["head_dim"], cfg["ffn"] // ws
    nh, nkv = cfg["n_heads"] // ws, cfg["n_kv_heads"] // ws
    wbytes = {"qkv": (nh + 2 * nkv) * hd * d * 2, "o": d * nh * hd * 2, "gate_up": 2 * F * d * 2, "down": d * F * 2,
              "lm_head": cfg["vocab"] // ws * d * 2}
    K = args.steps
    # phase stamps of the short-cache attention (tags 2301-2304, first round of each CTA)
    ph = recs[(recs["tag"] > 2300) & (recs["tag"] < 2400)]
    recs = recs[(recs["tag"] <= 2300) | (recs["tag"] >= 2400)]
    att_phases = {}
    for tag, name in ((2301, "release_to_staged"), (2302, "scores"), (2303, "softmax"), (2304, "p_v")):
        r = ph[ph["tag"] == tag]
        if len(r):
            att_phases[name] = round(float(np.median((r["t1"] - r["t0"]).astype(np.int64))) / 1e3, 2)
    launches = []  # (replay, id, role-tag, records)
    for lid in np.unique(recs["id"]):
        r = recs[recs["id"] == lid]
        r = r[np.argsort(r["t0"], kind="stable")]
        n = len(r) // K
        if n * K != len(r):
            continue
        for k in range(K):
            launches.append((k, int(lid), r[k * n:(k + 1) * n]))
    roles = {}
    step_us = []
    for k in range(K):
        seq = sorted([x for x in launches if x[0] == k], key=lambda x: int(x[2]["t1"].min()))
        prev_end, after_attn = None, False
        step_us.append((max(int(x[2]["t2"].max()) for x in seq) - min(int(x[2]["t0"].min()) for x in seq)) / 1e3)
        for _, _, r in seq:
            tag = int(r["tag"].max())
            if 900 <= tag < 1000 and (r["tag"] != 900).any():
                r = r[r["tag"] != 900]  # empty splits only prefetch; their stamps have no release
            if 900 <= tag < 1000:
                role = "attention"
                after_attn = True
            elif tag == 1001:
                role = "argmax_exchange"
            elif tag >= 1000:
                role = "allreduce"
            else:
                ek, norm = tag // 100, (tag // 10) % 10
                if ek == 3:
                    role = "qkv"
                elif ek == 2:
                    role = "gate_up"
                elif ek == 4:
                    role = "lm_head"
                elif ek in (0, 1) and not norm:
                    role = "o" if after_attn else "down"
                    after_attn = False
                else:
                    role = "other"
            t2max, t1min = int(r["t2"].max()), int(r["t1"].min())
            a = roles.setdefault(role, {"launches": 0, "span": 0.0, "release": 0.0, "ramp": 0.0, "tail": 0.0,
                                        "cta_us": 0.0, "ctas": 0})
            a["launches"] += 1
            if prev_end is not None:
                a["span"] += (t2max - prev_end) / 1e3
                a["release"] += (t1min - prev_end) / 1e3
            a["ramp"] += (int(r["t1"].max()) - t1min) / 1e3
            a["tail"] += (t2max - float(np.median(r["t2"]))) / 1e3
            a["cta_us"] += float(np.median(r["t2"] - r["t1"])) / 1e3
            a["ctas"] += len(r)
            prev_end = t2max
    out = {}
    for role in ROLE_ORDER:
        if role not in roles:
            continue
        a = roles[role]
        c = a["launches"]
        e = {"per_step": round(c / K, 2), "span_us": round(a["span"] / c, 2), "release_us": round(a["release"] / c, 2),
             "ramp_us": round(a["ramp"] / c, 2), "tail_us": round(a["tail"] / c, 2),
             "cta_us_p50": round(a["cta_us"] / c, 2), "ctas": round(a["ctas"] / c, 1)}
        if role in wbytes:
            e["weight_gbs_over_span"] = round(wbytes[role] / (a["span"] / c * 1e-6) / 1e9, 1)
        out[role] = e
    line = {"timeline": ("decode step, 70B fp16 bs1 after 2048 positions" if w70 else "decode step, 7B fp16 bs1") +
                        (f" ({cfg['n_layers']} layers)" if args.layers else ""),
            "tp": ws, "rank": rank, "steps": K, "step_us_p50": round(float(np.median(step_us)), 1),
            "step_span_note": "first CTA entry to last CTA exit of the traced kernels in one graph replay",
            "roles": out, "library": "lib/libvsl_trace.so (trace build; timings perturbed slightly by the stamps)"}
    if att_phases:
        line["attention_phases_us_p50"] = att_phases
    print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.timeline_prefill:
        return run_timeline_prefill(args)
    if args.timeline:
        return run_timeline(args)
    if args.profile_case:
        return run_profile_case(args)
    if args.sweep:
        return run_sweep(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
