"""Host-side tensor-parallel plumbing on CPU ranks (gloo, world size 2): the NCCL id
broadcast, max-over-ranks timing, and a rank that fails before the collective -- the
survivor must get an error from the short process-group timeout, not hang."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, mode, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "vulkan-symbiote-loader_b200"))
    os.environ.update(RANK=str(rank), WORLD_SIZE="2", LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    from vsl import dist as vdist
    try:
        d = vdist.init(2, timeout_s=8.0)
        if mode == "ok":
            nid = vdist.nccl_id(d, make_id=lambda: bytes(range(128)))
            m = vdist.max_over_ranks(d, 1.5 + rank)
            q.put((rank, "ok", nid == bytes(range(128)), m))
            d.barrier()
            d.destroy_process_group()
        else:
            if rank == 1:
                raise RuntimeError("injected failure on rank 1 before the broadcast")
            vdist.nccl_id(d, make_id=lambda: bytes(128))
            q.put((rank, "no-error", False, 0.0))
    except Exception as ex:  # reported to the parent, never swallowed silently
        q.put((rank, "error", type(ex).__name__, str(ex)[:200]))


def _run(mode, timeout):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    out = {}
    while not q.empty():
        r = q.get()
        out[r[0]] = r[1:]
    return out, alive


def test_nccl_id_broadcast_and_max_over_ranks():
    out, alive = _run("ok", 60)
    assert not alive
    assert out[0] == ("ok", True, 2.5) and out[1] == ("ok", True, 2.5)


def test_failed_rank_surfaces_as_error_not_hang():
    out, alive = _run("fail", 60)
    assert not alive, "a rank hung instead of failing"
    assert out[1][0] == "error" and "injected" in out[1][2]
    assert out[0][0] == "error"  # the survivor's collective ended with an error
