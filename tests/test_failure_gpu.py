"""Failure handling on one GPU without faulting it.

* The peer-memory all-reduce's bounded wait runs out: a 2-rank exchange whose second rank never
  takes part (none of its epoch-tagged words arrive) returns VSL_ERR_TIMEOUT in the status word
  within the wait bound, leaves the message unreduced and still advances every chunk's epoch; the
  device stays usable, and a following call whose peer words were placed by the host (standing in
  for a live peer, so no kernel waits on another kernel) completes with the rank-ordered sum, bit
  for bit.
* The engine reports a kernel's sticky status (injected on the host) as the error of the next
  host-facing call, and generate takes exactly max_seq positions (the last sampled token never
  takes a KV position).
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

import vsl  # noqa: E402
from vsl import synth  # noqa: E402

CHUNKS = 64  # epoch counters per call at most


def _layout(cap_bytes):
    """Slot stride and chunk size (32-bit pieces) of the exchange's receive buffer."""
    words = cap_bytes // 4
    slot = ((words + 1) // 2 * 16 + 255) // 256 * 256
    per = -(-((words + 1) // 2 * 2) // CHUNKS)
    chunk = max(256, (per + 1) // 2 * 2)
    return slot, chunk


def _tag(epoch):
    return (epoch & 0x7FFFFFFF) | 0x80000000


def _words(pieces_u32, epoch, n_words):
    """The 8-byte words a rank writes: (piece, tag) pairs, padded to an even count."""
    m = (n_words + 1) // 2 * 2
    w = np.zeros(m, np.uint64)
    w[:n_words] = pieces_u32.astype(np.uint64)
    w |= np.uint64(_tag(epoch)) << np.uint64(32)
    return w


@pytest.mark.parametrize("op,n", [(0, 4096), (0, 4099), (1, 3)])
def test_p2p_wait_times_out_then_recovers(op, n):
    dev = torch.device("cuda:0")
    es = 4 if op == 0 else 8
    cap = n * es
    slot, chunk = _layout(cap)
    n_words = cap // 4
    nchunks = -(-n_words // chunk)
    size = vsl.p2p_buffer_size(2, cap)
    assert size == 2 * 2 * slot
    bufs = [torch.zeros(size // 8, dtype=torch.int64, device=dev) for _ in range(2)]
    assert all(b.data_ptr() % 256 == 0 for b in bufs)
    epochs = torch.zeros(CHUNKS, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    g = torch.Generator(device="cpu").manual_seed(5)
    if op == 0:
        mine = torch.randn(n, generator=g)
        peer = torch.randn(n, generator=g)
    else:
        mine = torch.randint(0, 2**62, (n,), generator=g, dtype=torch.int64)
        peer = torch.randint(0, 2**62, (n,), generator=g, dtype=torch.int64)
    data = torch.zeros((n_words + 3) // 4 * 4, dtype=torch.int32, device=dev)  # 16-byte aligned storage
    data_view = data.view(torch.float32 if op == 0 else torch.int64)[:n]
    data_view.copy_(mine.to(dev))
    torch.cuda.synchronize()

    # 1. rank 1 never arrives: bounded wait of 50 ms
    t0 = time.perf_counter()
    vsl.p2p_allreduce(bufs, 0, cap, data, n, op, epochs, status, wait_ns=50_000_000)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert status.item() == -4  # VSL_ERR_TIMEOUT
    assert 0.04 < elapsed < 5.0, elapsed
    ep = epochs.cpu().numpy()
    assert (ep[:nchunks] == 1).all() and (ep[nchunks:] == 0).all()
    assert torch.equal(data_view.cpu(), mine)  # left unreduced: no word of rank 1 arrived
    # rank 0's message reached rank 1's buffer (slot [parity 1][rank 0]) as (piece, epoch) words
    pieces = mine.numpy().view(np.uint32)[:n_words]
    m = (n_words + 1) // 2 * 2
    got = bufs[1].cpu().numpy().view(np.uint64)[(1 * 2 + 0) * slot // 8:(1 * 2 + 0) * slot // 8 + m]
    assert np.array_equal(got, _words(pieces, 1, n_words))

    # 2. the device is still usable; the host stands in for a live rank 1 at epoch 2 (parity 0)
    status.zero_()
    w = torch.from_numpy(_words(peer.numpy().view(np.uint32)[:n_words], 2, n_words).view(np.int64))
    bufs[0][(0 * 2 + 1) * slot // 8:(0 * 2 + 1) * slot // 8 + m].copy_(w.to(dev))
    torch.cuda.synchronize()
    vsl.p2p_allreduce(bufs, 0, cap, data, n, op, epochs, status, wait_ns=1_000_000_000)
    torch.cuda.synchronize()
    assert status.item() == 0
    want = (mine + peer) if op == 0 else torch.maximum(mine, peer)
    assert torch.equal(data_view.cpu(), want)  # rank order: own piece first, then rank 1 (fp32 adds)
    ep = epochs.cpu().numpy()
    assert (ep[:nchunks] == 2).all() and (ep[nchunks:] == 0).all()
    assert float(torch.ones(8, device=dev).sum()) == 8.0


def test_p2p_arguments_checked():
    dev = torch.device("cuda:0")
    size = vsl.p2p_buffer_size(2, 1024)
    bufs = [torch.zeros(size, dtype=torch.uint8, device=dev) for _ in range(2)]
    epochs = torch.zeros(CHUNKS, dtype=torch.int64, device=dev)
    data = torch.zeros(512, device=dev)
    with pytest.raises(vsl.VslError) as e:
        vsl.p2p_allreduce(bufs, 0, 1024, data, 512, 0, epochs)  # 2 KB message in a 1 KB buffer
    assert e.value.code == -1
    with pytest.raises(vsl.VslError) as e:
        vsl.p2p_allreduce(bufs, 2, 1024, data, 16, 0, epochs)  # rank out of range
    assert e.value.code == -1
    with pytest.raises(vsl.VslError) as e:
        vsl.p2p_allreduce(bufs, 0, 1024, data[1:], 16, 0, epochs)  # unaligned message
    assert e.value.code == -1


CFG = dict(n_layers=2, d_model=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512, vocab=1024, rope_theta=1e4,
           rms_eps=1e-5, wdtype=vsl.F16)


def test_device_status_is_returned_by_host_calls():
    with vsl.Engine.synthetic(CFG, seed=3, max_seq=128) as e:
        prompt = synth.synth_ids(3, 0, 10, CFG["vocab"]).tolist()
        nxt = e.prefill(prompt)[0]
        e.inject_status(-4)  # as a bounded wait that expired
        with pytest.raises(vsl.VslError) as err:
            e.step_host(np.array([nxt], np.int32))
        assert err.value.code == -4
        assert e.device_status() == -4
        e.reset()  # clears the word
        assert e.device_status() == 0
        e.prefill(prompt)
        e.inject_status(-5)
        with pytest.raises(vsl.VslError) as err:
            e.prefill(prompt[:3], seq=0)
        assert err.value.code == -5
        e.reset()
        ids = e.generate(prompt, 5)
        assert len(ids) == 5 and e.device_status() == 0


def test_generate_fills_exactly_max_seq():
    max_seq = 64
    with vsl.Engine.synthetic(CFG, seed=3, max_seq=max_seq) as e:
        prompt = synth.synth_ids(3, 1, 40, CFG["vocab"]).tolist()
        ids = e.generate(prompt, max_seq - len(prompt) + 1)  # the last sampled token takes no position
        assert len(ids) == max_seq - len(prompt) + 1
        assert e.positions(1)[0] == max_seq
        with pytest.raises(vsl.VslError) as err:
            e.generate(prompt, max_seq - len(prompt) + 2)
        assert err.value.code == -5
        # generate_batch takes the same bound
        n_out = e.generate_batch([prompt], max_seq - len(prompt) + 1)
        assert [len(x) for x in n_out] == [max_seq - len(prompt) + 1]
        assert n_out[0] == ids
