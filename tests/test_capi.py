"""C ABI surface checks that need no GPU: the library loads, exports every function that
include/vsl.h declares, and rejects invalid arguments before touching the device."""
import ctypes as C
import subprocess

import pytest

import vsl


def test_library_exports_every_header_function():
    names = vsl.header_functions()
    assert len(names) >= 25
    L = vsl.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", vsl.LIB_PATH], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
    assert set(names) <= exported
    # the C ABI (vsl_*) and the C++ API classes (namespace vk_symbiote) are the only exports
    stray = [n for n in exported if not n.startswith("vsl_") and "11vk_symbiote" not in n]
    assert not stray, stray[:10]


def test_version_and_error_string():
    assert vsl.lib().vsl_version() >= 1
    with pytest.raises(vsl.VslError) as e:
        vsl.gemv(vsl.F16, 0, 16, 16, 0, 1, 0)
    assert e.value.code == -1 and "null" in str(e.value)


def test_invalid_arguments_rejected_without_device():
    with pytest.raises(vsl.VslError) as e:
        vsl.gemv(99, 16, 16, 16, 16, 1, 16)
    assert e.value.code == -9
    with pytest.raises(vsl.VslError) as e:
        vsl.flash_decode(0, 0, 0, vsl.F16, 0, 1, 64, 0, 1, 8, 2, 128, 64, 64, 0, 0, 0)
    assert e.value.code == -1
    with pytest.raises(vsl.VslError):
        vsl.flash_decode_workspace_size(0, 8, 2, 128, 64, 64)
    assert vsl.flash_decode_workspace_size(2, 8, 2, 128, 300, 64) > 2 * 8 * 5 * 128 * 4
    with pytest.raises(vsl.VslError) as e:
        vsl.qkv_rope_append(vsl.F16, 16, 6, 4, 64, 64, 16, 16, 1e-5, 1, 16, 16, 16, 16, 16, 16, vsl.F16, 16, 1, 64)
    assert e.value.code == -1  # 6 heads over 4 KV heads is not a valid grouping


def test_engine_config_validation_without_device():
    base = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1376, vocab=4096,
                rope_theta=1e4, rms_eps=1e-5, wdtype=vsl.F16)
    for bad, code in [(dict(head_dim=96), -9), (dict(n_kv_heads=3), -9), (dict(wdtype=5), -9),
                      (dict(n_layers=0), -1)]:
        with pytest.raises(vsl.VslError) as e:
            vsl.Engine.synthetic({**base, **bad})
        assert e.value.code == code, bad
    with pytest.raises(vsl.VslError) as e:
        vsl.Engine.synthetic(base, tp_size=3, tp_rank=0)
    assert e.value.code == -9  # 8 heads do not split over 3 ranks
    with pytest.raises(vsl.VslError) as e:
        vsl.Engine.synthetic(base, tp_size=2, tp_rank=0)  # no NCCL id
    assert e.value.code in (-1, -2)


def test_default_options():
    o = vsl.default_options()
    assert o.max_batch == 1 and o.tp_size == 1 and o.use_graph == 1 and o.kv_dtype == -1 and o.page_size == 64
    # tensor parallel: peer-memory all-reduce kernel by default; a bounded host wait on the ranks
    assert o.use_p2p == 1 and o.use_pdl == 1 and o.use_fused == 0 and o.nccl_timeout_ms == 120000


@pytest.mark.parametrize("change,code", [
    (dict(n_kv_heads=3), -9),                  # query heads not a multiple of KV heads
    (dict(n_layers=0), -1), (dict(vocab=-5), -1), (dict(d_model=0), -1),
    (dict(head_dim=63), -9),                   # head_dim 64 or 128
    (dict(wdtype=77), -9),                     # not a weight type
    (dict(wdtype=vsl.Q8_0, ffn=1370), -9),     # quantized rows need K % 32 == 0
])
def test_invalid_model_configs_refused_before_device_work(change, code):
    cfg = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1376, vocab=4096,
               rope_theta=10000.0, rms_eps=1e-5, wdtype=vsl.F16)
    cfg.update(change)
    with pytest.raises(vsl.VslError) as e:
        vsl.Engine.synthetic(cfg, seed=0, device=0, max_seq=128)
    assert e.value.code == code, str(e.value)
