"""Every engine and tokenizer entry point of the C ABI refuses a NULL handle (and NULL output
pointers) with an error status instead of dereferencing it. No GPU is needed: the calls are
checked before any device work. They run in a child process, so a crash fails the test."""
import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import ctypes as C, os, sys
    sys.path.insert(0, os.path.join(sys.argv[1], "vulkan-symbiote-loader_b200"))
    import vsl
    L = vsl.lib()
    N = None
    i32 = (C.c_int32 * 8)()
    i = C.c_int()
    u32 = C.c_uint32()
    u64 = C.c_uint64()
    d = C.c_double()
    sz = C.c_size_t()
    f = (C.c_float * 8)()
    cfg = vsl.ModelConfig()
    calls = {
        "vsl_engine_get_config": (N, C.byref(cfg)),
        "vsl_engine_reset": (N,),
        "vsl_engine_fill_kv_synthetic": (N, C.c_uint64(1), C.c_double(1.0), 4, 1),
        "vsl_engine_set_forced": (N, i32, 1, 1),
        "vsl_engine_run": (N, 1, 1, C.c_float(0.0), C.c_uint64(0)),
        "vsl_engine_step_host": (N, i32, 1, i32, f),
        "vsl_engine_read_tokens": (N, 1, 1, i32),
        "vsl_engine_positions": (N, 1, i32),
        "vsl_engine_generate": (N, i32, 2, 2, C.c_float(0.0), C.c_uint64(0), i32, 1, i32, C.byref(i)),
        "vsl_engine_step_stats": (N, 1, C.byref(i), C.byref(d)),
        "vsl_engine_memory_stats": (N, C.byref(sz), C.byref(sz), C.byref(sz)),
        "vsl_engine_prefill": (N, i32, 2, 0, i32, f),
        "vsl_engine_generate_batch": (N, i32, i32, 1, 2, C.c_float(0.0), C.c_uint64(0), i32, 1, i32, i32),
        "vsl_engine_reset_seq": (N, 0),
        "vsl_engine_residency": (N, C.byref(u32), C.byref(u32), C.byref(u64), C.byref(u64)),
        "vsl_engine_device_status": (N, C.byref(i)),
        "vsl_tokenizer_info": (N, C.byref(i), C.byref(i), i32, i32),
        "vsl_tokenize": (N, b"ab", 2, i32, 8, C.byref(i)),
        "vsl_detokenize": (N, i32, 1, C.create_string_buffer(8), 8, C.byref(sz)),
        "vsl_tokenizer_create_gguf": (N, N),
        "vsl_engine_create_gguf": (N, N, N),
        "vsl_engine_create_synthetic": (N, C.c_uint64(0), C.c_double(0.02), N, N),
        "vsl_gguf_model_config": (N, N),
    }
    bad = []
    for name, args in calls.items():
        rc = getattr(L, name)(*args)
        if rc >= 0:
            bad.append((name, rc))
    L.vsl_engine_destroy(N)     # destroying NULL is a no-op (status ignored)
    L.vsl_tokenizer_destroy(N)
    if L.vsl_engine_stream(N):
        bad.append(("vsl_engine_stream", "non-null"))
    print("bad", bad)
""")


def test_null_handles_are_refused():
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.returncode, r.stderr[-2000:])
    assert r.stdout.strip().splitlines()[-1] == "bad []", r.stdout
