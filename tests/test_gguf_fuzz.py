"""The C++ GGUF reader on damaged files, no GPU needed: a small model file with a vocabulary and
merges, with random bytes of its header and metadata overwritten or the file cut short, goes
through GGUFLoader (model config, tensor lookup) and Tokenizer::from_gguf. Every call must
return (an error status is fine); the loop runs in a child process with a bounded address
space, so a crash or a runaway allocation fails the test instead of the suite."""
import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import os, random, resource, sys
    resource.setrlimit(resource.RLIMIT_AS, (8 << 30, 8 << 30))
    sys.path.insert(0, os.path.join(sys.argv[1], "vulkan-symbiote-loader_b200"))
    import numpy as np
    import vsl
    from vsl import gguf, synth
    tmp = sys.argv[2]
    shape = gguf.LlamaShape(1, 64, 2, 2, 128, 40)
    toks = [f"t{i}" for i in range(40)]
    meta = gguf.llama_metadata(shape) + [
        ("tokenizer.ggml.model", gguf.T_STR, "gpt2"),
        ("tokenizer.ggml.pre", gguf.T_STR, "llama-bpe"),
        ("tokenizer.ggml.tokens", gguf.T_ARR, (gguf.T_STR, toks)),
        ("tokenizer.ggml.token_type", gguf.T_ARR, (gguf.T_I32, [1] * 40)),
        ("tokenizer.ggml.merges", gguf.T_ARR, (gguf.T_STR, ["t 1", "t 2", "t1 0"])),
        ("tokenizer.ggml.scores", gguf.T_ARR, (gguf.T_F32, [0.0] * 40))]
    tensors = [("token_embd.weight", np.zeros((40, 64), np.float16), synth.GGML_F16),
               ("output_norm.weight", np.ones(64, np.float32), synth.GGML_F32)]
    src = os.path.join(tmp, "base.gguf")
    gguf.write_gguf(src, meta, tensors)
    data = bytearray(open(src, "rb").read())
    head = min(len(data), 2048)  # header, metadata and tensor infos
    rng = random.Random(int(sys.argv[3]))
    n_err = 0
    for it in range(int(sys.argv[4])):
        d = bytearray(data)
        mode = rng.random()
        if mode < 0.7:
            for _ in range(rng.randrange(1, 6)):
                d[rng.randrange(8, head)] = rng.randrange(256)
        elif mode < 0.9:  # a length or count field set huge
            p = rng.randrange(8, head - 8)
            d[p:p + 8] = rng.choice([b"\\xff" * 8, b"\\xff\\xff\\xff\\x7f" + b"\\0" * 4, (1 << 40).to_bytes(8, "little")])
        else:
            d = d[:rng.randrange(0, len(d))]
        p = os.path.join(tmp, "m.gguf")
        open(p, "wb").write(bytes(d))
        for call in (lambda: vsl.gguf_model_config(p), lambda: vsl.gguf_tensor_info(p, "token_embd.weight")):
            try:
                call()
            except vsl.VslError:
                n_err += 1
        t = vsl.Tokenizer(p)
        t.decode(t.encode("t1 t2 hello"))
        t.close()
    print("done", n_err, flush=True)
""")


def test_damaged_gguf_files_never_crash_the_reader(tmp_path):
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT, str(tmp_path), "1", "400"], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, (r.returncode, r.stderr[-2000:])
    last = r.stdout.strip().splitlines()[-1].split()
    assert last[0] == "done" and int(last[1]) > 100  # most damaged files are refused
