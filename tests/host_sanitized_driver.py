"""Drives the host C code of a libdiolkos build given on the command line (the AddressSanitizer + UBSan
build of tests/test_host_sanitized.py) through the CPU paths of the reference API: the tokenizer on
random and malformed text, the safetensors / JSON loader reading a Q8_0 cache, the tensor helpers and
the random stream.  Results are checked against the oracle's restatements; the sanitizers check every
access on the way.  Usage: python tests/host_sanitized_driver.py <library> <scratch dir>."""
import ctypes as C
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from diolkos_b200 import _native  # noqa: E402

_native.LIB_PATH = os.path.abspath(sys.argv[1])
scratch = sys.argv[2]

import numpy as np  # noqa: E402

from diolkos_b200 import refapi, synth  # noqa: E402
from oracle import Port  # noqa: E402
from oracle import tokenizer_port as TP  # noqa: E402
from tests import test_host_api as H  # noqa: E402

L = refapi.lib()
with open("/proc/self/maps") as f:
    maps = f.read()
assert "libasan" in maps and "libubsan" in maps, "the sanitizer runtimes are not loaded"
assert os.path.basename(_native.LIB_PATH) in maps, "the library under test is not the one loaded"

# tokenizer: random text, malformed UTF-8, byte fallback, empty strings
pieces, scores, words = H.make_vocab(11)
vocab_path = os.path.join(scratch, "tokenizer.bin")
H.write_tokenizer_bin(vocab_path, pieces, scores)
tok = refapi.load_tokenizer(vocab_path)
f32_scores = [np.float32(s) for s in scores]
for text in H.random_texts(3, words, n=40):
    for bos, eos in ((True, False), (False, True)):
        got = refapi.encode(tok, text, bos, eos)
        assert got == TP.encode(pieces, f32_scores, text, bos, eos), text
        prev = 1
        for t in got:
            refapi.decode(tok, prev, t)
            prev = t

# loader: config.json with nested members, every Q8_0 tensor from the cache, F32 norms widened and cached
port = Port()
d = H._write_small_model(scratch)
cache = os.path.join(scratch, "cache", "small-model")
want = H._expected_tensors(port)
for name, v in want.items():
    if v[0] == "q8":
        synth.write_q8_cache(cache, name, v[1], v[2])
old = os.getcwd()
os.chdir(scratch)
try:
    m = L.load_safetensors(d.encode()).contents
    got = H._model_tensors(m)
    for name, t in got.items():
        if want[name][0] == "q8":
            q, s = t.q8()
            assert np.array_equal(q, want[name][1]) and np.array_equal(s.view(np.uint32), want[name][2].view(np.uint32))
        else:
            assert np.array_equal(t.f32(), want[name][1])
    # the same directory again: now every tensor, the norms included, comes from the cache
    m2 = L.load_safetensors(d.encode()).contents
    for name, t in H._model_tensors(m2).items():
        if want[name][0] == "f32":
            assert np.array_equal(t.f32(), want[name][1])
finally:
    os.chdir(old)

# tensor helpers
for n in (32, 64, 4096):
    t = L.tensor_create(n, refapi.Q8_0)
    assert L.Tensor_storage_size(t) == n + (n // 32) * 4
    L.tensor_destroy(t)
    t = L.tensor_create(n, refapi.F32)
    assert L.convert(t, refapi.F32).contents.data == t.contents.data
    L.tensor_destroy(t)

# random stream
for seed in (1, 0x123456789ABCDEF):
    a = C.c_ulonglong(seed)
    s = seed
    for _ in range(100):
        u = L.random_u32(C.byref(a))
        w, s = TP.random_u32(s)
        assert u == w

print("host code ok")
