"""The blob loaders (loader.cpp, loader_react.cpp) built with AddressSanitizer,
LeakSanitizer and UndefinedBehaviorSanitizer, host only
(tests/san/loader_harness.cpp stubs the device engine), over corrupted blobs.

The corruptions are seeded:
- truncations;
- overwritten header and record words (tags, shapes, counts, including
  negative and huge values);
- single-byte flips;
- trailing bytes.

Every case must end with no sanitizer report and no leak. It must also give
the same status and message as the shipped library gives in-process for the
same bytes. The checks restated are the reference loaders'
(csrc/bnn_model.c:27-96, csrc/bnn_model_stem.c, csrc/bnn_model_react.c:42-135).
The reference exits on every error; here each one is a status."""

import ctypes
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

import bnns_to_c_b200 as bn

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLD = os.path.join(HERE, "golden")
CSRC = os.path.join(ROOT, "bnns_to_c_b200", "csrc")
BLOBS = {"v1": "unet_c8_mixed_s1.blob", "stem": "stem_c8_mixed_s3.blob", "react": "react_c8_s3.blob"}
SAN = "-fsanitize=address,undefined"


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no g++")
    exe = str(tmp_path_factory.mktemp("san") / "loader_harness")
    cmd = [cxx, "-std=c++17", "-O1", "-g", SAN, "-fno-sanitize-recover=all", "-fno-omit-frame-pointer",
           "-I" + os.path.join(ROOT, "include"), os.path.join(CSRC, "loader.cpp"),
           os.path.join(CSRC, "loader_react.cpp"), os.path.join(HERE, "san", "loader_harness.cpp"), "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return exe


def _lib_status(kind, data):
    """Status and message of the shipped library's loader for `data`."""
    L = bn.lib()
    load, free = {"v1": (L.bnn_load_mem, L.bnn_free), "stem": (L.bnn_stem_load_mem, L.bnn_stem_free),
                  "react": (L.bnn_react_load_mem, L.bnn_free_react)}[kind]
    out = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(data, max(len(data), 1))
    load.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]
    load.restype = ctypes.c_int
    rc = load(buf, len(data), ctypes.byref(out))
    msg = L.bnn_last_error().decode()
    if out.value:
        free.argtypes = [ctypes.c_void_p]
        free(out)
    return rc, msg


def _mutants(data, seed):
    """Seeded corruptions of one blob: (label, bytes)."""
    rng = np.random.RandomState(seed)
    n = len(data)
    out = [("trail0", data + b"\0"), ("trail7", data + bytes(rng.randint(0, 256, 7).astype(np.uint8)))]
    cuts = {0, 1, 3, 4, 8, 20, 23, 24, 27, 28, 36, 52, n - 4, n - 1}
    cuts |= set(int(c) for c in rng.randint(0, n, 40))
    out += [(f"cut{c}", data[:c]) for c in sorted(c for c in cuts if 0 <= c < n)]
    vals = [-1, 0, 1, 2, 3, 7, 9, 255, 65536, 2**31 - 1, -2**31, 1 << 20]
    # header and the first records' words, then words anywhere
    offs = list(range(0, min(n - 4, 256), 4)) + [int(o) * 4 for o in rng.randint(0, (n - 4) // 4, 60)]
    for o in offs:
        v = vals[rng.randint(len(vals))] if rng.rand() < 0.8 else int(rng.randint(-2**31, 2**31 - 1))
        out.append((f"w{o}={v}", data[:o] + struct.pack("<i", v) + data[o + 4:]))
    for _ in range(40):
        o = int(rng.randint(n))
        out.append((f"b{o}", data[:o] + bytes([data[o] ^ (1 << int(rng.randint(8)))]) + data[o + 1:]))
    return out


@pytest.mark.parametrize("kind", sorted(BLOBS))
def test_loader_sanitized_on_corrupted_blobs(kind, harness, tmp_path):
    data = open(os.path.join(GOLD, BLOBS[kind]), "rb").read()
    cases = [("intact", data)] + _mutants(data, seed={"v1": 1, "stem": 2, "react": 3}[kind])
    paths = []
    for i, (_, b) in enumerate(cases):
        p = tmp_path / f"m{i:04d}.blob"
        p.write_bytes(b)
        paths.append(str(p))
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0:exitcode=99",
               UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1:exitcode=98")
    r = subprocess.run([harness, kind] + paths, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-4000:]
    assert "Sanitizer" not in r.stderr and "runtime error" not in r.stderr, r.stderr[-4000:]
    lines = r.stdout.rstrip("\n").split("\n")
    assert len(lines) == len(cases)
    rejected = 0
    for (label, b), line in zip(cases, lines):
        rc_s, _, msg = line.partition("\t")
        want = _lib_status(kind, b)
        assert (int(rc_s), msg) == want, (label, line, want)
        rejected += want[0] != 0
        if label.startswith(("cut", "trail")):
            assert want[0] != 0, label  # a blob of the wrong length never loads
    assert lines[0] == "0\t"
    # many overwritten words land in weight data and still load; the rest are refused
    assert rejected >= len(cases) // 3
