"""Host-side checks that need no GPU: the C-ABI library loads and exports
every declared entry point, the blob parser reproduces the reference
loader's accept/reject behaviour (csrc/bnn_model.c:66-96), the drop-in
bnn_load exits(1) with the reference's messages, and the Python blob
writer/reader round-trips."""

import ctypes
import os
import re
import struct
import subprocess
import sys

import numpy as np
import pytest

import bnns_to_c_b200 as bn
from bnns_to_c_b200 import blob as B

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
GOLD = os.path.join(ROOT, "tests", "golden")
C8 = os.path.join(GOLD, "unet_c8_mixed_s1.blob")
S8 = os.path.join(GOLD, "stem_c8_mixed_s3.blob")


def declared_functions():
    names = []
    for h in ("bnn_model.h", "bnn_b200.h", "bnn_model_stem.h", "bnn_model_react.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(bnn_\w+)\s*\(", src, flags=re.M):
            if "typedef" not in src[max(0, m.start() - 20):m.start() + 10]:
                names.append(m.group(1))
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(bn.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", bn.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    # only the C ABI is exported (no C++ or CUDA runtime internals)
    assert all(s.startswith("bnn_") for s in exported), sorted(s for s in exported if not s.startswith("bnn_"))


def test_load_parses_header_without_gpu():
    m = bn.Model(C8)
    assert (m.version, m.base_channels, m.n_bands, m.n_classes, m.upsampler) == (1, 8, 120, 3, 0)
    m.close()


def _status(data):
    L = bn.lib()
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(data, len(data))
    rc = L.bnn_load_mem(buf, len(data), ctypes.byref(h))
    if rc == 0:
        L.bnn_free(h.value)
    return rc, L.bnn_last_error().decode()


def test_loader_rejections_match_reference():
    data = open(C8, "rb").read()
    assert _status(data) == (0, "")
    assert _status(data[:100])[1] == "short read"
    assert _status(data[:-1])[1] == "short read"
    assert _status(data + b"\0")[1] == "trailing bytes in blob"
    assert _status(b"XNNC" + data[4:])[1] == "bad magic"
    assert _status(b"")[1] == "short read"
    # first conv tag -> 7
    bad = data[:24] + struct.pack("<i", 7) + data[28:]
    assert _status(bad)[1] == "bad conv tag 7"
    # locate the first act record: conv header 7 ints + wsign + alpha
    cout, cin = struct.unpack("<2i", data[28:36])
    act_off = 24 + 28 + cout * cin * 9 + cout * 4
    assert struct.unpack("<i", data[act_off:act_off + 4])[0] == 3
    bad = data[:act_off] + struct.pack("<i", 9) + data[act_off + 4:]
    assert _status(bad)[1] == "bad act tag 9"
    bad = data[:-(3 * 4 + 8 * 3 * 4 + 3 * 4)] + struct.pack("<i", 5) + data[-(2 * 4 + 8 * 3 * 4 + 3 * 4):]
    assert _status(bad)[1] == "bad head tag 5"


def test_loader_topology_validation():
    m = B.random_model(8, 120, 3, seed=4)
    m["enc2.act1"] = dict(m["enc2.act1"])
    good = B.blob_bytes(m)
    assert _status(good)[0] == 0
    # a real fold where the forward has an integer accumulator: the
    # reference would pass xreal = NULL to apply_fold_real
    m2 = B.random_model(8, 120, 3, seed=4)
    c = len(m2["enc2.act1"]["type"])
    m2["enc2.act1"] = {"kind": "real", "A": np.ones(c, np.float32), "B": np.zeros(c, np.float32),
                       "slope": np.ones(c, np.float32), "rsign": np.zeros(c, np.float32)}
    rc, msg = _status(B.blob_bytes(m2))
    assert rc == bn.BNN_ERR_UNSUPPORTED and "enc2.act1" in msg
    # channel chain broken: head sized for a different width
    m3 = B.random_model(8, 120, 3, seed=4)
    m3["head"]["W"] = np.zeros((3, 9), np.float32)
    rc, msg = _status(B.blob_bytes(m3))
    assert rc == bn.BNN_ERR_UNSUPPORTED and "head" in msg
    # 1x1 conv where the forward needs 3x3
    m4 = B.random_model(8, 120, 3, seed=4)
    m4["enc3.conv2"] = {"tag": "bin", "wsign": m4["enc3.conv2"]["wsign"][:, :, :1, :1], "pad": 0}
    rc, msg = _status(B.blob_bytes(m4))
    assert rc == bn.BNN_ERR_UNSUPPORTED and "enc3.conv2" in msg


def test_dropin_bnn_load_exits_like_reference(tmp_path):
    p = tmp_path / "t.blob"
    p.write_bytes(open(C8, "rb").read() + b"x")
    code = ("import ctypes,sys; L=ctypes.CDLL(sys.argv[1]); L.bnn_load.restype=ctypes.c_void_p; "
            "L.bnn_load(sys.argv[2].encode()); print('returned')")
    r = subprocess.run([sys.executable, "-c", code, bn.LIB_PATH, str(p)], capture_output=True, text=True)
    assert r.returncode == 1 and "trailing bytes in blob" in r.stderr and "returned" not in r.stdout
    r = subprocess.run([sys.executable, "-c", code, bn.LIB_PATH, str(tmp_path / "nope.blob")],
                       capture_output=True, text=True)
    assert r.returncode == 1 and "cannot open" in r.stderr


def test_arena_poison_setting():
    """BNN_ARENA_POISON is read as the reference's arena reads it (integer
    value & 255, csrc/bnn_react_arena.c:30); the setter overrides it and
    checks its range. No GPU needed: the setting is host state."""
    code = "import bnns_to_c_b200 as b; print(b.arena_poison())"
    for val, want in ((None, "None"), ("165", "165"), ("421", str(421 & 255)), ("0", "0")):
        env = {k: v for k, v in os.environ.items() if k != "BNN_ARENA_POISON"}
        if val is not None:
            env["BNN_ARENA_POISON"] = val
        r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
        assert r.returncode == 0, r.stderr
        assert r.stdout.strip() == want, (val, r.stdout)
    try:
        bn.set_arena_poison(7)
        assert bn.arena_poison() == 7
        bn.set_arena_poison(None)
        assert bn.arena_poison() is None
        for bad in (256, -2):
            with pytest.raises(bn.BnnError) as e:
                bn.set_arena_poison(bad)
            assert e.value.code == bn.BNN_ERR_ARG
    finally:
        bn.set_arena_poison(None)


def test_forward_without_gpu_raises_not_falls_back():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    m = bn.Model(C8)
    with pytest.raises(bn.BnnError) as e:
        m.forward(np.zeros((120, 32, 32), np.float32))
    assert e.value.code == bn.BNN_ERR_CUDA


def test_blob_roundtrip_and_committed_bytes():
    for name, base, rules, seed in (("unet_c8_mixed_s1", 8, "mixed", 1), ("unet_c16_base_s2", 16, "baseline", 2)):
        data = B.blob_bytes(B.random_model(base, 120, 3, seed=seed, rules=rules))
        assert data == open(os.path.join(GOLD, name + ".blob"), "rb").read()
    r = B.read_blob(C8)
    assert len(r["convs"]) == 18 and len(r["acts"]) == 22
    m = B.random_model(8, 120, 3, seed=1, rules="mixed")
    w = m["enc2.conv1"]["wsign"]
    assert np.array_equal(B.unpack_kidx(r["convs"][2]["packed"], w.shape[1], 3, 3), w)


def test_pack_kidx_bit_order():
    w = -np.ones((2, 1, 3, 3), np.int8)
    w[0, 0, 0, 0] = 1   # kidx 0
    w[1, 0, 2, 2] = 1   # kidx 8
    p = B.pack_kidx(w)
    assert p.shape == (2, 1) and int(p[0, 0]) == 1 and int(p[1, 0]) == 1 << 8


def test_cli_usage_matches_reference():
    r = subprocess.run([bn.CLI_PATH], capture_output=True, text=True)
    assert r.returncode == 1 and "usage:" in r.stderr and "input.bin|rand output.bin [H W [reps]]" in r.stderr


# ------------------------------------------------------------------ v2 (spectral stem)
def _stem_status(data):
    L = bn.lib()
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(data, len(data))
    rc = L.bnn_stem_load_mem(buf, len(data), ctypes.byref(h))
    if rc == 0:
        L.bnn_stem_free(h.value)
    return rc, L.bnn_last_error().decode()


def test_stem_load_parses_without_gpu():
    m = bn.StemModel(S8)
    assert (m.version, m.base_channels, m.n_bands, m.n_classes, m.upsampler) == (2, 8, 120, 3, 0)
    assert m.stem_channels == 16
    # the engine handle reads as a Model with the v2 body, and bnn_free on it
    # is a no-op (the StemModel owns it)
    hdr = bn._ModelHeader.from_address(m.handle)
    assert (hdr.version, hdr.n_bands) == (2, 120)
    bn.lib().bnn_free(m.handle)
    assert bn.lib().bnn_forward_launches(m.handle, 4, 32, 32) == 20
    m.close()


def test_stem_loader_rejections_match_reference():
    data = open(S8, "rb").read()
    assert _stem_status(data) == (0, "")
    assert _stem_status(data[:-1])[1] == "short read"
    assert _stem_status(data + b"\0")[1] == "trailing bytes in blob"
    assert _stem_status(b"XNNC" + data[4:])[1] == "bad magic"
    # csrc/bnn_model_stem.c:84-85 and 89-92
    assert _stem_status(open(C8, "rb").read())[1] == (
        "bnn_stem: expected v2 blob, got v1 (use the v1 engine for non-stem models)")
    for hs, ns in ((0, 1), (1, 2)):
        bad = data[:24] + struct.pack("<2i", hs, ns) + data[32:]
        assert _stem_status(bad)[1] == "bnn_stem: only has_stem=1, n_stem_layers=1 supported"
    bad = data[:32] + struct.pack("<i", 7) + data[36:]
    assert _stem_status(bad)[1] == "bad conv tag 7"
    # a v2 blob through the v1 loader misparses and is refused, not run
    assert _status(data)[0] != 0


def test_stem_topology_validation():
    def status(mut):
        m = B.random_model(8, 120, 3, seed=6, rules="mixed", stem_channels=12)
        mut(m)
        return _stem_status(B.blob_bytes(m))

    assert status(lambda m: None) == (0, "")
    # a 3x3 stem: the reference would run it; this engine refuses it
    rc, msg = status(lambda m: m["stem.conv"].update(wsign=np.ones((12, 120, 3, 3), np.int8), pad=1))
    assert rc == bn.BNN_ERR_UNSUPPORTED and "stem.conv" in msg
    # stem weights other than -1 / 0 / +1
    def big(m):
        m["stem.conv"]["wsign"] = m["stem.conv"]["wsign"].copy()
        m["stem.conv"]["wsign"][3, 7, 0, 0] = 2
    rc, msg = status(big)
    assert rc == bn.BNN_ERR_UNSUPPORTED and "wsign" in msg
    # zero weights (np.sign of an exact 0.0) are accepted
    def zero(m):
        m["stem.conv"]["wsign"] = m["stem.conv"]["wsign"].copy()
        m["stem.conv"]["wsign"][:, ::5] = 0
    assert status(zero) == (0, "")
    # enc1.conv1 must be binary on the stem's channels
    def chain(m):
        m["stem.act"] = {k: (v[:10] if isinstance(v, np.ndarray) else v) for k, v in m["stem.act"].items()}
        m["stem.conv"] = dict(m["stem.conv"], wsign=m["stem.conv"]["wsign"][:10], alpha=m["stem.conv"]["alpha"][:10])
    rc, msg = status(chain)
    assert rc == bn.BNN_ERR_UNSUPPORTED and "enc1.conv1" in msg


def test_v1_first_conv_weights_checked():
    m = B.random_model(8, 120, 3, seed=4)
    m["enc1.conv1"] = dict(m["enc1.conv1"], wsign=m["enc1.conv1"]["wsign"].copy())
    m["enc1.conv1"]["wsign"][0, :, 1, 1] = 0
    assert _status(B.blob_bytes(m)) == (0, "")
    m["enc1.conv1"]["wsign"][0, 0, 0, 0] = -3
    rc, msg = _status(B.blob_bytes(m))
    assert rc == bn.BNN_ERR_UNSUPPORTED and "enc1.conv1" in msg


def test_dropin_bnn_stem_load_exits_like_reference(tmp_path):
    code = ("import ctypes,sys; L=ctypes.CDLL(sys.argv[1]); L.bnn_stem_load.restype=ctypes.c_void_p; "
            "L.bnn_stem_load(sys.argv[2].encode()); print('returned')")
    r = subprocess.run([sys.executable, "-c", code, bn.LIB_PATH, C8], capture_output=True, text=True)
    assert r.returncode == 1 and "expected v2 blob, got v1" in r.stderr and "returned" not in r.stdout


def test_stem_blob_writer_matches_committed_fixtures():
    for name, base, rules, seed in (("stem_c8_mixed_s3", 8, "mixed", 3), ("stem_c16_base_s4", 16, "baseline", 4)):
        data = B.blob_bytes(B.random_model(base, 120, 3, seed=seed, rules=rules, stem_channels=16))
        assert data == open(os.path.join(GOLD, name + ".blob"), "rb").read()
        rt = B.read_blob(os.path.join(GOLD, name + ".blob"))
        assert rt["has_stem"] == 1 and rt["stem_conv"]["wsign"].shape == (16, 120, 1, 1)


def test_stem_cli_usage_matches_reference():
    r = subprocess.run([bn.CLI_STEM_PATH], capture_output=True, text=True)
    assert r.returncode == 1 and "usage:" in r.stderr and "weights_stem.blob" in r.stderr


def test_cli_error_paths_match_reference(tmp_path):
    """The CLIs' host-side failures, reached before any forward (so no GPU):
    the reference's messages and exit statuses (csrc/main.c:36-46,
    csrc/main_stem.c, csrc/main_react.c)."""
    short = tmp_path / "short.bin"
    short.write_bytes(b"\0" * 64)
    out = str(tmp_path / "o.bin")
    for cli, blob in ((bn.CLI_PATH, C8), (bn.CLI_STEM_PATH, S8)):
        for inp in (str(short), str(tmp_path / "missing.bin")):
            r = subprocess.run([cli, blob, inp, out], capture_output=True, text=True, timeout=60)
            assert (r.returncode, r.stderr.strip()) == (1, "bad input file"), (cli, inp, r.stderr)
        r = subprocess.run([cli, str(tmp_path / "nope.blob"), "rand", out], capture_output=True, text=True)
        assert r.returncode == 1 and "cannot open" in r.stderr
    cases = [
        ([R8, "rand", out, "0", "32"], 2, "bad H/W/reps"),
        ([R8, "rand", out, "32", "32", "0"], 2, "bad H/W/reps"),
        ([R8, "patch:rand", out, "32", "32"], 2, "bad patch spec 'patch:rand' (use patch32:FILE)"),
        ([R8, "patch24:rand", out, "48", "48"], 2, "patch size must be a multiple of 16"),
        ([R8, "mem:" + str(short), out, "32", "32"], 1, f"bad input {short}"),
        ([R8, "mem:" + str(tmp_path / "missing.bin"), out, "32", "32"], 1, f"bad input {tmp_path / 'missing.bin'}"),
        ([R8, str(tmp_path / "missing.bin"), out, "32", "32"], 1, f"cannot open {tmp_path / 'missing.bin'}"),
        ([R8, str(short), out, "32", "32"], 1, "file_reader: short read of the [120,32,32] cube"),
        ([R8, "patch32:" + str(short), out, "32", "32"], 1, "file_reader: short read of the [120,32,32] cube"),
        ([str(tmp_path / "nope.blob"), "patch24:rand", out, "32", "32"], 1, f"cannot open {tmp_path / 'nope.blob'}"),
    ]
    for args, code, msg in cases:
        r = subprocess.run([bn.CLI_REACT_PATH] + args, capture_output=True, text=True, timeout=60)
        assert (r.returncode, r.stderr.strip()) == (code, msg), (args, r.stderr)
    r = subprocess.run([bn.CLI_REACT_PATH], capture_output=True, text=True)
    assert r.returncode == 2 and "usage:" in r.stderr


# ------------------------------------------------------------------ v3 ReActNet
R8 = os.path.join(GOLD, "react_c8_s3.blob")


def _react_status(data):
    L = bn.lib()
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(data, len(data))
    rc = L.bnn_react_load_mem(buf, len(data), ctypes.byref(h))
    if rc == 0:
        L.bnn_free_react(h.value)
    return rc, L.bnn_last_error().decode()


def test_react_loader_matches_reference():
    """csrc/bnn_model_react.c:42-135: messages and structural checks."""
    from bnns_to_c_b200 import blob_react as BR
    data = open(R8, "rb").read()
    assert _react_status(data) == (0, "")
    m = bn.ReactModel(R8)
    assert (m.version, m.base_channels, m.n_bands, m.n_classes) == (3, 8, 120, 3)
    m.close()
    assert _react_status(data[:-1])[1] == "short read"
    assert _react_status(data + b"\0")[1] == "trailing bytes in blob"
    assert _react_status(b"XNNC" + data[4:])[1] == "bad magic"
    assert _react_status(open(C8, "rb").read())[1] == "blob version 1, this engine reads v3 (ReActNet)"
    assert _react_status(data[:20] + struct.pack("<i", 1) + data[24:])[1] == "only nearest upsampler supported"
    # enc1's first record is its conv (no tap1): tag 7 there
    assert _react_status(data[:24] + struct.pack("<i", 7) + data[28:])[1] == "bad conv tag 7"
    # a tap whose width does not match its conv
    mdl = BR.random_react_model(8, 120, 3, seed=3)
    mdl["blocks"]["enc2"]["tap2"] = mdl["blocks"]["enc2"]["tap2"][:5]
    assert _react_status(BR.react_blob_bytes(mdl))[1] == "blob layout mismatch: tap2 channels"
    # a channel chain the forward cannot run: refused at load
    mdl = BR.random_react_model(8, 120, 3, seed=3)
    mdl["head"]["W"] = mdl["head"]["W"][:, :4]
    rc, msg = _react_status(BR.react_blob_bytes(mdl))
    assert rc == bn.BNN_ERR_UNSUPPORTED and "head" in msg


def test_react_dropin_load_exits_like_reference(tmp_path):
    code = ("import ctypes,sys; L=ctypes.CDLL(sys.argv[1]); L.bnn_load_react.restype=ctypes.c_void_p; "
            "L.bnn_load_react(sys.argv[2].encode()); print('returned')")
    r = subprocess.run([sys.executable, "-c", code, bn.LIB_PATH, S8], capture_output=True, text=True)
    assert r.returncode == 1 and "blob version 2, this engine reads v3" in r.stderr and "returned" not in r.stdout
