"""Generate the golden fixtures under tests/golden/ from the REFERENCE itself.

Run in a container that has the reference tree (--ref, or the BNN_REFERENCE
environment variable) and
the reference build from ``make -C oracle`` (oracle/_ref/). The GPU box has
neither; it only reads the committed outputs of this script.

What it records:
  * blob byte-identity: each fixture model is written twice, once by
    ``bnns_to_c_b200.blob`` and once by the reference's own record emitters
    (python/bnn2c/blob.py:67-114, driven in the order of its v1 writer
    :181-199) from equivalent torch modules; the script fails unless the
    bytes are identical, then saves the blob.
  * whole-net stages: the reference kernels, unmodified, chained in
    bnn_forward order by oracle/ref_stages.c (and, for the v2 spectral-stem
    models, in bnn_stem_forward order by oracle/ref_stages_stem.c, logits
    checked against the reference stem CLI csrc/main_stem.c) -> every P, every +-1 plane,
    the real conv output and the logits, for seeded synthetic inputs; plus
    the logits of the reference CLI (csrc/main.c) on the same input, which
    must equal the chained logits exactly.
  * v3 ReActNet models (csrc/bnn_model_react.c): blob bytes against the
    reference's writer (python/bnn2c/blob_react.py:write_blob_react_from_fold,
    fed the same folded parameters); every stage from the reference's ReAct
    kernels chained by oracle/ref_stages_react.c; the chain's logits must equal
    the reference's own bnn_forward_react (strip-processed enc1/dec1) and the
    reference CLI csrc/main_react.c (file input, streamed).
  * kernel cases: reference bconv_dispatch P on the edge-shape list of
    csrc/bench_bconv.c:103-107 and on the pad=0 self-test case of
    python/verify/bconv_harness.py:113-118; maxpool_P on the shapes of
    python/verify/maxpool_harness.py:77.

usage: python tests/golden/make_golden.py --ref <reference tree>
"""

from __future__ import annotations

import argparse
import ctypes
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, ROOT)

from bnns_to_c_b200 import blob as B  # noqa: E402
from bnns_to_c_b200 import blob_react as BR  # noqa: E402

sys.path.insert(0, os.path.join(ROOT, "tests"))
from oracle_util import bind_kernel_abi  # noqa: E402

STAGE_CB = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int,
                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p)
DT = {0: np.int8, 1: np.int32, 2: np.float32}

# (name, base, rules, model seed, [(H, W, synth seed, n patches)])
MODELS = [
    ("unet_c8_mixed_s1", 8, "mixed", 1, [(32, 32, 7, 2), (37, 23, 8, 1)]),
    ("unet_c16_base_s2", 16, "baseline", 2, [(32, 32, 9, 1), (16, 48, 10, 1)]),
]
# base 32 (benchmark widths): blob not committed (1 MB); pinned by sha256
C32 = ("unet_c32_base_s0", 32, "baseline", 0, [(32, 32, 11, 1)])
# v2 spectral-stem models (csrc/bnn_model_stem.c): (name, base, rules, seed,
# stem channels, runs); the reference default stem width is 16
# (python/bnn2c/export.py:120)
STEMS = [
    ("stem_c8_mixed_s3", 8, "mixed", 3, 16, [(32, 32, 12, 2), (37, 23, 13, 1)]),
    ("stem_c16_base_s4", 16, "baseline", 4, 16, [(32, 32, 14, 1), (16, 48, 15, 1)]),
]


# v3 ReActNet models: (name, base, model seed, [(H, W, synth seed, n patches)])
REACTS = [
    ("react_c16_s1", 16, 1, [(32, 32, 21, 1)]),
    ("react_c8_s3", 8, 3, [(50, 38, 23, 1)]),
    ("react_c12_s4", 12, 4, [(32, 32, 24, 1)]),
]


def ref_react_blob_bytes(model: dict, ref: str) -> bytes:
    """The reference's own v3 writer on the same folded parameters."""
    sys.path.insert(0, os.path.join(ref, "python", "bnn2c"))
    import blob_react as RR  # the reference's python/bnn2c/blob_react.py
    fold = {}
    for name in BR.BLOCKS:
        b = model["blocks"][name]
        f = {"input_real": b["input_real"], "conv1_wsign": b["conv1"]["wsign"],
             "conv1_alpha": b["conv1"].get("alpha"), "proj1_W": b["proj"], "epi1": b["epi1"],
             "tap1_rsign": b["tap1"], "tap2_rsign": b["tap2"], "conv2_wsign": b["conv2"]["wsign"]}
        if b["kind"] == "down":
            f["epi_skip"], f["epi_down"] = b["epi_a"], b["epi_b"]
        else:
            f["epi2"] = b["epi_a"]
        fold[name] = f
    fold["outc_W"], fold["outc_b"] = model["head"]["W"], model["head"]["bias"]
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "r.blob")
        RR.write_blob_react_from_fold(fold, p, model["base_channels"], model["n_bands"], model["n_classes"])
        return open(p, "rb").read()


def ref_react_lib():
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_react.so"))
    lib.ref_react_stages.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_void_p, STAGE_CB, ctypes.c_void_p]
    lib.ref_react_forward.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p]
    return lib


def react_fixtures(ref, manifest):
    lib = ref_react_lib()
    for name, base, seed, runs in REACTS:
        model = BR.random_react_model(base, 120, 3, seed=seed)
        data = BR.react_blob_bytes(model)
        if data != ref_react_blob_bytes(model, ref):
            raise SystemExit(f"{name}: v3 blob bytes differ from the reference writer's")
        sha = hashlib.sha256(data).hexdigest()
        bpath = os.path.join(HERE, name + ".blob")
        open(bpath, "wb").write(data)
        for H, W, sseed, n in runs:
            x = synth(sseed, 0, n, 120, H, W)
            out = {"H": np.int32(H), "W": np.int32(W), "seed": np.int32(sseed), "n": np.int32(n),
                   "blob_sha256": np.array(sha)}
            for p in range(n):
                xp = np.ascontiguousarray(x[p])
                stages = {}

                def cb(ctx, nm, kind, C, h, w, d):
                    k = C * h * w
                    arr = np.ctypeslib.as_array(ctypes.cast(d, ctypes.POINTER(
                        {0: ctypes.c_int8, 1: ctypes.c_int32, 2: ctypes.c_float}[kind])), shape=(max(k, 1),))
                    stages[nm.decode()] = arr[:k].copy().reshape(C, h, w)
                lg = np.zeros((3, H, W), np.float32)
                lib.ref_react_stages(bpath.encode(), xp.ctypes.data, H, W, lg.ctypes.data, STAGE_CB(cb), None)
                fw = np.zeros((3, H, W), np.float32)
                lib.ref_react_forward(bpath.encode(), xp.ctypes.data, H, W, fw.ctypes.data)
                if not np.array_equal(fw.view(np.int32), stages["logits"].view(np.int32)):
                    raise SystemExit(f"{name}: bnn_forward_react logits != chained stage logits")
                with tempfile.TemporaryDirectory() as d:
                    inp, o = os.path.join(d, "in.bin"), os.path.join(d, "out.bin")
                    xp.astype("<f4").tofile(inp)
                    subprocess.run([os.path.join(ROOT, "oracle", "_ref", "bnn_infer_react"), bpath, inp, o,
                                    str(H), str(W)], check=True, capture_output=True,
                                   env=dict(os.environ, OMP_NUM_THREADS="1"))
                    cli = np.fromfile(o, "<f4").reshape(3, H, W)
                if not np.array_equal(cli.view(np.int32), stages["logits"].view(np.int32)):
                    raise SystemExit(f"{name}: bnn_infer_react logits != chained stage logits")
                for k, v in stages.items():
                    out[f"p{p}/{k}"] = v
            np.savez_compressed(os.path.join(HERE, f"{name}_{H}x{W}.npz"), **out)
            manifest.append(f"{name} {H}x{W} seed={sseed} n={n} blob_sha256={sha}")


def ref_blob_bytes(model: dict, ref: str) -> bytes:
    """Write ``model`` through the reference's own emitters."""
    import torch
    sys.path.insert(0, os.path.join(ref, "python", "verify"))
    sys.path.insert(0, os.path.join(ref, "python", "bnn2c"))
    import blob as RB  # the reference's python/bnn2c/blob.py

    def conv_mod(c, alpha=None):
        w = c["wsign"].astype(np.float32)
        if alpha is not None:
            w = w * alpha[:, None, None, None]
        cout, cin, kh, kw = w.shape
        mod = torch.nn.Conv2d(cin, cout, (kh, kw), padding=c.get("pad", 1),
                              stride=c.get("stride", 1), bias=False)
        with torch.no_grad():
            mod.weight.copy_(torch.from_numpy(w))
        return mod

    def rule(a):
        if a["kind"] == "int":
            return ("int", None, a["type"], a["t"], a["lo"], a["hi"])
        return ("real", None, a["A"], a["B"], a["slope"], a["rsign"])

    path = tempfile.mktemp(suffix=".blob")
    import struct
    stem = "stem.conv" in model
    with open(path, "wb") as f:
        f.write(RB.MAGIC)
        if stem:  # the v2 header and stem records of python/bnn2c/blob.py:229-232
            f.write(struct.pack("<7i", RB.VERSION_STEM, model["base_channels"], model["n_bands"],
                                model["n_classes"], 0, 1, 1))
            sc = model["stem.conv"]
            RB._w_conv_real(f, conv_mod(sc, sc["alpha"]))
            RB._w_act(f, rule(model["stem.act"]))
        else:
            f.write(struct.pack("<5i", RB.VERSION, model["base_channels"], model["n_bands"],
                                model["n_classes"], 0))
        for i, st in enumerate(RB.ENC):
            c1 = model[f"{st}.conv1"]
            if i == 0 and not stem:
                RB._w_conv_real(f, conv_mod(c1, c1["alpha"]))
            else:
                RB._w_conv_bin(f, conv_mod(c1))
            RB._w_act(f, rule(model[f"{st}.act1"]))
            RB._w_conv_bin(f, conv_mod(model[f"{st}.conv2"]))
            RB._w_act(f, rule(model[f"{st}.act2_skip"]))
            RB._w_act(f, rule(model[f"{st}.act2_down"]))
        RB._w_conv_bin(f, conv_mod(model["bottleneck.conv1"]))
        RB._w_act(f, rule(model["bottleneck.act1"]))
        RB._w_conv_bin(f, conv_mod(model["bottleneck.conv2"]))
        RB._w_act(f, rule(model["bottleneck.act2"]))
        for st in RB.DEC:
            RB._w_conv_bin(f, conv_mod(model[f"{st}.conv1"]))
            RB._w_act(f, rule(model[f"{st}.act1"]))
            RB._w_conv_bin(f, conv_mod(model[f"{st}.conv2"]))
            RB._w_act(f, rule(model[f"{st}.act2"]))
        head = torch.nn.Conv2d(model["head"]["W"].shape[1], model["head"]["W"].shape[0], 1)
        with torch.no_grad():
            head.weight.copy_(torch.from_numpy(model["head"]["W"][:, :, None, None]))
            head.bias.copy_(torch.from_numpy(model["head"]["bias"]))
        RB._w_head(f, head)
    data = open(path, "rb").read()
    rt = RB.read_blob(path)  # the reference reader's round-trip asserts
    assert len(rt["convs"]) == 18 and len(rt["acts"]) == 22
    assert (rt["stem_conv"] is not None) == stem
    os.unlink(path)
    return data


def pinned_model(name, base, rules, seed, ref, stem=0):
    """random_model written by both writers and byte-compared (the
    reference emitter recomputes alpha = mean|w|; random_model's alphas are
    exact under that recomputation)."""
    m = B.random_model(base, 120, 3, seed=seed, rules=rules, stem_channels=stem)
    rb = ref_blob_bytes(m, ref)
    tmp = tempfile.mktemp(suffix=".blob")
    open(tmp, "wb").write(rb)
    rt = B.read_blob(tmp)
    real = m["stem.conv"] if stem else m["enc1.conv1"]
    assert np.array_equal(real["alpha"], (rt["stem_conv"] if stem else rt["convs"][0])["alpha"])
    os.unlink(tmp)
    ours = B.blob_bytes(m)
    if ours != rb:
        raise SystemExit(f"{name}: blob bytes differ from the reference writer")
    return m, ours


def ref_lib():
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref.so"))
    lib.bnn_load.restype = ctypes.c_void_p
    lib.bnn_load.argtypes = [ctypes.c_char_p]
    lib.bnn_free.argtypes = [ctypes.c_void_p]
    lib.ref_stages.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                               ctypes.c_void_p, STAGE_CB, ctypes.c_void_p]
    lib.bconv_dispatch.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 8
    lib.pack_weights.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 4
    lib.maxpool_P.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 5
    return lib


def ref_stem_lib():
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_stem.so"))
    lib.bnn_stem_load.restype = ctypes.c_void_p
    lib.bnn_stem_load.argtypes = [ctypes.c_char_p]
    lib.bnn_stem_free.argtypes = [ctypes.c_void_p]
    lib.ref_stem_stages.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_void_p, STAGE_CB, ctypes.c_void_p]
    return lib


def synth(seed, first, n, bands, H, W):
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "liboracle.so"))
    lib.oracle_synth.argtypes = [ctypes.c_uint32, ctypes.c_uint32] + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    out = np.empty((n, bands, H, W), np.float32)
    lib.oracle_synth(seed, first, n, bands, H, W, out.ctypes.data)
    return out


def run_stages(lib, blob_path, x, H, W, stem=False):
    m = (lib.bnn_stem_load if stem else lib.bnn_load)(blob_path.encode())
    stages = {}

    def cb(ctx, name, kind, C, h, w, data):
        n = C * h * w
        arr = np.ctypeslib.as_array(ctypes.cast(data, ctypes.POINTER(
            {0: ctypes.c_int8, 1: ctypes.c_int32, 2: ctypes.c_float}[kind])), shape=(max(n, 1),))
        stages[name.decode()] = arr[:n].copy().reshape(C, h, w)

    logits = np.zeros((3, H, W), np.float32)
    fn = STAGE_CB(cb)
    (lib.ref_stem_stages if stem else lib.ref_stages)(m, x.ctypes.data, H, W, logits.ctypes.data, fn, None)
    (lib.bnn_stem_free if stem else lib.bnn_free)(m)
    return stages


def ref_cli_logits(blob_path, x, H, W, stem=False):
    with tempfile.TemporaryDirectory() as d:
        inp, out = os.path.join(d, "in.bin"), os.path.join(d, "out.bin")
        x.astype("<f4").tofile(inp)
        cli = "bnn_infer_stem" if stem else "bnn_infer"
        subprocess.run([os.path.join(ROOT, "oracle", "_ref", cli), blob_path, inp, out,
                        str(H), str(W)], check=True, capture_output=True,
                       env=dict(os.environ, OMP_NUM_THREADS="1"))
        return np.fromfile(out, "<f4").reshape(3, H, W)


def kernel_cases(lib):
    rng = np.random.default_rng(1234)
    res = {}
    edge = [(1, 1, 1, 4), (3, 1, 5, 4), (5, 5, 1, 8), (7, 4, 4, 6), (16, 3, 3, 16),
            (17, 5, 7, 8), (130, 3, 10, 8), (192, 3, 12, 8), (63, 4, 6, 8), (64, 4, 6, 8),
            (65, 4, 6, 8), (130, 3, 3, 8), (48, 9, 9, 16)]
    cases = [(cin, h, w, cout, 1) for cin, h, w, cout in edge] + [(3, 6, 6, 5, 0)]
    for i, (cin, h, w, cout, pad) in enumerate(cases):
        a = rng.choice(np.array([-1, 1], np.int8), size=(cin, h, w))
        ws = rng.choice(np.array([-1, 1], np.int8), size=(cout, cin, 3, 3))
        nw = (cin * 9 + 63) // 64
        packed = np.zeros((cout, nw), np.uint64)
        lib.pack_weights(ws.ctypes.data, packed.ctypes.data, cout, cin, 3, 3)
        assert np.array_equal(packed, B.pack_kidx(ws))
        ho, wo = h + 2 * pad - 2, w + 2 * pad - 2
        P = np.zeros((cout, ho, wo), np.int32)
        lib.bconv_dispatch(a.ctypes.data, packed.ctypes.data, P.ctypes.data, cin, h, w, cout,
                           3, 3, pad, 1)
        res[f"bconv{i}_a"], res[f"bconv{i}_w"], res[f"bconv{i}_P"] = a, packed, P
        res[f"bconv{i}_shape"] = np.array([cin, h, w, cout, pad], np.int32)
    for i, (c, h, w) in enumerate([(8, 8, 8), (16, 6, 10), (4, 4, 4), (5, 7, 9)]):
        P = rng.integers(-300, 300, size=(c, h, w)).astype(np.int32)
        out = np.zeros((c, (h - 2) // 2 + 1, (w - 2) // 2 + 1), np.int32)
        lib.maxpool_P(P.ctypes.data, out.ctypes.data, c, h, w, 2, 2)
        res[f"pool{i}_in"], res[f"pool{i}_out"] = P, out
    return res


# (Cin, H, W, Cout, kh, kw, pad, stride) of the kernel-ABI binary convs: the
# forward's 3x3 stride-1 shapes and the general ones (strides, 1x1 / 5x5 /
# non-square kernels, pad > 1, pad > k where the reference's two packed
# kernels count the valid taps differently)
ABI_BCONV = [(3, 9, 7, 5, 3, 3, 1, 1), (64, 8, 8, 16, 3, 3, 0, 1), (7, 9, 7, 5, 3, 3, 1, 2),
             (100, 11, 13, 24, 3, 3, 1, 2), (5, 6, 9, 4, 1, 1, 0, 1), (20, 10, 10, 8, 5, 5, 2, 1),
             (36, 7, 6, 8, 3, 3, 2, 1), (65, 5, 5, 3, 2, 2, 0, 2), (4, 3, 3, 2, 1, 1, 2, 1),
             (12, 6, 5, 3, 3, 5, 1, 1), (40, 4, 4, 4, 1, 1, 3, 2), (8, 2, 2, 3, 3, 3, 2, 3)]
ABI_REALIN = [(120, 9, 7, 8, 3, 3, 1, 1), (7, 9, 7, 5, 3, 3, 1, 1), (5, 6, 9, 4, 1, 1, 0, 1),
              (6, 8, 8, 3, 3, 3, 0, 1), (9, 10, 11, 4, 5, 5, 2, 2), (300, 5, 5, 2, 3, 3, 1, 1),
              (4, 4, 4, 3, 1, 1, 1, 1)]
ABI_POOL = [(3, 9, 8, 2, 2), (2, 7, 7, 3, 1), (4, 6, 6, 2, 1), (2, 9, 9, 3, 2), (1, 5, 4, 1, 1)]


def out_dim(n, k, pad, stride):
    return (n + 2 * pad - k) // stride + 1


def kernel_abi_cases(lib):
    """Inputs and the reference's own outputs for every function of the
    kernel-level ABI (include/bnn_kernels.h), from the reference's sources
    compiled unmodified (oracle/_ref/libref.so)."""
    rng = np.random.default_rng(4321)
    res = {}
    for i, (cin, h, w, cout, kh, kw, pad, st) in enumerate(ABI_BCONV):
        a = rng.choice(np.array([-1, 0, 1], np.int8), size=(cin, h, w), p=[0.45, 0.1, 0.45])
        ws = rng.choice(np.array([-1, 1], np.int8), size=(cout, cin, kh, kw))
        nw = (cin * kh * kw + 63) // 64
        packed = np.zeros((cout, nw), np.uint64)
        lib.pack_weights(ws.ctypes.data, packed.ctypes.data, cout, cin, kh, kw)
        assert np.array_equal(packed, B.pack_kidx(ws))
        shape = (cout, out_dim(h, kh, pad, st), out_dim(w, kw, pad, st))
        outs = {}
        for fn in ("bconv_naive_int", "bconv_xnor", "bconv_xnor_packed", "bconv_dispatch"):
            P = np.zeros(shape, np.int32)
            wp = ws if fn == "bconv_naive_int" else packed
            getattr(lib, fn)(a.ctypes.data, wp.ctypes.data, P.ctypes.data, cin, h, w, cout, kh, kw, pad, st)
            outs[fn] = P
        res.update({f"bc{i}_a": a, f"bc{i}_ws": ws, f"bc{i}_packed": packed,
                    f"bc{i}_shape": np.array([cin, h, w, cout, kh, kw, pad, st], np.int32)})
        res.update({f"bc{i}_{fn}": P for fn, P in outs.items()})
    for i, (cin, h, w, cout, kh, kw, pad, st) in enumerate(ABI_REALIN):
        x = (rng.standard_normal((cin, h, w)) * 2).astype(np.float32)
        ws = rng.choice(np.array([-1, 1], np.int8), size=(cout, cin, kh, kw))
        alpha = rng.uniform(0.1, 2.0, cout).astype(np.float32)
        out = np.zeros((cout, out_dim(h, kh, pad, st), out_dim(w, kw, pad, st)), np.float32)
        lib.conv_realin_naive(x.ctypes.data, ws.ctypes.data, alpha.ctypes.data, out.ctypes.data, cin, h, w, cout,
                              kh, kw, pad, st)
        res.update({f"ri{i}_x": x, f"ri{i}_ws": ws, f"ri{i}_alpha": alpha, f"ri{i}_out": out,
                    f"ri{i}_shape": np.array([cin, h, w, cout, kh, kw, pad, st], np.int32)})
    for i, (c, h, w, k, st) in enumerate(ABI_POOL):
        P = rng.integers(-2**31, 2**31 - 1, size=(c, h, w), dtype=np.int64).astype(np.int32)
        out = np.zeros((c, (h - k) // st + 1, (w - k) // st + 1), np.int32)
        lib.maxpool_P(P.ctypes.data, out.ctypes.data, c, h, w, k, st)
        res.update({f"mp{i}_in": P, f"mp{i}_out": out, f"mp{i}_shape": np.array([c, h, w, k, st], np.int32)})
    # integer fold: every rule type, an unknown code, thresholds inside the P range
    C, h, w = 7, 6, 5
    P = rng.integers(-20, 20, size=(C, h, w)).astype(np.int32)
    ty = np.array([0, 0, 1, 2, 3, 4, 7], np.int32)
    t = np.array([1, -1, 3, -2, 0, 0, 0], np.int32)
    lo = np.array([0, 0, 0, 0, -5, -4, 0], np.int32)
    hi = np.array([0, 0, 0, 0, 6, 3, 0], np.int32)
    out = np.zeros((C, h, w), np.int8)
    lib.apply_fold_int(P.ctypes.data, out.ctypes.data, C, h, w, ty.ctypes.data, t.ctypes.data, lo.ctypes.data,
                       hi.ctypes.data)
    res.update({"fi_P": P, "fi_type": ty, "fi_t": t, "fi_lo": lo, "fi_hi": hi, "fi_out": out})
    # real fold on values spread around each channel's switching point
    C, h, w = 5, 9, 11
    A = rng.standard_normal(C).astype(np.float32)
    Bv = rng.standard_normal(C).astype(np.float32)
    slope = rng.uniform(0.0, 0.5, C).astype(np.float32)
    rs = (rng.standard_normal(C) * 0.1).astype(np.float32)
    x = (rng.standard_normal((C, h, w)) * 3).astype(np.float32)
    out = np.zeros((C, h, w), np.int8)
    lib.apply_fold_real(x.ctypes.data, out.ctypes.data, C, h, w, A.ctypes.data, Bv.ctypes.data, slope.ctypes.data,
                        rs.ctypes.data)
    res.update({"fr_x": x, "fr_A": A, "fr_B": Bv, "fr_slope": slope, "fr_rsign": rs, "fr_out": out})
    # head: the network's +-1 input, and arbitrary floats
    cin, h, w, cout = 37, 5, 7, 3
    Wt = rng.standard_normal((cout, cin)).astype(np.float32)
    bias = rng.standard_normal(cout).astype(np.float32)
    for tag, a in (("pm1", rng.choice(np.array([-1.0, 1.0], np.float32), size=(cin, h, w))),
                   ("f32", rng.standard_normal((cin, h, w)).astype(np.float32))):
        out = np.zeros((cout, h, w), np.float32)
        lib.head_1x1(a.ctypes.data, Wt.ctypes.data, bias.ctypes.data, out.ctypes.data, cin, h, w, cout)
        res.update({f"hd_{tag}_a": a, f"hd_{tag}_out": out})
    res.update({"hd_W": Wt, "hd_bias": bias})
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BNN_REFERENCE"),
                    help="the reference project's root (default: $BNN_REFERENCE)")
    ap.add_argument("--only", choices=["kernel_abi"],
                    help="write just this fixture set (kernel_abi.npz) and leave the others as they are")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(os.path.join(args.ref, "csrc")):
        ap.error("the reference tree is needed: pass --ref or set BNN_REFERENCE")
    abi = kernel_abi_cases(bind_kernel_abi(os.path.join(ROOT, "oracle", "_ref", "libref.so")))
    np.savez_compressed(os.path.join(HERE, "kernel_abi.npz"), **abi)
    if args.only:
        return
    lib, slib = ref_lib(), ref_stem_lib()
    manifest = []
    models = [(n, b, r, s, 0, runs) for n, b, r, s, runs in MODELS + [C32]] + STEMS
    for name, base, rules, seed, stem, runs in models:
        m, data = pinned_model(name, base, rules, seed, args.ref, stem)
        sha = hashlib.sha256(data).hexdigest()
        bpath = os.path.join(HERE, name + ".blob")
        tmpb = tempfile.mktemp(suffix=".blob")
        open(tmpb, "wb").write(data)
        if name != C32[0]:
            open(bpath, "wb").write(data)
        for H, W, sseed, n in runs:
            x = synth(sseed, 0, n, 120, H, W)
            out = {"H": np.int32(H), "W": np.int32(W), "seed": np.int32(sseed), "n": np.int32(n),
                   "blob_sha256": np.array(sha)}
            for p in range(n):
                st = run_stages(slib if stem else lib, tmpb, np.ascontiguousarray(x[p]), H, W, bool(stem))
                cli = ref_cli_logits(tmpb, x[p], H, W, bool(stem))
                if not np.array_equal(cli.view(np.int32), st["logits"].view(np.int32)):
                    raise SystemExit(f"{name}: CLI logits != chained stage logits")
                for k, v in st.items():
                    out[f"p{p}/{k}"] = v
            np.savez_compressed(os.path.join(HERE, f"{name}_{H}x{W}.npz"), **out)
            manifest.append(f"{name} {H}x{W} seed={sseed} n={n} blob_sha256={sha}")
        os.unlink(tmpb)
    react_fixtures(args.ref, manifest)
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **kernel_cases(lib))
    with open(os.path.join(HERE, "MANIFEST.txt"), "w") as f:
        f.write("# generated by tests/golden/make_golden.py from the reference build\n")
        f.write("\n".join(manifest) + "\n")
    print("\n".join(manifest))


if __name__ == "__main__":
    main()
