"""The reference's kernel-level C ABI under its own names
(lib/libbnn_kernels.so, include/bnn_kernels.h) against the reference's own
functions. The fixtures (tests/golden/kernel_abi.npz, written by
tests/golden/make_golden.py from the reference's sources compiled
unmodified) record the reference's outputs for:
- the forward's shapes and general ones: strides, 1x1, 5x5 and non-square
  kernels, pad > 1, and pad > k, where bconv_xnor and bconv_xnor_packed
  disagree;
- activations holding zeros, where bconv_naive_int and the XNOR kernels
  disagree.

Integer results are compared bit for bit, and so are float results wherever
the reference's rounding is fixed by its source order. On arbitrary float
input, head_1x1 is checked to a tolerance: the reference's own builds round
it differently there."""

import os
import re
import subprocess
import sys

import numpy as np
import pytest

import bnns_to_c_b200 as bn
from oracle_util import KERNEL_ABI, bind_kernel_abi

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
FIX = os.path.join(ROOT, "tests", "golden", "kernel_abi.npz")


def _declared():
    src = open(os.path.join(ROOT, "include", "bnn_kernels.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^void (\w+)\(", src, flags=re.M)))


def test_kernel_library_exports_the_reference_names():
    assert _declared() == sorted(KERNEL_ABI)
    out = subprocess.run(["nm", "-D", "--defined-only", bn.KERNELS_PATH], capture_output=True, text=True).stdout
    exported = sorted(ln.split()[-1] for ln in out.splitlines() if " T " in ln)
    assert exported == sorted(KERNEL_ABI)


def test_pack_weights_matches_reference_fixtures():
    """pack_weights is host-side format work in the reference too."""
    L = bind_kernel_abi(bn.KERNELS_PATH)
    z = np.load(FIX)
    for i in range(_count(z, "bc", "_shape")):
        cin, h, w, cout, kh, kw, pad, st = (int(v) for v in z[f"bc{i}_shape"])
        ws = np.ascontiguousarray(z[f"bc{i}_ws"])
        out = np.full(z[f"bc{i}_packed"].shape, 0xAB, np.uint64)  # pack_weights clears it first
        L.pack_weights(ws.ctypes.data, out.ctypes.data, cout, cin, kh, kw)
        assert np.array_equal(out, z[f"bc{i}_packed"]), i


def test_kernel_calls_without_gpu_exit_like_reference():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    code = ("import ctypes, sys, numpy as np; sys.path.insert(0, sys.argv[2]); from oracle_util import bind_kernel_abi;"
            "L = bind_kernel_abi(sys.argv[1]); P = np.zeros(64, np.int32); o = np.zeros(16, np.int32);"
            "L.maxpool_P(P.ctypes.data, o.ctypes.data, 1, 8, 8, 2, 2); print('returned')")
    r = subprocess.run([sys.executable, "-c", code, bn.KERNELS_PATH, os.path.join(ROOT, "tests")],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 1 and "returned" not in r.stdout
    assert r.stderr.strip().endswith("maxpool_P: no CUDA device available"), r.stderr


# ------------------------------------------------------------------ GPU
@pytest.fixture(scope="module")
def gpu_abi():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return bind_kernel_abi(bn.KERNELS_PATH), np.load(FIX)


def _count(z, prefix, suffix):
    return len([k for k in z if k.startswith(prefix) and k.endswith(suffix)])


@pytest.mark.gpu
@pytest.mark.parametrize("fn", ["bconv_naive_int", "bconv_xnor", "bconv_xnor_packed", "bconv_dispatch"])
def test_binary_convs_match_reference(gpu_abi, fn):
    L, z = gpu_abi
    for i in range(_count(z, "bc", "_shape")):
        cin, h, w, cout, kh, kw, pad, st = (int(v) for v in z[f"bc{i}_shape"])
        a = np.ascontiguousarray(z[f"bc{i}_a"])
        wts = np.ascontiguousarray(z[f"bc{i}_ws"] if fn == "bconv_naive_int" else z[f"bc{i}_packed"])
        want = z[f"bc{i}_{fn}"]
        P = np.full(want.shape, 0x5A5A5A5A, np.int32)
        getattr(L, fn)(a.ctypes.data, wts.ctypes.data, P.ctypes.data, cin, h, w, cout, kh, kw, pad, st)
        assert np.array_equal(P, want), (fn, i, z[f"bc{i}_shape"].tolist())


@pytest.mark.gpu
def test_conv_realin_naive_matches_reference(gpu_abi):
    L, z = gpu_abi
    for i in range(_count(z, "ri", "_shape")):
        cin, h, w, cout, kh, kw, pad, st = (int(v) for v in z[f"ri{i}_shape"])
        x, ws, al = (np.ascontiguousarray(z[f"ri{i}_{k}"]) for k in ("x", "ws", "alpha"))
        want = z[f"ri{i}_out"]
        out = np.full(want.shape, np.nan, np.float32)
        L.conv_realin_naive(x.ctypes.data, ws.ctypes.data, al.ctypes.data, out.ctypes.data, cin, h, w, cout, kh, kw,
                            pad, st)
        assert out.tobytes() == want.tobytes(), (i, z[f"ri{i}_shape"].tolist(), float(np.abs(out - want).max()))


@pytest.mark.gpu
def test_maxpool_and_folds_match_reference(gpu_abi):
    L, z = gpu_abi
    for i in range(_count(z, "mp", "_shape")):
        c, h, w, k, st = (int(v) for v in z[f"mp{i}_shape"])
        P = np.ascontiguousarray(z[f"mp{i}_in"])
        out = np.zeros(z[f"mp{i}_out"].shape, np.int32)
        L.maxpool_P(P.ctypes.data, out.ctypes.data, c, h, w, k, st)
        assert np.array_equal(out, z[f"mp{i}_out"]), i
    P = np.ascontiguousarray(z["fi_P"])
    C, h, w = P.shape
    out = np.zeros(P.shape, np.int8)
    args = [np.ascontiguousarray(z[f"fi_{k}"]) for k in ("type", "t", "lo", "hi")]
    L.apply_fold_int(P.ctypes.data, out.ctypes.data, C, h, w, *(a.ctypes.data for a in args))
    assert np.array_equal(out, z["fi_out"])
    x = np.ascontiguousarray(z["fr_x"])
    C, h, w = x.shape
    out = np.zeros(x.shape, np.int8)
    args = [np.ascontiguousarray(z[f"fr_{k}"]) for k in ("A", "B", "slope", "rsign")]
    L.apply_fold_real(x.ctypes.data, out.ctypes.data, C, h, w, *(a.ctypes.data for a in args))
    assert np.array_equal(out, z["fr_out"])


@pytest.mark.gpu
def test_head_matches_reference(gpu_abi):
    L, z = gpu_abi
    Wt, bias = np.ascontiguousarray(z["hd_W"]), np.ascontiguousarray(z["hd_bias"])
    cout, cin = Wt.shape
    for tag in ("pm1", "f32"):
        a = np.ascontiguousarray(z[f"hd_{tag}_a"])
        _, h, w = a.shape
        out = np.zeros((cout, h, w), np.float32)
        L.head_1x1(a.ctypes.data, Wt.ctypes.data, bias.ctypes.data, out.ctypes.data, cin, h, w, cout)
        want = z[f"hd_{tag}_out"]
        if tag == "pm1":  # the network's domain: every product exact, the reference's bits
            assert out.tobytes() == want.tobytes()
        else:
            # arbitrary floats: the reference build fuses the multiply-adds of
            # the Cin % 4 tail, this one does not; the bound is the rounding of
            # one fused step per element, relative to the sum of |terms|
            scale = np.abs(bias)[:, None, None] + np.einsum("oc,chw->ohw", np.abs(Wt), np.abs(a))
            assert np.all(np.abs(out - want) <= 4 * np.finfo(np.float32).eps * scale)
            assert np.mean(out == want) > 0.5
