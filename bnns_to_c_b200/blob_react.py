"""Version-3 (ReActNet real-highway) weights blob: writer, reader and a
seeded random model.

The byte layout is the reference's (python/bnn2c/blob_react.py:1-44, read by
csrc/bnn_model_react.c:86-135), little-endian:

  "BNNC" <5i> version 3, base_channels, n_bands, n_classes, upsampler (0)
  per encoder DownBlock enc1..enc4:
      [TAP tap1] (not for enc1) CONV conv1 (real for enc1, else binary)
      PROJ proj1  EPI epi1 (kind 1 for enc1, else 0)  TAP tap2  CONV conv2
      EPI epi_skip  EPI epi_down
  per PlainBlock bottleneck, dec4..dec1:
      TAP tap1  CONV conv1  PROJ proj1  EPI epi1  TAP tap2  CONV conv2  EPI epi2
  HEAD

  CONV bin  <8i> 1,Cout,Cin,kh,kw,pad,stride,nwords ; u64[Cout*nwords] (kidx bits)
  CONV real <7i> 2,Cout,Cin,kh,kw,pad,stride ; i8[Cout*Cin*kh*kw] ; f32[Cout]
  HEAD      <3i> 4,Cout,Cin ; f32[Cout*Cin] ; f32[Cout]
  PROJ      <3i> 5,Cout,Cin ; f32[Cout*Cin]
  EPI       <3i> 6,kind,C ; f32[C] x 4 (A, B, move1, prelu_w)
  TAP       <2i> 7,C ; f32[C] rsign

A model is a dict: base_channels, n_bands, n_classes, upsampler, "blocks"
{name: block} in arch order, "head" {"W", "bias"}. A block: kind ("down" |
"plain"), input_real, tap1 (rsign or None), conv1 {"wsign" int8
[Cout][Cin][3][3], "alpha" (real conv only)}, proj (f32 [Cout][Cin]), epi1,
tap2, conv2 {"wsign"}, epi_a (skip / epi2), epi_b (down blocks) — each epi
a tuple (A, B, move1, prelu_w).
"""

from __future__ import annotations

import struct

import numpy as np

from .blob import MAGIC, pack_kidx, unpack_kidx

VERSION_REACT = 3
TAG_CONV_BIN, TAG_CONV_REAL, TAG_HEAD, TAG_PROJ, TAG_EPI, TAG_TAP = 1, 2, 4, 5, 6, 7
BLOCKS = ("enc1", "enc2", "enc3", "enc4", "bottleneck", "dec4", "dec3", "dec2", "dec1")


def arch(c: int, bands: int = 120):
    """(name, Cin, Cout, kind) of the nine blocks (blob_react.py:arch)."""
    return [("enc1", bands, c, "down"), ("enc2", c, 2 * c, "down"), ("enc3", 2 * c, 4 * c, "down"),
            ("enc4", 4 * c, 8 * c, "down"), ("bottleneck", 8 * c, 16 * c, "plain"),
            ("dec4", 16 * c + 8 * c, 8 * c, "plain"), ("dec3", 8 * c + 4 * c, 4 * c, "plain"),
            ("dec2", 4 * c + 2 * c, 2 * c, "plain"), ("dec1", 2 * c + c, c, "plain")]


def _i32(*v):
    return struct.pack("<%di" % len(v), *v)


def _f32(a):
    return np.ascontiguousarray(a, "<f4").tobytes()


def _conv(c: dict, real: bool) -> bytes:
    ws = np.ascontiguousarray(c["wsign"], np.int8)
    cout, cin, kh, kw = ws.shape
    if real:
        return _i32(TAG_CONV_REAL, cout, cin, kh, kw, 1, 1) + ws.tobytes() + _f32(c["alpha"])
    packed = pack_kidx(ws)
    return _i32(TAG_CONV_BIN, cout, cin, kh, kw, 1, 1, packed.shape[1]) + \
        np.ascontiguousarray(packed, "<u8").tobytes()


def _epi(e, kind: int) -> bytes:
    A, B, m1, pw = e
    return _i32(TAG_EPI, kind, len(A)) + b"".join(_f32(a) for a in (A, B, m1, pw))


def _tap(r) -> bytes:
    return _i32(TAG_TAP, len(r)) + _f32(r)


def _proj(W) -> bytes:
    W = np.asarray(W, np.float32)
    return _i32(TAG_PROJ, W.shape[0], W.shape[1]) + _f32(W)


def react_blob_bytes(model: dict) -> bytes:
    """Serialise a v3 model in the reference's record order
    (blob_react.py:write_blob_react_from_fold)."""
    out = [MAGIC, _i32(VERSION_REACT, model["base_channels"], model["n_bands"], model["n_classes"],
                       model.get("upsampler", 0))]
    for name in BLOCKS:
        b = model["blocks"][name]
        if not b["input_real"]:
            out.append(_tap(b["tap1"]))
        out.append(_conv(b["conv1"], b["input_real"]))
        out.append(_proj(b["proj"]))
        out.append(_epi(b["epi1"], 1 if b["input_real"] else 0))
        out.append(_tap(b["tap2"]))
        out.append(_conv(b["conv2"], False))
        out.append(_epi(b["epi_a"], 0))
        if b["kind"] == "down":
            out.append(_epi(b["epi_b"], 0))
    W = np.asarray(model["head"]["W"], np.float32)
    out.append(_i32(TAG_HEAD, W.shape[0], W.shape[1]) + _f32(W) + _f32(model["head"]["bias"]))
    return b"".join(out)


def read_react_blob(data: bytes) -> dict:
    """Parse v3 bytes into the model dict (binary conv weights unpacked to
    int8 signs)."""
    off = 0

    def take(n):
        nonlocal off
        if off + n > len(data):
            raise ValueError("short read")
        b = data[off:off + n]
        off += n
        return b

    def ints(n):
        return struct.unpack("<%di" % n, take(4 * n))

    def f32(n):
        return np.frombuffer(take(4 * n), "<f4").copy()

    if take(4) != MAGIC:
        raise ValueError("bad magic")
    ver, base, bands, classes, ups = ints(5)
    if ver != VERSION_REACT:
        raise ValueError(f"blob version {ver}, expected {VERSION_REACT}")

    def conv():
        (tag,) = ints(1)
        if tag == TAG_CONV_BIN:
            cout, cin, kh, kw, pad, stride, nw = ints(7)
            packed = np.frombuffer(take(8 * cout * nw), "<u8").reshape(cout, nw).astype(np.uint64)
            return {"wsign": unpack_kidx(packed, cin, kh, kw)}
        if tag == TAG_CONV_REAL:
            cout, cin, kh, kw, pad, stride = ints(6)
            ws = np.frombuffer(take(cout * cin * kh * kw), np.int8).reshape(cout, cin, kh, kw).copy()
            return {"wsign": ws, "alpha": f32(cout)}
        raise ValueError(f"bad conv tag {tag}")

    def tagged(want):
        (tag,) = ints(1)
        if tag != want:
            raise ValueError(f"bad tag {tag}, expected {want}")

    def epi():
        tagged(TAG_EPI)
        kind, c = ints(2)
        return tuple(f32(c) for _ in range(4))

    def tap():
        tagged(TAG_TAP)
        (c,) = ints(1)
        return f32(c)

    def proj():
        tagged(TAG_PROJ)
        cout, cin = ints(2)
        return f32(cout * cin).reshape(cout, cin)

    blocks = {}
    for name, _, _, kind in arch(base, bands):
        real = name == "enc1"
        b = {"kind": kind, "input_real": real, "tap1": None if real else tap()}
        b["conv1"] = conv()
        b["proj"] = proj()
        b["epi1"] = epi()
        b["tap2"] = tap()
        b["conv2"] = conv()
        b["epi_a"] = epi()
        if kind == "down":
            b["epi_b"] = epi()
        blocks[name] = b
    tagged(TAG_HEAD)
    cout, cin = ints(2)
    head = {"W": f32(cout * cin).reshape(cout, cin), "bias": f32(cout)}
    if off != len(data):
        raise ValueError(f"{len(data) - off} trailing bytes")
    return {"base_channels": base, "n_bands": bands, "n_classes": classes, "upsampler": ups,
            "blocks": blocks, "head": head}


def random_react_model(base_channels: int = 16, n_bands: int = 120, n_classes: int = 3,
                       seed: int = 0) -> dict:
    """Random-weight v3 model with BASELINE config 4's distributions: tap
    shifts (RSign) ~N(0,0.1), RPReLU shifts ~N(0,0.1) and slopes U(0.1,0.3);
    conv weights' signs from N(0,0.3) draws, real-conv alpha = mean |w|; BN
    (gamma~N(1,.5), beta~N(0,.3), mean~N(0,.2), var~|N|*.5+.1) folded into
    (A, B) as the reference's exporter does (A = gamma/sqrt(var+eps) * alpha
    for binary convs, without alpha for the real conv); 1x1 projections and
    head ~N(0,0.3)."""
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731

    def bn_fold(c, alpha=None):
        g = f(c) * 0.5 + 1
        beta = f(c) * 0.3
        mean = f(c) * 0.2
        var = np.abs(f(c)) * 0.5 + 0.1
        s = g / np.sqrt(var + np.float32(1e-5))
        A = (s * alpha) if alpha is not None else s
        return A.astype(np.float32), (beta - s * mean).astype(np.float32)

    def epi(c, alpha=None):
        A, B = bn_fold(c, alpha)
        return (A, B, (f(c) * 0.1).astype(np.float32), rng.uniform(0.1, 0.3, c).astype(np.float32))

    blocks = {}
    for name, cin, co, kind in arch(base_channels, n_bands):
        real = name == "enc1"
        w1 = f(co, cin, 3, 3) * 0.3
        a1 = np.abs(w1).mean(axis=(1, 2, 3)).astype(np.float32)
        w2 = f(co, co, 3, 3) * 0.3
        a2 = np.abs(w2).mean(axis=(1, 2, 3)).astype(np.float32)
        b = {"kind": kind, "input_real": real, "tap1": None if real else (f(cin) * 0.1)}
        b["conv1"] = {"wsign": np.where(w1 >= 0, 1, -1).astype(np.int8)}
        if real:
            b["conv1"]["alpha"] = a1
        b["proj"] = f(co, cin) * 0.3
        b["epi1"] = epi(co, None if real else a1)
        b["tap2"] = f(co) * 0.1
        b["conv2"] = {"wsign": np.where(w2 >= 0, 1, -1).astype(np.int8)}
        b["epi_a"] = epi(co, a2)
        if kind == "down":
            b["epi_b"] = epi(co, a2)
        blocks[name] = b
    head = {"W": f(n_classes, base_channels) * 0.3, "bias": f(n_classes) * 0.3}
    return {"base_channels": base_channels, "n_bands": n_bands, "n_classes": n_classes, "upsampler": 0,
            "blocks": blocks, "head": head}
