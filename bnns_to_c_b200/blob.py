"""Blob v1 format (weights.blob) - writer, reader and seeded random models.

The byte layout is the reference's contract, so it is kept identical
(python/bnn2c/blob.py:36-44,67-114,181-199 and csrc/bnn_model.c:66-96 of the
reference): little-endian int32 fields; magic ``b"BNNC"``; header
``version=1, base_channels, n_bands, n_classes, upsampler``; then per encoder
stage CONV, ACT, CONV, ACT(skip), ACT(down); bottleneck CONV, ACT, CONV, ACT;
dec4..dec1 CONV, ACT, CONV, ACT; HEAD. A binary conv record is
``1, Cout, Cin, kh, kw, pad, stride, nwords`` + ``uint64[Cout*nwords]`` with
weight bit kidx = (ci*kh + ky)*kw + kx set iff the weight is +1. The real conv
is ``2, Cout, Cin, kh, kw, pad, stride`` + ``int8 wsign`` + ``f32 alpha``. An
ACT is ``3, kind, C`` then four int32 arrays (kind 0: type, t, lo, hi) or four
f32 arrays (kind 1: A, B, slope, rsign). HEAD is ``4, Cout, Cin`` + f32 W +
f32 bias.

Unlike the reference writer this one is torch-free: it writes from numpy
arrays held in a plain dict (the structure ``random_model`` returns), which is
what the benchmark and tests need (the trained checkpoint and the training
repository are not available).
"""

from __future__ import annotations

import struct

import numpy as np

MAGIC = b"BNNC"
VERSION = 1
VERSION_STEM = 2   # spectral stem (python/bnn2c/blob.py:203-245, csrc/bnn_model_stem.c)
TAG_CONV_BIN, TAG_CONV_REAL, TAG_ACT, TAG_HEAD = 1, 2, 3, 4
RULE = {"const": 0, "ge": 1, "lt": 2, "band_in": 3, "band_out": 4}
ENC = ["enc1", "enc2", "enc3", "enc4"]
DEC = ["dec4", "dec3", "dec2", "dec1"]


def pack_kidx(wsign: np.ndarray) -> np.ndarray:
    """int8 +-1 weights [Cout, Cin, kh, kw] -> uint64 [Cout, nwords], bit
    kidx = C-order flat index, set iff w > 0 (reference blob.py:47-58)."""
    cout = wsign.shape[0]
    flat = (wsign.reshape(cout, -1) > 0).astype(np.uint8)
    k = flat.shape[1]
    nwords = (k + 63) // 64
    padded = np.zeros((cout, nwords * 64), np.uint8)
    padded[:, :k] = flat
    # little bit order inside each little-endian 64-bit word
    by = np.packbits(padded.reshape(cout, nwords * 8, 8), axis=-1, bitorder="little")
    return by.reshape(cout, nwords * 8).view("<u8").reshape(cout, nwords).astype(np.uint64)


def unpack_kidx(packed: np.ndarray, cin: int, kh: int, kw: int) -> np.ndarray:
    cout, nwords = packed.shape
    by = np.ascontiguousarray(packed.astype("<u8")).view(np.uint8).reshape(cout, nwords * 8)
    bits = np.unpackbits(by, axis=-1, bitorder="little")[:, : cin * kh * kw]
    return np.where(bits > 0, 1, -1).astype(np.int8).reshape(cout, cin, kh, kw)


def _w_i32(f, *vals):
    f.write(struct.pack("<%di" % len(vals), *vals))


def _write_conv(f, conv):
    w = conv["wsign"]
    cout, cin, kh, kw = w.shape
    pad, stride = conv.get("pad", 1), conv.get("stride", 1)
    if conv["tag"] == "bin":
        packed = pack_kidx(w)
        _w_i32(f, TAG_CONV_BIN, cout, cin, kh, kw, pad, stride, packed.shape[1])
        f.write(np.ascontiguousarray(packed, "<u8").tobytes())
    else:
        _w_i32(f, TAG_CONV_REAL, cout, cin, kh, kw, pad, stride)
        f.write(np.ascontiguousarray(w, np.int8).tobytes())
        f.write(np.ascontiguousarray(conv["alpha"], "<f4").tobytes())


def _write_act(f, act):
    if act["kind"] == "int":
        _w_i32(f, TAG_ACT, 0, len(act["type"]))
        for k in ("type", "t", "lo", "hi"):
            f.write(np.ascontiguousarray(act[k], "<i4").tobytes())
    else:
        _w_i32(f, TAG_ACT, 1, len(act["A"]))
        for k in ("A", "B", "slope", "rsign"):
            f.write(np.ascontiguousarray(act[k], "<f4").tobytes())


def blob_bytes(model: dict) -> bytes:
    """Serialise a model dict (see ``random_model``) to blob bytes: v1, or v2
    when the model has a spectral stem ("stem.conv": the header gains
    has_stem = n_stem_layers = 1 and the stem conv + act records come first,
    python/bnn2c/blob.py:229-233)."""
    import io

    f = io.BytesIO()
    f.write(MAGIC)
    if "stem.conv" in model:
        _w_i32(f, VERSION_STEM, model["base_channels"], model["n_bands"], model["n_classes"],
               model.get("upsampler", 0), 1, 1)
        _write_conv(f, model["stem.conv"])
        _write_act(f, model["stem.act"])
    else:
        _w_i32(f, VERSION, model["base_channels"], model["n_bands"], model["n_classes"],
               model.get("upsampler", 0))
    for st in ENC:
        _write_conv(f, model[f"{st}.conv1"])
        _write_act(f, model[f"{st}.act1"])
        _write_conv(f, model[f"{st}.conv2"])
        _write_act(f, model[f"{st}.act2_skip"])
        _write_act(f, model[f"{st}.act2_down"])
    for i in (1, 2):
        _write_conv(f, model[f"bottleneck.conv{i}"])
        _write_act(f, model[f"bottleneck.act{i}"])
    for st in DEC:
        for i in (1, 2):
            _write_conv(f, model[f"{st}.conv{i}"])
            _write_act(f, model[f"{st}.act{i}"])
    head = model["head"]
    cout, cin = head["W"].shape
    _w_i32(f, TAG_HEAD, cout, cin)
    f.write(np.ascontiguousarray(head["W"], "<f4").tobytes())
    f.write(np.ascontiguousarray(head["bias"], "<f4").tobytes())
    return f.getvalue()


def write_blob(model: dict, path: str) -> str:
    with open(path, "wb") as f:
        f.write(blob_bytes(model))
    return path


def read_blob(path: str) -> dict:
    """Parse a v1 or v2 blob into the reference reader's dict shape
    (python/bnn2c/blob.py:251-313): convs (18), acts (22), head, and for v2
    stem_conv / stem_act."""
    with open(path, "rb") as f:
        data = f.read()
    off = 0

    def take(n):
        nonlocal off
        if off + n > len(data):
            raise ValueError("short read")
        b = data[off : off + n]
        off += n
        return b

    def ints(n):
        return struct.unpack("<%di" % n, take(4 * n))

    if take(4) != MAGIC:
        raise ValueError("bad magic")
    (version,) = ints(1)
    if version == VERSION:
        base, bands, classes, ups = ints(4)
        has_stem, n_stem = 0, 0
    elif version == VERSION_STEM:
        base, bands, classes, ups, has_stem, n_stem = ints(6)
    else:
        raise ValueError(f"unsupported blob version {version}")
    out = {"version": version, "base_channels": base, "n_bands": bands,
           "n_classes": classes, "upsampler": ups, "has_stem": has_stem, "n_stem_layers": n_stem,
           "convs": [], "acts": [], "head": None, "stem_conv": None, "stem_act": None}

    def conv():
        (tag,) = ints(1)
        if tag == TAG_CONV_BIN:
            cout, cin, kh, kw, pad, stride, nw = ints(7)
            packed = np.frombuffer(take(8 * cout * nw), "<u8").reshape(cout, nw).astype(np.uint64)
            return {"tag": "bin", "Cout": cout, "Cin": cin, "kh": kh, "kw": kw, "pad": pad,
                    "stride": stride, "packed": packed}
        if tag == TAG_CONV_REAL:
            cout, cin, kh, kw, pad, stride = ints(6)
            ws = np.frombuffer(take(cout * cin * kh * kw), np.int8).reshape(cout, cin, kh, kw).copy()
            alpha = np.frombuffer(take(4 * cout), "<f4").copy()
            return {"tag": "real", "Cout": cout, "Cin": cin, "kh": kh, "kw": kw, "pad": pad,
                    "stride": stride, "wsign": ws, "alpha": alpha}
        raise ValueError(f"bad conv tag {tag}")

    def act():
        tag, kind, c = ints(3)
        if tag != TAG_ACT:
            raise ValueError(f"bad act tag {tag}")
        if kind == 0:
            a = [np.frombuffer(take(4 * c), "<i4").copy() for _ in range(4)]
            return {"kind": "int", "C": c, "type": a[0], "t": a[1], "lo": a[2], "hi": a[3]}
        a = [np.frombuffer(take(4 * c), "<f4").copy() for _ in range(4)]
        return {"kind": "real", "C": c, "A": a[0], "B": a[1], "slope": a[2], "rsign": a[3]}

    if version == VERSION_STEM:
        out["stem_conv"] = conv()
        out["stem_act"] = act()
    for _ in ENC:
        out["convs"].append(conv()); out["acts"].append(act())
        out["convs"].append(conv()); out["acts"].append(act()); out["acts"].append(act())
    for _ in range(2):
        out["convs"].append(conv()); out["acts"].append(act())
    for _ in DEC:
        for _ in range(2):
            out["convs"].append(conv()); out["acts"].append(act())
    tag, cout, cin = ints(3)
    if tag != TAG_HEAD:
        raise ValueError(f"bad head tag {tag}")
    W = np.frombuffer(take(4 * cout * cin), "<f4").reshape(cout, cin).copy()
    bias = np.frombuffer(take(4 * cout), "<f4").copy()
    out["head"] = {"Cout": cout, "Cin": cin, "W": W, "bias": bias}
    if off != len(data):
        raise ValueError(f"{len(data) - off} trailing bytes")
    return out


# --------------------------------------------------------------------------
# seeded random models (benchmark config 0/2 weights; richer rule mixes for
# tests)
# --------------------------------------------------------------------------
def unet_widths(base: int):
    """(Cin, Cout) of the 18 convs in blob order for base width c:
    encoder c/2c/4c/8c, bottleneck 16c, decoder concat skip + previous."""
    enc = [base, 2 * base, 4 * base, 8 * base]
    return enc, 16 * base


def _int_rule(rng, C, cin, mode):
    K = 9 * cin
    if mode == "baseline":
        # thresholds uniform in [-K*Cin/4, K*Cin/4] (K=9 taps) with a random
        # ge/lt flip
        lim = K // 4
        t = rng.integers(-lim, lim + 1, size=C).astype(np.int32)
        typ = np.where(rng.random(C) < 0.5, RULE["ge"], RULE["lt"]).astype(np.int32)
        return {"kind": "int", "type": typ, "t": t, "lo": np.zeros(C, np.int32),
                "hi": np.zeros(C, np.int32)}
    # "mixed": thresholds near the P distribution's centre so bits are
    # balanced, every rule type present (including an unknown code -> -1)
    sd = max(1, int(np.sqrt(K)))
    typ = rng.choice(np.array([0, 1, 1, 2, 2, 3, 4, 7], np.int32), size=C).astype(np.int32)
    t = rng.integers(-sd, sd + 1, size=C).astype(np.int32)
    lo = rng.integers(-2 * sd, sd, size=C).astype(np.int32)
    hi = (lo + rng.integers(1, 3 * sd, size=C)).astype(np.int32)
    const = typ == 0
    t[const] = np.where(rng.random(int(const.sum())) < 0.5, 1, -1)
    return {"kind": "int", "type": typ, "t": t, "lo": lo, "hi": hi}


def random_model(base_channels: int = 32, n_bands: int = 120, n_classes: int = 3,
                 seed: int = 0, rules: str = "baseline", stem_channels: int = 0) -> dict:
    """Random-weight UNet with the distributions of the benchmark config:
    real conv signs Bernoulli(0.5), alpha U(0.5,1.5); binary weights
    Bernoulli(0.5); int folds per ``rules``; real fold A~N(1,.3), B~N(0,.3),
    slope~U(.1,.3), rsign~N(0,.1); head W~N(0,.1), bias~N(0,.1).
    ``stem_channels`` > 0 gives the v2 spectral-stem model: a real-input 1x1
    binary-weight stem of that many channels + real fold, and enc1.conv1
    binary (csrc/bnn_model_stem.c)."""
    rng = np.random.default_rng(seed)
    m = {"base_channels": base_channels, "n_bands": n_bands, "n_classes": n_classes,
         "upsampler": 0}
    enc, bott = unet_widths(base_channels)

    def sgn(*shape):
        return np.where(rng.random(shape) < 0.5, 1, -1).astype(np.int8)

    def real_fold(c):
        return {"kind": "real",
                "A": rng.normal(1.0, 0.3, c).astype(np.float32),
                "B": rng.normal(0.0, 0.3, c).astype(np.float32),
                "slope": rng.uniform(0.1, 0.3, c).astype(np.float32),
                "rsign": rng.normal(0.0, 0.1, c).astype(np.float32)}

    cin = n_bands
    if stem_channels:
        alpha = (np.round(rng.uniform(0.5, 1.5, stem_channels) * 256.0) / 256.0).astype(np.float32)
        m["stem.conv"] = {"tag": "real", "wsign": sgn(stem_channels, n_bands, 1, 1), "alpha": alpha,
                          "pad": 0, "stride": 1}
        m["stem.act"] = real_fold(stem_channels)
        cin = stem_channels
    for i, st in enumerate(ENC):
        c = enc[i]
        if i == 0 and not stem_channels:
            # alpha on a 1/256 grid: the reference writer recomputes alpha as
            # the float32 mean of |w| (blob.py:83), which is exact for these
            alpha = (np.round(rng.uniform(0.5, 1.5, c) * 256.0) / 256.0).astype(np.float32)
            m[f"{st}.conv1"] = {"tag": "real", "wsign": sgn(c, cin, 3, 3), "alpha": alpha}
            m[f"{st}.act1"] = {"kind": "real",
                               "A": rng.normal(1.0, 0.3, c).astype(np.float32),
                               "B": rng.normal(0.0, 0.3, c).astype(np.float32),
                               "slope": rng.uniform(0.1, 0.3, c).astype(np.float32),
                               "rsign": rng.normal(0.0, 0.1, c).astype(np.float32)}
        else:
            m[f"{st}.conv1"] = {"tag": "bin", "wsign": sgn(c, cin, 3, 3)}
            m[f"{st}.act1"] = _int_rule(rng, c, cin, rules)
        m[f"{st}.conv2"] = {"tag": "bin", "wsign": sgn(c, c, 3, 3)}
        m[f"{st}.act2_skip"] = _int_rule(rng, c, c, rules)
        m[f"{st}.act2_down"] = _int_rule(rng, c, c, rules)
        cin = c
    m["bottleneck.conv1"] = {"tag": "bin", "wsign": sgn(bott, cin, 3, 3)}
    m["bottleneck.act1"] = _int_rule(rng, bott, cin, rules)
    m["bottleneck.conv2"] = {"tag": "bin", "wsign": sgn(bott, bott, 3, 3)}
    m["bottleneck.act2"] = _int_rule(rng, bott, bott, rules)
    prev = bott
    for i, st in enumerate(DEC):
        skip = enc[3 - i]
        c = skip
        m[f"{st}.conv1"] = {"tag": "bin", "wsign": sgn(c, skip + prev, 3, 3)}
        m[f"{st}.act1"] = _int_rule(rng, c, skip + prev, rules)
        m[f"{st}.conv2"] = {"tag": "bin", "wsign": sgn(c, c, 3, 3)}
        m[f"{st}.act2"] = _int_rule(rng, c, c, rules)
        prev = c
    m["head"] = {"W": rng.normal(0.0, 0.1, (n_classes, prev)).astype(np.float32),
                 "bias": rng.normal(0.0, 0.1, n_classes).astype(np.float32)}
    return m
