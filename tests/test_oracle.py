"""The CPU oracle against the reference's own outputs (golden fixtures made
by tests/golden/make_golden.py from the reference sources compiled
unmodified). Pins the oracle before any GPU result is compared with it."""

import glob
import hashlib
import os

import numpy as np
import pytest

from bnns_to_c_b200 import blob as B
from bnns_to_c_b200 import blob_react as BR
from oracle_util import OModel, ORModel, bconv_P, bconv_P_bits, maxpool, pack_bits, synth

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def fixtures():
    out = []
    for f in sorted(glob.glob(os.path.join(GOLD, "unet_*_*x*.npz")) +
                    glob.glob(os.path.join(GOLD, "stem_*_*x*.npz"))):
        base = os.path.basename(f)
        name = base.rsplit("_", 1)[0]
        out.append((name, f))
    return out


def blob_for(name, tmp_path):
    """Committed blob, or (base-32 model) regenerated from its seed and
    checked against the recorded sha256."""
    p = os.path.join(GOLD, name + ".blob")
    if os.path.exists(p):
        return p
    assert name == "unet_c32_base_s0"
    data = B.blob_bytes(B.random_model(32, 120, 3, seed=0, rules="baseline"))
    q = tmp_path / (name + ".blob")
    q.write_bytes(data)
    return str(q)


@pytest.mark.parametrize("name,npz", fixtures(), ids=[os.path.basename(f) for _, f in fixtures()])
def test_oracle_matches_reference_stages(name, npz, tmp_path):
    g = np.load(npz)
    path = blob_for(name, tmp_path)
    assert hashlib.sha256(open(path, "rb").read()).hexdigest() == str(g["blob_sha256"])
    H, W, seed, n = int(g["H"]), int(g["W"]), int(g["seed"]), int(g["n"])
    x = synth(seed, 0, n, 120, H, W)
    m = OModel(path)
    for p in range(n):
        st = m.stages(x[p])
        keys = [k[len(f"p{p}/"):] for k in g.files if k.startswith(f"p{p}/")]
        assert set(keys) == set(st), set(keys) ^ set(st)
        for k in keys:
            ref = g[f"p{p}/{k}"]
            got = st[k]
            assert got.shape == ref.shape, k
            # every stage bit-exact, floats included (same operation order)
            assert np.array_equal(got.view(np.uint8), ref.view(np.uint8)), k


def test_oracle_bconv_edge_shapes():
    g = np.load(os.path.join(GOLD, "kernels.npz"))
    i = 0
    while f"bconv{i}_a" in g.files:
        cin, h, w, cout, pad = g[f"bconv{i}_shape"]
        P = bconv_P(g[f"bconv{i}_a"], g[f"bconv{i}_w"], int(cout), int(pad))
        assert np.array_equal(P, g[f"bconv{i}_P"]), (cin, h, w, cout, pad)
        i += 1
    assert i == 14


def test_oracle_packed_bconv_matches_fixtures_and_scalar():
    """The packed-word checker (used for the large sweep shapes) gives the
    reference's P: on every pad-1 fixture of the reference's edge-shape list,
    and against the scalar restatement on Cin tails and sweep widths."""
    g = np.load(os.path.join(GOLD, "kernels.npz"))
    i, seen = 0, 0
    while f"bconv{i}_a" in g.files:
        cin, h, w, cout, pad = (int(v) for v in g[f"bconv{i}_shape"])
        if pad == 1:
            a = g[f"bconv{i}_a"]
            P = bconv_P_bits(pack_bits(a), g[f"bconv{i}_w"], cin, cout)
            assert np.array_equal(P, g[f"bconv{i}_P"]), (cin, h, w, cout)
            seen += 1
        i += 1
    assert seen >= 12
    rng = np.random.default_rng(5)
    for cin, cout, H, W in [(1, 3, 1, 1), (31, 5, 2, 7), (33, 8, 6, 1), (64, 16, 5, 5), (96, 7, 4, 9),
                            (512, 4, 3, 3), (130, 9, 7, 4)]:
        a = np.where(rng.random((cin, H, W)) < 0.5, 1, -1).astype(np.int8)
        ws = np.where(rng.random((cout, cin, 3, 3)) < 0.5, 1, -1).astype(np.int8)
        packed = B.pack_kidx(ws)
        assert np.array_equal(bconv_P_bits(pack_bits(a), packed, cin, cout), bconv_P(a, packed, cout)), (cin, H, W)


def test_oracle_maxpool():
    g = np.load(os.path.join(GOLD, "kernels.npz"))
    for i in range(4):
        assert np.array_equal(maxpool(g[f"pool{i}_in"]), g[f"pool{i}_out"])


def test_oracle_refuses_tiny_sizes():
    m = OModel(os.path.join(GOLD, "unet_c8_mixed_s1.blob"))
    with pytest.raises(ValueError):
        m.stages(np.zeros((120, 8, 8), np.float32))


def test_synth_distribution_and_determinism():
    a = synth(3, 10, 2, 120, 16, 16)
    b = synth(3, 11, 1, 120, 16, 16)
    assert np.array_equal(a[1], b[0])  # a pure function of (seed, patch, element)
    v = synth(5, 0, 4, 120, 32, 32).ravel()
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1.0) < 0.01
    assert np.abs(v).max() <= 3.47
    # pinned value (guards the generator against silent changes)
    assert float(synth(0, 0, 1, 1, 1, 1)[0, 0, 0, 0]).hex() == "0x1.fd9d880000000p-1"


@pytest.mark.parametrize("H,W,P", [(70, 50, 32), (32, 32, 32), (20, 45, 16), (64, 96, 32)])
def test_oracle_patched_is_tiles_of_the_forward(H, W, P, tmp_path):
    """The scene tiler (csrc/bnn_model_react.c:454-476 semantics on the v1
    forward) equals cutting zero-padded PxP tiles by hand, running the pinned
    per-patch oracle forward on them and stitching the in-scene parts."""
    path = tmp_path / "m.blob"
    path.write_bytes(B.blob_bytes(B.random_model(8, 120, 3, seed=11, rules="baseline")))
    m = OModel(str(path))
    cube = synth(5, 0, 1, 120, H, W)[0]
    got = m.forward_patched(cube, P)
    ty, tx = -(-H // P), -(-W // P)
    tiles = np.zeros((ty * tx, 120, P, P), np.float32)
    for r in range(ty):
        for c in range(tx):
            blk = cube[:, r * P:(r + 1) * P, c * P:(c + 1) * P]
            tiles[r * tx + c, :, :blk.shape[1], :blk.shape[2]] = blk
    lt = m.forward_batch(tiles)
    want = np.zeros((3, H, W), np.float32)
    for r in range(ty):
        for c in range(tx):
            ph, pw = min(P, H - r * P), min(P, W - c * P)
            want[:, r * P:r * P + ph, c * P:c * P + pw] = lt[r * tx + c, :, :ph, :pw]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------ v3 ReActNet
def react_fixtures():
    return [(os.path.basename(f).rsplit("_", 1)[0], f)
            for f in sorted(glob.glob(os.path.join(GOLD, "react_*_*x*.npz")))]


@pytest.mark.parametrize("name,npz", react_fixtures(), ids=[os.path.basename(f) for _, f in react_fixtures()])
def test_react_oracle_matches_reference_stages(name, npz):
    """The v3 oracle against the reference's ReAct kernels chained in
    forward order (whose logits equal the reference's own strip-processed
    bnn_forward_react and its CLI): every stage, floats included, bit for
    bit. The blob itself is byte-identical to the reference writer's."""
    g = np.load(npz)
    data = open(os.path.join(GOLD, name + ".blob"), "rb").read()
    assert hashlib.sha256(data).hexdigest() == str(g["blob_sha256"])
    H, W, seed, n = int(g["H"]), int(g["W"]), int(g["seed"]), int(g["n"])
    x = synth(seed, 0, n, 120, H, W)
    m = ORModel(data)
    for p in range(n):
        st = m.stages(x[p])
        keys = [k[len(f"p{p}/"):] for k in g.files if k.startswith(f"p{p}/")]
        assert set(keys) == set(st), set(keys) ^ set(st)
        for k in keys:
            assert st[k].shape == g[f"p{p}/{k}"].shape, k
            assert np.array_equal(st[k].view(np.uint8), g[f"p{p}/{k}"].view(np.uint8)), k


def test_react_blob_roundtrip_and_committed_bytes():
    for name, base, seed in (("react_c16_s1", 16, 1), ("react_c8_s3", 8, 3), ("react_c12_s4", 12, 4)):
        data = BR.react_blob_bytes(BR.random_react_model(base, 120, 3, seed=seed))
        assert data == open(os.path.join(GOLD, name + ".blob"), "rb").read()
        assert BR.react_blob_bytes(BR.read_react_blob(data)) == data


def test_react_oracle_loader_messages():
    data = open(os.path.join(GOLD, "react_c8_s3.blob"), "rb").read()
    for bad, msg in ((data[:-1], "short read"), (data + b"x", "trailing bytes in blob"),
                     (b"XNNC" + data[4:], "bad magic"),
                     (data[:4] + (1).to_bytes(4, "little") + data[8:],
                      "blob version 1, this engine reads v3 (ReActNet)"),
                     (data[:20] + (1).to_bytes(4, "little") + data[24:], "only nearest upsampler supported")):
        with pytest.raises(ValueError) as e:
            ORModel(bad)
        assert str(e.value) == msg
