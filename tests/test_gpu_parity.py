"""GPU parity: every kernel and the whole forward, through the C ABI,
against the CPU oracle (itself pinned to the reference build) and the
reference's golden fixtures. Integer stages and +-1 planes must be
bit-exact; the float stages (first conv output, logits) are bit-exact too
because the kernels keep the reference's fp32 operation order (the
reference's own logits gate is 1e-5 absolute, which this exceeds)."""

import glob
import os
import subprocess

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import bnns_to_c_b200 as bn  # noqa: E402
from bnns_to_c_b200 import blob as B  # noqa: E402
from bnns_to_c_b200 import blob_react as BR  # noqa: E402
from oracle_util import OModel, ORModel, bconv_P, fold_int, maxpool, realin, synth  # noqa: E402

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def same_bits(a, b):
    return a.shape == b.shape and np.array_equal(np.ascontiguousarray(a).view(np.uint8),
                                                 np.ascontiguousarray(b).view(np.uint8))


@pytest.fixture(params=["tc", "tc8", "tc4", "tcx", "popc", "mma"])
def bconv_kind(request):
    """Every binary-conv implementation: the default (tcgen05, int8 with
    e2m1 for the deeper 64/128-channel layers, mma.sync where the staging
    does not fit), tcgen05 int8 throughout, tcgen05 e2m1 for every
    non-pooled layer, int8 with the column taps in N at 32 channels, XOR +
    POPC, and mma.sync throughout. No bounded device wait may have given up
    while it ran."""
    bn.set_bconv_kernel(request.param)
    before = bn.device_wait_timeouts(0)
    yield request.param
    bn.set_bconv_kernel("tc")
    torch.cuda.synchronize()
    assert bn.device_wait_timeouts(0) == before


# ------------------------------------------------------------------ kernels
def test_bconv_dispatch_edge_shapes(bconv_kind):
    """Reference bench_bconv.c edge-shape list + bconv_harness pad=0 case."""
    g = np.load(os.path.join(GOLD, "kernels.npz"))
    i = 0
    while f"bconv{i}_a" in g.files:
        cin, h, w, cout, pad = (int(v) for v in g[f"bconv{i}_shape"])
        P = bn.gpu_bconv_dispatch(g[f"bconv{i}_a"], g[f"bconv{i}_w"], cout, pad)
        assert np.array_equal(P, g[f"bconv{i}_P"]), (cin, h, w, cout, pad)
        i += 1


@pytest.mark.parametrize("cin,cout,H,W", [(120, 32, 32, 32), (120, 16, 37, 23), (7, 8, 16, 16),
                                          (121, 40, 20, 33), (64, 64, 17, 64), (3, 5, 5, 7)])
def test_realin_bit_exact(cin, cout, H, W):
    rng = np.random.default_rng(cin * 1000 + cout)
    x = synth(21, cout, 1, cin, H, W)[0]
    ws = np.where(rng.random((cout, cin, 3, 3)) < 0.5, 1, -1).astype(np.int8)
    alpha = rng.uniform(0.5, 1.5, cout).astype(np.float32)
    assert same_bits(bn.gpu_conv_realin(x, ws, alpha), realin(x, ws, alpha))


def _rand_fold(rng, c, cin):
    sd = max(1, int(np.sqrt(9 * cin)))
    return {"type": rng.choice(np.array([0, 1, 2, 3, 4, 9], np.int32), c),
            "t": rng.integers(-sd, sd + 1, c).astype(np.int32),
            "lo": rng.integers(-2 * sd, sd, c).astype(np.int32),
            "hi": rng.integers(-sd, 2 * sd, c).astype(np.int32)}


def _unpack(bits, n, c, H, W):
    d = torch.empty((n, c, H, W), dtype=torch.int8, device="cuda")
    bn.unpack_act_device(bits, n, c, H, W, d)
    torch.cuda.synchronize()
    return d.cpu().numpy()


@pytest.mark.parametrize("pool", [True, False], ids=["pool", "nopool"])
@pytest.mark.parametrize("cin,cout,H,W,n", [(64, 64, 16, 16, 2), (128, 128, 16, 16, 2), (256, 256, 8, 8, 3),
                                            (512, 512, 4, 4, 5), (64, 64, 32, 32, 1), (48, 40, 17, 13, 2),
                                            (32, 32, 2, 2, 40), (96, 32, 32, 32, 1), (768, 256, 4, 4, 3),
                                            (16, 200, 9, 70, 1), (32, 16, 4, 4, 150), (40, 96, 3, 5, 31),
                                            (64, 64, 130, 2, 2), (32, 48, 1, 1, 70), (64, 32, 2, 300, 1)])
def test_fused_layer_vs_oracle(cin, cout, H, W, n, pool, bconv_kind):
    """One fused layer against the oracle. Shapes cover the tcgen05 kernel's
    padded-grid tiling: several images per grid row with a ragged last row,
    grid rows split across CTAs, single-pixel images, wide rows."""
    rng = np.random.default_rng(cin + 7 * cout + H)
    a = np.where(rng.random((n, cin, H, W)) < 0.5, 1, -1).astype(np.int8)
    ws = np.where(rng.random((cout, cin, 3, 3)) < 0.5, 1, -1).astype(np.int8)
    packed = B.pack_kidx(ws)
    f1, f2 = _rand_fold(rng, cout, cin), _rand_fold(rng, cout, cin)
    L = bn.BconvLayer(0, cin, cout, packed, f1, f2)
    cwi, cwo = (cin + 31) // 32, (cout + 31) // 32
    da = torch.from_numpy(a).cuda()
    bits = torch.empty((n, H, W, cwi), dtype=torch.int32, device="cuda")
    bn.pack_act_device(da, n, cin, H, W, bits)
    out = torch.zeros((n, H, W, cwo), dtype=torch.int32, device="cuda")
    outp = torch.zeros((n, H // 2, W // 2, cwo), dtype=torch.int32, device="cuda")
    P = torch.zeros((n, cout, H, W), dtype=torch.int32, device="cuda")
    Pp = torch.zeros((n, cout, H // 2, W // 2), dtype=torch.int32, device="cuda")
    pool = pool and H >= 2 and W >= 2
    L.run(bits, n, H, W, out, outp if pool else None, P, Pp if pool else None)
    torch.cuda.synchronize()
    got_a = _unpack(out, n, cout, H, W)
    got_p = _unpack(outp, n, cout, H // 2, W // 2) if pool else None
    P, Pp = P.cpu().numpy(), Pp.cpu().numpy()
    for i in range(n):
        Pr = bconv_P(a[i], packed, cout)
        assert np.array_equal(P[i], Pr)
        assert np.array_equal(got_a[i], fold_int(Pr, f1))
        if pool:
            Pd = maxpool(Pr)
            assert np.array_equal(Pp[i], Pd)
            assert np.array_equal(got_p[i], fold_int(Pd, f2))
    # unused high bits of the last output word stay zero
    if cout % 32:
        w = out.cpu().numpy()[..., -1].view(np.uint32)
        assert not np.any(w >> (cout % 32))


# ------------------------------------------------------------------ whole net
def _fixtures():
    return sorted(glob.glob(os.path.join(GOLD, "unet_*_*x*.npz")) + glob.glob(os.path.join(GOLD, "stem_*_*x*.npz")))


def _blob_path(name, tmp_path):
    p = os.path.join(GOLD, name + ".blob")
    if os.path.exists(p):
        return p
    q = tmp_path / (name + ".blob")
    q.write_bytes(B.blob_bytes(B.random_model(32, 120, 3, seed=0, rules="baseline")))
    return str(q)


@pytest.mark.parametrize("npz", _fixtures(), ids=[os.path.basename(f) for f in _fixtures()])
def test_forward_stages_match_reference(npz, tmp_path, bconv_kind):
    g = np.load(npz)
    name = os.path.basename(npz).rsplit("_", 1)[0]
    H, W, seed, n = int(g["H"]), int(g["W"]), int(g["seed"]), int(g["n"])
    # v2 fixtures (stem_*) run through the stem engine, v1 through bnn_load's
    m = (bn.StemModel if name.startswith("stem_") else bn.Model)(_blob_path(name, tmp_path))
    x = synth(seed, 0, n, 120, H, W)
    for p in range(n):
        st = m.stages(x[p])
        keys = [k[len(f"p{p}/"):] for k in g.files if k.startswith(f"p{p}/")]
        assert set(keys) == set(st), set(keys) ^ set(st)
        for k in keys:
            assert same_bits(st[k], g[f"p{p}/{k}"]), k
    # the batched path gives the same logits as the stage-by-stage path
    lg = m.forward_batch(x)
    for p in range(n):
        assert same_bits(lg[p], g[f"p{p}/logits"])


def test_batch_chunks_and_device_api_agree():
    m = bn.Model(os.path.join(GOLD, "unet_c8_mixed_s1.blob"))
    om = OModel(os.path.join(GOLD, "unet_c8_mixed_s1.blob"))
    x = synth(99, 0, 7, 120, 32, 48)
    ref = om.forward_batch(x)
    m.set_chunk(3)  # 3 chunks, the last one partial
    assert same_bits(m.forward_batch(x), ref)
    m.set_chunk(512)
    assert same_bits(m.forward_batch(x), ref)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((7, 3, 32, 48), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    for _ in range(2):  # second call replays the captured graph
        dy.zero_()
        m.forward_device(0, dx, 7, 32, 48, dy, s)
        s.synchronize()
        assert same_bits(dy.cpu().numpy(), ref)


def test_synth_device_matches_host():
    d = torch.empty((3, 120, 32, 32), dtype=torch.float32, device="cuda")
    bn.synth_device(0, 1234, 4000, 3, 120, 32, 32, d)
    torch.cuda.synchronize()
    assert same_bits(d.cpu().numpy(), synth(1234, 4000, 3, 120, 32, 32))


def test_cli_matches_reference_logits(tmp_path):
    g = np.load(os.path.join(GOLD, "unet_c16_base_s2_16x48.npz"))
    x = synth(int(g["seed"]), 0, 1, 120, 16, 48)[0]
    inp, out = tmp_path / "in.bin", tmp_path / "out.bin"
    x.astype("<f4").tofile(inp)
    r = subprocess.run([bn.CLI_PATH, os.path.join(GOLD, "unet_c16_base_s2.blob"), str(inp), str(out), "16", "48", "3"],
                       capture_output=True, text=True, env=dict(os.environ, BNN_PROFILE="1"))
    assert r.returncode == 0, r.stderr
    assert "# forward   :" in r.stderr and "# per-op" in r.stderr
    got = np.fromfile(out, "<f4").reshape(3, 16, 48)
    assert same_bits(got, g["p0/logits"])


def test_refuses_sizes_the_reference_cannot_run():
    m = bn.Model(os.path.join(GOLD, "unet_c8_mixed_s1.blob"))
    with pytest.raises(bn.BnnError) as e:
        m.forward(np.zeros((120, 8, 32), np.float32))
    assert e.value.code == bn.BNN_ERR_ARG


def test_profiler_records_every_launch():
    m = bn.Model(os.path.join(GOLD, "unet_c8_mixed_s1.blob"))
    m.profile(True)
    m.forward_batch(synth(5, 0, 4, 120, 32, 32))
    recs = m.profile_records()
    # 19 profiled ops; the first conv's op is two kernels (tensor-core pass + exact fix-up)
    assert len(recs) == 19 and m.launches(4, 32, 32) == 20
    assert sum(r["op"] == "bconv" for r in recs) == 17
    assert all(r["ms"] > 0 and r["calls"] == 1 for r in recs)


@pytest.mark.slow
def test_full_batch_properties():
    """Benchmark size (c=32, 4096 patches of 32x32x120): sampled patches
    equal the oracle, and the result does not depend on how the batch is
    split (shard invariance, the property the multi-GPU split relies on)."""
    m = bn.Model.__new__(bn.Model)
    data = B.blob_bytes(B.random_model(32, 120, 3, seed=0, rules="baseline"))
    m.__init__(data=data)
    N, H, W = 4096, 32, 32
    dx = torch.empty((N, 120, H, W), dtype=torch.float32, device="cuda")
    bn.synth_device(0, 17, 0, N, 120, H, W, dx)
    full = torch.empty((N, 3, H, W), dtype=torch.float32, device="cuda")
    m.forward_device(0, dx, N, H, W, full)
    part = torch.empty_like(full)
    m.forward_device(0, dx[:1000], 1000, H, W, part[:1000])
    m.forward_device(0, dx[1000:], N - 1000, H, W, part[1000:])
    torch.cuda.synchronize()
    assert torch.equal(full.view(torch.int32), part.view(torch.int32))
    import tempfile
    with tempfile.NamedTemporaryFile(suffix=".blob") as f:
        f.write(data)
        f.flush()
        om = OModel(f.name)
        idx = [0, 1, 2047, 4095]
        ref = np.stack([om.forward_batch(synth(17, i, 1, 120, H, W))[0] for i in idx])
    got = full[idx].cpu().numpy()
    assert same_bits(got, ref)
    assert torch.isfinite(full).all()


def test_multi_device_shards_match_single():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    m = bn.Model(os.path.join(GOLD, "unet_c8_mixed_s1.blob"))
    x = synth(3, 0, 9, 120, 32, 32)
    ref = m.forward_batch(x)
    m.set_devices(list(range(torch.cuda.device_count())))
    assert same_bits(m.forward_batch(x), ref)


# ------------------------------------------------------------------ first conv: tensor-core path
@pytest.fixture(params=["tc", "mma", "tcn", "tx"])
def first_kind(request):
    """Every first-conv tensor-core kernel (tcgen05 nine-tap, mma.sync,
    tcgen05 with the column taps in N where W divides 32, tcgen05 with the
    weights in M and the positions in N); no bounded
    device wait may have given up while it ran."""
    bn.set_first_conv_kernel(request.param)
    before = bn.device_wait_timeouts(0)
    yield request.param
    bn.set_first_conv_kernel("tc")
    torch.cuda.synchronize()
    assert bn.device_wait_timeouts(0) == before


def _first_conv_bits(m, x, exact):
    n, _, H, W = x.shape
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    cw = (m.enc_c1_cout + 31) // 32
    bits = torch.zeros((n, H, W, cw), dtype=torch.int32, device="cuda")
    und = m.first_conv_device(0, dx, n, H, W, bits, exact=exact)
    torch.cuda.synchronize()
    return bits.cpu().numpy(), und


def _model(base=32, seed=0, mutate=None, bands=120):
    mdl = B.random_model(base, bands, 3, seed=seed, rules="baseline")
    if mutate:
        mutate(mdl)
    m = bn.Model(data=B.blob_bytes(mdl))
    m.enc_c1_cout = mdl["enc1.conv1"]["wsign"].shape[0]
    return m


def test_first_conv_tensor_path_matches_exact_order(first_kind):
    m = _model()
    x = synth(41, 0, 256, 120, 32, 32)
    fast, und = _first_conv_bits(m, x, False)
    exact, _ = _first_conv_bits(m, x, True)
    assert np.array_equal(fast, exact)
    outs = 256 * 32 * 32 * 32
    assert 0 <= und < outs // 500, und  # the error bound decides > 99.8% of the outputs


def test_first_conv_fixup_exercised_near_threshold(first_kind):
    """Folds tuned so r sits near 0 for many outputs: many undecided,
    all resolved exactly."""
    x = synth(42, 0, 16, 120, 32, 32)

    def near_zero(mdl):
        a = mdl["enc1.act1"]
        a["A"][:] = 1.0
        a["B"][:] = 0.0
        a["rsign"][:] = 0.0  # r = alpha*acc (or slope*alpha*acc): decided by sign(acc) alone
    m = _model(mutate=near_zero)
    # inputs whose window sums cancel: each band repeated with its sign flipped
    x[:, 60:] = -x[:, :60]
    fast, und = _first_conv_bits(m, x, False)
    exact, _ = _first_conv_bits(m, x, True)
    assert np.array_equal(fast, exact)
    assert und > 0


def test_first_conv_nonmonotone_channels_and_overflow(first_kind):
    def neg_slope(mdl):
        mdl["enc1.act1"]["slope"][::2] = -0.2  # half the channels: V-shaped fold
    m = _model(mutate=neg_slope)
    x = synth(43, 0, 8, 120, 32, 32)
    fast, und = _first_conv_bits(m, x, False)
    exact, _ = _first_conv_bits(m, x, True)
    assert np.array_equal(fast, exact) and und >= 8 * 1024 * 16
    # every channel non-monotone and a big batch: the list overflows, the
    # fix-up recomputes the whole batch
    def all_neg(mdl):
        mdl["enc1.act1"]["slope"][:] = -0.2
    m2 = _model(mutate=all_neg)
    x2 = synth(44, 0, 96, 120, 32, 32)
    fast, und = _first_conv_bits(m2, x2, False)
    exact, _ = _first_conv_bits(m2, x2, True)
    assert und == 0xFFFFFFFF and np.array_equal(fast, exact)


def test_first_conv_nonfinite_and_extreme_inputs(first_kind):
    m = _model()
    x = synth(45, 0, 6, 120, 32, 32)
    x[0, 5, 3, 7] = np.nan
    x[1, 100, 31, 31] = np.inf
    x[2] *= 1e30           # huge values
    x[3] *= 1e-38          # subnormal range
    x[4, :, :16] = 0.0     # exact zeros
    x[5, ::2] *= 1e6       # mixed dynamic range
    fast, _ = _first_conv_bits(m, x, False)
    exact, _ = _first_conv_bits(m, x, True)
    assert np.array_equal(fast, exact)
    om_bits = None  # the exact kernel itself is pinned to the oracle by test_realin_bit_exact
    del om_bits


@pytest.mark.parametrize("H,W", [(17, 40), (33, 33), (64, 16), (16, 16), (16, 100), (40, 64), (21, 252),
                                 (16, 124), (17, 16), (21, 16), (31, 32), (18, 32)])
def test_first_conv_tensor_path_odd_sizes(H, W, first_kind):
    """Sizes that exercise the tcgen05 kernels' row items (several per
    image, a short last one, one image per item, wide rows; the column-taps
    kernel's items of 8 rows at W = 16 and 4 rows at W = 32 with 1 to 3 rows
    left for the last) and the shapes handed back to the mma.sync kernel
    (W not a multiple of 4, boxes too big for shared memory)."""
    m = _model(base=16, seed=3)
    x = synth(46, 0, 3, 120, H, W)
    fast, _ = _first_conv_bits(m, x, False)
    exact, _ = _first_conv_bits(m, x, True)
    assert np.array_equal(fast, exact)


@pytest.mark.parametrize("bands", [1, 37, 64, 128])
def test_first_conv_tensor_path_band_counts(bands, first_kind):
    """Band counts that leave 1 to 4 K chunks, partly filled or full."""
    m = _model(seed=5, bands=bands)
    x = synth(47, 0, 4, bands, 32, 32)
    fast, und = _first_conv_bits(m, x, False)
    exact, _ = _first_conv_bits(m, x, True)
    assert np.array_equal(fast, exact)
    assert und < 4 * 32 * 32 * 32 // 100


# ------------------------------------------------------------------ whole-scene patched forward
@pytest.mark.parametrize("H,W,P", [(70, 50, 32), (20, 45, 16), (64, 96, 32), (33, 100, 32), (16, 16, 16)])
def test_patched_forward_matches_oracle(H, W, P, tmp_path):
    """bnn_forward_patched (the reference's tiler, csrc/bnn_model_react.c:454-476,
    on the v1 forward) against the oracle tiler, bit for bit, through the host
    and the device entry points; partial edge tiles included."""
    from oracle_util import OModel
    path = tmp_path / "m.blob"
    path.write_bytes(B.blob_bytes(B.random_model(16, 120, 3, seed=13, rules="baseline")))
    m, om = bn.Model(str(path)), OModel(str(path))
    cube = synth(9, 0, 1, 120, H, W)[0]
    want = om.forward_patched(cube, P)
    got = m.forward_patched(cube, P)
    assert same_bits(got, want)
    dc = torch.from_numpy(cube).cuda()
    dl = torch.full((3, H, W), float("nan"), dtype=torch.float32, device="cuda")
    m.forward_patched_device(0, dc, H, W, dl, P)
    torch.cuda.synchronize()
    assert same_bits(dl.cpu().numpy(), want)


def test_patched_forward_multi_device(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU")
    path = tmp_path / "m.blob"
    path.write_bytes(B.blob_bytes(B.random_model(16, 120, 3, seed=13, rules="baseline")))
    m = bn.Model(str(path))
    cube = synth(10, 0, 1, 120, 150, 90)[0]
    one = m.forward_patched(cube, 32)
    m.set_devices([0, 1])
    two = m.forward_patched(cube, 32)
    assert same_bits(one, two)


# ------------------------------------------------------------------ first conv: zero weights
def test_first_conv_zero_weights(first_kind, tmp_path):
    """wsign = 0 (np.sign of an exact 0.0 weight, which the reference's blob
    writer can emit): the tensor-core paths take it as a 0 product, as the
    reference's fp32 sum does."""
    def zeros(mdl):
        w = mdl["enc1.conv1"]["wsign"].copy()
        w[:, ::3] = 0
        w[5] = 0
        mdl["enc1.conv1"]["wsign"] = w
    mdl = B.random_model(32, 120, 3, seed=8, rules="baseline")
    zeros(mdl)
    path = tmp_path / "z.blob"
    path.write_bytes(B.blob_bytes(mdl))
    m = bn.Model(str(path))
    m.enc_c1_cout = 32
    x = synth(48, 0, 8, 120, 32, 32)
    fast, _ = _first_conv_bits(m, x, False)
    exact, _ = _first_conv_bits(m, x, True)
    assert np.array_equal(fast, exact)
    om = OModel(str(path))
    assert same_bits(m.forward_batch(x[:2]), om.forward_batch(x[:2]))


# ------------------------------------------------------------------ v2 spectral stem
def _stem(tmp_path, stem, base=8, seed=0, bands=120, rules="mixed", mutate=None):
    mdl = B.random_model(base, bands, 3, seed=seed, rules=rules, stem_channels=stem)
    if mutate:
        mutate(mdl)
    path = tmp_path / f"stem{stem}_{bands}.blob"
    path.write_bytes(B.blob_bytes(mdl))
    return bn.StemModel(str(path)), OModel(str(path))


def _same_stages(st, ost, skip_float=False):
    assert set(st) == set(ost), set(st) ^ set(ost)
    for k in ost:
        if skip_float and k == "stem.conv.out":
            continue
        assert same_bits(st[k], ost[k]), k


@pytest.mark.parametrize("stem,H,W", [(16, 32, 32), (8, 37, 23), (12, 16, 48), (24, 33, 34), (32, 16, 16),
                                      (40, 20, 36), (1, 17, 17), (70, 32, 18)])
def test_stem_widths_and_sizes_match_oracle(stem, H, W, tmp_path, bconv_kind):
    """Stem widths on every kernel shape (8/16/32-channel slices, 1-3
    words per pixel) and patch sizes on every pixel grouping (4, 2 or 1
    pixels per thread): every stage, the stem's float output included, and
    the batched logits equal the oracle's bit for bit."""
    m, om = _stem(tmp_path, stem, seed=stem)
    x = synth(stem + H, 0, 3, 120, H, W)
    _same_stages(m.stages(x[0]), om.stages(x[0]))
    assert same_bits(m.forward_batch(x), om.forward_batch(x))


@pytest.mark.parametrize("bands", [1, 37, 300])
def test_stem_band_counts_and_zero_weights(bands, tmp_path):
    def zeros(mdl):
        w = mdl["stem.conv"]["wsign"].copy()
        w[:, ::4] = 0
        w[2] = 0
        mdl["stem.conv"]["wsign"] = w
    m, om = _stem(tmp_path, 16, seed=bands, bands=bands, mutate=zeros)
    x = synth(bands, 0, 2, bands, 32, 32)
    _same_stages(m.stages(x[0]), om.stages(x[0]))
    assert same_bits(m.forward_batch(x), om.forward_batch(x))


def test_stem_nonfinite_and_extreme_inputs(tmp_path):
    """NaN / inf / huge / subnormal bands: the +-1 planes and the logits
    match (NaN payloads of the float stage are not compared)."""
    m, om = _stem(tmp_path, 16, seed=21)
    x = synth(49, 0, 5, 120, 32, 32)
    x[0, 5, 3, 7] = np.nan
    x[1, 100, 31, 31] = np.inf
    x[1, 101, 31, 31] = -np.inf
    x[2] *= 1e30
    x[3] *= 1e-38
    x[4, :, :16] = 0.0
    for p in range(5):
        _same_stages(m.stages(x[p]), om.stages(x[p]), skip_float=(p < 2))
    assert same_bits(m.forward_batch(x), om.forward_batch(x))


def test_stem_device_patched_and_profiler(tmp_path):
    m, om = _stem(tmp_path, 16, base=16, seed=22, rules="baseline")
    x = synth(50, 0, 6, 120, 32, 48)
    ref = om.forward_batch(x)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((6, 3, 32, 48), dtype=torch.float32, device="cuda")
    for _ in range(2):  # the second call replays the captured graph
        dy.zero_()
        m.forward_device(0, dx, 6, 32, 48, dy)
        torch.cuda.synchronize()
        assert same_bits(dy.cpu().numpy(), ref)
    cube = synth(51, 0, 1, 120, 70, 50)[0]
    assert same_bits(m.forward_patched(cube, 32), om.forward_patched(cube, 32))
    # the stem alone through the first-conv entry point
    bits = torch.zeros((6, 32, 48, 1), dtype=torch.int32, device="cuda")
    und = m.first_conv_device(0, dx, 6, 32, 48, bits)
    torch.cuda.synchronize()
    want = np.stack([om.stages(x[p])["stem.act"] for p in range(6)])  # [n][C][H][W] int8
    got = _unpack(bits, 6, 16, 32, 48)
    assert und == 0 and np.array_equal(got, want)
    m.profile(True)
    m.forward_batch(x)
    recs = m.profile_records()
    assert len(recs) == 20 and m.launches(6, 32, 48) == 20
    assert recs[0]["label"] == "stem.conv+act" and sum(r["op"] == "bconv" for r in recs) == 18


def test_stem_cli_matches_reference_logits(tmp_path):
    g = np.load(os.path.join(GOLD, "stem_c16_base_s4_16x48.npz"))
    x = synth(int(g["seed"]), 0, 1, 120, 16, 48)[0]
    inp, out = tmp_path / "in.bin", tmp_path / "out.bin"
    x.astype("<f4").tofile(inp)
    r = subprocess.run([bn.CLI_STEM_PATH, os.path.join(GOLD, "stem_c16_base_s4.blob"), str(inp), str(out), "16", "48",
                        "2"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "# [stem] H=16 W=48 bands=120 classes=3 stem_channels=16 reps=2" in r.stderr
    got = np.fromfile(out, "<f4").reshape(3, 16, 48)
    assert same_bits(got, g["p0/logits"])


def test_stem_multi_device(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU")
    m, _ = _stem(tmp_path, 16, seed=23)
    x = synth(52, 0, 9, 120, 32, 32)
    one = m.forward_batch(x)
    m.set_devices([0, 1])
    assert same_bits(m.forward_batch(x), one)


# ------------------------------------------------------------------ v3 ReActNet
# stages the GPU engine holds (the oracle also reports pool.P, poolr and the
# decoders' cat, which the engine never materialises)
REACT_REQUIRED = ["enc1.proj", "enc1.conv1.out", "enc1.h1", "enc1.tap2", "enc1.conv2.P", "enc1.skip", "enc1.down",
                  "enc3.tap1", "enc3.conv1.P", "bottleneck.h2", "dec4.proj", "dec4.tap1", "dec1.h2", "logits"]


def _react_same_stages(st, ref):
    for k in REACT_REQUIRED:
        assert k in st, k
    for k in st:
        assert k in ref, k
        assert same_bits(st[k], ref[k]), k


def _react_fixtures():
    return sorted(glob.glob(os.path.join(GOLD, "react_*_*x*.npz")))


@pytest.mark.parametrize("npz", _react_fixtures(), ids=[os.path.basename(f) for f in _react_fixtures()])
def test_react_stages_match_reference(npz, bconv_kind):
    """Every intermediate the engine holds (highway maps, taps, P, logits)
    equals the reference ReAct engine's bit for bit (golden fixtures from the
    reference's kernels, whose logits equal its own bnn_forward_react)."""
    g = np.load(npz)
    name = os.path.basename(npz).rsplit("_", 1)[0]
    m = bn.ReactModel(os.path.join(GOLD, name + ".blob"))
    H, W, seed, n = int(g["H"]), int(g["W"]), int(g["seed"]), int(g["n"])
    x = synth(seed, 0, n, 120, H, W)
    for p in range(n):
        ref = {k[len(f"p{p}/"):]: g[k] for k in g.files if k.startswith(f"p{p}/")}
        _react_same_stages(m.stages(x[p]), ref)
    lg = m.forward_batch(x)
    for p in range(n):
        assert same_bits(lg[p], g[f"p{p}/logits"])


@pytest.mark.parametrize("base,H,W", [(16, 64, 64), (16, 44, 60), (8, 50, 38), (24, 32, 32), (12, 33, 47),
                                      (16, 16, 16), (8, 17, 83)])
def test_react_sizes_and_widths_vs_oracle(base, H, W):
    """Odd sizes (floor pools, partly covered upsamples, pixel tails of the
    blocked projection), widths on both real-conv orders (Cout % 8) and
    several channel slices; batched logits and every held stage."""
    mdl = BR.random_react_model(base, 120, 3, seed=base + H)
    data = BR.react_blob_bytes(mdl)
    m, om = bn.ReactModel(data=data), ORModel(data)
    x = synth(base * 7 + W, 0, 3, 120, H, W)
    _react_same_stages(m.stages(x[0]), om.stages(x[0]))
    assert same_bits(m.forward_batch(x), om.forward_batch(x))


def test_react_device_graph_patched_and_profiler():
    data = open(os.path.join(GOLD, "react_c8_s3.blob"), "rb").read()
    m, om = bn.ReactModel(data=data), ORModel(data)
    x = synth(61, 0, 5, 120, 32, 48)
    ref = om.forward_batch(x)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((5, 3, 32, 48), dtype=torch.float32, device="cuda")
    for _ in range(2):  # the second call replays the captured graph
        dy.zero_()
        m.forward_device(0, dx, 5, 32, 48, dy)
        torch.cuda.synchronize()
        assert same_bits(dy.cpu().numpy(), ref)
    # the reference's tiler: zero-padded 32x32 tiles, each a standalone forward
    cube = synth(62, 0, 1, 120, 70, 50)[0]
    tiles, P = [], 32
    for y in range(0, 70, P):
        for xx in range(0, 50, P):
            t = np.zeros((120, P, P), np.float32)
            c = cube[:, y:y + P, xx:xx + P]
            t[:, :c.shape[1], :c.shape[2]] = c
            tiles.append(t)
    tl = om.forward_batch(np.stack(tiles))
    want = np.zeros((3, 70, 50), np.float32)
    k = 0
    for y in range(0, 70, P):
        for xx in range(0, 50, P):
            want[:, y:y + P, xx:xx + P] = tl[k][:, :min(P, 70 - y), :min(P, 50 - xx)]
            k += 1
    assert same_bits(m.forward_patched(cube, P), want)
    m.profile(True)
    m.forward_batch(x)
    recs = m.profile_records()
    assert len(recs) == m.launches(5, 32, 48) == 46
    assert sum(r["op"] == "bconv" for r in recs) == 17 and all(r["ms"] > 0 for r in recs)


@pytest.mark.parametrize("H,W", [(64, 64), (32, 32), (48, 72), (20, 36), (64, 96)])
def test_react_conv_kernels_agree(H, W):
    """enc1's real conv: the TMA-staged kernel (both tile widths, edge tiles,
    rows past the patch) equals the thread-staged one and the oracle; no
    bounded wait gives up."""
    data = open(os.path.join(GOLD, "react_c16_s1.blob"), "rb").read()
    m, om = bn.ReactModel(data=data), ORModel(data)
    x = synth(70 + H, 0, 2, 120, H, W)
    before = bn.react_wait_timeouts(0)
    st = m.stages(x[0])
    bn.set_react_conv_kernel("plain")
    try:
        st2 = m.stages(x[0])
    finally:
        bn.set_react_conv_kernel("tma")
    ref = om.stages(x[0])
    assert same_bits(st["enc1.conv1.out"], ref["enc1.conv1.out"])
    assert same_bits(st2["enc1.conv1.out"], ref["enc1.conv1.out"])
    assert same_bits(m.forward_batch(x), om.forward_batch(x))
    assert bn.react_wait_timeouts(0) == before


def test_react_cli_matches_reference_binary(tmp_path):
    """bnn_infer_react against the reference's own CLI (csrc/main_react.c,
    built from its sources into oracle/_ref when the tree was present): the
    same `rand` cube, whole-image and patch-wise, identical logits."""
    ref_cli = os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref", "bnn_infer_react")
    if not os.path.exists(ref_cli):
        pytest.skip("reference ReAct CLI not built")
    blob = os.path.join(GOLD, "react_c8_s3.blob")
    for spec, H, W in (("rand", 48, 40), ("patch16:rand", 40, 56)):
        ours, theirs = tmp_path / "o.bin", tmp_path / "t.bin"
        r = subprocess.run([bn.CLI_REACT_PATH, blob, spec, str(ours), str(H), str(W), "2"], capture_output=True,
                           text=True)
        assert r.returncode == 0, r.stderr
        assert f"# forward {H}x{W} reps=2" in r.stdout
        r2 = subprocess.run([ref_cli, blob, spec, str(theirs), str(H), str(W)], capture_output=True, text=True,
                            env=dict(os.environ, OMP_NUM_THREADS="1"))
        assert r2.returncode == 0, r2.stderr
        assert same_bits(np.fromfile(ours, "<f4"), np.fromfile(theirs, "<f4")), spec
