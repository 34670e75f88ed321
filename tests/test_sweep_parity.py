"""GPU parity at every shape of the isolated binary-conv sweep (BASELINE
config 1): Cin = Cout = C in {64, 128, 256, 512}, H = W in {16, 32, 64,
128}, with and without the 2x2 max-pool of P, at small batches. The fused
layer (reference bconv_dispatch -> apply_fold_int, and maxpool_P ->
apply_fold_int for the pooled branch: csrc/bnn_conv.c:216-223,
csrc/bnn_fold.c:37-60, csrc/bnn_maxpool.c:28-48) must match the CPU oracle
bit for bit, and must run on a tcgen05 kernel (no fall-back to the legacy
mma.sync path)."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import bnns_to_c_b200 as bn  # noqa: E402
from oracle_util import bconv_P_bits, fold_int, maxpool  # noqa: E402

BATCH = {128: 2, 64: 2, 32: 3, 16: 4}


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _fold(rng, C):
    """Every rule type of apply_fold_int (0..4 and an unknown code), the
    thresholds in the sweep's range [-2C, 2C]."""
    return {"type": rng.choice(np.array([0, 1, 2, 3, 4, 9], np.int32), C),
            "t": rng.integers(-2 * C, 2 * C + 1, C).astype(np.int32),
            "lo": rng.integers(-2 * C, C, C).astype(np.int32),
            "hi": rng.integers(-C, 2 * C + 1, C).astype(np.int32)}


def _unpack(words, n, C, H, W):
    d = torch.empty((n, C, H, W), dtype=torch.int8, device="cuda")
    bn.unpack_act_device(words, n, C, H, W, d)
    torch.cuda.synchronize()
    return d.cpu().numpy()


@pytest.mark.parametrize("pool", [False, True], ids=["nopool", "pool"])
@pytest.mark.parametrize("H", [16, 32, 64, 128])
@pytest.mark.parametrize("C", [64, 128, 256, 512])
def test_sweep_shape_vs_oracle(C, H, pool):
    n, W, cw = BATCH[H], H, C // 32
    rng = np.random.default_rng(C * 1000 + H * 10 + int(pool))
    nw = 9 * C // 64
    packed = np.frombuffer(rng.bytes(C * nw * 8), np.uint64).reshape(C, nw).copy()
    f1 = _fold(rng, C)
    f2 = _fold(rng, C) if pool else None
    bits = np.frombuffer(rng.bytes(n * H * W * cw * 4), np.uint32).reshape(n, H, W, cw).copy()
    L = bn.BconvLayer(0, C, C, packed, f1, f2)
    before = bn.device_wait_timeouts(0)
    din = torch.from_numpy(bits.view(np.int32)).cuda()
    out = torch.zeros((n, H, W, cw), dtype=torch.int32, device="cuda")
    outp = torch.zeros((n, H // 2, W // 2, cw), dtype=torch.int32, device="cuda") if pool else None
    # production epilogue (no accumulator output), then the debug run with P
    L.run(din, n, H, W, out, outp)
    kern = bn.bconv_last_kernel()
    assert "tcgen05" in kern, kern
    P = torch.zeros((n, C, H, W), dtype=torch.int32, device="cuda")
    Pp = torch.zeros((n, C, H // 2, W // 2), dtype=torch.int32, device="cuda") if pool else None
    out2 = torch.zeros_like(out)
    outp2 = torch.zeros_like(outp) if pool else None
    L.run(din, n, H, W, out2, outp2, P, Pp)
    torch.cuda.synchronize()
    assert bn.device_wait_timeouts(0) == before
    assert torch.equal(out, out2)
    got = _unpack(out, n, C, H, W)
    gotp = _unpack(outp, n, C, H // 2, W // 2) if pool else None
    P = P.cpu().numpy()
    Pp = Pp.cpu().numpy() if pool else None
    for i in range(n):
        Pr = bconv_P_bits(bits[i], packed, C, C)
        assert np.array_equal(P[i], Pr), (C, H, pool, i)
        assert np.array_equal(got[i], fold_int(Pr, f1)), (C, H, pool, i)
        if pool:
            Pd = maxpool(Pr)
            assert np.array_equal(Pp[i], Pd), (C, H, pool, i)
            assert np.array_equal(gotp[i], fold_int(Pd, f2)), (C, H, pool, i)
    if pool:
        assert torch.equal(outp, outp2)
    L.close()
