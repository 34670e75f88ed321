"""Failure detection on the GPU, with no GPU fault: a bounded device wait
that runs out (an mbarrier phase nothing completes), a synchronous call
that meets such a give-up and must report it, a device allocation that
fails, and a multi-device shard thread that fails. After each, the context
stays usable and the next forward is bit-exact against the CPU oracle.

The reference has no failure handling of its own (every error is a print
and exit(1), csrc/bnn_model.c:17-24); these are the library's status paths."""

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import bnns_to_c_b200 as bn  # noqa: E402
from bnns_to_c_b200 import blob as B  # noqa: E402
from oracle_util import OModel, bconv_P, synth  # noqa: E402

GOLD = os.path.join(os.path.dirname(__file__), "golden")
BLOB = os.path.join(GOLD, "unet_c8_mixed_s1.blob")


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    bn.inject_fault(0)


@pytest.fixture(autouse=True)
def no_pending_injection():
    """An injection that a failing test left pending must not fire in the next."""
    bn.inject_fault(0)
    yield
    bn.inject_fault(0)


@pytest.fixture(scope="module")
def ref():
    x = synth(31, 0, 3, 120, 32, 32)
    return x, OModel(BLOB).forward_batch(x)


def same(a, b):
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_bounded_wait_gives_up_and_is_counted(ref):
    before = bn.device_wait_timeouts(0)
    gave_up, after = bn.wait_probe(0, rounds=4096)
    assert gave_up
    assert after == before + 1
    assert bn.device_wait_timeouts(0) == before + 1
    # the context is still usable: a full forward is bit-exact
    x, want = ref
    assert same(bn.Model(BLOB).forward_batch(x), want)


def test_sync_forward_reports_a_wait_that_gave_up(ref):
    x, want = ref
    m = bn.Model(BLOB)
    assert same(m.forward_batch(x), want)
    bn.inject_fault(bn.FAULT_WAIT)
    with pytest.raises(bn.BnnError) as e:
        m.forward_batch(x)
    assert e.value.code == bn.BNN_ERR_CUDA and "gave up" in str(e.value)
    # the injection fires once; the next call is clean and exact
    assert same(m.forward_batch(x), want)
    # the whole-scene path reports it too
    cube = synth(32, 0, 1, 120, 40, 36)[0]
    good = m.forward_patched(cube)
    bn.inject_fault(bn.FAULT_WAIT)
    with pytest.raises(bn.BnnError) as e:
        m.forward_patched(cube)
    assert "gave up" in str(e.value)
    assert same(m.forward_patched(cube), good)


def test_dispatch_shims_report_a_wait_that_gave_up():
    rng = np.random.default_rng(3)
    cin, cout, H, W = 40, 24, 9, 11
    a = np.where(rng.random((cin, H, W)) < 0.5, 1, -1).astype(np.int8)
    ws = np.where(rng.random((cout, cin, 3, 3)) < 0.5, 1, -1).astype(np.int8)
    packed = B.pack_kidx(ws)
    want = bconv_P(a, packed, cout)
    for fn in ("bnn_gpu_bconv_dispatch", "bnn_gpu_bconv_dispatch_noalloc"):
        P = np.zeros((cout, H, W), np.int32)
        bn.inject_fault(bn.FAULT_WAIT)
        rc = getattr(bn.lib(), fn)(a.ctypes.data, packed.ctypes.data, P.ctypes.data, cin, H, W, cout, 3, 3, 1, 1)
        assert rc == bn.BNN_ERR_CUDA, fn
        assert b"gave up" in bn.lib().bnn_last_error()
        rc = getattr(bn.lib(), fn)(a.ctypes.data, packed.ctypes.data, P.ctypes.data, cin, H, W, cout, 3, 3, 1, 1)
        assert rc == 0 and np.array_equal(P, want), fn


@pytest.mark.parametrize("k", [1, 2, 6], ids=["weights", "staging", "arena"])
def test_allocation_failure_is_reported_without_leaks(ref, k):
    """The k-th device allocation of a fresh model's first batch fails (1:
    the weight arena, 2: the first host-batch staging slot, 6: the activation
    arena, allocated after the four staging buffers): the
    call returns BNN_ERR_OOM, the model stays usable, the retry is exact, and
    device memory comes back when the model is freed."""
    x, want = ref
    warm = bn.Model(BLOB)
    warm.forward_batch(x)
    warm.close()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    m = bn.Model(BLOB)
    bn.inject_fault(bn.FAULT_ALLOC, k)
    with pytest.raises(bn.BnnError) as e:
        m.forward_batch(x)
    assert e.value.code == bn.BNN_ERR_OOM, str(e.value)
    bn.inject_fault(0)
    assert same(m.forward_batch(x), want)
    m.close()
    torch.cuda.synchronize()
    assert abs(torch.cuda.mem_get_info()[0] - free0) <= (4 << 20)


def test_failing_shard_thread_surfaces_after_join(ref):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    x, want = ref
    m = bn.Model(BLOB)
    m.set_devices([0, 1])
    assert same(m.forward_batch(x), want)
    bn.inject_fault(bn.FAULT_SHARD, 1)
    out = np.full((3, 3, 32, 32), np.nan, np.float32)
    with pytest.raises(bn.BnnError) as e:
        m.forward_batch(x, out=out)
    assert "shard 1" in str(e.value)
    # shard 0 ran to completion on its own thread before the error came back
    n0 = bn.shard_range(3, 0, 2)[1]
    assert same(out[:n0], want[:n0])
    assert same(m.forward_batch(x), want)
