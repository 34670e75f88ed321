"""The allocation-free entry point bnn_gpu_bconv_dispatch_noalloc, through
the C ABI. It exists for callers that cannot let the library allocate device
memory (GPU memory fixed up front by their own allocator or budget; loops
that cannot take cudaFree's device-wide synchronisation), so its buffers come
from one static device array instead of cudaMalloc. Checked here: two calls
in a row give exactly the allocating bnn_gpu_bconv_dispatch's P (the
tolerance of every integer test in this suite: none), the second call leaves
the device's free memory unchanged, and a size beyond the static array is
refused up front. This file is collected last on purpose."""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import bnns_to_c_b200 as bn  # noqa: E402
from bnns_to_c_b200 import blob as B  # noqa: E402


def _case(seed, cin, H, W, cout):
    rng = np.random.default_rng(seed)
    a = np.where(rng.random((cin, H, W)) < 0.5, 1, -1).astype(np.int8)
    packed = B.pack_kidx(np.where(rng.random((cout, cin, 3, 3)) < 0.5, 1, -1).astype(np.int8))
    return a, packed


def _noalloc(a, packed, cout, pad):
    cin, H, W = a.shape
    P = np.full((cout, H + 2 * pad - 2, W + 2 * pad - 2), 0x5A5A5A5A, np.int32)  # sentinel
    rc = bn.lib().bnn_gpu_bconv_dispatch_noalloc(a.ctypes.data, packed.ctypes.data, P.ctypes.data,
                                                 cin, H, W, cout, 3, 3, pad, 1)
    return rc, P


def test_noalloc_matches_allocating_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    first = _case(1, 130, 12, 10, 40)
    second = _case(2, 64, 9, 9, 16)
    rc1, P1 = _noalloc(*first, 40, 1)
    assert rc1 == 0, bn.lib().bnn_last_error()
    free_before = torch.cuda.mem_get_info()[0]
    rc2, P2 = _noalloc(*second, 16, 0)
    free_after = torch.cuda.mem_get_info()[0]
    assert rc2 == 0, bn.lib().bnn_last_error()
    assert free_after == free_before
    assert np.array_equal(P1, bn.gpu_bconv_dispatch(first[0], first[1], 40, 1))
    assert np.array_equal(P2, bn.gpu_bconv_dispatch(second[0], second[1], 16, 0))


def test_noalloc_refuses_sizes_beyond_its_array():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    a = np.ones((64, 256, 256), np.int8)  # P alone is 128*256*256*4 bytes = 32 MiB
    packed = np.zeros((128, 9), np.uint64)
    rc, _ = _noalloc(a, packed, 128, 1)
    assert rc == bn.BNN_ERR_ARG and "static array" in bn.lib().bnn_last_error().decode()
