"""ctypes access to the CPU oracle (oracle/liboracle.so) for the tests.

Test infrastructure only: the oracle is the checker, never the thing run
as the product.
"""

import ctypes
import os

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
_CB = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                       ctypes.c_int, ctypes.c_void_p)
_lib = None


def olib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(os.path.join(ROOT, "oracle", "liboracle.so"))
        vp, ip = ctypes.c_void_p, ctypes.c_int
        L.oracle_load.restype = vp
        L.oracle_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ip]
        L.oracle_free.argtypes = [vp]
        for f in ("oracle_n_bands", "oracle_n_classes", "oracle_base_channels"):
            getattr(L, f).argtypes = [vp]
            getattr(L, f).restype = ip
        L.oracle_forward.argtypes = [vp, vp, ip, ip, vp, _CB, vp]
        L.oracle_forward.restype = ip
        L.oracle_forward_batch.argtypes = [vp, vp, ip, ip, ip, vp]
        L.oracle_forward_batch.restype = ip
        L.oracle_forward_patched.argtypes = [vp, vp, ip, ip, vp, ip]
        L.oracle_forward_patched.restype = ip
        L.oracle_pack_weights.argtypes = [vp, vp, ip, ip, ip, ip]
        L.oracle_bconv_P.argtypes = [vp, vp, vp] + [ip] * 8
        L.oracle_bconv_P_bits.argtypes = [vp, vp, vp] + [ip] * 4
        L.oracle_realin.argtypes = [vp, vp, vp, vp] + [ip] * 8
        L.oracle_fold_int.argtypes = [vp, vp, ip, ip, ip, vp, vp, vp, vp]
        L.oracle_fold_real.argtypes = [vp, vp, ip, ip, ip, vp, vp, vp, vp]
        L.oracle_maxpool.argtypes = [vp, vp, ip, ip, ip, ip, ip]
        L.oracle_up_cat.argtypes = [vp, ip, ip, ip, vp, ip, ip, ip, vp]
        L.oracle_head.argtypes = [vp, vp, vp, vp, ip, ip, ip, ip]
        L.oracle_synth.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ip, ip, ip, ip, vp]
        L.oracle_react_load_mem.restype = vp
        L.oracle_react_load_mem.argtypes = [vp, ctypes.c_size_t, ctypes.c_char_p, ip]
        L.oracle_react_free.argtypes = [vp]
        for f in ("oracle_react_n_bands", "oracle_react_n_classes"):
            getattr(L, f).argtypes = [vp]
            getattr(L, f).restype = ip
        L.oracle_react_forward.argtypes = [vp, vp, ip, ip, vp, _CB, vp]
        L.oracle_react_forward.restype = ip
        L.oracle_react_forward_batch.argtypes = [vp, vp, ip, ip, ip, vp]
        L.oracle_react_forward_batch.restype = ip
        L.oracle_react_proj.argtypes = [vp, vp, vp, ip, ip, ip, ip]
        L.oracle_react_conv3.argtypes = [vp, vp, vp, vp, ip, ip, ip, ip]
        _lib = L
    return _lib


class OModel:
    def __init__(self, path):
        err = ctypes.create_string_buffer(256)
        self.h = olib().oracle_load(os.fsencode(path), err, 256)
        if not self.h:
            raise ValueError(err.value.decode())
        self.n_bands = olib().oracle_n_bands(self.h)
        self.n_classes = olib().oracle_n_classes(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            olib().oracle_free(self.h)

    def stages(self, x):
        x = np.ascontiguousarray(x, np.float32)
        _, H, W = x.shape
        logits = np.zeros((self.n_classes, H, W), np.float32)
        out = {}
        ct = {0: ctypes.c_int8, 1: ctypes.c_int32, 2: ctypes.c_float}

        def cb(ctx, name, kind, C, h, w, data):
            n = C * h * w
            arr = np.ctypeslib.as_array(ctypes.cast(data, ctypes.POINTER(ct[kind])), shape=(max(n, 1),))
            out[name.decode()] = arr[:n].copy().reshape(C, h, w)

        fn = _CB(cb)
        rc = olib().oracle_forward(self.h, x.ctypes.data, H, W, logits.ctypes.data, fn, None)
        if rc:
            raise ValueError("oracle_forward refused the input")
        return out

    def forward_patched(self, cube, P=32):
        cube = np.ascontiguousarray(cube, np.float32)
        _, H, W = cube.shape
        out = np.zeros((self.n_classes, H, W), np.float32)
        rc = olib().oracle_forward_patched(self.h, cube.ctypes.data, H, W, out.ctypes.data, P)
        if rc:
            raise ValueError("oracle_forward_patched refused the input")
        return out

    def forward_batch(self, x):
        x = np.ascontiguousarray(x, np.float32)
        n, _, H, W = x.shape
        out = np.zeros((n, self.n_classes, H, W), np.float32)
        rc = olib().oracle_forward_batch(self.h, x.ctypes.data, n, H, W, out.ctypes.data)
        if rc:
            raise ValueError("oracle_forward refused the input")
        return out


def _stage_collector(out):
    ct = {0: ctypes.c_int8, 1: ctypes.c_int32, 2: ctypes.c_float}

    def cb(ctx, name, kind, C, h, w, data):
        n = C * h * w
        arr = np.ctypeslib.as_array(ctypes.cast(data, ctypes.POINTER(ct[kind])), shape=(max(n, 1),))
        out[name.decode()] = arr[:n].copy().reshape(C, h, w)
    return _CB(cb)


class ORModel:
    """The v3 ReAct oracle (oracle/bnn_oracle_react.c) on a blob given as bytes."""

    def __init__(self, data: bytes):
        err = ctypes.create_string_buffer(256)
        self._buf = ctypes.create_string_buffer(data, len(data))
        self.h = olib().oracle_react_load_mem(self._buf, len(data), err, 256)
        if not self.h:
            raise ValueError(err.value.decode())
        self.n_bands = olib().oracle_react_n_bands(self.h)
        self.n_classes = olib().oracle_react_n_classes(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            olib().oracle_react_free(self.h)

    def stages(self, x):
        x = np.ascontiguousarray(x, np.float32)
        _, H, W = x.shape
        logits = np.zeros((self.n_classes, H, W), np.float32)
        out = {}
        fn = _stage_collector(out)
        if olib().oracle_react_forward(self.h, x.ctypes.data, H, W, logits.ctypes.data, fn, None):
            raise ValueError("oracle_react_forward refused the input")
        return out

    def forward_batch(self, x):
        x = np.ascontiguousarray(x, np.float32)
        n, _, H, W = x.shape
        out = np.zeros((n, self.n_classes, H, W), np.float32)
        if olib().oracle_react_forward_batch(self.h, x.ctypes.data, n, H, W, out.ctypes.data):
            raise ValueError("oracle_react_forward refused the input")
        return out


def synth(seed, first, n, bands, H, W):
    out = np.empty((n, bands, H, W), np.float32)
    olib().oracle_synth(seed, first, n, bands, H, W, out.ctypes.data)
    return out


def bconv_P(a, packed, cout, pad=1):
    a = np.ascontiguousarray(a, np.int8)
    packed = np.ascontiguousarray(packed, np.uint64)
    cin, H, W = a.shape
    P = np.zeros((cout, H + 2 * pad - 2, W + 2 * pad - 2), np.int32)
    olib().oracle_bconv_P(a.ctypes.data, packed.ctypes.data, P.ctypes.data, cin, H, W, cout, 3, 3, pad, 1)
    return P


def pack_bits(a):
    """int8 +-1 [C][H][W] -> uint32 [H][W][ceil(C/32)] (channel c -> bit c&31
    of word c>>5, +1 -> 1), the engine's bit-plane layout."""
    C, H, W = a.shape
    cw = (C + 31) // 32
    b = np.zeros((H, W, cw * 32), np.uint64)
    b[:, :, :C] = (np.transpose(a, (1, 2, 0)) > 0)
    w = (b.reshape(H, W, cw, 32) << np.arange(32, dtype=np.uint64)).sum(-1)
    return w.astype(np.uint32)


def bconv_P_bits(bits, packed, cin, cout):
    """P [cout][H][W] of a 3x3 pad-1 binary conv on channel-packed bits
    [H][W][ceil(cin/32)] (the reference's packed kernel)."""
    bits = np.ascontiguousarray(bits, np.uint32)
    packed = np.ascontiguousarray(packed, np.uint64)
    H, W, _ = bits.shape
    P = np.zeros((cout, H, W), np.int32)
    olib().oracle_bconv_P_bits(bits.ctypes.data, packed.ctypes.data, P.ctypes.data, cin, H, W, cout)
    return P


def realin(x, wsign, alpha):
    x = np.ascontiguousarray(x, np.float32)
    wsign = np.ascontiguousarray(wsign, np.int8)
    alpha = np.ascontiguousarray(alpha, np.float32)
    cin, H, W = x.shape
    cout = wsign.shape[0]
    out = np.zeros((cout, H, W), np.float32)
    olib().oracle_realin(x.ctypes.data, wsign.ctypes.data, alpha.ctypes.data, out.ctypes.data, cin, H, W, cout,
                         3, 3, 1, 1)
    return out


def fold_int(P, rule):
    P = np.ascontiguousarray(P, np.int32)
    C, H, W = P.shape
    out = np.zeros((C, H, W), np.int8)
    arrs = [np.ascontiguousarray(rule[k], np.int32) for k in ("type", "t", "lo", "hi")]
    olib().oracle_fold_int(P.ctypes.data, out.ctypes.data, C, H, W, *[a.ctypes.data for a in arrs])
    return out


def maxpool(P):
    P = np.ascontiguousarray(P, np.int32)
    C, H, W = P.shape
    out = np.zeros((C, (H - 2) // 2 + 1, (W - 2) // 2 + 1), np.int32)
    olib().oracle_maxpool(P.ctypes.data, out.ctypes.data, C, H, W, 2, 2)
    return out


# The reference's kernel-level C ABI (csrc/bnn_model.h:7-23, csrc/bnn_conv.c):
# argument types per function, for binding the reference build
# (oracle/_ref/libref.so, fixtures) and lib/libbnn_kernels.so (tests) alike.
_V, _I = ctypes.c_void_p, ctypes.c_int
KERNEL_ABI = {
    "bconv_naive_int": [_V] * 3 + [_I] * 8,
    "pack_weights": [_V] * 2 + [_I] * 4,
    "bconv_xnor": [_V] * 3 + [_I] * 8,
    "bconv_xnor_packed": [_V] * 3 + [_I] * 8,
    "bconv_dispatch": [_V] * 3 + [_I] * 8,
    "conv_realin_naive": [_V] * 4 + [_I] * 8,
    "maxpool_P": [_V] * 2 + [_I] * 5,
    "apply_fold_int": [_V] * 2 + [_I] * 3 + [_V] * 4,
    "apply_fold_real": [_V] * 2 + [_I] * 3 + [_V] * 4,
    "head_1x1": [_V] * 4 + [_I] * 4,
}


def bind_kernel_abi(path):
    """ctypes handle on a library that exports KERNEL_ABI, argtypes set."""
    L = ctypes.CDLL(path)
    for name, args in KERNEL_ABI.items():
        f = getattr(L, name)
        f.argtypes, f.restype = args, None
    return L
