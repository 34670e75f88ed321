"""bnns_to_c_b200 - Python binding of the B200 binary-UNet engine.

The product is the C-ABI library ``lib/libbnn_b200.so`` (headers in
``include/``): a drop-in for the reference engine's ``bnn_load`` /
``bnn_forward`` / ``bnn_free`` (csrc/bnn_model.h of Sboyle132/BNNs_to_C),
plus batched, device-pointer, multi-GPU and kernel-level entry points. This
module is a thin ctypes layer over it with the reference's Python-side
names where the reference has them (``read_blob``/``write_blob`` live in
``bnns_to_c_b200.blob``).

There is no CPU fallback: importing works on a machine without a GPU (so
blobs can be parsed and validated), but every compute call goes to the CUDA
library and raises ``BnnError`` when no GPU is present.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libbnn_b200.so")
CLI_PATH = os.path.join(HERE, "lib", "bnn_infer")
CLI_STEM_PATH = os.path.join(HERE, "lib", "bnn_infer_stem")
CLI_REACT_PATH = os.path.join(HERE, "lib", "bnn_infer_react")
# the reference's kernel-level ABI under its own names (include/bnn_kernels.h)
KERNELS_PATH = os.path.join(HERE, "lib", "libbnn_kernels.so")

BNN_OK, BNN_ERR_IO, BNN_ERR_FORMAT, BNN_ERR_UNSUPPORTED, BNN_ERR_ARG, BNN_ERR_CUDA, BNN_ERR_OOM = range(7)

STAGE_CB = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                            ctypes.c_int, ctypes.c_int, ctypes.c_void_p)


class BnnError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class _ModelHeader(ctypes.Structure):
    # leading public fields of Model (include/bnn_model.h)
    _fields_ = [("version", ctypes.c_int), ("base_channels", ctypes.c_int),
                ("n_bands", ctypes.c_int), ("n_classes", ctypes.c_int),
                ("upsampler", ctypes.c_int)]


_lib = None


def lib():
    """Load libbnn_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} missing: build it with `make -C bnns_to_c_b200/csrc` "
                          "(or __graft_entry__.build())")
    L = ctypes.CDLL(LIB_PATH)
    vp, ip, cp = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
    sig = {
        "bnn_last_error": (cp, []),
        "bnn_load_ex": (ip, [cp, ctypes.POINTER(vp)]),
        "bnn_load_mem": (ip, [vp, ctypes.c_size_t, ctypes.POINTER(vp)]),
        "bnn_load": (vp, [cp]),
        "bnn_free": (None, [vp]),
        "bnn_forward": (None, [vp, vp, ip, ip, vp]),
        "bnn_forward_batch": (ip, [vp, vp, ip, ip, ip, vp]),
        "bnn_forward_device": (ip, [vp, ip, vp, ip, ip, ip, vp, vp]),
        "bnn_set_devices": (ip, [vp, ctypes.POINTER(ip), ip]),
        "bnn_get_devices": (ip, [vp, ctypes.POINTER(ip), ip]),
        "bnn_set_chunk": (ip, [vp, ip]),
        "bnn_forward_stages": (ip, [vp, vp, ip, ip, vp, STAGE_CB, vp]),
        "bnn_profile_enable": (ip, [vp, ip]),
        "bnn_profile_reset": (None, [vp]),
        "bnn_profile_count": (ip, [vp]),
        "bnn_profile_get": (ip, [vp, ip, ctypes.POINTER(cp), ctypes.POINTER(cp),
                                 ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                 ctypes.POINTER(ip)]),
        "bnn_profile_report": (None, [vp, vp]),
        "bnn_gpu_bconv_dispatch": (ip, [vp, vp, vp] + [ip] * 8),
        "bnn_gpu_conv_realin": (ip, [vp, vp, vp, vp] + [ip] * 8),
        "bnn_gpu_bconv_dispatch_noalloc": (ip, [vp, vp, vp] + [ip] * 8),
        "bnn_bconv_layer_create": (ip, [ip, ip, ip] + [vp] * 9 + [ctypes.POINTER(vp)]),
        "bnn_bconv_layer_run": (ip, [vp, vp, ip, ip, ip, vp, vp, vp, vp, vp]),
        "bnn_bconv_layer_destroy": (None, [vp]),
        "bnn_synth_device": (ip, [ip, ctypes.c_uint32, ctypes.c_uint32, ip, ip, ip, ip, vp, vp]),
        "bnn_pack_act_device": (ip, [vp, ip, ip, ip, ip, vp, vp]),
        "bnn_unpack_act_device": (ip, [vp, ip, ip, ip, ip, vp, vp]),
        "bnn_forward_launches": (ip, [vp, ip, ip, ip]),
        "bnn_set_bconv_kernel": (ip, [ip]),
        "bnn_device_error": (ip, [ip, ctypes.POINTER(ctypes.c_uint)]),
        "bnn_set_first_conv_kernel": (ip, [ip]),
        "bnn_forward_patched": (ip, [vp, vp, ip, ip, vp, ip]),
        "bnn_forward_patched_device": (ip, [vp, ip, vp, ip, ip, ip, vp, vp]),
        "bnn_first_conv_device": (ip, [vp, ip, vp, ip, ip, ip, vp, ip, ctypes.POINTER(ctypes.c_uint), vp]),
        "bnn_stem_load_ex": (ip, [cp, ctypes.POINTER(vp)]),
        "bnn_stem_load_mem": (ip, [vp, ctypes.c_size_t, ctypes.POINTER(vp)]),
        "bnn_stem_load": (vp, [cp]),
        "bnn_stem_free": (None, [vp]),
        "bnn_stem_forward": (None, [vp, vp, ip, ip, vp]),
        "bnn_stem_as_model": (vp, [vp]),
        "bnn_react_load_ex": (ip, [cp, ctypes.POINTER(vp)]),
        "bnn_react_load_mem": (ip, [vp, ctypes.c_size_t, ctypes.POINTER(vp)]),
        "bnn_load_react": (vp, [cp]),
        "bnn_free_react": (None, [vp]),
        "bnn_forward_react": (None, [vp, vp, ip, ip, vp]),
        "bnn_forward_react_batch": (ip, [vp, vp, ip, ip, ip, vp]),
        "bnn_forward_react_device": (ip, [vp, ip, vp, ip, ip, ip, vp, vp]),
        "bnn_forward_react_patched_ex": (ip, [vp, vp, ip, ip, vp, ip]),
        "bnn_forward_react_stages": (ip, [vp, vp, ip, ip, vp, STAGE_CB, vp]),
        "bnn_react_profile_enable": (ip, [vp, ip]),
        "bnn_react_profile_reset": (None, [vp]),
        "bnn_react_profile_count": (ip, [vp]),
        "bnn_react_profile_get": (ip, [vp, ip, ctypes.POINTER(cp), ctypes.POINTER(cp),
                                       ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                       ctypes.POINTER(ip)]),
        "bnn_react_forward_launches": (ip, [vp, ip, ip, ip]),
        "bnn_react_set_conv_kernel": (ip, [ip]),
        "bnn_react_device_error": (ip, [ip, ctypes.POINTER(ctypes.c_uint)]),
        "bnn_wait_probe": (ip, [ip, ip, ctypes.POINTER(ip), ctypes.POINTER(ctypes.c_uint)]),
        "bnn_debug_inject_fault": (ip, [ip, ip]),
        "bnn_bconv_last_kernel": (cp, []),
        "bnn_set_arena_poison": (ip, [ip]),
        "bnn_arena_poison": (ip, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(rc):
    if rc != BNN_OK:
        raise BnnError(rc, lib().bnn_last_error().decode())


def _ptr(a):
    if a is None:
        return None
    if hasattr(a, "data_ptr"):  # torch tensor
        return a.data_ptr()
    if isinstance(a, int):
        return a
    return a.ctypes.data


class Model:
    """A loaded blob (reference ``Model *bnn_load(path)``)."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        L = lib()
        h = ctypes.c_void_p()
        if data is not None:
            buf = ctypes.create_string_buffer(data, len(data))
            _check(L.bnn_load_mem(buf, len(data), ctypes.byref(h)))
        else:
            _check(L.bnn_load_ex(os.fsencode(path), ctypes.byref(h)))
        self.handle = h.value
        hdr = _ModelHeader.from_address(self.handle)
        self.version, self.base_channels = hdr.version, hdr.base_channels
        self.n_bands, self.n_classes, self.upsampler = hdr.n_bands, hdr.n_classes, hdr.upsampler

    def close(self):
        if getattr(self, "handle", None):
            lib().bnn_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- forwards ----------------------------------------------------
    def forward(self, x: np.ndarray) -> np.ndarray:
        """One patch [bands, H, W] float32 -> logits [classes, H, W]
        (reference ``bnn_forward``), through the status-returning batch
        entry point so errors raise instead of exiting."""
        return self.forward_batch(x[None])[0]

    def forward_batch(self, x: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, bands, H, W = x.shape
        if bands != self.n_bands:
            raise ValueError(f"input has {bands} bands, model expects {self.n_bands}")
        if out is None:
            out = np.empty((n, self.n_classes, H, W), np.float32)
        _check(lib().bnn_forward_batch(self.handle, _ptr(x), n, H, W, _ptr(out)))
        return out

    def forward_device(self, device: int, d_in, n: int, H: int, W: int, d_out, stream=None):
        """Enqueue on device memory (pointers or torch CUDA tensors)."""
        _check(lib().bnn_forward_device(self.handle, device, _ptr(d_in), n, H, W, _ptr(d_out),
                                        stream if stream is None or isinstance(stream, int)
                                        else stream.cuda_stream))

    def stages(self, x: np.ndarray):
        """Every intermediate of one forward, in order (name -> array)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        bands, H, W = x.shape
        logits = np.empty((self.n_classes, H, W), np.float32)
        out = {}
        ct = {0: ctypes.c_int8, 1: ctypes.c_int32, 2: ctypes.c_float}

        def cb(ctx, name, kind, C, h, w, data):
            n = C * h * w
            arr = np.ctypeslib.as_array(ctypes.cast(data, ctypes.POINTER(ct[kind])), shape=(max(n, 1),))
            out[name.decode()] = arr[:n].copy().reshape(C, h, w)

        fn = STAGE_CB(cb)
        _check(lib().bnn_forward_stages(self.handle, _ptr(x), H, W, _ptr(logits), fn, None))
        return out

    def first_conv_device(self, device, d_in, n, H, W, d_bits, exact=False, stream=None):
        """First conv + real fold alone on device memory; returns the number
        of outputs the production path sent to the exact fix-up."""
        und = ctypes.c_uint()
        _check(lib().bnn_first_conv_device(self.handle, device, _ptr(d_in), n, H, W, _ptr(d_bits),
                                           1 if exact else 0, ctypes.byref(und),
                                           stream if stream is None or isinstance(stream, int)
                                           else stream.cuda_stream))
        return und.value

    def set_devices(self, devices):
        arr = (ctypes.c_int * max(1, len(devices)))(*devices)
        _check(lib().bnn_set_devices(self.handle, arr, len(devices)))

    def forward_patched(self, cube, P=32, out=None):
        """Whole-scene patch-wise forward (the reference's tiler): host
        [bands, H, W] float32 -> [classes, H, W]."""
        cube = np.ascontiguousarray(cube, np.float32)
        _, H, W = cube.shape
        if out is None:
            out = np.empty((self.n_classes, H, W), np.float32)
        _check(lib().bnn_forward_patched(self.handle, cube.ctypes.data, H, W, out.ctypes.data, P))
        return out

    def forward_patched_device(self, device, d_cube, H, W, d_logits, P=32, stream=None):
        _check(lib().bnn_forward_patched_device(self.handle, device, _ptr(d_cube), H, W, P, _ptr(d_logits),
                                                stream if stream is None or isinstance(stream, int)
                                                else stream.cuda_stream))

    def set_chunk(self, n):
        _check(lib().bnn_set_chunk(self.handle, n))

    def launches(self, n, H, W):
        return lib().bnn_forward_launches(self.handle, n, H, W)

    # -- profiler ----------------------------------------------------
    def profile(self, on=True):
        _check(lib().bnn_profile_enable(self.handle, 1 if on else 0))

    def profile_reset(self):
        lib().bnn_profile_reset(self.handle)

    def profile_records(self):
        L = lib()
        recs = []
        for i in range(L.bnn_profile_count(self.handle)):
            lab, op = ctypes.c_char_p(), ctypes.c_char_p()
            work, ms, calls = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
            _check(L.bnn_profile_get(self.handle, i, ctypes.byref(lab), ctypes.byref(op),
                                     ctypes.byref(work), ctypes.byref(ms), ctypes.byref(calls)))
            recs.append({"label": lab.value.decode(), "op": op.value.decode(), "work": work.value,
                         "ms": ms.value, "calls": calls.value})
        return recs


class _ConvS(ctypes.Structure):
    # ConvS / Conv (include/bnn_model_stem.h, include/bnn_model.h)
    _fields_ = [("tag", ctypes.c_int), ("Cout", ctypes.c_int), ("Cin", ctypes.c_int),
                ("kh", ctypes.c_int), ("kw", ctypes.c_int), ("pad", ctypes.c_int),
                ("stride", ctypes.c_int), ("nwords", ctypes.c_int),
                ("packed", ctypes.c_void_p), ("wsign", ctypes.c_void_p), ("alpha", ctypes.c_void_p)]


class _StemHeader(ctypes.Structure):
    # leading public fields of StemModel (include/bnn_model_stem.h)
    _fields_ = [("version", ctypes.c_int), ("base_channels", ctypes.c_int),
                ("n_bands", ctypes.c_int), ("n_classes", ctypes.c_int),
                ("upsampler", ctypes.c_int), ("has_stem", ctypes.c_int),
                ("n_stem_layers", ctypes.c_int), ("stem_conv", _ConvS)]


class StemModel(Model):
    """A loaded v2 spectral-stem blob (reference ``StemModel
    *bnn_stem_load(path)``, csrc/bnn_model_stem.c). Every ``Model`` method
    runs the v2 forward, through the engine handle ``bnn_stem_as_model``;
    the stage dump starts with "stem.conv.out" and "stem.act"."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        L = lib()
        h = ctypes.c_void_p()
        if data is not None:
            buf = ctypes.create_string_buffer(data, len(data))
            _check(L.bnn_stem_load_mem(buf, len(data), ctypes.byref(h)))
        else:
            _check(L.bnn_stem_load_ex(os.fsencode(path), ctypes.byref(h)))
        self.stem_handle = h.value
        self.handle = L.bnn_stem_as_model(self.stem_handle)
        hdr = _StemHeader.from_address(self.stem_handle)
        self.version, self.base_channels = hdr.version, hdr.base_channels
        self.n_bands, self.n_classes, self.upsampler = hdr.n_bands, hdr.n_classes, hdr.upsampler
        self.stem_channels = hdr.stem_conv.Cout

    def close(self):
        if getattr(self, "stem_handle", None):
            lib().bnn_stem_free(self.stem_handle)
        self.stem_handle = None
        self.handle = None


class ReactModel:
    """A loaded v3 ReActNet blob (reference ``ModelR *bnn_load_react(path)``,
    csrc/bnn_model_react.c)."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        L = lib()
        h = ctypes.c_void_p()
        if data is not None:
            buf = ctypes.create_string_buffer(data, len(data))
            _check(L.bnn_react_load_mem(buf, len(data), ctypes.byref(h)))
        else:
            _check(L.bnn_react_load_ex(os.fsencode(path), ctypes.byref(h)))
        self.handle = h.value
        hdr = _ModelHeader.from_address(self.handle)
        self.version, self.base_channels = hdr.version, hdr.base_channels
        self.n_bands, self.n_classes, self.upsampler = hdr.n_bands, hdr.n_classes, hdr.upsampler

    def close(self):
        if getattr(self, "handle", None):
            lib().bnn_free_react(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x: np.ndarray) -> np.ndarray:
        return self.forward_batch(np.asarray(x, np.float32)[None])[0]

    def forward_batch(self, x: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        n, _, H, W = x.shape
        if out is None:
            out = np.empty((n, self.n_classes, H, W), np.float32)
        _check(lib().bnn_forward_react_batch(self.handle, x.ctypes.data, n, H, W, out.ctypes.data))
        return out

    def forward_device(self, device: int, d_in, n: int, H: int, W: int, d_out, stream=None):
        s = stream.cuda_stream if hasattr(stream, "cuda_stream") else stream
        _check(lib().bnn_forward_react_device(self.handle, device, _ptr(d_in), n, H, W, _ptr(d_out), s))

    def forward_patched(self, cube, P=32, out=None):
        cube = np.ascontiguousarray(cube, np.float32)
        _, H, W = cube.shape
        if out is None:
            out = np.empty((self.n_classes, H, W), np.float32)
        _check(lib().bnn_forward_react_patched_ex(self.handle, cube.ctypes.data, H, W, out.ctypes.data, P))
        return out

    def stages(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        _, H, W = x.shape
        logits = np.zeros((self.n_classes, H, W), np.float32)
        out = {}
        ct = {0: ctypes.c_int8, 1: ctypes.c_int32, 2: ctypes.c_float}

        def cb(ctx, name, kind, C, h, w, data):
            k = C * h * w
            arr = np.ctypeslib.as_array(ctypes.cast(data, ctypes.POINTER(ct[kind])), shape=(max(k, 1),))
            out[name.decode()] = arr[:k].copy().reshape(C, h, w)

        fn = STAGE_CB(cb)
        _check(lib().bnn_forward_react_stages(self.handle, x.ctypes.data, H, W, logits.ctypes.data, fn, None))
        return out

    def launches(self, n, H, W):
        return lib().bnn_react_forward_launches(self.handle, n, H, W)

    def profile(self, on=True):
        _check(lib().bnn_react_profile_enable(self.handle, 1 if on else 0))

    def profile_reset(self):
        lib().bnn_react_profile_reset(self.handle)

    def profile_records(self):
        L = lib()
        recs = []
        for i in range(L.bnn_react_profile_count(self.handle)):
            lab, op = ctypes.c_char_p(), ctypes.c_char_p()
            work, ms, calls = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
            _check(L.bnn_react_profile_get(self.handle, i, ctypes.byref(lab), ctypes.byref(op),
                                           ctypes.byref(work), ctypes.byref(ms), ctypes.byref(calls)))
            recs.append({"label": lab.value.decode(), "op": op.value.decode(), "work": work.value,
                         "ms": ms.value, "calls": calls.value})
        return recs


def set_react_conv_kernel(kind: str):
    """enc1 real-conv kernel of the ReAct engine: 'tma' (default) or 'plain'."""
    _check(lib().bnn_react_set_conv_kernel({"tma": 0, "plain": 1}[kind]))


def react_wait_timeouts(device=0):
    n = ctypes.c_uint()
    _check(lib().bnn_react_device_error(device, ctypes.byref(n)))
    return n.value


def load_stem(path: str) -> StemModel:
    """Reference ``bnn_stem_load`` (status-raising form)."""
    return StemModel(path)


def load(path: str) -> Model:
    return Model(path)


# ---------------- kernel-level helpers ----------------
def gpu_bconv_dispatch(a: np.ndarray, packed_w: np.ndarray, cout: int, pad: int = 1) -> np.ndarray:
    """Reference ``bconv_dispatch`` semantics on the GPU: int8 [Cin,H,W] ->
    int32 P [Cout, Ho, Wo]."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    w = np.ascontiguousarray(packed_w, dtype=np.uint64)
    cin, H, W = a.shape
    ho, wo = H + 2 * pad - 2, W + 2 * pad - 2
    P = np.zeros((cout, max(ho, 0), max(wo, 0)), np.int32)
    _check(lib().bnn_gpu_bconv_dispatch(_ptr(a), _ptr(w), _ptr(P), cin, H, W, cout, 3, 3, pad, 1))
    return P


def gpu_conv_realin(x: np.ndarray, wsign: np.ndarray, alpha: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    ws = np.ascontiguousarray(wsign, dtype=np.int8)
    al = np.ascontiguousarray(alpha, dtype=np.float32)
    cin, H, W = x.shape
    cout = ws.shape[0]
    out = np.zeros((cout, H, W), np.float32)
    _check(lib().bnn_gpu_conv_realin(_ptr(x), _ptr(ws), _ptr(al), _ptr(out), cin, H, W, cout, 3, 3, 1, 1))
    return out


class BconvLayer:
    """One fused binary conv layer on device memory (isolated-kernel API)."""

    def __init__(self, device, cin, cout, packed_kidx, fold, pool_fold=None):
        self._keep = [np.ascontiguousarray(packed_kidx, np.uint64)]
        f = [np.ascontiguousarray(fold[k], np.int32) for k in ("type", "t", "lo", "hi")]
        self._keep += f
        if pool_fold is not None:
            pf = [np.ascontiguousarray(pool_fold[k], np.int32) for k in ("type", "t", "lo", "hi")]
            self._keep += pf
        else:
            pf = [None] * 4
        h = ctypes.c_void_p()
        _check(lib().bnn_bconv_layer_create(device, cin, cout, _ptr(self._keep[0]), *[_ptr(v) for v in f],
                                            *[_ptr(v) for v in pf], ctypes.byref(h)))
        self.handle = h.value
        self.cin, self.cout, self.pool = cin, cout, pool_fold is not None

    def run(self, d_in, n, H, W, d_out, d_out_pool=None, d_P=None, d_Ppool=None, stream=None):
        _check(lib().bnn_bconv_layer_run(self.handle, _ptr(d_in), n, H, W, _ptr(d_out), _ptr(d_out_pool),
                                         _ptr(d_P), _ptr(d_Ppool),
                                         stream if stream is None or isinstance(stream, int)
                                         else stream.cuda_stream))

    def close(self):
        if getattr(self, "handle", None):
            lib().bnn_bconv_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def set_bconv_kernel(kind: str):
    """'tc' (default: tcgen05, int8 operands, e2m1 for the deeper non-pooled
    layers: 64/128 channels with at least 4 input words, 256 with at least
    16; mma.sync where the staging does not fit), 'tc8' (tcgen05 int8 throughout), 'tcx' (as
    'tc8', with the column taps in N for the non-pooled layers of at most 32
    channels), 'tc4' (tcgen05 e2m1 for every non-pooled layer), 'popc'
    (XOR + POPC) or 'mma' (mma.sync for every layer)."""
    _check(lib().bnn_set_bconv_kernel({"tc": 0, "popc": 1, "mma": 2, "tcx": 3, "tc8": 4, "tc4": 5}[kind]))


def set_first_conv_kernel(kind):
    """'tc' (tcgen05, nine shifted taps; default), 'mma' (mma.sync) or
    'tcn' (tcgen05 with the column taps in N where W divides 32) or 'tx'
    (tcgen05 with the weights in M and the positions in N) for the first
    conv."""
    _check(lib().bnn_set_first_conv_kernel({"tc": 0, "mma": 1, "tcn": 2, "tx": 3}[kind]))


def device_wait_timeouts(device=0):
    n = ctypes.c_uint()
    _check(lib().bnn_device_error(device, ctypes.byref(n)))
    return n.value


def set_arena_poison(byte):
    """Fill the activation arenas with `byte` (0..255) before every forward,
    or stop (None / -1): the debug mode BNN_ARENA_POISON turns on."""
    _check(lib().bnn_set_arena_poison(-1 if byte is None else int(byte)))


def arena_poison():
    """The poison byte in force, None when off."""
    b = lib().bnn_arena_poison()
    return None if b < 0 else b


def wait_probe(device=0, rounds=4096):
    """Run the bounded-wait self-test kernel (an mbarrier phase nothing
    completes). Returns (gave_up, device counter afterwards)."""
    g, n = ctypes.c_int(), ctypes.c_uint()
    _check(lib().bnn_wait_probe(device, rounds, ctypes.byref(g), ctypes.byref(n)))
    return bool(g.value), n.value


FAULT_ALLOC, FAULT_WAIT, FAULT_SHARD = 1, 2, 3


def inject_fault(kind: int, arg: int = 0):
    """Host-side fault injection (bnn_debug_inject_fault); kind 0 clears."""
    _check(lib().bnn_debug_inject_fault(kind, arg))


def bconv_last_kernel() -> str:
    """Name and template parameters of the last binary-conv kernel this
    thread launched."""
    return lib().bnn_bconv_last_kernel().decode()


def synth_device(device, seed, first, n, bands, H, W, d_out, stream=None):
    _check(lib().bnn_synth_device(device, seed, first, n, bands, H, W, _ptr(d_out),
                                  stream if stream is None or isinstance(stream, int) else stream.cuda_stream))


def pack_act_device(d_a, n, c, H, W, d_bits, stream=None):
    _check(lib().bnn_pack_act_device(_ptr(d_a), n, c, H, W, _ptr(d_bits), stream))


def unpack_act_device(d_bits, n, c, H, W, d_a, stream=None):
    _check(lib().bnn_unpack_act_device(_ptr(d_bits), n, c, H, W, _ptr(d_a), stream))


def shard_range(n: int, rank: int, world: int):
    """Contiguous patch-index slice of rank ``rank`` (same split as the
    library's multi-device batches and the benchmark's ranks)."""
    return (n * rank) // world, (n * (rank + 1)) // world
