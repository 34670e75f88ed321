"""Activation arenas filled with a poison byte before every forward (the
BNN_ARENA_POISON debug mode, the device-side form of
csrc/bnn_react_arena.c:30-32). The logits and every dumped stage must stay
the same bits for the v1, v2-stem and ReAct engines: a launch that read an
arena word that no earlier launch of the same forward wrote would change
them under one of the three bytes. The batch path is graph-replayed; the
stage dump and the first conv alone run eagerly."""

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import bnns_to_c_b200 as bn  # noqa: E402
from oracle_util import synth  # noqa: E402

GOLD = os.path.join(os.path.dirname(__file__), "golden")
BYTES = (0x00, 0xFF, 0xA5)
CASES = [
    ("unet_c8_mixed_s1", bn.Model, 37, 23),
    ("unet_c16_base_s2", bn.Model, 32, 32),
    ("stem_c8_mixed_s3", bn.StemModel, 37, 23),
    ("react_c8_s3", bn.ReactModel, 50, 38),
    ("react_c16_s1", bn.ReactModel, 32, 32),
]


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    bn.set_arena_poison(None)
    yield
    bn.set_arena_poison(None)


def same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and a.tobytes() == b.tobytes()


@pytest.mark.parametrize("name,cls,H,W", CASES, ids=[c[0] for c in CASES])
def test_poisoned_arena_changes_nothing(name, cls, H, W):
    m = cls(os.path.join(GOLD, name + ".blob"))
    try:
        x = synth(71, 0, 3, m.n_bands, H, W)
        bn.set_arena_poison(None)
        want = m.forward_batch(x)
        want_st = m.stages(x[1])
        for b in BYTES:
            bn.set_arena_poison(b)
            assert bn.arena_poison() == b
            assert same(m.forward_batch(x), want), f"logits, poison {b:#04x}"
            st = m.stages(x[1])
            assert set(st) == set(want_st)
            for k in want_st:
                assert same(st[k], want_st[k]), f"{k}, poison {b:#04x}"
    finally:
        bn.set_arena_poison(None)
        m.close()


def test_poisoned_arena_first_conv_alone():
    """The first conv's own entry point (its bits and the undecided list
    live in the arena too)."""
    m = bn.Model(os.path.join(GOLD, "unet_c8_mixed_s1.blob"))
    try:
        N, H, W = 4, 32, 32
        x = torch.from_numpy(synth(72, 0, N, m.n_bands, H, W)).cuda()
        cw = (m.base_channels + 31) // 32  # enc1.conv1 has base_channels outputs
        outs = []
        for b in (None,) + BYTES:
            bn.set_arena_poison(b)
            bits = torch.zeros(N * H * W * cw, dtype=torch.int32, device="cuda")
            m.first_conv_device(0, x.data_ptr(), N, H, W, bits.data_ptr())
            torch.cuda.synchronize()
            outs.append(bits.cpu().numpy())
        for o in outs[1:]:
            assert same(o, outs[0])
    finally:
        bn.set_arena_poison(None)
        m.close()
