"""CPU checks of the window-attention entry points: argument validation runs
before any CUDA call, so a bad shape is refused without a GPU."""

from __future__ import annotations

import ctypes

from altxs_b200 import _lib


def _fwd(L, T, H, Hkv, hd, ld=None):
    ld = ld if ld is not None else H * hd
    return L.altxs_window_attention(T, H, Hkv, hd, ctypes.c_float(1.0), None, ld, None, Hkv * hd, None, Hkv * hd,
                                    None, ld, None, None, 0, None)


def _bwd(L, T, H, Hkv, hd):
    d, kvd = H * hd, Hkv * hd
    return L.altxs_window_attention_backward(T, H, Hkv, hd, ctypes.c_float(1.0), None, d, None, kvd, None, kvd, None,
                                             d, None, None, d, None, d, None, kvd, None, kvd, None, 0, None)


def test_forward_refuses_bad_shapes_before_touching_the_device():
    L = _lib.lib()
    assert _fwd(L, 8, 3, 2, 32) == _lib.ALTXS_EINVAL      # H not a multiple of Hkv
    assert _fwd(L, 8, 4, 2, 32, ld=64) == _lib.ALTXS_EINVAL  # q rows narrower than H * hd
    assert _fwd(L, -1, 4, 2, 32) == _lib.ALTXS_EINVAL
    assert _fwd(L, 8, 2, 2, 128) == _lib.ALTXS_ENOTSUP    # head size without a kernel
    assert _fwd(L, 0, 4, 2, 64) == 0                       # nothing to do


def test_backward_refuses_bad_shapes_before_touching_the_device():
    L = _lib.lib()
    assert _bwd(L, 8, 3, 2, 32) == _lib.ALTXS_EINVAL
    assert _bwd(L, 8, 2, 2, 16) == _lib.ALTXS_ENOTSUP
    assert _bwd(L, 0, 4, 2, 64) == 0


def test_workspace_sizes():
    L = _lib.lib()
    assert L.altxs_window_attention_workspace_bytes(-1, 4, 2, 64) == -1
    assert L.altxs_window_attention_backward_workspace_bytes(2047, 8, 8, 64) > \
        L.altxs_window_attention_workspace_bytes(2047, 8, 8, 64) > 0
