"""The window attention kernel (tcgen05, online softmax per 128-key tile, no
T x T buffer) against a float64 causal softmax attention, and the context
prefill that runs on it against the materialised attention.

Reference: the causal attention of the reference's window forward
(F.scaled_dot_product_attention(q, k, v, is_causal=True) in
CausalSelfAttention.forward, src/xsa_ttt/model.py; train_attn.py:67).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

from altxs_b200 import _lib
from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = 1e-4  # hi/lo bf16 products keep 16 significand bits: ~1e-5 on unit-scale rows


def _ref(q, k, v, H, Hkv, hd, scale):
    T = q.shape[0]
    G = H // Hkv
    mask = torch.ones(T, T, dtype=torch.bool, device=q.device).tril()
    out = torch.empty(T, H * hd, dtype=torch.float64, device=q.device)
    for h in range(H):
        g = h // G
        s = (q[:, h * hd:(h + 1) * hd].double() @ k[:, g * hd:(g + 1) * hd].double().T) * scale
        p = torch.softmax(s.masked_fill(~mask, float("-inf")), dim=1)
        out[:, h * hd:(h + 1) * hd] = p @ v[:, g * hd:(g + 1) * hd].double()
    return out


def _run(T, H, Hkv, hd, scale, q, k, v, ldy=None, lse=None):
    L = _lib.lib()
    ldy = ldy or H * hd
    y = torch.full((max(T, 1), ldy), float("nan"), device=DEV)
    wsb = int(L.altxs_window_attention_workspace_bytes(T, H, Hkv, hd))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=DEV)
    rc = L.altxs_window_attention(T, H, Hkv, hd, ctypes.c_float(scale), q.data_ptr(), q.stride(0), k.data_ptr(),
                                  k.stride(0), v.data_ptr(), v.stride(0), y.data_ptr(), ldy,
                                  None if lse is None else lse.data_ptr(), ws.data_ptr(), wsb,
                                  torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, y


def _ref_grads(q, k, v, dy, H, Hkv, hd, scale):
    """float64 autograd of the causal attention: (dq, dk, dv)."""
    T, G = q.shape[0], H // Hkv
    qd, kd, vd = (x.detach().double().requires_grad_() for x in (q, k, v))
    mask = torch.ones(T, T, dtype=torch.bool, device=q.device).tril()
    outs = []
    for h in range(H):
        g = h // G
        s = (qd[:, h * hd:(h + 1) * hd] @ kd[:, g * hd:(g + 1) * hd].T) * scale
        outs.append(torch.softmax(s.masked_fill(~mask, float("-inf")), dim=1) @ vd[:, g * hd:(g + 1) * hd])
    torch.cat(outs, dim=1).backward(dy.double())
    return qd.grad, kd.grad, vd.grad


def _run_bwd(T, H, Hkv, hd, scale, q, k, v, y, lse, dy):
    L = _lib.lib()
    dq = torch.full((T, H * hd), float("nan"), device=DEV)
    dk = torch.full((T, Hkv * hd), float("nan"), device=DEV)
    dv = torch.full((T, Hkv * hd), float("nan"), device=DEV)
    wsb = int(L.altxs_window_attention_backward_workspace_bytes(T, H, Hkv, hd))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=DEV)
    rc = L.altxs_window_attention_backward(
        T, H, Hkv, hd, ctypes.c_float(scale), q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(),
        v.stride(0), y.data_ptr(), y.stride(0), lse.data_ptr(), dy.data_ptr(), dy.stride(0), dq.data_ptr(), dq.stride(0),
        dk.data_ptr(), dk.stride(0), dv.data_ptr(), dv.stride(0), ws.data_ptr(), wsb,
        torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, dq, dk, dv


@pytest.mark.parametrize("T,H,Hkv,hd", [(1, 4, 4, 32), (5, 4, 2, 32), (127, 4, 4, 64), (128, 8, 8, 64),
                                         (129, 8, 4, 64), (300, 4, 1, 32), (1000, 8, 2, 64), (2048, 8, 8, 64)])
def test_matches_float64(T, H, Hkv, hd):
    """Ragged and whole key tiles, GQA groups, the strided q/k/v views of a
    fused qkv row (as the window forward stores them)."""
    g = torch.Generator(device=DEV)
    g.manual_seed(T * 131 + hd)
    d, kvd = H * hd, Hkv * hd
    qkv = torch.randn(T, d + 2 * kvd, generator=g, device=DEV)
    q, k, v = qkv[:, :d], qkv[:, d:d + kvd], qkv[:, d + kvd:]
    scale = 1.0 / math.sqrt(hd)
    rc, y = _run(T, H, Hkv, hd, scale, q, k, v)
    assert rc == 0, (rc, _lib.lib().altxs_last_cuda_error())
    err = float((y.double() - _ref(q, k, v, H, Hkv, hd, scale)).abs().max())
    print(f"T={T} H={H} Hkv={Hkv} hd={hd}: max abs error {err:.2e}")
    assert err < TOL


def test_peaked_rows_and_padded_output():
    """Scores of std ~6 (near one-hot rows) and an output row stride wider than H*hd."""
    T, H, Hkv, hd = 400, 4, 2, 64
    g = torch.Generator(device=DEV)
    g.manual_seed(3)
    q = 6.0 * torch.randn(T, H * hd, generator=g, device=DEV)
    k = torch.randn(T, Hkv * hd, generator=g, device=DEV)
    v = torch.randn(T, Hkv * hd, generator=g, device=DEV)
    scale = 1.0 / math.sqrt(hd)
    rc, y = _run(T, H, Hkv, hd, scale, q, k, v, ldy=H * hd + 4)
    assert rc == 0
    ref = _ref(q, k, v, H, Hkv, hd, scale)
    err = float((y[:, :H * hd].double() - ref).abs().max())
    assert err < 4 * TOL, err
    assert bool(torch.isnan(y[:, H * hd:]).all())  # the padding columns are not written


@pytest.mark.parametrize("T,H,Hkv,hd", [(1, 4, 4, 32), (70, 4, 2, 32), (129, 8, 4, 64), (300, 4, 1, 32),
                                         (1000, 8, 2, 64), (2047, 8, 8, 64)])
def test_backward_matches_float64(T, H, Hkv, hd):
    """dq, dk, dv (GQA sums over a group's heads) against float64 autograd, from
    the forward's own output and log-sum-exp; two calls give the same bits."""
    g = torch.Generator(device=DEV)
    g.manual_seed(T * 17 + hd)
    d, kvd = H * hd, Hkv * hd
    qkv = torch.randn(T, d + 2 * kvd, generator=g, device=DEV)
    q, k, v = qkv[:, :d], qkv[:, d:d + kvd], qkv[:, d + kvd:]
    dy = torch.randn(T, d, generator=g, device=DEV)
    scale = 1.0 / math.sqrt(hd)
    lse = torch.empty(H, T, device=DEV)
    rc, y = _run(T, H, Hkv, hd, scale, q, k, v, lse=lse)
    assert rc == 0
    rc, dq, dk, dv = _run_bwd(T, H, Hkv, hd, scale, q, k, v, y, lse, dy)
    assert rc == 0, (rc, _lib.lib().altxs_last_cuda_error())
    ref = _ref_grads(q, k, v, dy, H, Hkv, hd, scale)
    for name, got, want in zip(("dq", "dk", "dv"), (dq, dk, dv), ref):
        # relative to the largest entry (at least 1: with one key dq and dk are 0 up to rounding)
        err = float((got.double() - want).abs().max()) / max(float(want.abs().max()), 1.0)
        print(f"T={T} H={H} Hkv={Hkv} hd={hd} {name}: max error / max(|ref|, 1) = {err:.2e}")
        assert err < 2e-4, name
    rc, dq2, dk2, dv2 = _run_bwd(T, H, Hkv, hd, scale, q, k, v, y, lse, dy)
    assert rc == 0
    for a, b in ((dq, dq2), (dk, dk2), (dv, dv2)):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_refuses_unsupported_shapes():
    q = torch.zeros(8, 256, device=DEV)
    rc, _ = _run(8, 2, 2, 128, 1.0, q, q, q)
    assert rc == _lib.ALTXS_ENOTSUP
    rc, _ = _run(8, 3, 2, 32, 1.0, q, q, q)
    assert rc == _lib.ALTXS_EINVAL


@pytest.mark.parametrize("hd", [32, 64])
def test_prefill_flash_matches_materialised(hd):
    """Context prefill (reset mode) of a 6-tile window on the flash kernel and
    on the materialised attention: the next step's logits agree to fp32
    rounding."""
    from altxs_b200.engine import ContextReset, DeviceModel, StreamBatch

    L = _lib.lib()
    cfg = ModelConfig(vocab_size=512, num_layers=3, model_dim=4 * hd, num_heads=4, num_kv_heads=2, mlp_mult=2.0,
                      rope_dims=16, block_size=700, online_retrain_every=700, seed=5, context_mode="reset")
    dm = DeviceModel(C.synth_weights(cfg, seed=4), DEV, tensor_cores=True)
    rng = np.random.default_rng(11)
    s = torch.as_tensor(rng.integers(0, cfg.vocab_size, size=700), dtype=torch.int32, device=DEV)
    got = []
    try:
        for on in (1, 0):
            assert L.altxs_set_flash(on) == 0
            b = StreamBatch(dm, 1, words_per_stream=8, keep_logits=True, hist_len=cfg.ctx + 2)
            b.hist[0, :700] = s
            ContextReset(dm)(b, [0], 700)
            b.tok.fill_(int(s[699]))
            b.step(_lib.STEP_LOGITS)
            got.append(b.logits[0].clone())
    finally:
        L.altxs_set_flash(1)
    err = float((got[0] - got[1]).abs().max())
    print(f"hd={hd}: flash vs materialised prefill, next-step logits max diff {err:.2e}")
    assert err < 1e-3
