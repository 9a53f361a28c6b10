"""One mixed-bit linear layer through ``altxs_linear``: tensor cores and CUDA
cores against a float64 product of the exact dequantised weights."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from altxs_b200 import codec as Cd
from altxs_b200.config import ModelConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")

CFG = dict(vocab_size=1000, num_layers=2, model_dim=256, num_heads=4, num_kv_heads=2, mlp_mult=4.0,
           rope_dims=16, block_size=32, seed=11)


@pytest.fixture(scope="module")
def model():
    from altxs_b200.engine import DeviceModel

    cfg = ModelConfig(**CFG)
    return DeviceModel(Cd.synth_weights(cfg, seed=21), DEV)


def _dense(dm, name):
    from altxs_b200 import _lib

    q = dm.q[name]
    t = torch.empty((q.rows, q.cols), dtype=torch.float32, device=DEV)
    _lib.check(_lib.lib().altxs_dequant(C.byref(q), t.data_ptr(), q.cols, None), "altxs_dequant")
    return t.cpu().numpy().astype(np.float64)


def _linear(dm, name, X, row0, N, tensor_cores):
    from altxs_b200 import _lib

    L = _lib.lib()
    q = dm.q[name]
    M = X.shape[0]
    Xd = torch.as_tensor(X, device=DEV).contiguous()
    Y = torch.full((M, N), float("nan"), dtype=torch.float32, device=DEV)
    ws_b = int(L.altxs_linear_workspace_bytes(M, q.cols))
    ws = torch.empty(max(ws_b, 1), dtype=torch.uint8, device=DEV)
    sp = dm._split
    hi = getattr(sp, f"{name}_hi") if tensor_cores else None
    lo = getattr(sp, f"{name}_lo") if tensor_cores else None
    rc = L.altxs_linear(C.byref(q), hi, lo, row0, N, Xd.data_ptr(), M, Y.data_ptr(), ws.data_ptr(), ws_b, None)
    assert rc == 0
    torch.cuda.synchronize()
    return Y.cpu().numpy()


def test_split_planes_are_exact_for_symmetric_levels(model):
    """hi + lo reproduces every dequantised weight of the 2/3/4-bit groups."""
    for name in ("qkv", "down", "emb"):
        W = _dense(model, name)
        hi = model._split_bufs[2 * ("emb", "qkv", "o", "up", "down").index(name)].float().cpu().numpy()
        lo = model._split_bufs[2 * ("emb", "qkv", "o", "up", "down").index(name) + 1].float().cpu().numpy()
        assert np.array_equal((hi.astype(np.float64) + lo), W), name


@pytest.mark.parametrize("tensor_cores", [True, False])
@pytest.mark.parametrize("name,row0,N,M", [("qkv", 0, 512, 1), ("qkv", 512, 512, 130), ("down", 256, 256, 300),
                                          ("emb", 0, 1000, 77), ("up", 1024, 136, 5)])
def test_linear_matches_float64(model, tensor_cores, name, row0, N, M):
    W = _dense(model, name)
    rng = np.random.default_rng(M + N)
    X = rng.normal(0, 1, size=(M, W.shape[1])).astype(np.float32)
    got = _linear(model, name, X, row0, N, tensor_cores)
    ref = X.astype(np.float64) @ W[row0: row0 + N].T
    bound = np.abs(X.astype(np.float64)) @ np.abs(W[row0: row0 + N]).T
    # tensor cores: products within 2^-16 relative; CUDA cores: fp32 rounding
    rel = 2.0 ** -15 if tensor_cores else 2.0 ** -18
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - ref) <= rel * bound + 1e-30), float(np.max(np.abs(got - ref) / (bound + 1e-30)))


def test_tensor_core_rows_do_not_depend_on_the_batch(model):
    """Row i of a 300-row call equals the same row computed alone, bit for bit."""
    rng = np.random.default_rng(5)
    X = rng.normal(0, 1, size=(300, 256)).astype(np.float32)
    full = _linear(model, "qkv", X, 0, 512, True)
    for i in (0, 127, 128, 255, 299):
        alone = _linear(model, "qkv", X[i: i + 1], 0, 512, True)
        assert np.array_equal(alone.view(np.uint32), full[i: i + 1].view(np.uint32)), i


def _gemm(A, B, M, N, K, tA, tB, batch, alpha=1.0, beta=0.0, C0=None, causal=0):
    from altxs_b200 import _lib

    L = _lib.lib()
    Ad = torch.as_tensor(A, device=DEV).contiguous()
    Bd = torch.as_tensor(B, device=DEV).contiguous()
    C = torch.as_tensor(C0 if C0 is not None else np.zeros((batch, M, N), np.float32), device=DEV).contiguous()
    lda, ldb = Ad.shape[-1], Bd.shape[-1]
    wsb = int(L.altxs_gemm_workspace_bytes(M, N, K, tA, tB, batch))
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    rc = L.altxs_gemm(M, N, K, Ad.data_ptr(), lda, Ad[0].numel(), tA, Bd.data_ptr(), ldb, Bd[0].numel(), tB,
                      C.data_ptr(), N, M * N, batch, alpha, beta, causal, ws.data_ptr(), wsb, None)
    assert rc == 0
    torch.cuda.synchronize()
    return C.cpu().numpy()


@pytest.mark.parametrize("tA,tB", [(0, 1), (0, 0), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K,batch", [(200, 96, 333, 3), (64, 64, 2048, 2), (300, 130, 64, 1)])
def test_gemm_transposes_match_float64(tA, tB, M, N, K, batch):
    """Every operand orientation (K-major and MN-major tensor-core tiles),
    ragged sizes, batches, alpha and beta, against float64."""
    rng = np.random.default_rng(M * 7 + N + K + 3 * tA + tB)
    A = rng.normal(0, 1, size=(batch, K, M) if tA else (batch, M, K)).astype(np.float32)
    B = rng.normal(0, 1, size=(batch, N, K) if tB else (batch, K, N)).astype(np.float32)
    C0 = rng.normal(0, 1, size=(batch, M, N)).astype(np.float32)
    got = _gemm(A, B, M, N, K, tA, tB, batch, alpha=0.5, beta=0.25, C0=C0)
    opA = np.swapaxes(A, 1, 2) if tA else A
    opB = np.swapaxes(B, 1, 2) if tB else B
    ref = 0.5 * np.einsum("bmk,bkn->bmn", opA.astype(np.float64), opB.astype(np.float64)) + 0.25 * C0
    bound = 0.5 * np.einsum("bmk,bkn->bmn", np.abs(opA).astype(np.float64), np.abs(opB).astype(np.float64))
    err = np.abs(got - ref)
    assert np.all(err <= 2.0 ** -15 * bound + 2.0 ** -22 * np.abs(ref) + 1e-30), float((err / (bound + 1e-30)).max())


@pytest.mark.parametrize("causal", [2, 3])
def test_gemm_triangular_operands(causal):
    """Modes 2/3 read only the K range a triangular op(A) can be nonzero in."""
    rng = np.random.default_rng(causal)
    T, N = 300, 64
    A = rng.normal(0, 1, size=(1, T, T)).astype(np.float32)
    A[0] = np.tril(A[0]) if causal == 2 else np.triu(A[0])
    B = rng.normal(0, 1, size=(1, T, N)).astype(np.float32)
    got = _gemm(A, B, T, N, T, 0, 0, 1, causal=causal)
    ref = A[0].astype(np.float64) @ B[0].astype(np.float64)
    bound = np.abs(A[0]).astype(np.float64) @ np.abs(B[0]).astype(np.float64)
    assert np.all(np.abs(got[0] - ref) <= 2.0 ** -15 * bound + 1e-30)


def test_rows_do_not_depend_on_tile_width():
    """At the 33M shapes a 2048-row call runs 128-wide output tiles and a
    1-row call 64-wide ones: rows must agree bit for bit all the same."""
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel

    dm = DeviceModel(Cd.synth_weights(c3_config(), seed=5), DEV)
    rng = np.random.default_rng(9)
    for name, N in (("qkv", 1536), ("emb", 16384)):
        X = rng.normal(0, 1, size=(2048, 512)).astype(np.float32)
        full = _linear(dm, name, X, 0, N, True)
        for i in (0, 700, 2047):
            alone = _linear(dm, name, X[i: i + 1], 0, N, True)
            assert np.array_equal(alone.view(np.uint32), full[i: i + 1].view(np.uint32)), (name, i)


def _linear_tc(dm, name, X, row0, N):
    """The step's tensor-core linear: packed weights expanded by the GEMM's
    producer warps, K split by layer shape."""
    from altxs_b200 import _lib

    L = _lib.lib()
    t = getattr(dm.tiles, name)
    M = X.shape[0]
    Xd = torch.as_tensor(X, device=DEV).contiguous()
    Y = torch.full((M, N), float("nan"), dtype=torch.float32, device=DEV)
    ws_b = int(L.altxs_linear_tc_workspace_bytes(M, N, t.cols))
    ws = torch.empty(max(ws_b, 1), dtype=torch.uint8, device=DEV)
    assert L.altxs_linear_tc(C.byref(t), row0, N, Xd.data_ptr(), M, Y.data_ptr(), ws.data_ptr(), ws_b, None) == 0
    torch.cuda.synchronize()
    return Y.cpu().numpy()


@pytest.mark.parametrize("name,row0,N,M", [("qkv", 0, 512, 1), ("qkv", 512, 512, 130), ("down", 256, 256, 300),
                                          ("down", 0, 256, 1), ("emb", 0, 1000, 77), ("up", 1024, 136, 5),
                                          ("o", 0, 256, 260)])
def test_packed_weight_gemm_matches_planes_and_float64(model, name, row0, N, M):
    """Expanding the packed codes in the GEMM's producer warps gives the same
    products as the dequantised planes: bit-identical output (where a layer's
    K loop is split the bits may differ: then within the tensor-core bound of
    float64, which every output meets)."""
    from altxs_b200 import _lib

    W = _dense(model, name)
    rng = np.random.default_rng(M + N + 1)
    X = rng.normal(0, 1, size=(M, W.shape[1])).astype(np.float32)
    got = _linear_tc(model, name, X, row0, N)
    planes = _linear(model, name, X, row0, N, True)
    assert np.all(np.isfinite(got))
    if _lib.lib().altxs_linear_tc_workspace_bytes(M, N, W.shape[1]) == _lib.lib().altxs_linear_workspace_bytes(
            M, W.shape[1]):  # no split scratch: the layer is not split
        assert np.array_equal(got.view(np.uint32), planes.view(np.uint32)), name
    ref = X.astype(np.float64) @ W[row0: row0 + N].T
    bound = np.abs(X.astype(np.float64)) @ np.abs(W[row0: row0 + N]).T
    assert np.all(np.abs(got - ref) <= 2.0 ** -15 * bound + 1e-30)


@pytest.mark.parametrize("name,N", [("qkv", 1536), ("o", 512), ("down", 512), ("up", 2048), ("emb", 16384)])
def test_packed_weight_gemm_rows_do_not_depend_on_the_batch(name, N):
    """33M shapes (split o and down layers included): rows of a 2048-row call
    and of a 256-row call equal the rows computed alone, bit for bit."""
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel

    dm = DeviceModel(Cd.synth_weights(c3_config(), seed=5), DEV)
    K = dm.q[name].cols
    rng = np.random.default_rng(11)
    X = rng.normal(0, 1, size=(2048, K)).astype(np.float32)
    full = _linear_tc(dm, name, X, 0, N)
    part = _linear_tc(dm, name, X[:256], 0, N)
    assert np.array_equal(part.view(np.uint32), full[:256].view(np.uint32)), name
    for i in (0, 129, 2047):
        alone = _linear_tc(dm, name, X[i: i + 1], 0, N)
        assert np.array_equal(alone.view(np.uint32), full[i: i + 1].view(np.uint32)), (name, i)
    from altxs_b200 import _lib

    L = _lib.lib()
    if L.altxs_linear_tc_workspace_bytes(2048, N, K) == L.altxs_linear_workspace_bytes(2048, K):
        planes = _linear(dm, name, X, 0, N, True)  # unsplit layer: the same bits as the plane path
        assert np.array_equal(full.view(np.uint32), planes.view(np.uint32)), name
    W = _dense(dm, name)
    ref = X[:64].astype(np.float64) @ W[:N].T
    bound = np.abs(X[:64].astype(np.float64)) @ np.abs(W[:N]).T
    assert np.all(np.abs(full[:64] - ref) <= 2.0 ** -15 * bound + 1e-30)


@pytest.mark.parametrize("c3", [False, True])
def test_step_with_packed_linears_is_bit_identical(model, c3):
    """The decode step with its tensor-core linears reading the packed codes
    (altxs_set_linear_packed(1)) gives the same logits, bit for bit, as with
    the dense planes."""
    from altxs_b200 import _lib
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel
    from tests.test_gpu_step import _run_logits

    dm = DeviceModel(Cd.synth_weights(c3_config(), seed=5), DEV) if c3 else model
    assert dm.tiles is not None
    rng = np.random.default_rng(4)
    toks = [rng.integers(0, dm.cfg.vocab_size, size=12) for _ in range(40 if c3 else 7)]
    L = _lib.lib()
    try:
        assert L.altxs_set_linear_packed(0) == 0
        planes = _run_logits(dm, toks)
        assert L.altxs_set_linear_packed(1) == 0
        packed = _run_logits(dm, toks)
    finally:
        L.altxs_set_linear_packed(0)
    assert np.isfinite(packed).all()
    assert np.array_equal(planes.view(np.uint32), packed.view(np.uint32))
