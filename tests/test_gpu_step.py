"""The CUDA model step against the torch oracle, and encode/decode round trips."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig, c3_config
from oracle import coder as oc
from oracle.model import OracleLoRA, OracleModel, OracleWeights

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
TOL = 2e-3  # max-abs logits tolerance vs the fp32 reference path

SMALL = dict(
    vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2,
    mlp_mult=4.0, rope_dims=16, block_size=32, online_retrain_every=64, seed=11,
    ttt_lora_rank=4, ttt_lora_lr=1e-3, ttt_k_lora=True, ttt_o_lora=True,
)


def _small(**kw) -> ModelConfig:
    d = dict(SMALL)
    d.update(kw)
    return ModelConfig(**d)


def _run_logits(dm, toks_by_stream, lora_vec=None):
    """Feed tokens through the device step in LOGITS mode; return [n][T][V]."""
    from altxs_b200 import _lib
    from altxs_b200.engine import StreamBatch

    n = len(toks_by_stream)
    T = len(toks_by_stream[0])
    b = StreamBatch(dm, n, words_per_stream=8, keep_logits=True)
    if lora_vec is not None:
        b.lora.copy_(torch.as_tensor(lora_vec, device=DEV).expand_as(b.lora))
    out = np.zeros((n, T, dm.cfg.vocab_size), dtype=np.float32)
    toks = torch.as_tensor(np.stack(toks_by_stream).astype(np.int32), device=DEV)
    for t in range(T):
        b.tok.copy_(toks[:, t])
        b.step(_lib.STEP_LOGITS)
        out[:, t] = b.logits.cpu().numpy()
        b.pos.add_(1)
    return out


def _lora_vec(cfg, rng):
    """Random adapters (nonzero B) as a flat arena + the oracle equivalent."""
    from altxs_b200.lora import lora_shapes

    lo = OracleLoRA()
    flat = []
    for name, (a_shape, b_shape) in lora_shapes(cfg).items():
        A = rng.uniform(-0.1, 0.1, size=a_shape).astype(np.float32)
        B = rng.normal(0, 0.02, size=b_shape).astype(np.float32)
        lo.A[name], lo.B[name] = torch.from_numpy(A), torch.from_numpy(B)
        flat += [A.reshape(-1), B.reshape(-1)]
    return np.concatenate(flat), lo


@pytest.mark.parametrize("tensor_cores", [True, False])
@pytest.mark.parametrize("use_lora", [False, True])
def test_step_logits_match_oracle(use_lora, tensor_cores):
    from altxs_b200.engine import DeviceModel

    cfg = _small()
    w = C.synth_weights(cfg, seed=7)
    dm = DeviceModel(w, DEV, tensor_cores=tensor_cores)
    om = OracleModel(OracleWeights.from_model_weights(w))
    rng = np.random.default_rng(1)
    T = 80  # > ctx: exercises the sliding window
    toks = rng.integers(0, cfg.vocab_size, size=T)
    vec, lo = _lora_vec(cfg, rng) if use_lora else (None, None)
    got = _run_logits(dm, [toks], vec)[0]
    st = om.new_stream()
    ref = np.stack([om.step(st, int(t), lo).numpy() for t in toks])
    err = float(np.abs(got - ref).max())
    assert err < TOL, err


def test_step_matches_reference_golden(golden):
    """Device logits vs the reference GPT's sliding-window logits (golden)."""
    from altxs_b200.engine import DeviceModel

    g = golden("model_small.npz")
    cfg = _small()
    dm = DeviceModel(C.synth_weights(cfg, seed=7), DEV)
    got = _run_logits(dm, [g["tokens"]])[0]
    err = float(np.abs(got - g["logits"]).max())
    assert err < TOL, err


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_step_is_batch_independent(tensor_cores):
    """A stream's logits are bit-identical alone and inside batches of 40 and
    200 (first slot; slot 137, i.e. the second 128-row tile and another
    tensor-memory lane), whatever the other streams hold.  On CUDA cores this
    also crosses the GEMV/tiled split."""
    from altxs_b200.engine import DeviceModel

    cfg = _small(block_size=64)
    dm = DeviceModel(C.synth_weights(cfg, seed=3), DEV, tensor_cores=tensor_cores)
    rng = np.random.default_rng(2)
    T = 24
    base = rng.integers(0, cfg.vocab_size, size=T)
    alone = _run_logits(dm, [base])[0]
    others = [rng.integers(0, cfg.vocab_size, size=T) for _ in range(199)]
    batched = _run_logits(dm, [base] + others[:39])[0]
    assert np.array_equal(alone.view(np.uint32), batched.view(np.uint32))
    big = _run_logits(dm, others[:137] + [base] + others[137:199])[137]
    assert np.array_equal(alone.view(np.uint32), big.view(np.uint32))


def test_fused_cdf_and_coder_bit_exact_vs_oracle():
    """The in-step CDF + coder equal the oracle coder run on the step's own logits."""
    from altxs_b200 import _lib
    from altxs_b200.engine import DeviceModel, StreamBatch

    for mode in ("fixed", "ref"):
        cfg = _small(cdf_mode=mode)
        dm = DeviceModel(C.synth_weights(cfg, seed=5), DEV)
        rng = np.random.default_rng(4)
        n, T = 3, 50
        syms = rng.integers(0, cfg.vocab_size, size=(n, T)).astype(np.int32)
        b = StreamBatch(dm, n, words_per_stream=T + 8, keep_logits=True)
        lg = np.zeros((n, T, cfg.vocab_size), dtype=np.float32)
        for t in range(T):
            b.sym.copy_(torch.as_tensor(syms[:, t], device=DEV))
            b.step(_lib.STEP_ENCODE)
            lg[:, t] = b.logits.cpu().numpy()
        b.ac_flush()
        b.check_status()
        got = b.segment_bytes(list(range(n)))
        for i in range(n):
            cum = oc.cum_from_logits(lg[i], mode, cfg.cdf_bits)
            assert got[i] == oc.encode_cum(cum, syms[i]), (mode, i)
        assert np.all(lg[:, 0] == 0.0)  # first symbol: uniform row


@pytest.mark.parametrize("n_streams", [1, 5])
def test_engine_roundtrip_segments(n_streams):
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.synth import zipf_markov

    cfg = _small(online_retrain_every=64, retrain_mode="none")
    dm = DeviceModel(C.synth_weights(cfg, seed=9), DEV)
    lens = [200, 0, 1, 64, 129][:n_streams]
    src = zipf_markov(max(lens), cfg.vocab_size, np.arange(n_streams) + 100)
    streams = [src[i, : lens[i]] for i in range(n_streams)]
    enc = Engine(dm).encode(streams)
    dec = Engine(dm).decode([r.payload for r in enc], lens)
    for s, d in zip(streams, dec):
        assert np.array_equal(s, d)


def test_incremental_entry_points_roundtrip():
    from altxs_b200.incremental import compress_full_sha_incremental, decompress_full_sha_incremental
    from altxs_b200.synth import zipf_markov

    cfg = _small(online_retrain_every=100, retrain_mode="none")
    w = C.synth_weights(cfg, seed=2)
    data = zipf_markov(350, cfg.vocab_size, [5])[0]
    res = compress_full_sha_incremental(w, data, cfg=cfg, device=DEV, online_retrain_enabled=False,
                                        progress=False, verify_decode=True)
    assert res["roundtrip_ok"] and res["first_mismatch"] is None
    assert len(res["chunk_bpb_rows"]) == 4
    dec = decompress_full_sha_incremental(w, res["payload"], 350, cfg=cfg, device=DEV,
                                          online_retrain_enabled=False, progress=False)
    assert dec["decoded_sha256"] == res["sha256"]


def test_c3_shape_step_runs_and_is_batch_independent():
    """Full 33M shapes (8L/512d/V16384, ctx 2048): finite logits, M-independence."""
    from altxs_b200.engine import DeviceModel

    cfg = c3_config()
    dm = DeviceModel(C.synth_weights(cfg, seed=1), DEV)
    rng = np.random.default_rng(0)
    T = 6
    toks = [rng.integers(0, cfg.vocab_size, size=T) for _ in range(20)]
    one = _run_logits(dm, toks[:1])[0]
    many = _run_logits(dm, toks)[0]
    assert np.isfinite(one).all()
    assert np.array_equal(one.view(np.uint32), many.view(np.uint32))
    om = OracleModel(OracleWeights.from_model_weights(C.synth_weights(cfg, seed=1)))
    st = om.new_stream()
    ref = np.stack([om.step(st, int(t)).numpy() for t in toks[0]])
    assert float(np.abs(one - ref).max()) < TOL


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_c3_full_window_logits_match_oracle(tensor_cores):
    """The 33M model with the window full: 2100 symbols of one stream, so the
    KV ring wraps and every fixed 256-key attention split is full; every
    position from 2040 on against the fp32 oracle (one causal prefill of the
    first 2040 symbols, then sliding-window steps), on both linear paths."""
    from altxs_b200.engine import DeviceModel
    from altxs_b200.synth import zipf_markov

    cfg = c3_config()
    w = C.synth_weights(cfg, seed=1)
    T, first = 2100, 2040
    toks = zipf_markov(T, cfg.vocab_size, [5])[0]
    dm = DeviceModel(w, DEV, tensor_cores=tensor_cores)
    got = _run_logits(dm, [toks[: T - 1]])[0]
    om = OracleModel(OracleWeights.from_model_weights(w))
    st = om.new_stream()
    ref = [om.prefill(st, toks[:first]).numpy()]
    for t in range(first, T - 1):
        ref.append(om.step(st, int(toks[t])).numpy())
    err = np.abs(got[first - 1:] - np.stack(ref)).max(axis=1)
    print(f"33M full window, tensor_cores={tensor_cores}: max |logit - oracle| = {err.max():.2e}")
    assert float(err.max()) < TOL


def test_graph_replay_matches_launches():
    """StreamBatch(graphs=True) replays captured steps: same symbols, same bytes."""
    from altxs_b200 import _lib
    from altxs_b200.engine import DeviceModel, StreamBatch

    cfg = _small()
    dm = DeviceModel(C.synth_weights(cfg, seed=5), DEV)
    rng = np.random.default_rng(8)
    n, T = 5, 30
    syms = rng.integers(0, cfg.vocab_size, size=(n, T)).astype(np.int32)
    out = []
    for graphs in (False, True):
        b = StreamBatch(dm, n, words_per_stream=T + 8, graphs=graphs)
        b.ac_init()
        for t in range(T):
            b.sym.copy_(torch.as_tensor(syms[:, t], device=DEV))
            b.step(_lib.STEP_ENCODE)
        b.ac_flush()
        b.check_status()
        out.append(b.segment_bytes(list(range(n))))
        if graphs:
            assert b.replays == T - 1
    assert out[0] == out[1]


def test_bpe_token_file_roundtrip(tmp_path):
    """A BPE token file (uint16 ids, sidecar vocabulary) through the
    reference-named entry points: encode, decode, identical tokens."""
    import json

    from altxs_b200.data import load_symbols
    from altxs_b200.incremental import compress_full_sha_incremental, decompress_full_sha_incremental
    from altxs_b200.synth import zipf_markov

    cfg = _small()
    toks = zipf_markov(150, cfg.vocab_size, np.array([77]))[0].astype("<u2")
    p = tmp_path / "tokens.bin"
    p.write_bytes(toks.tobytes())
    (tmp_path / "tokens.bin.json").write_text(json.dumps({"format": "blsmc-bpe-v1", "vocab_size": cfg.vocab_size}))
    arr, info = load_symbols(p)
    assert info.vocab_size == cfg.vocab_size
    w = C.synth_weights(cfg, seed=12)
    enc = compress_full_sha_incremental(w, np.asarray(arr), cfg=cfg, progress=False)
    dec = decompress_full_sha_incremental(w, enc["payload"], enc["n_symbols"], cfg=cfg, progress=False)
    assert dec["decoded_sha256"] == enc["sha256"]
