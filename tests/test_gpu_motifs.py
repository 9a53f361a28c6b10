"""Reference motifs in the CUDA step (smear gate, XSA, sparse attention gate,
asymmetric softcap, depth-loop schedule, parallel lanes) against the
reference GPT's golden logits and the torch oracle."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from altxs_b200 import _lib
from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig
from oracle.model import OracleModel, OracleWeights

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
TOL = 2e-3  # max-abs logits tolerance vs the fp32 reference path

BASE = dict(
    vocab_size=384, num_layers=6, model_dim=128, num_heads=4, num_kv_heads=2, mlp_mult=2.0,
    rope_dims=16, block_size=32, online_retrain_every=64, seed=5, retrain_mode="none",
)

# one case per motif, then all of them together
CASES = {
    "smear": dict(smear_gate_enabled=True),
    "xsa": dict(xsa_last_n=2),
    "gate": dict(sparse_attn_gate_enabled=True),
    "asym": dict(asym_logit_rescale=True),
    "loop": dict(num_loops=2, loop_start=1, loop_end=3),
    "par_mean": dict(parallel_start_layer=3, parallel_final_lane="mean"),
    "par_attn": dict(parallel_start_layer=4, parallel_final_lane="attn"),
    "par_mlp": dict(parallel_start_layer=3, parallel_final_lane="mlp"),
    "all": dict(smear_gate_enabled=True, xsa_last_n=3, sparse_attn_gate_enabled=True, asym_logit_rescale=True,
                num_loops=1, loop_start=1, loop_end=2, parallel_start_layer=4),
}


def _golden_model(g):
    cfg = ModelConfig(**json.loads(bytes(g["config"])))
    tensors = {k[2:]: g[k].astype(np.float32) for k in g.files if k.startswith("w/")}
    return cfg, C.dense_weights(cfg, tensors)


def _case_model(name: str):
    """Mixed-bit synthetic weights with random motif parameters."""
    kw = dict(BASE)
    kw.update(CASES[name])
    cfg = ModelConfig(**kw)
    w = C.synth_weights(cfg, seed=9)
    rng = np.random.default_rng(len(name))
    s = w.small
    s["smear_gate"] = rng.normal(0, 0.5, s["smear_gate"].shape).astype(np.float32)
    s["smear_lambda"] = np.array([0.7], dtype=np.float32)
    s["attn_gate_w"] = rng.normal(0, 0.5, s["attn_gate_w"].shape).astype(np.float32)
    s["softcap"] = np.array([12.0, 20.0], dtype=np.float32)
    s["parallel_post"] = (s["parallel_post"] + rng.normal(0, 0.1, s["parallel_post"].shape)).astype(np.float32)
    s["parallel_resid"] = (s["parallel_resid"] + rng.normal(0, 0.1, s["parallel_resid"].shape)).astype(np.float32)
    return cfg, w


def _logits_mode(dm, toks_by_stream, lora=None):
    """LOGITS mode (the stream is not advanced: the test moves pos and prev_tok);
    ``lora``: one adapter vector for every stream."""
    from altxs_b200.engine import StreamBatch

    n, T = len(toks_by_stream), len(toks_by_stream[0])
    b = StreamBatch(dm, n, words_per_stream=8, keep_logits=True)
    if lora is not None:
        b.lora.copy_(lora.expand_as(b.lora))
    toks = torch.as_tensor(np.stack(toks_by_stream).astype(np.int32), device=DEV)
    out = np.zeros((n, T, dm.cfg.vocab_size), dtype=np.float32)
    for t in range(T):
        b.tok.copy_(toks[:, t])
        b.step(_lib.STEP_LOGITS)
        out[:, t] = b.logits.cpu().numpy()
        b.pos.add_(1)
        if b.prev_tok is not None:
            b.prev_tok.copy_(toks[:, t])
    return out


def _encode_mode(dm, toks_by_stream):
    """ENCODE mode: the step itself advances tok, pos and prev_tok.  Returns
    the logits that coded symbol t+1 (after consuming symbol t)."""
    from altxs_b200.engine import StreamBatch

    n, T = len(toks_by_stream), len(toks_by_stream[0])
    b = StreamBatch(dm, n, words_per_stream=T + 8, keep_logits=True)
    toks = torch.as_tensor(np.stack(toks_by_stream).astype(np.int32), device=DEV)
    b.tok.copy_(toks[:, 0])
    out = np.zeros((n, T - 1, dm.cfg.vocab_size), dtype=np.float32)
    for t in range(T - 1):
        b.sym.copy_(toks[:, t + 1])
        b.step(_lib.STEP_ENCODE)
        out[:, t] = b.logits.cpu().numpy()
    torch.cuda.synchronize()
    b.check_status()
    return out


def _oracle(w, toks):
    om = OracleModel(OracleWeights.from_model_weights(w))
    st = om.new_stream()
    return np.stack([om.step(st, int(t)).numpy() for t in toks])


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_motifs_match_reference_golden(golden, tensor_cores):
    """Every supported motif on at once; the reference GPT's own logits."""
    from altxs_b200.engine import DeviceModel

    g = golden("model_motifs.npz")
    cfg, w = _golden_model(g)
    dm = DeviceModel(w, DEV, tensor_cores=tensor_cores)
    got = _logits_mode(dm, [g["tokens"]])[0]
    err = float(np.abs(got - g["logits"]).max())
    assert err < TOL, err


@pytest.mark.parametrize("case", sorted(CASES))
def test_motif_step_matches_oracle(case):
    """Each motif alone (and all together) on mixed-bit weights, past the
    window so the ring wraps on every KV set, three streams."""
    from altxs_b200.engine import DeviceModel

    cfg, w = _case_model(case)
    dm = DeviceModel(w, DEV)
    rng = np.random.default_rng(4)
    T = cfg.block_size + 20
    toks = [rng.integers(0, cfg.vocab_size, size=T) for _ in range(3)]
    got = _logits_mode(dm, toks)
    for i in range(3):
        err = float(np.abs(got[i] - _oracle(w, toks[i])).max())
        assert err < TOL, (case, i, err)


def test_motif_encode_mode_advances_prev_token():
    """In the coding modes the kernel carries the smear gate's previous token:
    ENCODE-mode logits equal the oracle's step logits."""
    from altxs_b200.engine import DeviceModel

    cfg, w = _case_model("all")
    dm = DeviceModel(w, DEV)
    rng = np.random.default_rng(6)
    T = 50
    toks = [rng.integers(0, cfg.vocab_size, size=T) for _ in range(2)]
    got = _encode_mode(dm, toks)
    for i in range(2):
        err = float(np.abs(got[i] - _oracle(w, toks[i])[: T - 1]).max())
        assert err < TOL, (i, err)


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_motif_round_trip_and_batch_independence(tensor_cores):
    """Encode -> decode restores every stream (several segments); a stream's
    bytes are the same coded alone and inside a batch."""
    from altxs_b200.engine import DeviceModel, Engine

    cfg, w = _case_model("all")
    dm = DeviceModel(w, DEV, tensor_cores=tensor_cores)
    eng = Engine(dm)
    rng = np.random.default_rng(8)
    streams = [rng.integers(0, cfg.vocab_size, size=n).astype(np.int32) for n in (150, 97, 1, 64)]
    res = eng.encode(streams)
    back = eng.decode([r.payload for r in res], [len(s) for s in streams])
    for s, d in zip(streams, back):
        assert np.array_equal(s, d)
    alone = eng.encode([streams[1]])[0]
    assert alone.payload == res[1].payload


def test_motif_desc_accepted_by_update_and_prefill():
    """A motif desc with adapters sizes a workspace for the LoRA update and the
    reset prefill (both compute the motifs); the full-parameter gradient
    refuses a desc with adapters."""
    import ctypes
    import dataclasses

    from altxs_b200.engine import DeviceModel

    cfg, w = _case_model("xsa")
    cfg = dataclasses.replace(cfg, retrain_mode="lora", ttt_lora_rank=4)
    w.cfg = cfg
    dm = DeviceModel(w, DEV)
    L = _lib.lib()
    assert L.altxs_prefill_workspace_bytes(ctypes.byref(dm.desc), 8) > 0
    assert L.altxs_ttt_workspace_bytes(ctypes.byref(dm.desc), 8) > 0
    assert L.altxs_full_workspace_bytes(ctypes.byref(dm.desc), 8) == -1  # the full gradient trains no adapters


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_shipped_format_codec_runs_on_the_step(golden, tensor_cores):
    """The reference-format V=256 codec (residual over Init(seed), lloyd
    codebooks, motifs) loaded by read_codec and run by the CUDA step: logits
    within 2e-3 of the reference GPT's; encode -> decode round trip."""
    from altxs_b200.engine import DeviceModel, Engine
    from tests.conftest import GOLDEN

    g = golden("codec_ref_v256.npz")
    w = C.read_codec(GOLDEN / "codec_ref_v256.safetensors")
    dm = DeviceModel(w, DEV, tensor_cores=tensor_cores)
    got = _logits_mode(dm, [g["tokens"]])[0]
    err = float(np.abs(got - g["logits"]).max())
    assert err < TOL, err
    rng = np.random.default_rng(2)
    streams = [rng.integers(0, 256, size=n).astype(np.int32) for n in (300, 77)]
    eng = Engine(dm)
    res = eng.encode(streams)
    back = eng.decode([r.payload for r in res], [len(s) for s in streams])
    for s, d in zip(streams, back):
        assert np.array_equal(s, d)


def test_shipped_format_codec_with_its_retrain_mode(golden):
    """The reference-format codec keeps its config's retrain mode ("full", the
    reference default) and the entry points run it: every weight, the motifs'
    own included, updated at each boundary on both sides; round trip exact."""
    from altxs_b200.incremental import compress_full_sha_incremental, decompress_full_sha_incremental
    from tests.conftest import GOLDEN

    w = C.read_codec(GOLDEN / "codec_ref_v256.safetensors")
    assert w.cfg.retrain_mode == "full" and w.cfg.motifs
    data = np.random.default_rng(4).integers(0, 256, size=300).astype(np.uint8)
    res = compress_full_sha_incremental(w, data, cfg=w.cfg, device=DEV, progress=False, verify_decode=True)
    assert res["sha256_ok"] and res["roundtrip_ok"] and res["retrain_count"] == 2
    dec = decompress_full_sha_incremental(w, res["payload"], len(data), cfg=w.cfg, device=DEV, progress=False)
    assert dec["decoded_sha256"] == res["sha256"]
