"""The handle-based runtime API (altxs_create ... altxs_destroy) against the
Python engine: the same segments byte for byte, with the test-time LoRA
update at every boundary, and a decode through the context that restores the
streams."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from altxs_b200 import _lib
from altxs_b200 import codec as CO
from altxs_b200.config import ModelConfig

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
CFG = dict(vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2, mlp_mult=4.0, rope_dims=16,
           block_size=32, online_retrain_every=64, seed=11, ttt_lora_rank=4, ttt_lora_lr=1e-3, ttt_k_lora=True,
           ttt_o_lora=True)


def _init_adapters(cfg) -> torch.Tensor:
    from altxs_b200.lora import init_lora_A, lora_shapes

    A = init_lora_A(cfg)
    flat = []
    for name, (_, b_shape) in lora_shapes(cfg).items():
        flat += [A[name].reshape(-1), np.zeros(b_shape[0] * b_shape[1], dtype=np.float32)]
    return torch.from_numpy(np.concatenate(flat).astype(np.float32)).to(DEV)


class Ctx:
    """Thin ctypes driver of the context API."""

    def __init__(self, dm, n: int, tensor_cores: bool):
        L = self.L = _lib.lib()
        cfg = dm.cfg
        st = C.c_int(0)
        self.h = L.altxs_create(C.byref(dm.desc), DEV.index or 0, C.byref(st))
        assert self.h and st.value == 0
        view = dm.weights_struct
        saved = view.split
        view.split = None
        try:
            assert L.altxs_load_weights(self.h, C.byref(view), int(tensor_cores)) == 0
        finally:
            view.split = saved
        self.init = _init_adapters(cfg)
        assert L.altxs_set_adapters(self.h, self.init.data_ptr()) == 0
        hp = _lib.TttHparams(lr=cfg.ttt_lora_lr, beta1=cfg.ttt_beta1, beta2=cfg.ttt_beta2, eps=1e-8,
                             weight_decay=cfg.ttt_weight_decay, grad_clip=cfg.grad_clip)
        assert L.altxs_set_ttt(self.h, C.byref(hp)) == 0
        assert L.altxs_set_segment(self.h, cfg.online_retrain_every) == 0
        assert L.altxs_streams_init(self.h, n, None) == 0
        self.n = n
        self.words = int(L.altxs_ctx_words_per_stream(self.h))
        self.bits = torch.zeros((n, self.words), dtype=torch.int32, device=DEV)
        self.nbits = torch.zeros(n, dtype=torch.int64, device=DEV)
        self.s = torch.cuda.current_stream().cuda_stream

    def flush(self) -> list[bytes]:
        assert self.L.altxs_flush(self.h, self.bits.data_ptr(), self.nbits.data_ptr(), self.s) == 0
        bits = self.bits.cpu().numpy().view(np.uint8)
        nb = self.nbits.cpu().numpy()
        return [bits[i, : (int(nb[i]) + 7) // 8].tobytes() for i in range(self.n)]

    def load(self, segs: list[bytes]) -> None:
        host = np.zeros((self.n, self.words * 4), dtype=np.uint8)
        nb = np.zeros(self.n, dtype=np.int64)
        for i, p in enumerate(segs):
            host[i, : len(p)] = np.frombuffer(p, dtype=np.uint8)
            nb[i] = len(p) * 8
        self.bits.copy_(torch.from_numpy(host.view(np.int32)))
        self.nbits.copy_(torch.from_numpy(nb))
        assert self.L.altxs_begin_decode(self.h, self.bits.data_ptr(), self.nbits.data_ptr(), self.s) == 0

    def close(self) -> None:
        self.L.altxs_destroy(self.h)


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_context_api_matches_engine(tensor_cores):
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.ttt import LoraTTT

    cfg = ModelConfig(**CFG)
    dm = DeviceModel(CO.synth_weights(cfg, seed=7), DEV, tensor_cores=tensor_cores)
    n, T, every = 3, 150, cfg.online_retrain_every
    rng = np.random.default_rng(9)
    streams = [rng.integers(0, cfg.vocab_size, size=T).astype(np.int32) for _ in range(n)]
    ref = Engine(dm, ttt=LoraTTT(dm)).encode(streams)

    syms = torch.as_tensor(np.stack(streams, axis=1).copy(), device=DEV)  # [T][n]
    enc = Ctx(dm, n, tensor_cores)
    segs = [[] for _ in range(n)]
    for t in range(T):
        if t > 0 and t % every == 0:
            for i, p in enumerate(enc.flush()):
                segs[i].append(p)
            assert enc.L.altxs_ttt_boundary(enc.h, enc.s) == 0
        assert enc.L.altxs_step_encode(enc.h, syms[t].data_ptr(), enc.s) == 0
    for i, p in enumerate(enc.flush()):
        segs[i].append(p)
    assert enc.L.altxs_get_status(enc.h, None) == 0
    enc.close()
    for i in range(n):
        assert segs[i] == ref[i].segments, i

    dec = Ctx(dm, n, tensor_cores)
    out = torch.zeros((T, n), dtype=torch.int32, device=DEV)
    dec.load([segs[i][0] for i in range(n)])
    for t in range(T):
        if t > 0 and t % every == 0:
            assert dec.L.altxs_ttt_boundary(dec.h, dec.s) == 0
            dec.load([segs[i][t // every] for i in range(n)])
        assert dec.L.altxs_step_decode(dec.h, out[t].data_ptr(), dec.s) == 0
    status = (C.c_int32 * n)()
    assert dec.L.altxs_get_status(dec.h, status) == 0 and list(status) == [0] * n
    dec.close()
    back = out.cpu().numpy()
    for i in range(n):
        assert np.array_equal(back[:, i], streams[i])


def test_context_api_refuses_misuse():
    """Calls out of order or with bad arguments return error codes, not faults."""
    from altxs_b200.engine import DeviceModel

    cfg = ModelConfig(**CFG)
    dm = DeviceModel(CO.synth_weights(cfg, seed=7), DEV)
    L = _lib.lib()
    st = C.c_int(0)
    h = L.altxs_create(C.byref(dm.desc), DEV.index or 0, C.byref(st))
    assert h
    s = torch.cuda.current_stream().cuda_stream
    tok = torch.zeros(2, dtype=torch.int32, device=DEV)
    assert L.altxs_step_encode(h, tok.data_ptr(), s) == _lib.ALTXS_EINVAL  # no streams yet
    assert L.altxs_streams_init(h, 2, None) == _lib.ALTXS_EINVAL           # no weights, no segment size
    L.altxs_destroy(h)


def test_context_refuses_a_decoder_with_other_settings():
    """The encoder's lockstep id given to a decoder context on the other
    linear path (or with other weights) makes altxs_begin_decode refuse
    (ALTXS_EMISMATCH) instead of desyncing; the matching context accepts."""
    from altxs_b200.engine import DeviceModel

    cfg = ModelConfig(**CFG)
    dm = DeviceModel(CO.synth_weights(cfg, seed=7), DEV)
    enc = Ctx(dm, 2, True)
    L = enc.L
    assert L.altxs_set_lockstep(enc.h, 1234, 0) == 0
    eid = C.c_uint64(0)
    assert L.altxs_lockstep_id(enc.h, C.byref(eid)) == 0 and eid.value != 0
    enc.close()
    for tensor_cores, wid, ok in ((False, 1234, False), (True, 99, False), (True, 1234, True)):
        dec = Ctx(dm, 2, tensor_cores)
        assert L.altxs_set_lockstep(dec.h, wid, eid.value) == 0
        rc = L.altxs_begin_decode(dec.h, dec.bits.data_ptr(), dec.nbits.data_ptr(), dec.s)
        assert rc == (0 if ok else -71), (tensor_cores, wid, rc)
        dec.close()
