"""Device range coder with the reference ``GpuRangeCoder`` interface.

Mirrors altxs ``src/xsa_ttt/gpu_ac.py:397-479`` (same constructor arguments,
``encode_symbol`` / ``finish`` / ``begin_decode`` / ``decode_symbol``, same
bytes out) on top of the C-ABI coder in ``libaltxs_b200.so``.  Differences
that are deliberate: bits are packed 32 per word instead of one int64 per
bit, and a full bit buffer raises instead of silently dropping bits
(gpu_ac.py:44-51).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib


class GpuRangeCoder:
    """One-stream coder on the device; probs rows use the reference mass rule."""

    def __init__(self, device: torch.device, *, max_bits: int, vocab: int):
        self.device = torch.device(device)
        self.vocab = int(vocab)
        self.max_bits = int(max_bits)
        self.words = (self.max_bits + 31) // 32 + 2
        self.state = torch.zeros((1, 8), dtype=torch.int64, device=self.device)
        self.bits = torch.zeros(self.words, dtype=torch.int32, device=self.device)
        self.sym = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._n_in = torch.zeros(1, dtype=torch.int64, device=self.device)
        self._lib = _lib.lib()
        _lib.check(self._lib.altxs_ac_init(1, None, self.state.data_ptr(), self._stream()), "ac_init")

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    @staticmethod
    def _probs_arg(probs: torch.Tensor) -> torch.Tensor:
        p = probs.reshape(-1)
        if p.dtype == torch.float32 and p.is_contiguous():
            return p
        return p.float().contiguous()

    def encode_symbol(self, probs: torch.Tensor, symbol: torch.Tensor) -> None:
        p = self._probs_arg(probs)
        if p.numel() != self.vocab:
            raise ValueError(f"probs must have {self.vocab} entries")
        self.sym.copy_(symbol.reshape(-1)[:1].to(torch.int32))
        _lib.check(
            self._lib.altxs_ac_encode_probs(1, None, self.vocab, p.data_ptr(), self.vocab, self.sym.data_ptr(),
                                            self.state.data_ptr(), self.bits.data_ptr(), self.words,
                                            self._stream()), "ac_encode_probs")

    def finish(self) -> bytes:
        _lib.check(self._lib.altxs_ac_flush(1, None, self.state.data_ptr(), self.bits.data_ptr(), self.words,
                                            self._stream()), "ac_flush")
        st = self.state.cpu().numpy()[0]
        self._raise_status(int(st[7]) & 0xFFFFFFFF)
        nbits = int(st[3])
        raw = self.bits.cpu().numpy().view(np.uint8)
        return raw[: (nbits + 7) // 8].tobytes()

    def begin_decode(self, payload: bytes) -> None:
        n_bits = len(payload) * 8
        if n_bits > self.words * 32:
            raise ValueError(f"decode payload has {n_bits} bits, capacity is {self.words * 32}")
        buf = np.zeros(self.words * 4, dtype=np.uint8)
        buf[: len(payload)] = np.frombuffer(bytes(payload), dtype=np.uint8)
        self.bits.copy_(torch.from_numpy(buf.view(np.int32)))
        self._n_in.fill_(n_bits)
        _lib.check(self._lib.altxs_ac_begin_decode(1, None, self.state.data_ptr(), self.bits.data_ptr(),
                                                   self._n_in.data_ptr(), self.words, self._stream()),
                   "ac_begin_decode")

    def decode_symbol(self, probs: torch.Tensor) -> torch.Tensor:
        p = self._probs_arg(probs)
        _lib.check(
            self._lib.altxs_ac_decode_probs(1, None, self.vocab, p.data_ptr(), self.vocab, self.sym.data_ptr(),
                                            self.state.data_ptr(), self.bits.data_ptr(), self.words,
                                            self._stream()), "ac_decode_probs")
        return self.sym.to(torch.int64)

    def status(self) -> int:
        return int(self.state.cpu().numpy()[0, 7]) & 0xFFFFFFFF

    @staticmethod
    def _raise_status(st: int) -> None:
        if st:
            from .engine import ST_NAMES

            raise RuntimeError(f"range coder status {st:#x}: " + ", ".join(v for k, v in ST_NAMES.items() if st & k))


def can_gpu_ac(device: torch.device) -> bool:
    """True when the device coder can run (CUDA device and library present)."""
    if torch.device(device).type != "cuda":
        return False
    _lib.lib()
    return True
