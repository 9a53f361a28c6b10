"""Device range coder and CDF kernels against the reference goldens and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import coder as oc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _lib():
    from altxs_b200 import _lib

    return _lib, _lib.lib()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def test_gpu_range_coder_matches_reference_coder(golden):
    """Mirror of the reference test_gpu_ac_matches_host_coder (n=64, V=256, rng(0))."""
    from altxs_b200.gpu_ac import GpuRangeCoder

    g = golden("coder_probs.npz")
    for case in ("a", "b"):
        rows, syms, ref = g[f"{case}_probs"], g[f"{case}_syms"], g[f"{case}_bits"].tobytes()
        n, v = rows.shape
        coder = GpuRangeCoder(DEV, max_bits=n * 48 + 4096, vocab=v)
        probs = torch.as_tensor(rows, device=DEV)
        tok = torch.as_tensor(syms.astype(np.int64), device=DEV)
        for i in range(n):
            coder.encode_symbol(probs[i], tok[i])
        got = coder.finish()
        assert got == ref, case
        dec = GpuRangeCoder(DEV, max_bits=len(got) * 8 + 64, vocab=v)
        dec.begin_decode(got)
        out = torch.stack([dec.decode_symbol(probs[i]).clone() for i in range(n)]).reshape(-1)
        assert np.array_equal(out.cpu().numpy(), syms.astype(np.int64)), case
        assert dec.status() == 0


def _encode_cum_streams(cums: list[np.ndarray], symss: list[np.ndarray]):
    """Lockstep multi-stream encode through altxs_ac_encode_cum."""
    L, lib = _lib()
    n = len(cums)
    T = max(len(s) for s in symss)
    V = cums[0].shape[1] - 1
    wps = T + 8
    st = torch.zeros((n, 8), dtype=torch.int64, device=DEV)
    bits = torch.zeros((n, wps), dtype=torch.int32, device=DEV)
    L.check(lib.altxs_ac_init(n, None, st.data_ptr(), _stream()), "init")
    for t in range(T):
        rows = [i for i in range(n) if t < len(symss[i])]
        cum = np.stack([cums[i][t] for i in rows]).astype(np.uint32)
        sy = np.array([symss[i][t] for i in rows], dtype=np.int32)
        cd, sd = torch.as_tensor(cum.view(np.int32), device=DEV), torch.as_tensor(sy, device=DEV)
        rd = torch.as_tensor(np.array(rows, np.int32), device=DEV)
        L.check(lib.altxs_ac_encode_cum(len(rows), rd.data_ptr(), V, cd.data_ptr(), V + 1, sd.data_ptr(),
                                        st.data_ptr(), bits.data_ptr(), wps, _stream()), "enc")
    L.check(lib.altxs_ac_flush(n, None, st.data_ptr(), bits.data_ptr(), wps, _stream()), "flush")
    s = st.cpu().numpy()
    b = bits.cpu().numpy().view(np.uint8)
    assert (s[:, 7] == 0).all()
    return [b[i, : (int(s[i, 3]) + 7) // 8].tobytes() for i in range(n)]


def _decode_cum_streams(cums, payloads, lens):
    L, lib = _lib()
    n = len(cums)
    V = cums[0].shape[1] - 1
    wps = max(len(p) for p in payloads) // 4 + 8
    host = np.zeros((n, wps * 4), dtype=np.uint8)
    for i, p in enumerate(payloads):
        host[i, : len(p)] = np.frombuffer(p, np.uint8)
    bits = torch.as_tensor(host.view(np.int32), device=DEV)
    nb = torch.as_tensor(np.array([len(p) * 8 for p in payloads], np.int64), device=DEV)
    st = torch.zeros((n, 8), dtype=torch.int64, device=DEV)
    L.check(lib.altxs_ac_begin_decode(n, None, st.data_ptr(), bits.data_ptr(), nb.data_ptr(), wps, _stream()), "bd")
    out = [[] for _ in range(n)]
    sd = torch.zeros(n, dtype=torch.int32, device=DEV)
    for t in range(max(lens)):
        rows = [i for i in range(n) if t < lens[i]]
        cum = np.stack([cums[i][t] for i in rows]).astype(np.uint32)
        cd = torch.as_tensor(cum.view(np.int32), device=DEV)
        rd = torch.as_tensor(np.array(rows, np.int32), device=DEV)
        L.check(lib.altxs_ac_decode_cum(len(rows), rd.data_ptr(), V, cd.data_ptr(), V + 1, sd.data_ptr(),
                                        st.data_ptr(), bits.data_ptr(), wps, _stream()), "dec")
        got = sd.cpu().numpy()
        for j, r in enumerate(rows):
            out[r].append(int(got[j]))
    return [np.array(o, dtype=np.int32) for o in out]


def test_gpu_coder_given_integer_cdfs_matches_reference(golden):
    g = golden("coder_cum.npz")
    cases = [
        (oc.cum_from_logits(g["a_logits"], "fixed", 20), g["a_syms"], g["a_bits"]),
        (oc.cum_from_logits(g["a_logits"], "ref"), g["a_syms"], g["b_bits"]),
        (g["c_cum"], g["c_syms"], g["c_bits"]),
        (g["d_cum"], g["d_syms"], g["d_bits"]),
    ]
    for cum, syms, ref in cases:
        got = _encode_cum_streams([cum], [syms])[0]
        assert got == ref.tobytes()
        dec = _decode_cum_streams([cum], [got], [len(syms)])[0]
        assert np.array_equal(dec, syms)


def test_gpu_coder_many_streams_ragged():
    """Independent streams of different lengths in one launch == oracle per stream."""
    rng = np.random.default_rng(3)
    V = 300
    lens = [0, 1, 2, 17, 64, 200, 333]
    cums, symss = [], []
    for ln in lens:
        lg = rng.normal(0, 5, size=(max(ln, 1), V)).astype(np.float32)
        cums.append(oc.cum_from_logits(lg, "fixed", 20))
        symss.append(rng.integers(0, V, size=ln).astype(np.int32))
    got = _encode_cum_streams(cums, symss)
    for c, s, p in zip(cums, symss, got):
        assert p == oc.encode_cum(c[: len(s)], s)
    dec = _decode_cum_streams(cums, got, lens)
    for s, d in zip(symss, dec):
        assert np.array_equal(s, d)


@pytest.mark.parametrize("mode,bits", [("fixed", 20), ("fixed", 16), ("fixed", 30), ("ref", 20)])
@pytest.mark.parametrize("V", [2, 257, 4096, 16384])
def test_gpu_cdf_kernel_bit_exact(mode, bits, V):
    if mode == "fixed" and (1 << bits) <= V:
        pytest.skip("vocab too large for this total")
    L, lib = _lib()
    rng = np.random.default_rng(V + bits)
    n = 24
    lg = (30 * np.tanh(rng.normal(0, 4, size=(n, V)) / 30)).astype(np.float32)
    lg[0] = 0.0  # uniform row
    lg[1, :] = -30.0
    lg[1, 0] = 30.0  # one dominant symbol
    ld = torch.as_tensor(lg, device=DEV)
    cum = torch.zeros((n, V + 1), dtype=torch.int32, device=DEV)
    L.check(lib.altxs_cdf_from_logits(n, V, ld.data_ptr(), V, 0 if mode == "fixed" else 1, bits,
                                      cum.data_ptr(), V + 1, _stream()), "cdf")
    got = cum.cpu().numpy().view(np.uint32).astype(np.uint64)
    ref = oc.cum_from_logits(lg, mode, bits)
    assert np.array_equal(got, ref)


def test_gpu_coder_overflow_is_flagged_not_fatal():
    """A bit buffer that is too small sets the overflow status; the GPU stays usable."""
    L, lib = _lib()
    V, T = 64, 200
    rng = np.random.default_rng(0)
    cum = oc.cum_from_logits(rng.normal(0, 1, size=(T, V)).astype(np.float32), "fixed", 20)
    syms = rng.integers(0, V, size=T).astype(np.int32)
    wps = 2  # 64 bits for ~1200 bits of output
    st = torch.zeros((1, 8), dtype=torch.int64, device=DEV)
    bits = torch.zeros((1, wps), dtype=torch.int32, device=DEV)
    L.check(lib.altxs_ac_init(1, None, st.data_ptr(), _stream()), "init")
    for t in range(T):
        cd = torch.as_tensor(cum[t:t + 1].astype(np.uint32).view(np.int32), device=DEV)
        sd = torch.as_tensor(syms[t:t + 1], device=DEV)
        L.check(lib.altxs_ac_encode_cum(1, None, V, cd.data_ptr(), V + 1, sd.data_ptr(), st.data_ptr(),
                                        bits.data_ptr(), wps, _stream()), "enc")
    s = st.cpu().numpy()[0]
    assert int(s[7]) & L.ST_OVERFLOW
    # a bad symbol is flagged too
    st.zero_()
    L.check(lib.altxs_ac_init(1, None, st.data_ptr(), _stream()), "init")
    sd = torch.as_tensor(np.array([V + 5], np.int32), device=DEV)
    cd = torch.as_tensor(cum[:1].astype(np.uint32).view(np.int32), device=DEV)
    L.check(lib.altxs_ac_encode_cum(1, None, V, cd.data_ptr(), V + 1, sd.data_ptr(), st.data_ptr(),
                                    bits.data_ptr(), wps, _stream()), "enc")
    assert int(st.cpu().numpy()[0, 7]) & L.ST_BAD_SYMBOL
    torch.cuda.synchronize()
