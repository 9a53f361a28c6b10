"""CPU checks of the C-ABI library: it loads and exports every declared symbol."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> list[str]:
    text = (ROOT / "include" / "altxs_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|uint32_t|void|const char \*|altxs_ctx \*)\s*(altxs_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib_path():
    from altxs_b200 import build

    try:
        return build.build()
    except Exception as e:  # pragma: no cover - nvcc missing
        pytest.skip(f"nvcc build unavailable: {e}")


def test_header_declares_entry_points():
    names = _declared()
    assert "altxs_step" in names and "altxs_ac_encode_cum" in names
    from altxs_b200 import _lib

    assert set(_lib.EXPORTS) == set(names)


def test_library_loads_and_exports_every_symbol(lib_path):
    lib = ctypes.CDLL(str(lib_path))
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True).stdout
    for name in _declared():
        assert re.search(rf"\bT {name}\b", out), name


def test_host_queries_without_gpu(lib_path):
    """Pure host functions (no device work) answer on a CPU-only machine."""
    from altxs_b200 import _lib
    from altxs_b200.config import c3_config
    from altxs_b200.lora import lora_shapes

    L = _lib.lib()
    cfg = c3_config()
    d = _lib.ModelDesc(vocab=cfg.vocab_size, n_layers=cfg.num_layers, d_model=cfg.model_dim,
                       n_heads=cfg.num_heads, n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                       mlp_hidden=cfg.mlp_hidden, ctx=cfg.ctx, rope_dims=cfg.rope_dims, skip_gates=1,
                       lora_rank=cfg.ttt_lora_rank, lora_mask=1 | 2 | 4 | 8 | 16, cdf_mode=0, cdf_bits=20,
                       logit_softcap=30.0, lora_scale=cfg.lora_scale)
    n_floats = sum(a[0] * a[1] + b[0] * b[1] for a, b in lora_shapes(cfg).values())
    assert L.altxs_lora_floats(ctypes.byref(d)) == n_floats
    assert L.altxs_workspace_bytes(ctypes.byref(d), 256) > 0
    assert L.altxs_version().startswith(b"altxs_b200")
    bad = _lib.ModelDesc.from_buffer_copy(d)
    bad.d_model = 100
    assert L.altxs_workspace_bytes(ctypes.byref(bad), 4) < 0
