"""ctypes binding of ``libaltxs_b200.so`` (declarations in include/altxs_b200.h).

The product path has no fallback: if the library is missing or fails to
load, every entry point raises.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libaltxs_b200.so"

ALTXS_OK = 0
ALTXS_EINVAL, ALTXS_ENOSPC, ALTXS_ENOTSUP, ALTXS_ECUDA, ALTXS_ENOMEM = -22, -28, -95, -5, -12
ST_OVERFLOW, ST_BAD_SYMBOL, ST_BAD_TOTAL, ST_NONFINITE, ST_TIMEOUT, ST_BAD_POS = 1, 2, 4, 8, 16, 32
CDF_FIXED, CDF_REF = 0, 1
STEP_LOGITS, STEP_ENCODE, STEP_DECODE = 0, 1, 2

EXPORTS = (
    "altxs_ac_init", "altxs_ac_encode_probs", "altxs_ac_encode_cum", "altxs_ac_flush",
    "altxs_ac_begin_decode", "altxs_ac_decode_probs", "altxs_ac_decode_cum",
    "altxs_cdf_from_logits", "altxs_workspace_bytes", "altxs_lora_floats", "altxs_step",
    "altxs_launch_count", "altxs_profile", "altxs_profile_read", "altxs_version",
    "altxs_ttt_workspace_bytes", "altxs_ttt_update", "altxs_step_noalloc", "altxs_step_noalloc_max_bytes",
    "altxs_dequant", "altxs_split_weights", "altxs_linear_workspace_bytes", "altxs_linear",
    "altxs_linear_tc_workspace_bytes", "altxs_linear_tc", "altxs_set_lockstep", "altxs_lockstep_id",
    "altxs_set_linear_packed",
    "altxs_set_flash", "altxs_window_attention_workspace_bytes", "altxs_window_attention", "altxs_last_cuda_error",
    "altxs_window_attention_backward_workspace_bytes", "altxs_window_attention_backward",
    "altxs_gemm_workspace_bytes", "altxs_gemm", "altxs_profile_mask", "altxs_prefill",
    "altxs_prefill_workspace_bytes", "altxs_set_wait_limit", "altxs_default_wait_limit", "altxs_set_step_fusion",
    "altxs_param_layout_of", "altxs_full_workspace_bytes", "altxs_full_loss_grad", "altxs_adamw",
    "altxs_params_axpy", "altxs_params_anchor", "altxs_split_params",
    "altxs_create", "altxs_load_weights", "altxs_set_adapters", "altxs_set_ttt", "altxs_set_segment",
    "altxs_streams_init", "altxs_step_encode", "altxs_step_decode", "altxs_ttt_boundary", "altxs_flush",
    "altxs_begin_decode", "altxs_get_status", "altxs_ctx_words_per_stream", "altxs_destroy",
)
KERNEL_CLASSES = ("embed", "prenorm", "linear", "qkv_post", "attn_partial", "attn_merge", "post_attn",
                  "final_norm", "cdf_code", "coder", "ttt", "fused_step")


class AcState(C.Structure):
    _fields_ = [
        ("low", C.c_uint64), ("high", C.c_uint64), ("pending", C.c_uint64), ("nbits", C.c_uint64),
        ("value", C.c_uint64), ("bpos", C.c_uint64), ("n_in_bits", C.c_uint64),
        ("status", C.c_uint32), ("reserved", C.c_uint32),
    ]


class QMat(C.Structure):
    _fields_ = [
        ("codes", C.c_void_p), ("row_off8", C.c_void_p), ("gdesc", C.c_void_p),
        ("lut", C.c_void_p), ("glut", C.c_void_p), ("rows", C.c_int32), ("cols", C.c_int32),
    ]


class ModelDesc(C.Structure):
    _fields_ = [
        ("vocab", C.c_int32), ("n_layers", C.c_int32), ("d_model", C.c_int32), ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("mlp_hidden", C.c_int32),
        ("ctx", C.c_int32), ("rope_dims", C.c_int32), ("skip_gates", C.c_int32),
        ("lora_rank", C.c_int32), ("lora_mask", C.c_int32), ("cdf_mode", C.c_int32),
        ("cdf_bits", C.c_int32), ("logit_softcap", C.c_float), ("lora_scale", C.c_float),
        ("n_virtual", C.c_int32), ("n_encoder", C.c_int32), ("schedule", C.c_void_p),
        ("smear_gate", C.c_int32), ("gate_window", C.c_int32), ("xsa_last_n", C.c_int32),
        ("sparse_gate", C.c_int32), ("sparse_gate_scale", C.c_float), ("asym_softcap", C.c_int32),
        ("parallel_start", C.c_int32), ("parallel_final", C.c_int32),
    ]


class SplitPlanes(C.Structure):
    _fields_ = [(f"{m}_{h}", C.c_void_p) for m in ("emb", "qkv", "o", "up", "down") for h in ("hi", "lo")]


class QTiles(C.Structure):
    _fields_ = [("data", C.c_void_p), ("rows", C.c_int32), ("cols", C.c_int32)]


class TileWeights(C.Structure):
    _fields_ = [(k, QTiles) for k in ("emb", "qkv", "o", "up", "down")]


class Weights(C.Structure):
    _fields_ = [
        ("emb", QMat), ("qkv", QMat), ("o", QMat), ("up", QMat), ("down", QMat),
        ("q_gain", C.c_void_p), ("attn_scale", C.c_void_p), ("mlp_scale", C.c_void_p),
        ("resid_mix", C.c_void_p), ("ln_scale", C.c_void_p), ("skip_weights", C.c_void_p),
        ("skip_gates", C.c_void_p), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
        ("rope_positions", C.c_int64), ("split", C.POINTER(SplitPlanes)),
        ("smear_gate", C.c_void_p), ("smear_lambda", C.c_void_p), ("attn_gate_w", C.c_void_p),
        ("softcap", C.c_void_p), ("parallel_post", C.c_void_p), ("parallel_resid", C.c_void_p),
        ("emb_dense", C.c_void_p), ("planes_live", C.c_int32), ("tiles", C.POINTER(TileWeights)),
    ]


class ParamLayout(C.Structure):
    """Segments (floats) of a full parameter arena (altxs_param_layout)."""

    _fields_ = [(k, C.c_int64) for k in ("emb", "qkv", "o", "up", "down", "q_gain", "attn_scale", "mlp_scale",
                                         "resid_mix", "skip_weights", "skip_gates", "smear_gate", "smear_lambda",
                                         "attn_gate_w", "softcap", "parallel_post", "parallel_resid", "total")]


class TttHparams(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
                ("weight_decay", C.c_float), ("grad_clip", C.c_float)]


class DenseWeights(C.Structure):
    _fields_ = [("emb", C.c_void_p), ("qkv", C.c_void_p), ("o", C.c_void_p), ("up", C.c_void_p),
                ("down", C.c_void_p)]


class Batch(C.Structure):
    _fields_ = [
        ("n_streams", C.c_int32), ("tok", C.c_void_p), ("pos", C.c_void_p), ("active", C.c_void_p),
        ("kv", C.c_void_p), ("lora", C.c_void_p), ("lora_stride", C.c_int64), ("ac", C.c_void_p),
        ("bits", C.c_void_p), ("words_per_stream", C.c_int64), ("sym", C.c_void_p),
        ("hist", C.c_void_p), ("hist_len", C.c_int32), ("logits_out", C.c_void_p),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_int64), ("pos_base", C.c_void_p),
        ("prev_tok", C.c_void_p),
    ]


_lib = None


def lib():
    """Load the library (raises if it is not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m altxs_b200.build` "
                "(there is no CPU fallback)"
            )
        L = C.CDLL(str(LIB_PATH))
        i64, vp = C.c_int64, C.c_void_p
        sig = {
            "altxs_ac_init": (C.c_int, [C.c_int, vp, vp, vp]),
            "altxs_ac_encode_probs": (C.c_int, [C.c_int, vp, C.c_int, vp, i64, vp, vp, vp, i64, vp]),
            "altxs_ac_decode_probs": (C.c_int, [C.c_int, vp, C.c_int, vp, i64, vp, vp, vp, i64, vp]),
            "altxs_ac_encode_cum": (C.c_int, [C.c_int, vp, C.c_int, vp, i64, vp, vp, vp, i64, vp]),
            "altxs_ac_decode_cum": (C.c_int, [C.c_int, vp, C.c_int, vp, i64, vp, vp, vp, i64, vp]),
            "altxs_ac_flush": (C.c_int, [C.c_int, vp, vp, vp, i64, vp]),
            "altxs_ac_begin_decode": (C.c_int, [C.c_int, vp, vp, vp, vp, i64, vp]),
            "altxs_cdf_from_logits": (C.c_int, [C.c_int, C.c_int, vp, i64, C.c_int, C.c_int, vp, i64, vp]),
            "altxs_workspace_bytes": (i64, [C.POINTER(ModelDesc), C.c_int]),
            "altxs_lora_floats": (i64, [C.POINTER(ModelDesc)]),
            "altxs_step": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(Weights), C.POINTER(Batch), C.c_int, vp]),
            "altxs_version": (C.c_char_p, []),
            "altxs_launch_count": (i64, []),
            "altxs_profile": (C.c_int, [C.c_int]),
            "altxs_profile_mask": (C.c_int, [C.c_uint32]),
            "altxs_set_wait_limit": (C.c_int, [C.c_uint32]),
            "altxs_default_wait_limit": (C.c_uint32, []),
            "altxs_set_step_fusion": (C.c_int, [C.c_int]),
            "altxs_set_linear_packed": (C.c_int, [C.c_int]),
            "altxs_set_flash": (C.c_int, [C.c_int]),
            "altxs_last_cuda_error": (C.c_int, []),
            "altxs_window_attention_workspace_bytes": (i64, [C.c_int, C.c_int, C.c_int, C.c_int]),
            "altxs_window_attention": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, vp, i64, vp, i64, vp,
                                                 i64, vp, i64, vp, vp, i64, vp]),
            "altxs_window_attention_backward_workspace_bytes": (i64, [C.c_int, C.c_int, C.c_int, C.c_int]),
            "altxs_window_attention_backward": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, vp, i64, vp,
                                                          i64, vp, i64, vp, i64, vp, vp, i64, vp, i64, vp, i64, vp,
                                                          i64, vp, i64, vp]),
            "altxs_profile_read": (C.c_int, [C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
            "altxs_step_noalloc": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(Weights), C.POINTER(Batch), C.c_int,
                                             vp]),
            "altxs_step_noalloc_max_bytes": (i64, []),
            "altxs_ttt_workspace_bytes": (i64, [C.POINTER(ModelDesc), C.c_int]),
            "altxs_ttt_update": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(Weights), C.POINTER(DenseWeights),
                                           C.POINTER(TttHparams), vp, C.c_int, vp, vp, vp, C.c_int, vp, vp, i64,
                                           vp]),
            "altxs_dequant": (C.c_int, [C.POINTER(QMat), vp, i64, vp]),
            "altxs_prefill_workspace_bytes": (i64, [C.POINTER(ModelDesc), C.c_int]),
            "altxs_prefill": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(Weights), C.POINTER(DenseWeights), vp,
                                        C.c_int, vp, vp, vp, i64, vp]),
            "altxs_split_weights": (C.c_int, [C.POINTER(QMat), vp, vp, vp]),
            "altxs_linear_workspace_bytes": (i64, [C.c_int, C.c_int]),
            "altxs_linear": (C.c_int, [C.POINTER(QMat), vp, vp, C.c_int, C.c_int, vp, C.c_int, vp, vp, i64, vp]),
            "altxs_linear_tc_workspace_bytes": (i64, [C.c_int, C.c_int, C.c_int]),
            "altxs_linear_tc": (C.c_int, [C.POINTER(QTiles), C.c_int, C.c_int, vp, C.c_int, vp, vp, i64, vp]),
            "altxs_gemm_workspace_bytes": (i64, [C.c_int] * 6),
            "altxs_param_layout_of": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(ParamLayout)]),
            "altxs_create": (vp, [C.POINTER(ModelDesc), C.c_int, C.POINTER(C.c_int)]),
            "altxs_load_weights": (C.c_int, [vp, C.POINTER(Weights), C.c_int]),
            "altxs_set_adapters": (C.c_int, [vp, vp]),
            "altxs_set_ttt": (C.c_int, [vp, C.POINTER(TttHparams)]),
            "altxs_set_segment": (C.c_int, [vp, i64]),
            "altxs_streams_init": (C.c_int, [vp, C.c_int, vp]),
            "altxs_step_encode": (C.c_int, [vp, vp, vp]),
            "altxs_step_decode": (C.c_int, [vp, vp, vp]),
            "altxs_ttt_boundary": (C.c_int, [vp, vp]),
            "altxs_flush": (C.c_int, [vp, vp, vp, vp]),
            "altxs_begin_decode": (C.c_int, [vp, vp, vp, vp]),
            "altxs_set_lockstep": (C.c_int, [vp, C.c_uint64, C.c_uint64]),
            "altxs_lockstep_id": (C.c_int, [vp, C.POINTER(C.c_uint64)]),
            "altxs_get_status": (C.c_int, [vp, vp]),
            "altxs_ctx_words_per_stream": (i64, [vp]),
            "altxs_destroy": (None, [vp]),
            "altxs_full_workspace_bytes": (i64, [C.POINTER(ModelDesc), C.c_int]),
            "altxs_full_loss_grad": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(Weights), C.POINTER(DenseWeights), vp,
                                               C.c_int, C.c_int, vp, vp, vp, i64, vp]),
            "altxs_adamw": (C.c_int, [i64, vp, vp, vp, vp, C.POINTER(TttHparams), C.c_int, vp, vp]),
            "altxs_params_axpy": (C.c_int, [i64, vp, C.c_float, vp, vp, vp]),
            "altxs_params_anchor": (C.c_int, [i64, vp, vp, vp, vp]),
            "altxs_split_params": (C.c_int, [C.POINTER(ModelDesc), vp, C.POINTER(SplitPlanes), vp]),
            "altxs_gemm": (C.c_int, [C.c_int, C.c_int, C.c_int, vp, i64, i64, C.c_int, vp, i64, i64, C.c_int, vp, i64,
                                     i64, C.c_int, C.c_float, C.c_float, C.c_int, vp, i64, vp]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != ALTXS_OK:
        raise RuntimeError(f"{what} failed with code {rc}")
