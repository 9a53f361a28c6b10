"""Host side of the B200 model-and-code loop.

``DeviceModel`` uploads one model (packed mixed-bit weights + small params +
RoPE tables) to a GPU.  ``StreamBatch`` owns the device state of n
independent symbol streams (KV rings, LoRA adapters, coder states, bit
buffers) and drives the C-ABI step.  ``Engine`` runs whole streams: symbols
are coded in segments of ``online_retrain_every`` symbols, each segment
flushed separately and framed as ``<u64 LE len><segment bytes>`` like the
reference (altxs src/xsa_ttt/incremental.py:1721-1722, 1782-1796); the
test-time LoRA update runs at every segment boundary on both sides.

Stream semantics (identical on encode and decode): symbol 0 is coded with the
uniform distribution (reference ``uniform_probs``, compress.py:53-56);
symbol t >= 1 is coded with the model's distribution after consuming symbols
0..t-1, attending over the last ``block_size`` positions.
"""

from __future__ import annotations

import ctypes as C
import math
import struct
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, lockstep
from .codec import ModelWeights, PackedMatrix, tile_stream
from .config import ModelConfig
from .lora import init_lora_A, lora_shapes, rope_tables

ST_NAMES = {1: "bit buffer overflow", 2: "bad symbol", 4: "bad CDF total", 8: "non-finite logits",
            16: "device wait timeout", 32: "position beyond the RoPE table"}


def _i32(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.int32)


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def lora_mask(cfg: ModelConfig) -> int:
    if not cfg.lora_enabled:
        return 0
    m = 1 | 4 | 16  # q, v, lm_head always (reference TTTLoRA)
    if cfg.ttt_k_lora:
        m |= 2
    if cfg.ttt_o_lora:
        m |= 8
    if cfg.ttt_mlp_lora:
        m |= 32
    if cfg.ttt_o_lora and cfg.ttt_o_lora_on_y:
        m |= 64
    return m


# small parameters held in the arena (segment names of altxs_param_layout)
_ARENA_SMALL = ("q_gain", "attn_scale", "mlp_scale", "resid_mix", "skip_weights", "skip_gates", "smear_gate",
                "smear_lambda", "attn_gate_w", "softcap", "parallel_post", "parallel_resid")


class DeviceModel:
    """One model resident on one GPU.

    ``tensor_cores=True`` (default) also keeps the hi/lo bf16 planes of every
    mixed-bit matrix (4 bytes per weight) and runs the step's linear layers on
    the tensor cores; ``False`` runs them on CUDA cores from the packed codes.
    The two differ in the last bits of the logits, so an encoder and its
    decoder must use the same setting.
    """

    def __init__(self, weights: ModelWeights, device: torch.device | str, *, rope_positions: int = 1 << 16,
                 tensor_cores: bool = True, full_params: bool = False):
        """``full_params=True`` keeps every parameter in one fp32 arena
        (``self.params``, layout ``self.layout``) that the step reads — the
        embedding rows, the small parameters and the tensor-core planes
        (re-split by ``refresh()``) — so that a full-parameter update
        (``replenish.ReplenishTTT``) can change the model between segments."""
        self.cfg = cfg = weights.cfg
        cfg.validate()
        self.device = device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("the B200 engine needs a CUDA device (there is no CPU path)")
        _lib.lib()
        self._keep: list[torch.Tensor] = []
        packed = weights.packed()
        self.weight_bytes = sum(p.nbytes for p in packed.values())
        self.weights_sha256 = lockstep.weights_digest(packed, weights.small)
        self.q = {k: self._qmat(v) for k, v in packed.items()}
        # the packed codes in the tensor-core GEMM's tile-stream layout (when every
        # group is 0/2/3/4-bit symmetric), read by the packed tensor-core linears
        self.tiles = None
        if tensor_cores:
            ts = {k: tile_stream(v) for k, v in packed.items()}
            if all(t is not None for t in ts.values()):
                self.tiles = _lib.TileWeights(**{k: _lib.QTiles(data=self._up(t).data_ptr(), rows=packed[k].rows,
                                                                cols=packed[k].cols) for k, t in ts.items()})
        s = weights.small
        L = cfg.num_layers
        f32 = lambda a: self._up(np.ascontiguousarray(a, dtype=np.float32))  # noqa: E731
        self.small = {
            "q_gain": f32(s["q_gain"]),
            "attn_scale": f32(s["attn_scale"]),
            "mlp_scale": f32(s["mlp_scale"]),
            "resid_mix": f32(s["resid_mix"]),
            "ln_scale": f32(
                np.array([1.0 / math.sqrt(i + 1) if cfg.ln_scale else 1.0 for i in range(L)], dtype=np.float32)
            ),
            "skip_weights": f32(s["skip_weights"] if s["skip_weights"].size else np.zeros((1, cfg.model_dim))),
            "skip_gates": f32(s["skip_gates"] if s["skip_gates"].size else np.zeros((1, cfg.model_dim))),
        }
        # reference motifs: parameters uploaded only for the motifs that are on
        motif_on = {
            "smear_gate": cfg.smear_gate_enabled, "smear_lambda": cfg.smear_gate_enabled,
            "attn_gate_w": cfg.sparse_attn_gate_enabled, "softcap": cfg.asym_logit_rescale,
            "parallel_post": cfg.parallel_start_layer > 0, "parallel_resid": cfg.parallel_start_layer > 0,
        }
        for k, on in motif_on.items():
            if on:
                self.small[k] = f32(s[k])
        enc, dec = cfg.layer_schedule
        sched = enc + dec
        self._schedule = (C.c_int32 * len(sched))(*sched)
        self.n_virtual = len(sched)
        self.rope_positions = 0
        self.ensure_rope(rope_positions)
        self.desc = _lib.ModelDesc(
            vocab=cfg.vocab_size, n_layers=L, d_model=cfg.model_dim, n_heads=cfg.num_heads,
            n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, mlp_hidden=cfg.mlp_hidden,
            ctx=cfg.kv_len, rope_dims=cfg.rope_dims, skip_gates=int(cfg.skip_gates_enabled),
            lora_rank=cfg.ttt_lora_rank if cfg.lora_enabled else 0, lora_mask=lora_mask(cfg),
            cdf_mode=_lib.CDF_FIXED if cfg.cdf_mode == "fixed" else _lib.CDF_REF, cdf_bits=cfg.cdf_bits,
            logit_softcap=cfg.logit_softcap, lora_scale=cfg.lora_scale if cfg.lora_enabled else 0.0,
            n_virtual=self.n_virtual, n_encoder=len(enc),
            schedule=C.cast(self._schedule, C.c_void_p) if cfg.num_loops > 0 else None,
            smear_gate=int(cfg.smear_gate_enabled), gate_window=cfg.gate_window, xsa_last_n=cfg.xsa_last_n,
            sparse_gate=int(cfg.sparse_attn_gate_enabled), sparse_gate_scale=cfg.sparse_attn_gate_scale,
            asym_softcap=int(cfg.asym_logit_rescale), parallel_start=cfg.parallel_start_layer,
            parallel_final={"mean": 0, "attn": 1, "mlp": 2}[cfg.parallel_final_lane],
        )
        self.lora_floats = int(_lib.lib().altxs_lora_floats(C.byref(self.desc)))
        self.tensor_cores = bool(tensor_cores)
        self.full_params = bool(full_params)
        self.params = None
        if self.full_params:
            self._build_arena()
        self._split = self._split_planes() if self.tensor_cores else None

    def _build_arena(self) -> None:
        """Every parameter in one device arena: the five matrices dequantised
        exactly, the small parameters copied; ``small`` then views the arena."""
        L = _lib.lib()
        lay = _lib.ParamLayout()
        _lib.check(L.altxs_param_layout_of(C.byref(self.desc), C.byref(lay)), "altxs_param_layout_of")
        self.layout = lay
        self.params = torch.zeros(lay.total, dtype=torch.float32, device=self.device)
        base = self.params.data_ptr()
        st = _stream_handle(self.device)
        for name in ("emb", "qkv", "o", "up", "down"):
            q = self.q[name]
            _lib.check(L.altxs_dequant(C.byref(q), base + 4 * getattr(lay, name), q.cols, st), "altxs_dequant")
        for name in _ARENA_SMALL:
            if name not in self.small or self._arena_size(name) == 0:
                continue  # no skips, or a motif that is off
            src = self.small[name].reshape(-1)
            off = getattr(lay, name)
            view = self.params[off: off + src.numel()]
            view.copy_(src)
            self.small[name] = view
        self.params_initial = self.params.clone()  # the shipped weights: every stream starts from them
        if not self.tensor_cores:
            # the CUDA-core step reads the live arena as 32-bit groups (raw fp32
            # values, scale 1): the same group-order dot products, on the updated weights
            for name in ("emb", "qkv", "o", "up", "down"):
                q = self.q[name]
                rows, cols = q.rows, q.cols
                G = cols // 64
                row_off8 = (np.arange(rows, dtype=np.int64) * (cols // 2)).astype(np.uint32)
                gd = (np.uint32(0x3C00) | np.uint32(4 << 16)
                      | (np.arange(G, dtype=np.uint32) * np.uint32(32)) << np.uint32(20))
                gdesc = np.broadcast_to(gd, (rows, G)).astype(np.uint32)
                ro, gdt = self._up(_i32(row_off8)), self._up(_i32(gdesc))
                self.q[name] = _lib.QMat(codes=base + 4 * getattr(lay, name), row_off8=ro.data_ptr(),
                                         gdesc=gdt.data_ptr(), lut=None, glut=None, rows=rows, cols=cols)
        self._weights_struct = None

    def _arena_size(self, name: str) -> int:
        cfg, L, d = self.cfg, self.cfg.num_layers, self.cfg.model_dim
        gw = cfg.gate_window
        sizes = {"emb": cfg.vocab_size * d, "qkv": L * (d + 2 * cfg.kv_dim) * d, "o": L * d * d,
                 "up": L * cfg.mlp_hidden * d, "down": L * d * cfg.mlp_hidden, "q_gain": L * cfg.num_heads,
                 "attn_scale": L * d, "mlp_scale": L * d, "resid_mix": L * 2 * d,
                 "skip_weights": cfg.num_skip_weights * d, "skip_gates": cfg.num_skip_weights * d,
                 "smear_gate": gw if cfg.smear_gate_enabled else 0,
                 "smear_lambda": 1 if cfg.smear_gate_enabled else 0,
                 "attn_gate_w": L * cfg.num_heads * gw if cfg.sparse_attn_gate_enabled else 0,
                 "softcap": 2 if cfg.asym_logit_rescale else 0,
                 "parallel_post": L * 4 if cfg.parallel_start_layer > 0 else 0,
                 "parallel_resid": L * 2 if cfg.parallel_start_layer > 0 else 0}
        return sizes[name]

    def arena(self, name: str) -> torch.Tensor:
        """The segment ``name`` of the parameter arena (a view)."""
        off = getattr(self.layout, name)
        return self.params[off: off + self._arena_size(name)]

    def refresh(self) -> None:
        """After the arena changed: rewrite the step's tensor-core planes."""
        if self.full_params and self._split is not None:
            _lib.check(_lib.lib().altxs_split_params(C.byref(self.desc), self.params.data_ptr(),
                                                     C.byref(self._split), _stream_handle(self.device)),
                       "altxs_split_params")

    def _up(self, a: np.ndarray) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(a)).to(self.device)
        self._keep.append(t)
        return t

    def _qmat(self, p: PackedMatrix) -> _lib.QMat:
        codes = self._up(p.codes)
        ro = self._up(_i32(p.row_off8))
        gd = self._up(_i32(p.gdesc))
        lut = self._up(p.lut.view(np.int16)) if p.lut is not None else None
        glut = self._up(_i32(p.glut)) if p.glut is not None else None
        return _lib.QMat(
            codes=codes.data_ptr(), row_off8=ro.data_ptr(), gdesc=gd.data_ptr(),
            lut=lut.data_ptr() if lut is not None else None,
            glut=glut.data_ptr() if glut is not None else None,
            rows=p.rows, cols=p.cols,
        )

    def _split_planes(self) -> _lib.SplitPlanes:
        L = _lib.lib()
        fields = {}
        self._split_bufs = []
        for name in ("emb", "qkv", "o", "up", "down"):
            q = self.q[name]
            hi = torch.empty((q.rows, q.cols), dtype=torch.bfloat16, device=self.device)
            lo = torch.empty_like(hi)
            if not self.full_params:
                _lib.check(L.altxs_split_weights(C.byref(q), hi.data_ptr(), lo.data_ptr(),
                                                 _stream_handle(self.device)), "altxs_split_weights")
            self._split_bufs += [hi, lo]
            fields[f"{name}_hi"], fields[f"{name}_lo"] = hi.data_ptr(), lo.data_ptr()
        planes = _lib.SplitPlanes(**fields)
        if self.full_params:
            _lib.check(L.altxs_split_params(C.byref(self.desc), self.params.data_ptr(), C.byref(planes),
                                            _stream_handle(self.device)), "altxs_split_params")
        return planes

    def ensure_rope(self, n_pos: int) -> None:
        """RoPE tables must cover every absolute position a stream reaches."""
        if n_pos <= self.rope_positions:
            return
        n = 1 << max(12, (int(n_pos) - 1).bit_length())
        cos, sin = rope_tables(self.cfg, n)
        self.rope_cos = self._up(cos)
        self.rope_sin = self._up(sin)
        self.rope_positions = n
        self._weights_struct = None

    def dense_weights(self) -> _lib.DenseWeights:
        """Dense fp32 copies of the frozen base for the test-time update
        (built once on first use, exact values; 4 bytes per weight)."""
        if getattr(self, "_dense", None) is None and self.full_params:
            base, lay = self.params.data_ptr(), self.layout
            self._dense = _lib.DenseWeights(**{k: base + 4 * getattr(lay, k) for k in ("emb", "qkv", "o", "up", "down")})
        if getattr(self, "_dense", None) is None:
            L = _lib.lib()
            bufs = {}
            for name in ("emb", "qkv", "o", "up", "down"):
                q = self.q[name]
                t = torch.empty((q.rows, q.cols), dtype=torch.float32, device=self.device)
                _lib.check(L.altxs_dequant(C.byref(q), t.data_ptr(), q.cols, _stream_handle(self.device)),
                           "altxs_dequant")
                bufs[name] = t
            self._dense_bufs = bufs
            self._dense = _lib.DenseWeights(**{k: v.data_ptr() for k, v in bufs.items()})
        return self._dense

    @property
    def weights_struct(self) -> _lib.Weights:
        if getattr(self, "_weights_struct", None) is None:
            s = self.small
            self._weights_struct = _lib.Weights(
                emb=self.q["emb"], qkv=self.q["qkv"], o=self.q["o"], up=self.q["up"], down=self.q["down"],
                q_gain=s["q_gain"].data_ptr(), attn_scale=s["attn_scale"].data_ptr(),
                mlp_scale=s["mlp_scale"].data_ptr(), resid_mix=s["resid_mix"].data_ptr(),
                ln_scale=s["ln_scale"].data_ptr(), skip_weights=s["skip_weights"].data_ptr(),
                skip_gates=s["skip_gates"].data_ptr(), rope_cos=self.rope_cos.data_ptr(),
                rope_sin=self.rope_sin.data_ptr(), rope_positions=self.rope_positions,
                split=C.pointer(self._split) if self._split is not None else None,
                **{k: s[k].data_ptr() for k in ("smear_gate", "smear_lambda", "attn_gate_w", "softcap",
                                                "parallel_post", "parallel_resid") if k in s},
                emb_dense=self.params.data_ptr() + 4 * self.layout.emb if self.full_params else None,
                planes_live=1 if self.full_params else 0,
                tiles=C.pointer(self.tiles) if self.tiles is not None else None,
            )
        return self._weights_struct


class StreamBatch:
    """Device state of n independent streams on one GPU."""

    def __init__(self, dm: DeviceModel, n: int, *, words_per_stream: int, hist_len: int = 0,
                 keep_logits: bool = False, graphs: bool = False):
        """``graphs=True`` replays each step mode from a CUDA graph captured on
        its second call (every call still runs exactly one step): the step's
        kernels read their per-step inputs from device memory, so one capture
        serves every later step of this batch."""
        cfg, dev = dm.cfg, dm.device
        self.graphs = bool(graphs)
        self._graphs: dict = {}
        self._graph_seen: set = set()
        self.graph_kernels: dict = {}  # kernels per captured step, by key
        self.replays = 0
        self.dm, self.n, self.cfg = dm, int(n), cfg
        self.words_per_stream = int(words_per_stream)
        L, Hkv, hd = dm.n_virtual, cfg.num_kv_heads, cfg.head_dim
        self.tok = torch.full((n,), -1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(n, dtype=torch.int64, device=dev)
        self.active = torch.ones(n, dtype=torch.uint8, device=dev)
        # sliding-window ring, rows in the 24-bit split format (3 bytes/value)
        self.kv = torch.zeros((n, L, 2, Hkv, cfg.kv_len, 3 * hd), dtype=torch.uint8, device=dev)
        self.pos_base = torch.zeros(n, dtype=torch.int64, device=dev)  # absolute index of position 0
        # smear gate: the token each stream consumed last (-1: none yet)
        self.prev_tok = torch.full((n,), -1, dtype=torch.int32, device=dev) if cfg.smear_gate_enabled else None
        self.ac = torch.zeros((n, 8), dtype=torch.int64, device=dev)
        self.bits = torch.zeros((n, self.words_per_stream), dtype=torch.int32, device=dev)
        self.sym = torch.zeros(n, dtype=torch.int32, device=dev)
        self.hist_len = int(hist_len)
        self.hist = torch.zeros((n, max(1, self.hist_len)), dtype=torch.int32, device=dev) if hist_len else None
        self.lora = None
        if dm.lora_floats > 0:
            self.lora = torch.zeros((n, dm.lora_floats), dtype=torch.float32, device=dev)
            self.reset_lora()
        self.logits = torch.zeros((n, cfg.vocab_size), dtype=torch.float32, device=dev) if keep_logits else None
        wsb = int(_lib.lib().altxs_workspace_bytes(C.byref(dm.desc), n))
        if wsb < 0:
            raise ValueError("model shape not supported by the kernels")
        self.workspace = torch.empty(wsb, dtype=torch.uint8, device=dev)
        self.rows_all = None
        self._batch = _lib.Batch(
            n_streams=n, tok=self.tok.data_ptr(), pos=self.pos.data_ptr(), active=self.active.data_ptr(),
            kv=self.kv.data_ptr(), lora=self.lora.data_ptr() if self.lora is not None else None,
            lora_stride=dm.lora_floats, ac=self.ac.data_ptr(), bits=self.bits.data_ptr(),
            words_per_stream=self.words_per_stream, sym=self.sym.data_ptr(),
            hist=self.hist.data_ptr() if self.hist is not None else None, hist_len=self.hist_len,
            pos_base=self.pos_base.data_ptr(),
            prev_tok=self.prev_tok.data_ptr() if self.prev_tok is not None else None,
            logits_out=self.logits.data_ptr() if self.logits is not None else None,
            workspace=self.workspace.data_ptr(), workspace_bytes=wsb,
        )
        self.ac_init()

    # ---- adapters -----------------------------------------------------------
    def reset_lora(self) -> None:
        """Reference init: A ~ U(+-1/sqrt(in)) from the seeded generator, B = 0."""
        if self.lora is None:
            return
        flat = []
        A = init_lora_A(self.cfg)
        for name, (a_shape, b_shape) in lora_shapes(self.cfg).items():
            flat.append(A[name].reshape(-1))
            flat.append(np.zeros(b_shape[0] * b_shape[1], dtype=np.float32))
        vec = torch.from_numpy(np.concatenate(flat))
        if vec.numel() != self.dm.lora_floats:
            raise RuntimeError("LoRA layout mismatch between host and library")
        self.lora.copy_(vec.to(self.lora.device).expand_as(self.lora))

    # ---- coder --------------------------------------------------------------
    def _rows(self, rows):
        if rows is None:
            return None, self.n
        r = torch.as_tensor(np.asarray(rows, dtype=np.int32), device=self.dm.device)
        self._rows_keep = r
        return r.data_ptr(), int(r.numel())

    def ac_init(self, rows=None) -> None:
        rp, n = self._rows(rows)
        _lib.check(_lib.lib().altxs_ac_init(n, rp, self.ac.data_ptr(), _stream_handle(self.dm.device)), "ac_init")

    def ac_flush(self, rows=None) -> None:
        rp, n = self._rows(rows)
        _lib.check(
            _lib.lib().altxs_ac_flush(n, rp, self.ac.data_ptr(), self.bits.data_ptr(), self.words_per_stream,
                                      _stream_handle(self.dm.device)), "ac_flush")

    def begin_decode(self, payloads: dict[int, bytes]) -> None:
        """Load one segment payload per listed stream and seed its decoder."""
        rows = sorted(payloads)
        host = np.zeros((len(rows), self.words_per_stream), dtype=np.uint32)
        nb = np.zeros(len(rows), dtype=np.uint64)
        for j, r in enumerate(rows):
            p = payloads[r]
            if len(p) > self.words_per_stream * 4:
                raise ValueError(f"segment of {len(p)} bytes exceeds the bit buffer")
            buf = np.zeros(self.words_per_stream * 4, dtype=np.uint8)
            buf[: len(p)] = np.frombuffer(p, dtype=np.uint8)
            host[j] = buf.view(np.uint32)
            nb[j] = len(p) * 8
        idx = torch.as_tensor(np.asarray(rows, dtype=np.int64), device=self.dm.device)
        self.bits.index_copy_(0, idx, torch.from_numpy(host.view(np.int32)).to(self.dm.device))
        nbt = torch.from_numpy(nb.view(np.int64)).to(self.dm.device)
        rp, n = self._rows(rows)
        _lib.check(
            _lib.lib().altxs_ac_begin_decode(n, rp, self.ac.data_ptr(), self.bits.data_ptr(), nbt.data_ptr(),
                                             self.words_per_stream, _stream_handle(self.dm.device)),
            "ac_begin_decode")
        self._nbt_keep = nbt

    def segment_bytes(self, rows) -> dict[int, bytes]:
        """Bytes written by the listed (flushed) encoders."""
        ac = self.ac[rows].cpu().numpy()
        nbits = ac[:, 3].astype(np.int64)
        bits = self.bits[rows].cpu().numpy().view(np.uint8)
        return {int(r): bits[j, : (int(nbits[j]) + 7) // 8].tobytes() for j, r in enumerate(rows)}

    def status(self) -> np.ndarray:
        return (self.ac[:, 7].cpu().numpy() & 0xFFFFFFFF).astype(np.uint32)

    def check_status(self) -> None:
        st = self.status()
        bad = np.flatnonzero(st)
        if bad.size:
            i = int(bad[0])
            names = [v for k, v in ST_NAMES.items() if st[i] & k]
            raise RuntimeError(f"stream {i}: device status {int(st[i]):#x} ({', '.join(names)})")

    # ---- step ---------------------------------------------------------------
    def step(self, mode: int) -> None:
        if self.graphs:
            key = (int(mode), id(self.dm.weights_struct))
            g = self._graphs.get(key)
            if g is None and key in self._graph_seen:
                dev = self.dm.device
                g = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream(device=dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                n0 = _lib.lib().altxs_launch_count()
                with torch.cuda.graph(g, stream=side):
                    self._launch(mode)
                self.graph_kernels[key] = int(_lib.lib().altxs_launch_count() - n0)
                torch.cuda.current_stream(dev).wait_stream(side)
                self._graphs[key] = g
            if g is not None:
                g.replay()
                self.replays += 1
                return
            self._graph_seen.add(key)
        self._launch(mode)

    def _launch(self, mode: int) -> None:
        rc = _lib.lib().altxs_step(
            C.byref(self.dm.desc), C.byref(self.dm.weights_struct), C.byref(self._batch), int(mode),
            _stream_handle(self.dm.device),
        )
        _lib.check(rc, "altxs_step")

    # ---- chunk API: one flushed segment per stream ---------------------------
    def encode_chunk(self, symbols: torch.Tensor) -> list[bytes]:
        """Code ``symbols[t][i]`` (host or device, [n_steps][n]) as one segment
        per stream, continuing every stream's model state; returns the bytes."""
        dev = self.dm.device
        syms = symbols.to(dev, non_blocking=True)
        self.ac_init()
        for t in range(syms.shape[0]):
            self.sym.copy_(syms[t])
            self.step(_lib.STEP_ENCODE)
        self.ac_flush()
        out = self.segment_bytes(list(range(self.n)))
        self.check_status()
        return [out[i] for i in range(self.n)]

    def pack_payloads(self, payloads: list[bytes], pin: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
        """Host staging of one segment per stream: ([n][words] int32, [n] bits)."""
        host = np.zeros((self.n, self.words_per_stream * 4), dtype=np.uint8)
        nb = np.zeros(self.n, dtype=np.int64)
        for i, p in enumerate(payloads):
            if len(p) > host.shape[1]:
                raise ValueError(f"segment of {len(p)} bytes exceeds the bit buffer")
            host[i, : len(p)] = np.frombuffer(p, dtype=np.uint8)
            nb[i] = len(p) * 8
        words = torch.from_numpy(host.view(np.int32))
        nbits = torch.from_numpy(nb)
        if pin:
            words, nbits = words.pin_memory(), nbits.pin_memory()
        return words, nbits

    def decode_chunk(self, words: torch.Tensor, nbits: torch.Tensor, n_steps: int,
                     out: torch.Tensor | None = None) -> torch.Tensor:
        """Decode ``n_steps`` symbols per stream from one segment per stream.

        ``words``/``nbits`` are host (ideally pinned) buffers from
        ``pack_payloads``; the result is a host tensor [n_steps][n] (int32).
        Host->device copy, the decode steps and the device->host copy are
        all enqueued on the current stream."""
        dev = self.dm.device
        self.bits.copy_(words, non_blocking=True)
        nb = nbits.to(dev, non_blocking=True)
        _lib.check(
            _lib.lib().altxs_ac_begin_decode(self.n, None, self.ac.data_ptr(), self.bits.data_ptr(), nb.data_ptr(),
                                             self.words_per_stream, _stream_handle(dev)), "ac_begin_decode")
        dsyms = torch.empty((n_steps, self.n), dtype=torch.int32, device=dev)
        for t in range(n_steps):
            self.step(_lib.STEP_DECODE)
            dsyms[t].copy_(self.sym)
        if out is None:
            out = torch.empty((n_steps, self.n), dtype=torch.int32).pin_memory()
        out.copy_(dsyms, non_blocking=True)
        self._nb_keep = nb
        return out

    def set_active(self, mask: np.ndarray | None) -> None:
        if mask is None:
            self.active.fill_(1)
        else:
            self.active.copy_(torch.from_numpy(np.asarray(mask, dtype=np.uint8)).to(self.dm.device))


def words_for_segment(every: int, cdf_bits: int = 20) -> int:
    """Bit-buffer words that always hold one segment (<= cdf_bits+2 bits/symbol)."""
    return int(every) * (max(int(cdf_bits), 20) + 2) // 32 + 4


@dataclass
class StreamResult:
    payload: bytes
    segments: list
    n_symbols: int


class ContextReset:
    """Segment-reset context (``context_mode="reset"``): at a boundary
    ``start`` (after the update) each row's context becomes its last
    ``n = min(block_size, start)`` symbols at positions 0..n-1 (reference
    ``reset_segment`` with ``_chunk_ctx_start``, incremental.py:858-897,
    compress.py:122-125).  ``altxs_prefill`` writes the K/V rows of the first
    n-1 of them with the row's adapters; the row's pending token is already
    the n-th, so the next step at position n-1 gives the segment's first
    distribution.  ``pos_base`` keeps the symbol ring in absolute order."""

    def __init__(self, dm: DeviceModel):
        self.dm = dm
        self.t_max = max(1, int(dm.cfg.block_size) - 1)
        self.ws_bytes = int(_lib.lib().altxs_prefill_workspace_bytes(C.byref(dm.desc), self.t_max))
        if self.ws_bytes < 0:
            raise ValueError("model shape not supported by the prefill kernels")
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dm.device)
        self.dense = None if dm.tensor_cores else dm.dense_weights()

    def __call__(self, b: StreamBatch, rows, start: int) -> None:
        if b.hist is None:
            raise RuntimeError("the batch was built without a symbol ring")
        n = min(int(self.dm.cfg.block_size), int(start))
        if n < 1:
            return
        dev = self.dm.device
        idx = torch.arange(start - n, start, device=dev) % b.hist_len
        L = _lib.lib()
        for r in rows:
            ctx = b.hist[r].index_select(0, idx).contiguous()
            lora = b.lora[r].data_ptr() if b.lora is not None else None
            rc = L.altxs_prefill(
                C.byref(self.dm.desc), C.byref(self.dm.weights_struct),
                C.byref(self.dense) if self.dense is not None else None, ctx.data_ptr(), n - 1, lora,
                b.kv[r].data_ptr(), self.ws.data_ptr(), self.ws_bytes, _stream_handle(dev))
            _lib.check(rc, "altxs_prefill")
        ri = torch.as_tensor(list(rows), dtype=torch.int64, device=dev)
        b.pos.index_fill_(0, ri, n - 1)
        b.pos_base.index_fill_(0, ri, int(start) - n)


class Engine:
    """Encode / decode many independent streams in lockstep on one GPU."""

    def __init__(self, dm: DeviceModel, *, ttt=None, on_logits=None, header: bool = True):
        self.dm = dm
        self.cfg = dm.cfg
        self.ttt = ttt  # optional callable(batch, rows, hist_end) for the boundary update
        # payloads carry (and decoding checks) the lockstep fingerprint of the run
        self.header = bool(header)
        self.settings = lockstep.run_settings(dm, ttt is not None)
        self.reset = ContextReset(dm) if dm.cfg.context_mode == "reset" else None
        # optional callable(t, logits [n, V] on the device) after each encode step:
        # the logits every stream's symbol t was coded with (before the CDF rule)
        self.on_logits = on_logits

    def _new_batch(self, n: int, max_len: int) -> StreamBatch:
        cfg = self.cfg
        self.dm.ensure_rope(max_len + 2)
        hist = cfg.ctx + 2 if (self.ttt is not None or self.reset is not None) else 0
        return StreamBatch(self.dm, n, words_per_stream=words_for_segment(cfg.online_retrain_every, cfg.cdf_bits),
                           hist_len=hist, keep_logits=self.on_logits is not None)

    def _per_stream(self) -> bool:
        """A full-parameter update changes the model itself: one stream at a time."""
        return bool(getattr(self.ttt, "per_stream_model", False))

    def _update(self, b: StreamBatch, rows, t: int, prefix: torch.Tensor) -> None:
        if getattr(self.ttt, "needs_prefix", False):
            self.ttt(b, rows, t, prefix=prefix)
        else:
            self.ttt(b, rows, t)

    def encode(self, streams: list[np.ndarray]) -> list[StreamResult]:
        if self._per_stream():
            out = []
            for s in streams:
                self.ttt.reset()
                out += self._encode(list([s]))
            return out
        return self._encode(streams)

    def _encode(self, streams: list[np.ndarray]) -> list[StreamResult]:
        cfg, dev = self.cfg, self.dm.device
        n = len(streams)
        lens = np.array([len(s) for s in streams], dtype=np.int64)
        T = int(lens.max()) if n else 0
        every = max(1, int(cfg.online_retrain_every))
        b = self._new_batch(n, T)
        symsT = np.zeros((max(T, 1), n), dtype=np.int32)
        for i, s in enumerate(streams):
            symsT[: len(s), i] = np.asarray(s, dtype=np.int32)
        if n and (symsT.min() < 0 or symsT.max() >= cfg.vocab_size):
            raise ValueError("symbol outside the alphabet")
        symsT_d = torch.from_numpy(symsT).to(dev)
        segs: list[list[bytes]] = [[] for _ in range(n)]
        for t in range(T):
            if t > 0 and t % every == 0:
                rows = [i for i in range(n) if lens[i] > t]
                self._boundary_encode(b, rows, segs, t, symsT_d)
            active = lens > t
            if not active.all():
                b.set_active(active)
            b.sym.copy_(symsT_d[t])
            b.step(_lib.STEP_ENCODE)
            if self.on_logits is not None:
                self.on_logits(t, b.logits)
        rows = [i for i in range(n) if lens[i] > 0]
        if rows:
            b.set_active(None)
            b.ac_flush(rows)
            for r, p in b.segment_bytes(rows).items():
                segs[r].append(p)
        torch.cuda.synchronize(dev)
        b.check_status()
        out = []
        head = lockstep.header_frame(self.settings) if self.header else b""
        for i in range(n):
            payload = head + b"".join(struct.pack("<Q", len(p)) + p for p in segs[i])
            out.append(StreamResult(payload=payload, segments=segs[i], n_symbols=int(lens[i])))
        return out

    def _boundary_encode(self, b: StreamBatch, rows, segs, t: int, prefix: torch.Tensor) -> None:
        b.set_active(None)
        b.ac_flush(rows)
        for r, p in b.segment_bytes(rows).items():
            segs[r].append(p)
        b.ac_init(rows)
        if self.ttt is not None:
            self._update(b, rows, t, prefix)
        if self.reset is not None:
            self.reset(b, rows, t)

    def decode(self, payloads: list[bytes], n_symbols: list[int]) -> list[np.ndarray]:
        if self._per_stream():
            out = []
            for p, k in zip(payloads, n_symbols):
                self.ttt.reset()
                out += self._decode([p], [k])
            return out
        return self._decode(payloads, n_symbols)

    def _decode(self, payloads: list[bytes], n_symbols: list[int]) -> list[np.ndarray]:
        cfg, dev = self.cfg, self.dm.device
        n = len(payloads)
        lens = np.asarray(n_symbols, dtype=np.int64)
        T = int(lens.max()) if n else 0
        every = max(1, int(cfg.online_retrain_every))
        segs = []
        for p in payloads:
            enc_settings, fp, body = lockstep.split_header(p)
            lockstep.check(enc_settings, fp, self.settings)  # raises on a mismatch
            segs.append(list(iter_framed_segments(body)))
        for i in range(n):
            need = (int(lens[i]) + every - 1) // every
            if len(segs[i]) != need:
                raise ValueError(f"stream {i}: {len(segs[i])} segments, expected {need}")
        b = self._new_batch(n, T)
        out = torch.zeros((max(T, 1), n), dtype=torch.int32, device=dev)
        first = {i: segs[i][0] for i in range(n) if lens[i] > 0}
        if first:
            b.begin_decode(first)
        for t in range(T):
            if t > 0 and t % every == 0:
                rows = [i for i in range(n) if lens[i] > t]
                if rows:
                    b.set_active(None)
                    if self.ttt is not None:
                        self._update(b, rows, t, out)
                    if self.reset is not None:
                        self.reset(b, rows, t)
                    b.begin_decode({i: segs[i][t // every] for i in rows})
            active = lens > t
            if not active.all():
                b.set_active(active)
            b.step(_lib.STEP_DECODE)
            out[t].copy_(b.sym)
        torch.cuda.synchronize(dev)
        b.check_status()
        host = out.cpu().numpy()
        return [host[: int(lens[i]), i].copy() for i in range(n)]


def iter_framed_segments(payload: bytes):
    """Walk the ``<u64 len><segment bytes>`` framing (incremental.py:1782-1796)."""
    off, total = 0, len(payload)
    while off < total:
        if off + 8 > total:
            raise ValueError(f"truncated segment header at offset {off}")
        (ln,) = struct.unpack_from("<Q", payload, off)
        off += 8
        if off + ln > total:
            raise ValueError(f"truncated segment at offset {off}: need {ln}, have {total - off}")
        yield payload[off: off + ln]
        off += ln
