"""Decoder stages over the C ABI: the host mirror of the reference's
`Transformer` (spm::Forwarder, dial-core/src/models/qwen3_vl/text.rs:1599-1707)
and of the generator's embed / ln_f / lm_head / argmax path
(qwen3_vl.rs:2143-2463, :130-143).

A `Stage` owns a contiguous range of decoder layers (the unit the reference's
topology assigns to a worker, spm/topology.rs:54-110), optionally the token
embedding (first stage) and the final norm + output head (last stage), their
KV caches (one slot per sequence, llama3/cache.rs:149-217) and a workspace.
Weights are random-initialised on the device from a seed per (layer, tensor),
so any split of the layers into stages holds exactly the weights of the
single-stage model.  torch provides device memory and streams only; every
kernel is in libdial_cuda.so.
"""
from __future__ import annotations

import ctypes
import hashlib
from dataclasses import dataclass, field
from typing import Optional

from . import (BF16, F16, F32, GgufLinear, W8A16Linear, _torch, check, dtype_code, lib,
               stream_ptr)

WFMT_W8A16, WFMT_W8A16_F16S, WFMT_Q4_0, WFMT_Q8_0 = 0, 1, 2, 8


class DecoderDims(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("vocab", ctypes.c_int32),
                ("qk_norm", ctypes.c_int32), ("weight_format", ctypes.c_int32),
                ("head_format", ctypes.c_int32), ("act_dtype", ctypes.c_int32),
                ("rms_eps", ctypes.c_float), ("max_seq", ctypes.c_int64),
                ("n_slots", ctypes.c_int32)]


class LinearRef(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("s", ctypes.c_void_p)]


class LayerWeights(ctypes.Structure):
    _fields_ = [("qkv", LinearRef), ("o", LinearRef), ("gate_up", LinearRef), ("down", LinearRef),
                ("input_norm", ctypes.c_void_p), ("post_norm", ctypes.c_void_p),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
                ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p)]


_SIGS = {
    "dial_decoder_workspace_bytes": ([ctypes.POINTER(DecoderDims), ctypes.c_int64, ctypes.c_int64],
                                     ctypes.c_size_t),
    "dial_decoder_layers": ([ctypes.POINTER(DecoderDims), ctypes.POINTER(LayerWeights), ctypes.c_int,
                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                             ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                             ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "dial_decoder_head": ([ctypes.POINTER(DecoderDims), ctypes.c_void_p, LinearRef, ctypes.c_void_p,
                           ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                           ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "dial_decoder_head_shard": ([ctypes.POINTER(DecoderDims), ctypes.c_void_p, LinearRef, ctypes.c_int64,
                                 ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                 ctypes.c_void_p], ctypes.c_int),
}


def _bind():
    L = lib()
    for name, (a, r) in _SIGS.items():
        fn = getattr(L, name)
        fn.argtypes, fn.restype = a, r
    return L


@dataclass
class ModelConfig:
    """Decoder shape.  Defaults: the Qwen3-8B text decoder (W8A16, QK-norm)."""
    n_layers: int = 36
    hidden: int = 4096
    intermediate: int = 12288
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    qk_norm: bool = True
    weight_format: int = WFMT_W8A16       # layer linears
    head_format: int = WFMT_W8A16         # output head (Q8_0 for the GGUF Llama config)
    act_dtype: str = "f16"
    init_std: float = 0.02

    @staticmethod
    def llama3_8b_q4_0() -> "ModelConfig":
        """Llama-3-8B shape, Q4_0 layers, Q8_0 head, no QK-norm."""
        return ModelConfig(n_layers=32, intermediate=14336, vocab=128256, rope_theta=5e5,
                           qk_norm=False, weight_format=WFMT_Q4_0, head_format=WFMT_Q8_0)


def _seed(base: int, *key) -> int:
    h = hashlib.sha256(("/".join(map(str, (base,) + key))).encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


class _Linear:
    """A quantised linear held by a stage (W8A16 or GGUF device layout)."""

    def __init__(self, fmt: int, weight_f32):
        torch = _torch()
        self.fmt = fmt
        if fmt in (WFMT_W8A16, WFMT_W8A16_F16S):
            sd = torch.float32 if fmt == WFMT_W8A16 else torch.float16
            self.lin = W8A16Linear.from_linear("", weight_f32, scale_dtype=sd)
            self.ref = LinearRef(self.lin.qweight.data_ptr(), self.lin.scales.data_ptr())
        else:
            self.lin = GgufLinear.quantize(weight_f32, fmt)
            self.ref = LinearRef(self.lin.qs.data_ptr(), self.lin.d.data_ptr())

    @property
    def weight_bytes(self) -> int:
        return self.lin.weight_bytes


class Stage:
    """Layers [first, last) of the model, plus embedding (first == 0) and head
    (last == n_layers) when `with_embed` / `with_head`."""

    def __init__(self, cfg: ModelConfig, first: int, last: int, n_slots: int, max_seq: int,
                 seed: int = 299792458, device=None, with_embed: Optional[bool] = None,
                 with_head: Optional[bool] = None, weights: Optional[dict] = None,
                 head_rows: Optional[tuple] = None):
        torch = _torch()
        self.L = _bind()
        self.cfg, self.first, self.last = cfg, first, last
        self.n_slots, self.max_seq = n_slots, max_seq
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.dt = {"f16": torch.float16, "bf16": torch.bfloat16}[cfg.act_dtype]
        self.with_embed = first == 0 if with_embed is None else with_embed
        self.with_head = last == cfg.n_layers if with_head is None else with_head
        c = cfg
        self.dims = DecoderDims(c.hidden, c.intermediate, c.n_heads, c.n_kv_heads, c.head_dim,
                                c.vocab, int(c.qk_norm), c.weight_format, c.head_format,
                                dtype_code(self.dt), c.rms_eps, max_seq, n_slots)
        self._keep = []
        self.layers = []
        self.linears = []
        self.layer_linears = []  # per layer: {"qkv", "o", "gate_up", "down"} -> _Linear
        self.layer_norms = []    # per layer: {"input_norm", "post_norm", "q_norm", "k_norm"}
        gen = torch.Generator(device=self.device)

        def rand(shape, *key, std=None):
            if weights is not None:
                return weights[key].to(self.device, torch.float32)
            gen.manual_seed(_seed(seed, *key))
            return torch.randn(shape, generator=gen, device=self.device, dtype=torch.float32) * (
                c.init_std if std is None else std)

        def ones(n, *key):
            if weights is not None and key in weights:
                return weights[key].to(self.device, self.dt).contiguous()
            return torch.ones(n, device=self.device, dtype=self.dt)

        D, H, I = c.head_dim, c.hidden, c.intermediate
        QKV = (c.n_heads + 2 * c.n_kv_heads) * D
        kv_shape = (n_slots, c.n_kv_heads, max_seq, D)
        self.k_caches, self.v_caches = [], []
        arr = (LayerWeights * max(1, last - first))()
        for i, li in enumerate(range(first, last)):
            lin = {}
            # fused projections as the reference builds them (text.rs:1428-1432, 634-637)
            for name, shape in (("qkv", (QKV, H)), ("o", (H, c.n_heads * D)),
                                ("gate_up", (2 * I, H)), ("down", (H, I))):
                w = rand(shape, li, name)
                lin[name] = _Linear(c.weight_format, w)
                del w
            norms = {n: ones(H if n in ("input_norm", "post_norm") else D, li, n)
                     for n in ("input_norm", "post_norm", "q_norm", "k_norm")}
            kc = torch.zeros(kv_shape, device=self.device, dtype=self.dt)
            vc = torch.zeros(kv_shape, device=self.device, dtype=self.dt)
            self.k_caches.append(kc)
            self.v_caches.append(vc)
            self._keep += [lin, norms]
            self.linears += list(lin.values())
            self.layer_linears.append(lin)
            self.layer_norms.append(norms)
            arr[i] = LayerWeights(lin["qkv"].ref, lin["o"].ref, lin["gate_up"].ref, lin["down"].ref,
                                  norms["input_norm"].data_ptr(), norms["post_norm"].data_ptr(),
                                  norms["q_norm"].data_ptr(), norms["k_norm"].data_ptr(),
                                  kc.data_ptr(), vc.data_ptr())
        self.layer_arr = arr
        self.embed = None
        if self.with_embed:
            e = rand((c.vocab, H), "embed")
            self.embed = e.to(self.dt)
            del e
        self.head = None
        # head_rows = (v0, v1): this stage's share of a vocabulary-parallel head
        # (rows v0..v1 of the same seeded head), used by head_shard_forward
        self.head_rows = tuple(head_rows) if head_rows is not None else None
        self.head_shard = None
        if self.with_head or (self.head_rows is not None and self.head_rows[1] > self.head_rows[0]):
            self.final_norm = ones(H, "final_norm")
            w = rand((c.vocab, H), "lm_head")
            if self.head_rows is not None:
                v0, v1 = self.head_rows
                self.head_shard = _Linear(c.head_format, w[v0:v1].contiguous())
            if self.with_head:
                self.head = _Linear(c.head_format, w)
            del w
        # RoPE tables (llama3/cache.rs:24-64) in the activation dtype
        self.cos = torch.empty((max_seq, D // 2), device=self.device, dtype=self.dt)
        self.sin = torch.empty_like(self.cos)
        check(self.L.dial_rope_tables(self.cos.data_ptr(), self.sin.data_ptr(), dtype_code(self.dt),
                                      max_seq, D, c.rope_theta, stream_ptr()), "dial_rope_tables")
        self._ws = None
        torch.cuda.synchronize(self.device)

    # -------------------------------------------------------------- sizes
    @property
    def weight_bytes(self) -> int:
        b = sum(l.weight_bytes for l in self.linears)
        if self.head is not None:
            b += self.head.weight_bytes
        if self.head_shard is not None:
            b += self.head_shard.weight_bytes
        return b

    def workspace(self, tokens: int, max_len: int):
        torch = _torch()
        need = self.L.dial_decoder_workspace_bytes(ctypes.byref(self.dims), tokens, max_len)
        if self._ws is None or self._ws.numel() < need:
            # zero-filled: the stream-K counters at its start must begin at zero
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._ws, need

    # -------------------------------------------------------------- forward pieces
    def embed_tokens(self, ids, out):
        """out[t] = embedding[ids[t]] (ids int32 on the device)."""
        check(lib().dial_embedding(self.embed.data_ptr(), ids.data_ptr(), out.data_ptr(),
                                   dtype_code(self.dt), ids.numel(), self.cfg.vocab, self.cfg.hidden,
                                   stream_ptr()), "dial_embedding")

    def layers_forward(self, hidden, positions, slots, max_len: int):
        """Runs this stage's layers on hidden [T, H] in place."""
        if self.last == self.first:
            return hidden
        T = hidden.shape[0]
        ws, need = self.workspace(T, max_len)
        check(self.L.dial_decoder_layers(ctypes.byref(self.dims), self.layer_arr,
                                         self.last - self.first, hidden.data_ptr(),
                                         positions.data_ptr(), slots.data_ptr(), T, max_len,
                                         self.cos.data_ptr(), self.sin.data_ptr(), ws.data_ptr(),
                                         need, stream_ptr()), "dial_decoder_layers")
        return hidden

    def head_forward(self, hidden, out_ids, row_index=None, logits=None):
        rows = out_ids.numel()
        ws, need = self.workspace(max(rows, hidden.shape[0]), 1)
        check(self.L.dial_decoder_head(ctypes.byref(self.dims), self.final_norm.data_ptr(),
                                       self.head.ref, hidden.data_ptr(),
                                       row_index.data_ptr() if row_index is not None else None,
                                       rows, out_ids.data_ptr(),
                                       logits.data_ptr() if logits is not None else None,
                                       ws.data_ptr(), need, stream_ptr()), "dial_decoder_head")
        return out_ids


    def head_shard_forward(self, hidden, keys_out, row_index=None, logits=None):
        """This stage's share of a vocabulary-parallel head: keys_out (int64
        [rows], the unsigned greedy keys' bits) of head rows head_rows over
        rmsnorm(hidden) (dial_decoder_head_shard); logits [rows, v1 - v0]."""
        rows = keys_out.numel()
        v0, v1 = self.head_rows
        ws, need = self.workspace(max(rows, hidden.shape[0]), 1)
        check(self.L.dial_decoder_head_shard(ctypes.byref(self.dims), self.final_norm.data_ptr(),
                                             self.head_shard.ref, v0, v1 - v0, hidden.data_ptr(),
                                             row_index.data_ptr() if row_index is not None else None,
                                             rows, keys_out.data_ptr(),
                                             logits.data_ptr() if logits is not None else None,
                                             ws.data_ptr(), need, stream_ptr()), "dial_decoder_head_shard")
        return keys_out


def head_merge(keys, out_ids):
    """keys int64 [n_shards, rows] (the shards' greedy keys) -> out_ids int32 [rows]."""
    n, rows = keys.shape
    check(lib().dial_head_merge(keys.data_ptr(), n, rows, out_ids.data_ptr(), stream_ptr()),
          "dial_head_merge")
    return out_ids


def vocab_shards(vocab: int, weights) -> list:
    """Splits the head's rows over stages in proportion to `weights` (a stage
    with weight 0 holds none), each share a multiple of 16 rows (one GEMV tile)
    except the last non-empty one; returns [(v0, v1)] per stage."""
    tot = float(sum(weights))
    if tot <= 0:
        raise ValueError("no stage takes a share of the head")
    out, v0, acc = [], 0, 0.0
    last = max(i for i, w in enumerate(weights) if w > 0)
    for i, w in enumerate(weights):
        acc += w
        v1 = vocab if i >= last else min(vocab, int(round(vocab * acc / tot / 16)) * 16)
        v1 = max(v0, v1)
        out.append((v0, v1))
        v0 = v1
    return out


class Decoder:
    """All layers on one GPU: prefill + greedy decode (the reference's token
    loop, Qwen3Vl::next_token qwen3_vl.rs:3240-3392, with greedy sampling)."""

    def __init__(self, cfg: ModelConfig, n_slots: int, max_seq: int, seed: int = 299792458,
                 weights: Optional[dict] = None):
        self.stage = Stage(cfg, 0, cfg.n_layers, n_slots, max_seq, seed=seed, weights=weights)
        self.cfg = cfg

    def prefill(self, ids, slot: int):
        """ids int32 [T] on the device -> first generated token (int32 [1])."""
        torch = _torch()
        st = self.stage
        T = ids.numel()
        hidden = torch.empty((T, self.cfg.hidden), device=st.device, dtype=st.dt)
        st.embed_tokens(ids, hidden)
        pos = torch.arange(T, device=st.device, dtype=torch.int32)
        slots = torch.full((T,), slot, device=st.device, dtype=torch.int32)
        st.layers_forward(hidden, pos, slots, T)
        out = torch.empty(1, device=st.device, dtype=torch.int32)
        last = torch.tensor([T - 1], device=st.device, dtype=torch.int32)
        st.head_forward(hidden, out, row_index=last)
        return out

    def decode_step(self, ids, positions, slots, max_len: int, out_ids, hidden=None):
        """One token per sequence: ids/positions/slots int32 [B] -> out_ids [B]."""
        torch = _torch()
        st = self.stage
        B = ids.numel()
        if hidden is None:
            hidden = torch.empty((B, self.cfg.hidden), device=st.device, dtype=st.dt)
        st.embed_tokens(ids, hidden)
        st.layers_forward(hidden, positions, slots, max_len)
        st.head_forward(hidden, out_ids)
        return out_ids
