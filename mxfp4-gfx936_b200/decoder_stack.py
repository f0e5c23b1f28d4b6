"""Qwen3-30B-A3B-shaped decoder stack on the MXFP4 backend.

Every linear of the stack is an MXFP4 W4A16 call of this backend: the qkv
projection (2048 -> 5120), the output projection (4096 -> 2048), the router
(2048 -> 128) and the experts (the ``_moe_apply`` composition of the reference
adapter, vllm:233-265, as ``moe_layer_mxfp4``).  Around them sit the layer's
PyTorch ops: RMSNorm (input, post-attention, per-head q/k norms), rotary
embeddings, attention through ``torch.nn.functional.scaled_dot_product_attention``
(causal over each prefill sequence, over the KV cache when decoding) and the
residual adds.  The routing between router and experts is the device router
(``moe_router``: softmax, top-8, renormalised).  Weights are random-init in
the checkpoint's layout (packed ``[N, K/2]`` uint8, E8M0 ``[N, K/32]``).

Several GPUs (one process per GPU, ``torch.distributed`` over NCCL):

* dense linears (qkv, o) column-sharded with the all-gather fused into the
  GEMM epilogue (``ColumnParallelLinear``, ``fused=True``), so every rank holds
  the full projection outputs;
* attention sharded by sequence (each rank attends for its own sequences and
  holds only their KV cache); the attention outputs are all-gathered (NCCL)
  before the output projection;
* experts expert-parallel (``ExpertParallelMoE``: E/G experts per rank, the
  rank's own tokens dispatched to the experts' owners and combined back over
  NVLink); the router is replicated (128 outputs);
* the residual stream of the rank's tokens is all-gathered (NCCL) after the
  MoE block, so every layer starts from the full hidden states.

``audit`` (optional) is called as ``audit(name, layer_index, inputs, output)``
after every MXFP4 call with the exact tensors the call saw: the same-input
audit of the reference's release gate (results/release_validation.json,
``same_input_dense_gate``), where each call is re-run through the reference
path on the same input and compared.  ``ops`` (optional, one GPU) replaces the
operator module (``linear_mxfp4_soft``, ``moe_router``, ``moe_layer_mxfp4``),
e.g. by a restatement of the reference path for a whole-stack comparison.
"""

from __future__ import annotations

import importlib.util
import sys
from dataclasses import dataclass, field
from pathlib import Path

import torch
import torch.nn.functional as F

_HERE = Path(__file__).resolve().parent


def _module(name: str, file: str):
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, _HERE / file)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def _soft():
    return _module("moe_op_mxfp4_soft", "moe_op_mxfp4_soft.py")


@dataclass(frozen=True)
class StackConfig:
    """Shape of the stack (defaults: Qwen3-30B-A3B)."""

    layers: int = 48
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    inter: int = 768
    rope_theta: float = 1.0e6
    eps: float = 1.0e-6

    @property
    def q_size(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    def layer_flops(self, tokens: int, ctx_per_token: float) -> float:
        """Linear FLOPs of one layer (2*M*N*K per MXFP4 call, experts at top_k
        routes per token) plus attention (QK^T and PV over ctx_per_token keys
        on average per query)."""
        h = self.hidden
        dense = 2.0 * tokens * h * (self.qkv_size + self.experts) + 2.0 * tokens * self.q_size * h
        moe = 2.0 * tokens * self.top_k * (h * 2 * self.inter + self.inter * h)
        attn = 4.0 * tokens * self.heads * self.head_dim * ctx_per_token
        return dense + moe + attn


@dataclass
class LayerWeights:
    """One decoder layer in the compressed-tensors layout: packed E2M1 bytes
    ``[N, K/2]`` and E8M0 scales ``[N, K/32]`` for every linear; BF16 norms."""

    qkv_w: torch.Tensor
    qkv_s: torch.Tensor
    o_w: torch.Tensor
    o_s: torch.Tensor
    router_w: torch.Tensor
    router_s: torch.Tensor
    w13: torch.Tensor
    s13: torch.Tensor
    w2: torch.Tensor
    s2: torch.Tensor
    ln1: torch.Tensor
    ln2: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor


def random_layer(cfg: StackConfig, device, seed: int) -> LayerWeights:
    """Random-init layer: packed bytes uniform over all codes, scales uniform in
    118..130 (BASELINE's distributions); norm weights near one."""
    g = torch.Generator(device=device).manual_seed(seed)
    h, e, i = cfg.hidden, cfg.experts, cfg.inter

    def packed(*shape):
        return torch.randint(0, 256, shape, generator=g, device=device, dtype=torch.uint8)

    def scales(*shape):
        return torch.randint(118, 131, shape, generator=g, device=device, dtype=torch.uint8)

    def norm(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)

    return LayerWeights(
        qkv_w=packed(cfg.qkv_size, h // 2), qkv_s=scales(cfg.qkv_size, h // 32),
        o_w=packed(h, cfg.q_size // 2), o_s=scales(h, cfg.q_size // 32),
        router_w=packed(e, h // 2), router_s=scales(e, h // 32),
        w13=packed(e, 2 * i, h // 2), s13=scales(e, 2 * i, h // 32),
        w2=packed(e, h, i // 2), s2=scales(e, h, i // 32),
        ln1=norm(h), ln2=norm(h), q_norm=norm(cfg.head_dim), k_norm=norm(cfg.head_dim))


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm in FP32, rounded back to the input dtype (Qwen3)."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * weight.float()).to(x.dtype)


def rope_tables(cfg: StackConfig, positions: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, device=device, dtype=torch.float32) / cfg.head_dim))
    t = torch.arange(positions, device=device, dtype=torch.float32)
    ang = torch.outer(t, inv)
    ang = torch.cat((ang, ang), dim=-1)
    return ang.cos(), ang.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding (rotate-half form) on [T, heads, head_dim] with
    per-token tables [T, head_dim]."""
    d = x.shape[-1] // 2
    xf = x.float()
    rot = torch.cat((-xf[..., d:], xf[..., :d]), dim=-1)
    return (xf * cos[:, None, :] + rot * sin[:, None, :]).to(x.dtype)


@dataclass
class KVCache:
    """Per-layer key/value cache of this rank's sequences: [seqs, kv_heads, ctx, head_dim]."""

    k: list = field(default_factory=list)
    v: list = field(default_factory=list)
    length: int = 0


class DecoderStack:
    """The stack on ``world`` GPUs (rank ``rank``; ``world == 1``: one GPU).

    ``layers`` holds full (unsharded) weights; the constructor shards them for
    the rank.  ``prefill(h, seqs)`` runs ``seqs`` equal-length sequences whose
    hidden states are stacked as ``h [seqs * seq_len, hidden]`` and fills this
    rank's KV cache; ``decode(h)`` appends one token to every sequence.  Both
    return the full hidden states of all tokens on every rank."""

    def __init__(self, cfg: StackConfig, layers: list[LayerWeights], rank: int = 0, world: int = 1, group=None,
                 audit=None, max_ctx: int = 4096, ops=None, max_tokens: int | None = None):
        self.cfg, self.rank, self.world, self.group = cfg, rank, world, group
        self.audit = audit
        self.soft = ops if ops is not None else _soft()
        if ops is not None and world > 1:
            raise ValueError("operator overrides are for one GPU")
        self.layers = []
        # the layers run one after another on every rank, so they share one set
        # of peer-mapped output and exchange buffers (sized by the largest call)
        tp_pool, ep_pool = {}, {}
        ep_max = None if max_tokens is None else -(-max_tokens // world)
        for L in layers:
            entry = {"w": L}
            if world > 1:
                cp = _module("mxfp4_column_parallel", "column_parallel.py")
                ep = _module("mxfp4_expert_parallel", "expert_parallel.py")
                entry["qkv"] = cp.ColumnParallelLinear.from_full(L.qkv_w, L.qkv_s, rank, world, group=group, fused=True,
                                                                 buffer_pool=tp_pool)
                entry["o"] = cp.ColumnParallelLinear.from_full(L.o_w, L.o_s, rank, world, group=group, fused=True,
                                                               buffer_pool=tp_pool)
                entry["moe"] = ep.ExpertParallelMoE.from_full(L.w13, L.s13, L.w2, L.s2, rank, world, group=group,
                                                              fused=True, max_tokens=ep_max, buffer_pool=ep_pool)
                # the shards are copies: keep only what this rank needs of the full layer
                entry["w"] = LayerWeights(qkv_w=None, qkv_s=None, o_w=None, o_s=None, router_w=L.router_w,
                                          router_s=L.router_s, w13=None, s13=None, w2=None, s2=None, ln1=L.ln1,
                                          ln2=L.ln2, q_norm=L.q_norm, k_norm=L.k_norm)
            self.layers.append(entry)
        device = layers[0].ln1.device
        self.cos, self.sin = rope_tables(cfg, max_ctx, device)
        self.max_ctx = max_ctx
        self.cache = KVCache()

    # ------------------------------------------------------------------ pieces
    def _linear(self, name, li, x, w, s):
        y = self.soft.linear_mxfp4_soft(x, w, s)
        if self.audit is not None:
            self.audit(name, li, (x, w, s), y)
        return y

    def _tp_linear(self, name, li, entry, x):
        if self.world == 1:
            L = entry["w"]
            w, s = (L.qkv_w, L.qkv_s) if name == "qkv" else (L.o_w, L.o_s)
            return self._linear(name, li, x, w, s)
        y = entry[name](x)
        if self.audit is not None:
            self.audit(name, li, (x, entry[name]), y)
        return y

    def _moe(self, li, entry, x):
        L = entry["w"]
        logits = self._linear("router", li, x, L.router_w, L.router_s)
        tw, tid = self.soft.moe_router(logits, self.cfg.top_k)
        if self.world == 1:
            y = self.soft.moe_layer_mxfp4(x, L.w13, L.s13, L.w2, L.s2, tw, tid)
            if self.audit is not None:
                self.audit("experts", li, (x, L.w13, L.s13, L.w2, L.s2, tw, tid), y)
        else:
            y = entry["moe"](x, tw, tid)
            if self.audit is not None:
                self.audit("experts", li, (x, entry["moe"], tw, tid), y)
        return y

    def _own_seqs(self, seqs: int) -> tuple[int, int]:
        """Sequences [lo, hi) this rank attends for (all of them on one GPU,
        or when they do not divide over the ranks)."""
        if self.world == 1 or seqs % self.world:
            return 0, seqs
        per = seqs // self.world
        return self.rank * per, (self.rank + 1) * per

    def _gather_rows(self, local: torch.Tensor, total_rows: int) -> torch.Tensor:
        """Concatenate every rank's equal-size row block (NCCL all-gather)."""
        import torch.distributed as dist
        out = torch.empty((total_rows, local.shape[1]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
        return out

    # ------------------------------------------------------------------ blocks
    def _attention(self, li, entry, h, seqs, seq_len, pos0):
        cfg = self.cfg
        L = entry["w"]
        t = seqs * seq_len
        x = rms_norm(h, L.ln1, cfg.eps)
        qkv = self._tp_linear("qkv", li, entry, x)
        lo, hi = self._own_seqs(seqs)
        rows = slice(lo * seq_len, hi * seq_len)
        mine = qkv[rows]
        n_own = hi - lo
        q = mine[:, :cfg.q_size].reshape(-1, cfg.heads, cfg.head_dim)
        k = mine[:, cfg.q_size:cfg.q_size + cfg.kv_size].reshape(-1, cfg.kv_heads, cfg.head_dim)
        v = mine[:, cfg.q_size + cfg.kv_size:].reshape(-1, cfg.kv_heads, cfg.head_dim)
        q = rms_norm(q, L.q_norm, cfg.eps)
        k = rms_norm(k, L.k_norm, cfg.eps)
        pos = torch.arange(pos0, pos0 + seq_len, device=h.device).repeat(n_own)
        q = apply_rope(q, self.cos[pos], self.sin[pos])
        k = apply_rope(k, self.cos[pos], self.sin[pos])
        # [seqs, heads, seq_len, head_dim]
        q4 = q.reshape(n_own, seq_len, cfg.heads, cfg.head_dim).transpose(1, 2)
        k4 = k.reshape(n_own, seq_len, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        v4 = v.reshape(n_own, seq_len, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        kc, vc = self.cache.k[li], self.cache.v[li]
        kc[:, :, pos0:pos0 + seq_len] = k4
        vc[:, :, pos0:pos0 + seq_len] = v4
        if pos0 == 0:
            attn = F.scaled_dot_product_attention(q4, k4, v4, is_causal=True, enable_gqa=True)
        else:
            end = pos0 + seq_len
            mask = None
            if seq_len > 1:  # queries at pos0.. see the cache up to themselves
                qpos = torch.arange(pos0, end, device=h.device)[:, None]
                mask = torch.arange(end, device=h.device)[None, :] <= qpos
            attn = F.scaled_dot_product_attention(q4, kc[:, :, :end], vc[:, :, :end], attn_mask=mask,
                                                  enable_gqa=True)
        attn = attn.transpose(1, 2).reshape(n_own * seq_len, cfg.q_size)
        if n_own != seqs:
            attn = self._gather_rows(attn, t)
        o = self._tp_linear("o", li, entry, attn)
        return h + o

    def _moe_block(self, li, entry, h):
        L = entry["w"]
        t = h.shape[0]
        if self.world == 1:
            return h + self._moe(li, entry, rms_norm(h, L.ln2, self.cfg.eps))
        per = -(-t // self.world)
        lo, hi = min(t, self.rank * per), min(t, (self.rank + 1) * per)
        mine = h[lo:hi]
        out_mine = mine + self._moe(li, entry, rms_norm(mine, L.ln2, self.cfg.eps))
        if per * self.world == t:
            return self._gather_rows(out_mine, t)
        padded = torch.zeros((per, h.shape[1]), dtype=h.dtype, device=h.device)
        padded[: hi - lo] = out_mine
        return self._gather_rows(padded, per * self.world)[:t]

    # ------------------------------------------------------------------ public
    def allocate_cache(self, seqs: int, ctx: int) -> None:
        """KV cache of this rank's sequences for up to ``ctx`` positions."""
        cfg = self.cfg
        lo, hi = self._own_seqs(seqs)
        device = self.cos.device
        shape = (hi - lo, cfg.kv_heads, ctx, cfg.head_dim)
        self.cache = KVCache(k=[torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in self.layers],
                             v=[torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in self.layers],
                             length=0)
        self._seqs = seqs

    def forward(self, h: torch.Tensor, seqs: int, seq_len: int, pos0: int) -> torch.Tensor:
        """``seq_len`` new tokens of each of ``seqs`` sequences at positions
        ``pos0 ..``; h is [seqs * seq_len, hidden] BF16 (sequence-major)."""
        if pos0 + seq_len > self.max_ctx:
            raise ValueError("positions beyond the rotary table")
        for li, entry in enumerate(self.layers):
            h = self._attention(li, entry, h, seqs, seq_len, pos0)
            h = self._moe_block(li, entry, h)
        self.cache.length = pos0 + seq_len
        return h

    def prefill(self, h: torch.Tensor, seqs: int) -> torch.Tensor:
        return self.forward(h, seqs, h.shape[0] // seqs, 0)

    def decode(self, h: torch.Tensor, pos: int) -> torch.Tensor:
        return self.forward(h, h.shape[0], 1, pos)


def attention_ctx_per_token(seq_len: int, pos0: int) -> float:
    """Mean number of keys a query attends to: causal prefill or decode."""
    if pos0 == 0:
        return (seq_len + 1) / 2.0
    return pos0 + (seq_len + 1) / 2.0


__all__ = ["StackConfig", "LayerWeights", "random_layer", "rms_norm", "rope_tables", "apply_rope", "DecoderStack",
           "attention_ctx_per_token"]
