"""Qwen3 decoder with the reference's attention ops replaced by the sm_100a
kernels — the engine integration of the attention backend.

Same architecture and math as leaninfer/qwen3/model.py (Qwen3MLP :25-33,
Qwen3Attention :36-69, Qwen3DecoderLayer :72-83, Qwen3Model :87-101,
Qwen3ForCausalLM :104-112, lm_head tied to the embedding). Differences are
confined to how the work is launched:
  * q/k/v projections run as one GEMM on concatenated weights (and gate/up as
    one), the same products in bf16;
  * q_norm/k_norm + apply_rope + cache.write (model.py:50-55) are one launch
    of qk_norm_rope_paged_write, with rope from a position-indexed table
    instead of build_rope per forward (model.py:98);
  * decode attention (model.py:60-67) is flash_attn_with_kvcache from this
    package; prefill attention (model.py:56-57) is flash_attn_varlen_func;
  * each residual add and the RMSNorm after it are one launch
    (add_rms_norm), and SiLU(gate) * up is one launch (silu_mul);
  * the greedy next token, logits[:, -1].argmax(-1)
    (leaninfer/engine/llm_engine.py:86), is one launch (argmax_rows).
Weights are random-init bf16 (no checkpoint is loaded: the benchmark runs on
synthetic data).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

import ctypes

from . import _lib
from . import flash_attn_interface as fai
from .cache import BlockCache


def add_rms_norm(h: torch.Tensor, a: torch.Tensor | None, weight: torch.Tensor, eps: float,
                 inplace: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """(h + a, RMSNorm(h + a) * weight) for bf16 rows [T, n] in one launch
    (la_add_rms_norm); with a None: (h, RMSNorm(h) * weight). The sum is
    written into h when inplace."""
    T, n = h.shape
    x = torch.empty_like(h)
    h_out = (h if inplace else torch.empty_like(h)) if a is not None else None
    if T:
        _lib.call("la_add_rms_norm", ctypes.c_void_p(h.data_ptr()), h.stride(0),
                  ctypes.c_void_p(a.data_ptr() if a is not None else 0), a.stride(0) if a is not None else n,
                  ctypes.c_void_p(h_out.data_ptr() if h_out is not None else 0),
                  h_out.stride(0) if h_out is not None else n, ctypes.c_void_p(x.data_ptr()), x.stride(0),
                  ctypes.c_void_p(weight.data_ptr()), T, n, ctypes.c_float(eps),
                  ctypes.c_void_p(torch.cuda.current_stream(h.device).cuda_stream))
    return (h_out if h_out is not None else h), x


def silu_mul(gate_up: torch.Tensor, n: int) -> torch.Tensor:
    """SiLU(gate_up[:, :n]) * gate_up[:, n:] in one launch (la_silu_mul)."""
    T = gate_up.shape[0]
    out = torch.empty(T, n, dtype=gate_up.dtype, device=gate_up.device)
    if T:
        _lib.call("la_silu_mul", ctypes.c_void_p(gate_up.data_ptr()), gate_up.stride(0),
                  ctypes.c_void_p(out.data_ptr()), out.stride(0), T, n,
                  ctypes.c_void_p(torch.cuda.current_stream(gate_up.device).cuda_stream))
    return out


def argmax_rows(x: torch.Tensor) -> torch.Tensor:
    """x.argmax(-1) for a bf16 matrix [rows, cols] with unit column stride, in
    one launch (la_argmax_rows): int64 [rows], the first index of each row's
    maximum, NaN above every number — torch.argmax's rules."""
    assert x.dim() == 2 and x.dtype == torch.bfloat16 and x.stride(1) == 1
    out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    if x.shape[0]:
        _lib.call("la_argmax_rows", ctypes.c_void_p(x.data_ptr()), x.stride(0), x.shape[0], x.shape[1],
                  ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    return out


@dataclass(frozen=True)
class ModelConfig:
    """Field-for-field leaninfer.qwen3.model_config.ModelConfig
    (model_config.py:20-31); defaults are Qwen3-0.6B."""
    num_hidden_layers: int = 28
    hidden_size: int = 1024
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6


class Qwen3Attention(nn.Module):
    def __init__(self, cfg: ModelConfig, head_offset: int = 0, num_kv_heads: int | None = None) -> None:
        super().__init__()
        self.cfg = cfg
        self.hkv = cfg.num_key_value_heads if num_kv_heads is None else num_kv_heads
        self.hq = self.hkv * (cfg.num_attention_heads // cfg.num_key_value_heads)
        D = cfg.head_dim
        self.qkv_proj = nn.Linear(cfg.hidden_size, (self.hq + 2 * self.hkv) * D, bias=False)
        self.q_norm = nn.Parameter(torch.ones(D))
        self.k_norm = nn.Parameter(torch.ones(D))
        self.o_proj = nn.Linear(cfg.num_attention_heads * D, cfg.hidden_size, bias=False)

    def attend(self, x: torch.Tensor, cache: BlockCache, layer: int, block_tables: torch.Tensor, pos: torch.Tensor,
               cache_seqlens: torch.Tensor | None, rope, cu_seqlens: torch.Tensor | None = None,
               max_seqlen: int = 0) -> torch.Tensor:
        """Attention output [T, hq*D] before o_proj. x: [T, hidden]."""
        T = x.shape[0]
        D = self.cfg.head_dim
        qkv = self.qkv_proj(x)
        q = qkv[:, : self.hq * D].view(T, self.hq, D)
        k = qkv[:, self.hq * D: (self.hq + self.hkv) * D].view(T, self.hkv, D)
        v = qkv[:, (self.hq + self.hkv) * D:].view(T, self.hkv, D)
        kc, vc = cache.k[layer], cache.v[layer]
        if cache_seqlens is not None:  # decode: one token per sequence
            q = fai.qk_norm_rope_paged_write(q, k, v, self.q_norm, self.k_norm, rope[0], rope[1], pos, block_tables,
                                             kc, vc, eps=self.cfg.rms_norm_eps)
            o = fai.flash_attn_with_kvcache(q.view(T, 1, self.hq, D), kc, vc, cache_seqlens=cache_seqlens,
                                            block_table=block_tables, causal=True, num_splits=1)
        else:  # prefill of packed prompts starting at pos
            k_out = torch.empty_like(k)
            q = fai.qk_norm_rope_paged_write(q, k, v, self.q_norm, self.k_norm, rope[0], rope[1], pos, block_tables,
                                             kc, vc, eps=self.cfg.rms_norm_eps, cu_seqlens=cu_seqlens, k_out=k_out)
            o = fai.flash_attn_varlen_func(q, k_out, v, cu_seqlens, cu_seqlens, max_seqlen, max_seqlen, causal=True)
        return o.reshape(T, self.hq * D)

    def forward(self, x, cache, layer, block_tables, pos, cache_seqlens, rope, cu_seqlens=None, max_seqlen=0):
        return self.o_proj(self.attend(x, cache, layer, block_tables, pos, cache_seqlens, rope, cu_seqlens,
                                       max_seqlen))


class Qwen3MLP(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.gate_up_proj = nn.Linear(cfg.hidden_size, 2 * cfg.intermediate_size, bias=False)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)
        self.inter = cfg.intermediate_size

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(silu_mul(self.gate_up_proj(x), self.inter))


class Qwen3DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.self_attn = Qwen3Attention(cfg)
        self.mlp = Qwen3MLP(cfg)
        self.input_layernorm = nn.Parameter(torch.ones(cfg.hidden_size))
        self.post_attention_layernorm = nn.Parameter(torch.ones(cfg.hidden_size))
        self.eps = cfg.rms_norm_eps

    def forward(self, h, x, next_norm, cache, layer, block_tables, pos, cache_seqlens, rope, cu_seqlens=None,
                max_seqlen=0):
        """h: residual stream [T, hidden]; x = RMSNorm(h) * input_layernorm
        (produced by the previous layer's last fused add). Returns the new h
        and RMSNorm(h) * next_norm (the next layer's input norm, or the
        model's final norm)."""
        a = self.self_attn(x, cache, layer, block_tables, pos, cache_seqlens, rope, cu_seqlens, max_seqlen)
        h, x = add_rms_norm(h, a, self.post_attention_layernorm, self.eps)
        return add_rms_norm(h, self.mlp(x), next_norm, self.eps)


class Qwen3ForCausalLM(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.config = cfg
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(Qwen3DecoderLayer(cfg) for _ in range(cfg.num_hidden_layers))
        self.norm = nn.Parameter(torch.ones(cfg.hidden_size))
        self.max_pos = 0
        self._rope = None

    def rope(self, max_pos: int):
        dev = self.embed_tokens.weight.device
        if self._rope is None or self.max_pos < max_pos:
            self.max_pos = max(max_pos, 4096)
            self._rope = fai.rope_tables(self.max_pos, self.config.head_dim, self.config.rope_theta, dev)
        return self._rope

    def forward(self, input_ids: torch.Tensor, cache: BlockCache, block_tables: torch.Tensor, pos: torch.Tensor,
                cache_seqlens: torch.Tensor | None, cu_seqlens: torch.Tensor | None = None,
                max_seqlen: int = 0) -> torch.Tensor:
        """Decode: input_ids [B, 1], cache_seqlens [B] -> logits [B, 1, vocab].
        Prefill: input_ids [T] packed, cu_seqlens [S+1] -> logits [T, vocab].
        The rope table must already cover every position (call rope() before
        capturing a graph)."""
        ids = input_ids.reshape(-1)
        h = self.embed_tokens(ids)
        rope = self._rope if self._rope is not None else self.rope(4096)
        eps = self.config.rms_norm_eps
        _, x = add_rms_norm(h, None, self.layers[0].input_layernorm, eps)
        for i, layer in enumerate(self.layers):
            nxt = self.layers[i + 1].input_layernorm if i + 1 < len(self.layers) else self.norm
            h, x = layer(h, x, nxt, cache, i, block_tables, pos, cache_seqlens, rope, cu_seqlens, max_seqlen)
        logits = F.linear(x, self.embed_tokens.weight)  # x = final RMSNorm(h) * norm
        return logits.view(input_ids.shape[0], -1, logits.shape[-1]) if cache_seqlens is not None else logits


def random_model(cfg: ModelConfig, device, seed: int = 0, dtype=torch.bfloat16) -> Qwen3ForCausalLM:
    """Random-init weights (nn defaults; norm weights near 1) in `dtype`."""
    torch.manual_seed(seed)
    with torch.device(device):
        m = Qwen3ForCausalLM(cfg)
    with torch.no_grad():
        g = torch.Generator(device=device).manual_seed(seed)
        for layer in m.layers:
            layer.self_attn.q_norm.copy_(1 + 0.1 * torch.randn(cfg.head_dim, generator=g, device=device))
            layer.self_attn.k_norm.copy_(1 + 0.1 * torch.randn(cfg.head_dim, generator=g, device=device))
    # inference only: no autograd bookkeeping in eager calls or graph captures
    return m.to(dtype).eval().requires_grad_(False)


def staging_views(buf: torch.Tensor, n_slots: int, max_blocks: int):
    """(ids [B, 1] i64, pos [B] i64, ctx [B] i32, bt [B, max_blocks] i32) as
    views of one uint8 buffer of staging_bytes(B, max_blocks) bytes, laid out
    ids | pos | ctx | bt, so that the four inputs move in a single copy."""
    B = n_slots
    o_pos, o_ctx, o_bt = 8 * B, 16 * B, 20 * B
    assert buf.dtype == torch.uint8 and buf.numel() == staging_bytes(B, max_blocks)
    return (buf[:o_pos].view(torch.long).view(B, 1), buf[o_pos:o_ctx].view(torch.long),
            buf[o_ctx:o_bt].view(torch.int32), buf[o_bt:].view(torch.int32).view(B, max_blocks))


def staging_bytes(n_slots: int, max_blocks: int) -> int:
    return 20 * n_slots + 4 * n_slots * max_blocks


class DecodeGraph:
    """Fixed-B decode step captured in a CUDA graph — the engine's DecodeGraph
    (leaninfer/engine/llm_engine.py:23-86): pinned host staging buffers,
    static device buffers ids [B,1] i64, pos [B] i64, bt [B, max_blocks] i32,
    ctx [B] i32; three warm-up forwards on a side stream, then capture. Idle
    rows get pos 0, ctx 1 and block 0 (the trash block). The four host
    buffers are views of one pinned allocation and the four device buffers
    views of one device allocation with the same layout, so a step's inputs
    go up in a single copy."""

    def __init__(self, model: Qwen3ForCausalLM, cache: BlockCache, n_slots: int, max_blocks: int) -> None:
        self.model, self.cache = model, cache
        dev = cache.device
        nbytes = staging_bytes(n_slots, max_blocks)
        self._host_buf = torch.zeros(nbytes, dtype=torch.uint8, pin_memory=True)
        self._dev_buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self.host_ids, self.host_pos, self.host_ctx, self.host_bt = staging_views(self._host_buf, n_slots, max_blocks)
        self.ids, self.pos, self.ctx, self.bt = staging_views(self._dev_buf, n_slots, max_blocks)
        self.host_ctx.fill_(1)
        self.ctx.fill_(1)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.logits: torch.Tensor | None = None
        self.next_tokens: torch.Tensor | None = None
        model.rope(max_blocks * cache.block_size)

    @property
    def h2d_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.host_ids, self.host_pos, self.host_bt, self.host_ctx))

    def _forward(self):
        logits = self.model(self.ids, self.cache, self.bt, self.pos, self.ctx)
        return logits, argmax_rows(logits[:, -1])

    def capture(self) -> None:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                self._forward()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits, self.next_tokens = self._forward()

    def stage(self, ids, pos, bt, ctx) -> None:
        """Fill the pinned host buffers (numpy-style views, as the engine does)."""
        self.host_ids.copy_(ids)
        self.host_pos.copy_(pos)
        self.host_bt.zero_()
        self.host_bt[:, : bt.shape[1]].copy_(bt)
        self.host_ctx.copy_(ctx)

    def upload(self) -> None:
        self._dev_buf.copy_(self._host_buf, non_blocking=True)  # ids, pos, ctx, bt in one copy

    def replay(self) -> None:
        if self.graph is None:
            self.capture()
        self.graph.replay()

    def step(self) -> list[int]:
        """H2D copy of the staged inputs, graph replay, D2H of the next tokens
        (llm_engine.py:65-86)."""
        self.upload()
        self.replay()
        return self.next_tokens.tolist()

    def release(self) -> None:
        self.graph = None


class BucketedDecodeGraph:
    """Decode steps captured for several batch sizes over one set of static
    buffers. The reference captures a single graph at B = n_slots and points
    idle rows at the trash block 0 with position 0 and context 1
    (llm_engine.py:23-86); here a step replays the smallest captured bucket
    that holds the active rows, and the idle rows inside that bucket are
    masked — start position -1 and context 0 — so they write no cache slot
    (la_qk_norm_rope_paged_write skips them) and attend to nothing
    (la_paged_decode returns zeros): no trash block is needed and a small
    batch does not pay for n_slots rows."""

    def __init__(self, model: Qwen3ForCausalLM, cache: BlockCache, buckets, max_blocks: int) -> None:
        self.model, self.cache = model, cache
        self.buckets = sorted({int(b) for b in buckets})
        if not self.buckets or self.buckets[0] <= 0:
            raise ValueError("buckets must be positive batch sizes")
        n = self.buckets[-1]
        dev = cache.device
        self.host_ids = torch.zeros(n, 1, dtype=torch.long, pin_memory=True)
        self.host_pos = torch.full((n,), -1, dtype=torch.long, pin_memory=True)
        self.host_bt = torch.zeros(n, max_blocks, dtype=torch.int32, pin_memory=True)
        self.host_ctx = torch.zeros(n, dtype=torch.int32, pin_memory=True)
        self.ids = torch.zeros(n, 1, dtype=torch.long, device=dev)
        self.pos = torch.full((n,), -1, dtype=torch.long, device=dev)
        self.bt = torch.zeros(n, max_blocks, dtype=torch.int32, device=dev)
        self.ctx = torch.zeros(n, dtype=torch.int32, device=dev)
        self.graphs: dict[int, tuple] = {}
        self.bucket = n
        self.active = 0
        model.rope(max_blocks * cache.block_size)

    def bucket_for(self, rows: int) -> int:
        for b in self.buckets:
            if b >= rows:
                return b
        raise ValueError(f"{rows} active rows exceed the largest bucket {self.buckets[-1]}")

    def h2d_bytes(self, bucket: int) -> int:
        return bucket * (8 + 8 + 4 + self.host_bt.shape[1] * 4)

    def _forward(self, b: int):
        logits = self.model(self.ids[:b], self.cache, self.bt[:b], self.pos[:b], self.ctx[:b])
        return logits, argmax_rows(logits[:, -1])

    def capture(self) -> None:
        """Three warm-up forwards per bucket on a side stream, then one graph
        per bucket (all rows idle while capturing: nothing is written)."""
        self.pos.fill_(-1)
        self.ctx.zero_()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for b in self.buckets:
                for _ in range(3):
                    self._forward(b)
        torch.cuda.current_stream().wait_stream(side)
        for b in self.buckets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                logits, nxt = self._forward(b)
            self.graphs[b] = (g, logits, nxt)

    def stage(self, ids, pos, bt, ctx) -> int:
        """Stage the active rows (the first len(ids) rows) and mask the rest
        of the chosen bucket; returns the bucket."""
        n = int(ids.shape[0])
        b = self.bucket_for(n)
        self.host_ids[:n].copy_(ids.view(n, 1))
        self.host_ids[n:b].zero_()
        self.host_pos[:n].copy_(pos)
        self.host_pos[n:b].fill_(-1)
        self.host_bt[:b].zero_()
        self.host_bt[:n, : bt.shape[1]].copy_(bt)
        self.host_ctx[:n].copy_(ctx)
        self.host_ctx[n:b].zero_()
        self.active, self.bucket = n, b
        return b

    def step(self) -> list[int]:
        """H2D copy of the bucket's staged rows, replay of its graph, D2H of
        the active rows' next tokens."""
        b = self.bucket
        if not self.graphs:
            self.capture()
        self.ids[:b].copy_(self.host_ids[:b], non_blocking=True)
        self.pos[:b].copy_(self.host_pos[:b], non_blocking=True)
        self.bt[:b].copy_(self.host_bt[:b], non_blocking=True)
        self.ctx[:b].copy_(self.host_ctx[:b], non_blocking=True)
        g, _, nxt = self.graphs[b]
        g.replay()
        return nxt[: self.active].tolist()

    def logits(self) -> torch.Tensor:
        """Logits of the last step's active rows [n, 1, vocab]."""
        return self.graphs[self.bucket][1][: self.active]

    def release(self) -> None:
        self.graphs = {}
