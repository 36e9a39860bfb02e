"""CPU fp32 restatement of the reference model's decode step — the CPU
baseline of the benchmark. Test and CPU-baseline infrastructure only.

Follows leaninfer/qwen3/model.py:25-112 op for op in fp32 on the host cores:
embedding, per layer input RMSNorm, q/k/v projections, q_norm/k_norm,
build_rope + apply_rope (layers.py:7-23), BlockCache.write
(cache_manager.py:63-76), paged decode attention (the flash_attn_with_kvcache
contract, computed as gather-by-block_table + one masked fp32 SDPA per layer),
o_proj, post-attention RMSNorm, SwiGLU MLP, final norm and the tied lm_head.

Weights are random (the benchmark runs on synthetic data). A bounded sample
can run `sample_layers` of the model's layers: decode_step() then reports the
time of the layer loop and of the embedding/head separately, and
full_step_seconds() scales the layer part to the full depth (every layer does
identical work). All sampled layers share one KV pool (the work per layer is
unchanged; the host memory footprint drops).
"""
from __future__ import annotations

import time

import torch
import torch.nn.functional as F

from . import paged_attention as opa
from . import pre_attention as opre


def seeded_weights(layers, hidden, heads, kv_heads, head_dim, inter, vocab, seed):
    """fp32 weights drawn in a fixed order from one seeded generator, in the
    dict form CpuQwen3Decode.from_weights takes. The golden-fixture script
    loads the same values into the reference's own Qwen3ForCausalLM
    (model.py:104-112), so the port and the reference run identical weights.
    Linear weights are N(0, 1/fan_in); norm weights 1 + N(0, 0.1^2)."""
    g = torch.Generator().manual_seed(seed)

    def lin(o, i):
        return torch.randn(o, i, generator=g) / i ** 0.5

    def norm(n):
        return 1.0 + 0.1 * torch.randn(n, generator=g)

    w = {"embed": torch.randn(vocab, hidden, generator=g), "norm": norm(hidden)}
    names = ("wq", "wk", "wv", "wo", "qn", "kn", "wg", "wu", "wd", "ln1", "ln2")
    for k in names:
        w[k] = []
    for _ in range(layers):
        w["wq"].append(lin(heads * head_dim, hidden))
        w["wk"].append(lin(kv_heads * head_dim, hidden))
        w["wv"].append(lin(kv_heads * head_dim, hidden))
        w["wo"].append(lin(hidden, heads * head_dim))
        w["qn"].append(norm(head_dim))
        w["kn"].append(norm(head_dim))
        w["wg"].append(lin(inter, hidden))
        w["wu"].append(lin(inter, hidden))
        w["wd"].append(lin(hidden, inter))
        w["ln1"].append(norm(hidden))
        w["ln2"].append(norm(hidden))
    return w


REFERENCE_NAMES = dict(wq="self_attn.q_proj", wk="self_attn.k_proj", wv="self_attn.v_proj",
                       wo="self_attn.o_proj", qn="self_attn.q_norm", kn="self_attn.k_norm", wg="mlp.gate_proj",
                       wu="mlp.up_proj", wd="mlp.down_proj", ln1="input_layernorm",
                       ln2="post_attention_layernorm")


def reference_state_dict(w: dict) -> dict:
    """The weights of seeded_weights() under the parameter names of the
    reference's Qwen3ForCausalLM (the checkpoint names at model.py:10-22)."""
    sd = {"model.embed_tokens.weight": w["embed"], "model.norm.weight": w["norm"]}
    for i in range(len(w["wq"])):
        for k, n in REFERENCE_NAMES.items():
            sd[f"model.layers.{i}.{n}.weight"] = w[k][i]
    return sd


class CpuQwen3Decode:
    def __init__(self, num_layers=28, hidden=1024, heads=16, kv_heads=8, head_dim=128, inter=3072, vocab=151936,
                 eps=1e-6, theta=1e6, num_blocks=512, block_size=256, seed=0, sample_layers=None):
        g = torch.Generator().manual_seed(seed)
        self.L, self.H, self.Hq, self.Hkv, self.D = num_layers, hidden, heads, kv_heads, head_dim
        self.eps, self.theta = eps, theta
        self.n_alloc = num_layers if sample_layers is None else min(sample_layers, num_layers)

        # Seeded noise, tiled from a 1 Mi-element block: seeding every element
        # of ~2 GB with the host RNG would take longer than the timed work.
        noise = torch.randn(1 << 20, generator=g)

        def fill(shape, scale):
            n = 1
            for d in shape:
                n *= d
            reps = -(-n // noise.numel())
            return (noise.repeat(reps)[:n] * scale).view(*shape)

        def lin(o, i):
            return fill((o, i), 1.0 / i ** 0.5)

        self.embed = fill((vocab, hidden), 1.0)
        self.layers = []
        for _ in range(self.n_alloc):
            self.layers.append(dict(
                wq=lin(heads * head_dim, hidden), wk=lin(kv_heads * head_dim, hidden),
                wv=lin(kv_heads * head_dim, hidden), wo=lin(hidden, heads * head_dim),
                qn=torch.ones(head_dim), kn=torch.ones(head_dim),
                wg=lin(inter, hidden), wu=lin(inter, hidden), wd=lin(hidden, inter),
                ln1=torch.ones(hidden), ln2=torch.ones(hidden)))
        self.norm = torch.ones(hidden)
        self.k_pool = fill((num_blocks, block_size, kv_heads, head_dim), 1.0)
        self.v_pool = fill((num_blocks, block_size, kv_heads, head_dim), 1.0).roll(7, dims=0)
        self.last_times = (0.0, 0.0)

    @classmethod
    def from_weights(cls, w: dict, cfg: dict, num_blocks: int, block_size: int):
        """Build the oracle model from explicit fp32 weights (the same values
        a GPU model holds) instead of random ones. `w` holds embed [V, H],
        norm [H] and per-layer lists wq, wk, wv, wo, qn, kn, wg, wu, wd, ln1,
        ln2; the KV pools start at zero and are written by decode_step /
        prefill. Every layer gets its own pool."""
        m = cls.__new__(cls)
        m.L, m.H, m.Hq, m.Hkv, m.D = cfg["layers"], cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
        m.eps, m.theta = cfg["eps"], cfg["theta"]
        m.n_alloc = m.L
        m.embed, m.norm = w["embed"], w["norm"]
        m.layers = [dict((k, w[k][i]) for k in ("wq", "wk", "wv", "wo", "qn", "kn", "wg", "wu", "wd", "ln1", "ln2"))
                    for i in range(m.L)]
        shape = (m.L, num_blocks, block_size, m.Hkv, m.D)
        m.k_pools, m.v_pools = torch.zeros(shape), torch.zeros(shape)
        m.k_pool = m.v_pool = None
        m.last_times = (0.0, 0.0)
        return m

    @torch.no_grad()
    def forward(self, ids, pos, block_table, cache_seqlens):
        """Reference forward (model.py:95-112) for B rows of q_len tokens
        starting at pos: writes the per-layer pools, returns fp32 logits
        [B, q_len, V]. Attention: causal SDPA over the fresh q/k/v when
        cache_seqlens is None (prefill, model.py:56-57), else paged decode over
        the pool (the flash_attn_with_kvcache contract, q_len = 1)."""
        B, n = ids.shape
        Hq, Hkv, D = self.Hq, self.Hkv, self.D
        h = self.embed[ids]
        cos, sin = opre.build_rope(pos, n, D, self.theta, h.dtype)  # model.py:98
        for i in range(self.L):
            w = self.layers[i]
            x = F.rms_norm(h, (self.H,), w["ln1"], self.eps)
            q = F.rms_norm((x @ w["wq"].T).view(B, n, Hq, D), (D,), w["qn"], self.eps).transpose(1, 2)
            k = F.rms_norm((x @ w["wk"].T).view(B, n, Hkv, D), (D,), w["kn"], self.eps).transpose(1, 2)
            v = (x @ w["wv"].T).view(B, n, Hkv, D).transpose(1, 2)
            q = opre.apply_rope(q, cos, sin)
            k = opre.apply_rope(k, cos, sin)
            opre.block_cache_write(self.k_pools[i], self.v_pools[i], block_table, pos, k, v)
            if cache_seqlens is None:
                o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True).transpose(1, 2)
            else:
                o = opa.paged_decode(q.transpose(1, 2), self.k_pools[i], self.v_pools[i], block_table,
                                     cache_seqlens)
            h = h + o.reshape(B, n, Hq * D) @ w["wo"].T
            x = F.rms_norm(h, (self.H,), w["ln2"], self.eps)
            h = h + (F.silu(x @ w["wg"].T) * (x @ w["wu"].T)) @ w["wd"].T
        h = F.rms_norm(h, (self.H,), self.norm, self.eps)
        return h @ self.embed.T

    def full_step_seconds(self) -> float:
        """Time of the last step scaled to all num_layers layers."""
        t_layers, t_rest = self.last_times
        return t_rest + t_layers * self.L / self.n_alloc

    @torch.no_grad()
    def decode_step(self, ids, pos, block_table, cache_seqlens):
        """ids [B, 1] int64, pos [B] int64, block_table [B, nb] int32,
        cache_seqlens [B] int32 -> logits [B, 1, vocab] (fp32). Runs the
        allocated layers (all of them unless sample_layers was given)."""
        B = ids.shape[0]
        Hq, Hkv, D = self.Hq, self.Hkv, self.D
        t0 = time.perf_counter()
        h = self.embed[ids]  # [B, 1, H]
        cos, sin = opre.build_rope(pos, 1, D, self.theta, torch.float32)
        t1 = time.perf_counter()
        kp, vp = self.k_pool, self.v_pool
        for i in range(self.n_alloc):
            w = self.layers[i]
            x = F.rms_norm(h, (self.H,), w["ln1"], self.eps)
            q = F.rms_norm((x @ w["wq"].T).view(B, 1, Hq, D), (D,), w["qn"], self.eps).transpose(1, 2)
            k = F.rms_norm((x @ w["wk"].T).view(B, 1, Hkv, D), (D,), w["kn"], self.eps).transpose(1, 2)
            v = (x @ w["wv"].T).view(B, 1, Hkv, D).transpose(1, 2)
            q = opre.apply_rope(q, cos, sin)
            k = opre.apply_rope(k, cos, sin)
            opre.block_cache_write(kp, vp, block_table, pos, k, v)
            o = opa.paged_decode_padded(q.transpose(1, 2), kp, vp, block_table, cache_seqlens)
            h = h + o.reshape(B, 1, Hq * D) @ w["wo"].T
            x = F.rms_norm(h, (self.H,), w["ln2"], self.eps)
            h = h + (F.silu(x @ w["wg"].T) * (x @ w["wu"].T)) @ w["wd"].T
        t2 = time.perf_counter()
        h = F.rms_norm(h, (self.H,), self.norm, self.eps)
        logits = h @ self.embed.T
        t3 = time.perf_counter()
        self.last_times = (t2 - t1, (t1 - t0) + (t3 - t2))
        return logits
