"""Generate golden fixtures by running the reference's own code on the CPU.

Usage: python tests/golden/make_golden.py /path/to/lean-infer-checkout

Imports leaninfer.qwen3.model / layers / model_config and
leaninfer.engine.cache_manager / engine_config from the reference checkout
(read-only) and runs Qwen3Attention.forward on seeded inputs, capturing the
tensors at the boundaries the kernels replace:

  pre_attention_decode.npz   bf16 decode step, B=4 rows at positions that cross
                             block boundaries: raw q/k/v projections, q_norm /
                             k_norm weights, positions, block table -> post-rope
                             q and k (the inputs of the attention call) and the
                             KV pool after BlockCache.write. The flash-attn call
                             (CUDA only) is replaced by a capturing stub.
  pre_attention_prefill.npz  the same for a bf16 prefill (B=1, pos=0, q_len=37).
  attention_prefill.npz      fp32 prefill, B=1, L=80: the q/k/v handed to
                             F.scaled_dot_product_attention(is_causal=True,
                             enable_gqa=True) and its output (model.py:56-57).
  rope.npz                   build_rope(...) cos/sin in bf16 at positions up to
                             40000 (layers.py:7-15).
  model_step.npz             the whole Qwen3ForCausalLM (model.py:87-112) in
                             fp32, 2 layers of Qwen3-0.6B shapes (vocab cut to
                             2048), weights from oracle.qwen3_step.seeded_weights:
                             two prompts prefilled one at a time through its
                             SDPA path, then one decode step of both rows with
                             its flash-attn call (CUDA only) answered by the
                             oracle's paged decode. Saved: prefill logits of
                             each prompt's last 3 tokens, the decode logits, and
                             K/V pool rows of both layers at sampled positions.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if len(sys.argv) < 2:
    sys.exit("usage: make_golden.py /path/to/lean-infer-checkout")
REF = Path(sys.argv[1])
sys.path.insert(0, str(REF))
sys.path.insert(0, str(HERE.parent.parent))  # the oracle package (seeded weights, paged decode)

from leaninfer.engine import cache_manager, engine_config  # noqa: E402
from leaninfer.qwen3 import layers, model  # noqa: E402
from leaninfer.qwen3.model_config import ModelConfig  # noqa: E402

CFG = ModelConfig(num_hidden_layers=1, hidden_size=1024, num_attention_heads=16, num_key_value_heads=8,
                  head_dim=128, intermediate_size=3072, vocab_size=151936, rms_norm_eps=1e-6, rope_theta=1e6)


def bf16_to_u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


class Capture:
    """Wraps the attention call and BlockCache.write of a Qwen3Attention run."""

    def __init__(self):
        self.items = {}

    def sdpa(self, orig):
        def f(q, k, v, **kw):
            o = orig(q, k, v, **kw)
            self.items.update(sdpa_q=q.detach().clone(), sdpa_k=k.detach().clone(), sdpa_v=v.detach().clone(),
                              sdpa_o=o.detach().clone())
            return o
        return f

    def fa(self, q, k_cache, v_cache, cache_seqlens=None, block_table=None, **kw):
        self.items.update(fa_q=q.detach().clone(), fa_seqlens=cache_seqlens.clone(), fa_bt=block_table.clone())
        return torch.zeros_like(q)

    def write(self, orig):
        def f(layer, block_tables, pos, k, v):
            self.items.update(write_k=k.detach().clone(), write_v=v.detach().clone())
            return orig(layer, block_tables, pos, k, v)
        return f


def run_attention(dtype, B, q_len, pos, block_tables, num_blocks, block_size, seed, decode):
    torch.manual_seed(seed)
    attn = model.Qwen3Attention(CFG).to(dtype)
    with torch.no_grad():
        attn.q_norm.weight.copy_((1.0 + 0.3 * torch.randn(128)).to(dtype))
        attn.k_norm.weight.copy_((1.0 + 0.3 * torch.randn(128)).to(dtype))
    ecfg = engine_config.EngineConfig(num_blocks=num_blocks, block_size=block_size, device=torch.device("cpu"),
                                      dtype=dtype)
    cache = cache_manager.BlockCache(CFG, ecfg)  # zero-filled pools, as the engine allocates them
    x = (torch.randn(B, q_len, CFG.hidden_size) * 0.5).to(dtype)
    cap = Capture()
    hooks = []
    raw = {}
    hooks.append(attn.q_proj.register_forward_hook(lambda m, i, o: raw.__setitem__("q", o.detach().clone())))
    hooks.append(attn.k_proj.register_forward_hook(lambda m, i, o: raw.__setitem__("k", o.detach().clone())))
    hooks.append(attn.v_proj.register_forward_hook(lambda m, i, o: raw.__setitem__("v", o.detach().clone())))
    orig_sdpa = model.F.scaled_dot_product_attention
    orig_fa = model.flash_attn_with_kvcache
    cache.write = cap.write(cache.write)
    try:
        model.F.scaled_dot_product_attention = cap.sdpa(orig_sdpa)
        model.flash_attn_with_kvcache = cap.fa
        cos, sin = layers.build_rope(CFG, pos, q_len, dtype)
        seqlens = (pos + q_len).to(torch.int32) if decode else None
        with torch.no_grad():
            attn(x, cos, sin, cache, 0, block_tables, pos, seqlens)
    finally:
        model.F.scaled_dot_product_attention = orig_sdpa
        model.flash_attn_with_kvcache = orig_fa
        for h in hooks:
            h.remove()
    return attn, cache, raw, cap.items


def pre_attention_fixture(name, B, q_len, pos, num_blocks, block_size, seed, decode):
    g = torch.Generator().manual_seed(seed + 1)
    alloc = cache_manager.BlockAllocator(num_blocks)
    perm = torch.randperm(num_blocks - 1, generator=g).tolist()
    alloc.free = type(alloc.free)([p + 1 for p in perm])
    max_blocks = int(((pos + q_len).max() + block_size - 1) // block_size)
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    for b in range(B):
        need = int((pos[b] + q_len + block_size - 1) // block_size)
        bt[b, :need] = torch.tensor(alloc.allocate(need), dtype=torch.int32)
    attn, cache, raw, items = run_attention(torch.bfloat16, B, q_len, pos, bt, num_blocks, block_size, seed,
                                                    decode)
    out = dict(
        q_raw=bf16_to_u16(raw["q"].view(B * q_len, 16, 128)),
        k_raw=bf16_to_u16(raw["k"].view(B * q_len, 8, 128)),
        v_raw=bf16_to_u16(raw["v"].view(B * q_len, 8, 128)),
        q_norm_w=bf16_to_u16(attn.q_norm.weight.detach()),
        k_norm_w=bf16_to_u16(attn.k_norm.weight.detach()),
        pos=pos.numpy(), q_len=np.int64(q_len), block_table=bt.numpy(), block_size=np.int64(block_size),
        # post-rope q/k as [tokens, heads, D]
        k_rope=bf16_to_u16(items["write_k"].transpose(1, 2).reshape(B * q_len, 8, 128)),
        pool_k_after=bf16_to_u16(cache.k[0]), pool_v_after=bf16_to_u16(cache.v[0]),
    )
    if decode:
        out["q_rope"] = bf16_to_u16(items["fa_q"].reshape(B * q_len, 16, 128))
    else:
        out["q_rope"] = bf16_to_u16(items["sdpa_q"].transpose(1, 2).reshape(B * q_len, 16, 128))
    np.savez_compressed(HERE / name, **out)
    print(name, {k: v.shape for k, v in out.items()})


def attention_fixture(name, L, seed):
    bt = torch.tensor([[1]], dtype=torch.int32)
    pos = torch.zeros(1, dtype=torch.long)
    attn, cache, raw, items = run_attention(torch.float32, 1, L, pos, bt, 2, 256, seed, decode=False)
    out = dict(q=items["sdpa_q"][0].numpy(), k=items["sdpa_k"][0].numpy(), v=items["sdpa_v"][0].numpy(),
               o=items["sdpa_o"][0].numpy())
    np.savez_compressed(HERE / name, **out)
    print(name, {k: v.shape for k, v in out.items()})


def rope_fixture(name):
    pos = torch.tensor([0, 1, 255, 256, 767, 1023, 4095, 8191, 16384, 32767, 40000], dtype=torch.long)
    cos, sin = layers.build_rope(CFG, pos, 1, torch.bfloat16)
    np.savez_compressed(HERE / name, pos=pos.numpy(), cos=bf16_to_u16(cos[:, 0, 0]), sin=bf16_to_u16(sin[:, 0, 0]))
    print(name, cos.shape)


MODEL_CFG = dict(layers=2, hidden=1024, heads=16, kv_heads=8, head_dim=128, inter=3072, vocab=2048, eps=1e-6,
                 theta=1e6, seed=21, num_blocks=8, block_size=256, prompts=(300, 77))


def model_fixture(name):
    from oracle import paged_attention as opa
    from oracle.qwen3_step import reference_state_dict, seeded_weights

    c = MODEL_CFG
    cfg = ModelConfig(num_hidden_layers=c["layers"], hidden_size=c["hidden"], num_attention_heads=c["heads"],
                      num_key_value_heads=c["kv_heads"], head_dim=c["head_dim"], intermediate_size=c["inter"],
                      vocab_size=c["vocab"], rms_norm_eps=c["eps"], rope_theta=c["theta"])
    w = seeded_weights(c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["inter"], c["vocab"],
                       c["seed"])
    m = model.Qwen3ForCausalLM(cfg).float()
    m.load_state_dict(reference_state_dict(w), strict=True)
    ecfg = engine_config.EngineConfig(num_blocks=c["num_blocks"], block_size=c["block_size"],
                                      device=torch.device("cpu"), dtype=torch.float32)
    cache = cache_manager.BlockCache(cfg, ecfg)
    alloc = cache_manager.BlockAllocator(c["num_blocks"])
    g = torch.Generator().manual_seed(c["seed"] + 1)
    lens = list(c["prompts"])
    tables = [alloc.allocate(-(-(L + 1) // c["block_size"])) for L in lens]
    bt = torch.zeros(len(lens), max(len(t) for t in tables), dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    prompts = [torch.randint(0, c["vocab"], (L,), generator=g) for L in lens]
    out = {"block_table": bt.numpy(), "lens": np.array(lens)}
    for i, p in enumerate(prompts):
        out[f"prompt{i}"] = p.numpy()
    orig_fa = model.flash_attn_with_kvcache

    def fa_stub(q, k_cache, v_cache, cache_seqlens=None, block_table=None, **kw):
        return opa.paged_decode(q, k_cache, v_cache, block_table, cache_seqlens).to(q.dtype)

    try:
        model.flash_attn_with_kvcache = fa_stub
        with torch.no_grad():
            nxt = []
            for i, p in enumerate(prompts):  # the engine prefills one prompt per step (B=1)
                lg = m(p.view(1, -1), cache, bt[i:i + 1], torch.zeros(1, dtype=torch.long), None)[0]
                out[f"prefill_logits{i}"] = lg[-3:].numpy()
                nxt.append(int(lg[-1].argmax()))
            ids = torch.tensor(nxt).view(-1, 1)
            pos = torch.tensor(lens, dtype=torch.long)
            lg = m(ids, cache, bt, pos, (pos + 1).to(torch.int32))
            out["decode_ids"] = ids.numpy()
            out["decode_logits"] = lg[:, 0].numpy()
    finally:
        model.flash_attn_with_kvcache = orig_fa
    # pool rows (both layers, K and V) at sampled positions of each sequence
    sample = []
    for i, L in enumerate(lens):
        for t in (0, L // 2, L - 1, L):  # L: the token the decode step wrote
            sample.append((i, t))
    out["pool_positions"] = np.array(sample)
    ks, vs = [], []
    for i, t in sample:
        blk, off = int(bt[i, t // c["block_size"]]), t % c["block_size"]
        ks.append(cache.k[:, blk, off].numpy())
        vs.append(cache.v[:, blk, off].numpy())
    out["pool_k"] = np.stack(ks)
    out["pool_v"] = np.stack(vs)
    np.savez_compressed(HERE / name, **out)
    print(name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    pre_attention_fixture("pre_attention_decode.npz", B=4, q_len=1,
                          pos=torch.tensor([0, 255, 256, 700], dtype=torch.long), num_blocks=8, block_size=256,
                          seed=11, decode=True)
    pre_attention_fixture("pre_attention_prefill.npz", B=1, q_len=37, pos=torch.tensor([0], dtype=torch.long),
                          num_blocks=4, block_size=16, seed=12, decode=False)
    attention_fixture("attention_prefill.npz", L=80, seed=13)
    rope_fixture("rope.npz")
    model_fixture("model_step.npz")
