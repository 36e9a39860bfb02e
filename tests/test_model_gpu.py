"""Engine-level parity: the Qwen3 decoder with the sm_100a kernels (fused
pre-attention, varlen prefill, paged decode in the CUDA-graph DecodeGraph)
against the CPU fp32 restatement of the reference model
(leaninfer/qwen3/model.py) holding the same weights. A small depth and vocab
keep the oracle fast; the shapes per layer are Qwen3-0.6B's.

Tolerance: the model computes in bf16, the oracle in fp32. Run on the CPU,
the reference's own model differs between fp32 and bf16 by ~0.5 % relative L2
on these logits (max |diff| ~4 on logits up to ~1000, argmax identical), so
the bound is relative L2 <= 2 % and >= 90 % argmax agreement."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(got, want):
    rel = ((got - want).norm() / want.norm()).item()
    agree = (got.argmax(-1) == want.argmax(-1)).float().mean().item()
    return rel, agree


def _weights(model):
    """fp32 CPU copies of the GPU model's weights, split as the reference
    holds them (separate q/k/v and gate/up projections)."""
    cfg = model.config
    Hq, Hkv, D, I = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.intermediate_size
    w = {k: [] for k in ("wq", "wk", "wv", "wo", "qn", "kn", "wg", "wu", "wd", "ln1", "ln2")}
    for layer in model.layers:
        a = layer.self_attn
        qkv = a.qkv_proj.weight.float().cpu()
        w["wq"].append(qkv[: Hq * D])
        w["wk"].append(qkv[Hq * D:(Hq + Hkv) * D])
        w["wv"].append(qkv[(Hq + Hkv) * D:])
        w["wo"].append(a.o_proj.weight.float().cpu())
        w["qn"].append(a.q_norm.float().cpu())
        w["kn"].append(a.k_norm.float().cpu())
        gu = layer.mlp.gate_up_proj.weight.float().cpu()
        w["wg"].append(gu[:I])
        w["wu"].append(gu[I:])
        w["wd"].append(layer.mlp.down_proj.weight.float().cpu())
        w["ln1"].append(layer.input_layernorm.float().cpu())
        w["ln2"].append(layer.post_attention_layernorm.float().cpu())
    w["embed"] = model.embed_tokens.weight.float().cpu()
    w["norm"] = model.norm.float().cpu()
    return w


@pytest.mark.parametrize("NB,BS", [(24, 256), (64, 16)])
def test_prefill_then_graph_decode_matches_reference_model(pkg, cuda_dev, NB, BS):
    """256-token blocks (the engine's) and 16-token blocks (row f2: the
    kernels lift flash-attn's 256 minimum), same prompts and weights."""
    from lean_infer_b200 import qwen3
    from lean_infer_b200.cache import BlockAllocator, BlockCache
    from oracle.qwen3_step import CpuQwen3Decode

    cfg = qwen3.ModelConfig(num_hidden_layers=2, vocab_size=4096)
    model = qwen3.random_model(cfg, cuda_dev, seed=5)
    cache = BlockCache(cfg.num_hidden_layers, NB, BS, 8, 128, cuda_dev)
    ref = CpuQwen3Decode.from_weights(_weights(model), dict(layers=2, hidden=1024, heads=16, kv_heads=8,
                                                            head_dim=128, eps=1e-6, theta=1e6), NB, BS)
    g = torch.Generator().manual_seed(6)
    lens = [300, 57, 513]
    alloc = BlockAllocator(NB)
    tables = [alloc.allocate(-(-(L + 8) // BS)) for L in lens]
    max_blocks = max(len(t) for t in tables)
    bt = torch.zeros(len(lens), max_blocks, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, : len(t)] = torch.tensor(t)
    prompts = [torch.randint(0, cfg.vocab_size, (L,), generator=g) for L in lens]

    # prefill: packed on the GPU, one prompt at a time (B=1) on the oracle, as the engine does
    ids = torch.cat(prompts)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0)), dtype=torch.int32)
    model.rope(4096)
    pos0 = torch.zeros(len(lens), dtype=torch.long)
    logits = model(ids.to(cuda_dev), cache, bt.to(cuda_dev), pos0.to(cuda_dev), None, cu_seqlens=cu.to(cuda_dev),
                   max_seqlen=max(lens))
    for i, L in enumerate(lens):
        lr = ref.forward(prompts[i].view(1, L), pos0[i:i + 1], bt[i:i + 1], None)[0]
        lg = logits[int(cu[i]):int(cu[i + 1])].float().cpu()
        rel, agree = _close(lg, lr)
        assert rel <= 0.02 and agree >= 0.9, (i, rel, agree)
    # K/V written by prefill
    for layer in range(cfg.num_hidden_layers):
        for i, L in enumerate(lens):
            blk = bt[i, 0].item()
            n = min(L, BS)
            got, want = cache.k[layer, blk, :n].float().cpu(), ref.k_pools[layer, blk, :n]
            assert ((got - want).norm() / want.norm()).item() <= 0.02

    # 4 decode steps through the captured DecodeGraph
    dg = qwen3.DecodeGraph(model, cache, len(lens), max_blocks)
    nxt = torch.tensor([int(logits[int(cu[i + 1]) - 1].argmax()) for i in range(len(lens))])
    pos = torch.tensor(lens, dtype=torch.long)
    for _ in range(4):
        dg.stage(nxt.view(-1, 1), pos, bt, (pos + 1).to(torch.int32))
        toks = dg.step()
        lr = ref.forward(nxt.view(-1, 1), pos, bt, (pos + 1).to(torch.int32))[:, 0]
        lg = dg.logits[:, 0].float().cpu()
        rel, _ = _close(lg, lr)
        assert rel <= 0.02, rel
        assert (torch.tensor(toks) == lr.argmax(-1)).float().mean().item() >= 2 / 3
        nxt = lr.argmax(-1)  # follow the oracle's tokens so both stay on the same path
        pos = pos + 1
    pkg.check_device_errors(cuda_dev.index)
    dg.release()


def test_bucketed_decode_graph_masks_idle_rows(pkg, cuda_dev):
    """5 active rows replayed in the 8-row bucket: the same logits as a plain
    5-row decode graph, and the 3 masked rows write no cache slot (no trash
    block: block 0 and every unused block keep their bytes)."""
    from lean_infer_b200 import qwen3
    from lean_infer_b200.cache import BlockAllocator, BlockCache

    cfg = qwen3.ModelConfig(num_hidden_layers=2, vocab_size=4096)
    model = qwen3.random_model(cfg, cuda_dev, seed=9)
    NB, BS = 40, 256
    cache_a = BlockCache(cfg.num_hidden_layers, NB, BS, 8, 128, cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(10)
    cache_a.k.copy_(torch.randn(cache_a.k.shape, generator=g, device=cuda_dev).to(torch.bfloat16))
    cache_a.v.copy_(torch.randn(cache_a.v.shape, generator=g, device=cuda_dev).to(torch.bfloat16))
    cache_b = BlockCache(cfg.num_hidden_layers, NB, BS, 8, 128, cuda_dev)
    cache_b.k.copy_(cache_a.k)
    cache_b.v.copy_(cache_a.v)
    k0, v0 = cache_a.k.clone(), cache_a.v.clone()
    lens = [100, 300, 1000, 7, 520]
    alloc = BlockAllocator(NB)
    tables = [alloc.allocate(-(-(L + 2) // BS)) for L in lens]
    max_blocks = max(len(t) for t in tables)
    bt = torch.zeros(len(lens), max_blocks, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, : len(t)] = torch.tensor(t)
    used = sorted({b for t in tables for b in t})
    unused = [b for b in range(NB) if b not in used]
    ids = torch.randint(0, cfg.vocab_size, (len(lens), 1), generator=torch.Generator().manual_seed(11))
    pos = torch.tensor(lens, dtype=torch.long)
    ctx = (pos + 1).to(torch.int32)

    ref = qwen3.DecodeGraph(model, cache_b, len(lens), max_blocks)
    ref.stage(ids, pos, bt, ctx)
    toks_ref = ref.step()
    bg = qwen3.BucketedDecodeGraph(model, cache_a, [2, 8, 16], max_blocks)
    assert bg.stage(ids, pos, bt, ctx) == 8
    toks = bg.step()
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    la, lb = bg.logits()[:, 0].float(), ref.logits[:, 0].float()
    assert ((la - lb).norm() / lb.norm()).item() <= 1e-2
    assert sum(int(a == b) for a, b in zip(toks, toks_ref)) >= 4
    for blk in unused:  # block 0 included: idle rows wrote nothing
        assert torch.equal(cache_a.k[:, blk], k0[:, blk]) and torch.equal(cache_a.v[:, blk], v0[:, blk])
    # the active rows did write their slot
    assert not torch.equal(cache_a.k[:, bt[0, 0]], k0[:, bt[0, 0]])
    # a 2-row step uses the 2-row bucket
    assert bg.stage(ids[:2], pos[:2] + 1, bt[:2], ctx[:2] + 1) == 2
    assert len(bg.step()) == 2
    ref.release()
    bg.release()
