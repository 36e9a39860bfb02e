"""Host-side logic of the decode step that runs without a GPU: the packed
staging layout DecodeGraph uploads in one copy."""
import pytest
import torch


@pytest.mark.parametrize("B,max_blocks", [(128, 4), (1, 1), (7, 33), (256, 128)])
def test_staging_views_layout(pkg, B, max_blocks):
    """ids, pos, ctx and the block table are disjoint, aligned views of one
    byte buffer covering it exactly, so a byte copy of the buffer moves all
    four (llm_engine.py:23-86 uploads them as four copies)."""
    from lean_infer_b200 import qwen3

    n = qwen3.staging_bytes(B, max_blocks)
    buf = torch.zeros(n, dtype=torch.uint8)
    ids, pos, ctx, bt = qwen3.staging_views(buf, B, max_blocks)
    assert (ids.shape, ids.dtype) == ((B, 1), torch.int64)
    assert (pos.shape, pos.dtype) == ((B,), torch.int64)
    assert (ctx.shape, ctx.dtype) == ((B,), torch.int32)
    assert (bt.shape, bt.dtype) == ((B, max_blocks), torch.int32)
    base = buf.data_ptr()
    spans = sorted((t.data_ptr() - base, t.data_ptr() - base + t.numel() * t.element_size()) for t in (ids, pos, ctx, bt))
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))  # back to back, no overlap
    for t in (ids, pos, ctx, bt):
        assert (t.data_ptr() - base) % t.element_size() == 0 and t.is_contiguous()

    # Writing through the views and copying the bytes carries every field.
    g = torch.Generator().manual_seed(B)
    want = (torch.randint(0, 151936, (B, 1), generator=g), torch.randint(-1, 4096, (B,), generator=g),
            torch.randint(0, 4096, (B,), generator=g, dtype=torch.int32),
            torch.randint(0, 512, (B, max_blocks), generator=g, dtype=torch.int32))
    for v, w in zip((ids, pos, ctx, bt), want):
        v.copy_(w)
    other = buf.clone()
    for v, w in zip(qwen3.staging_views(other, B, max_blocks), want):
        assert torch.equal(v, w)


def test_staging_views_rejects_wrong_size(pkg):
    from lean_infer_b200 import qwen3

    with pytest.raises(AssertionError):
        qwen3.staging_views(torch.zeros(qwen3.staging_bytes(4, 2) + 8, dtype=torch.uint8), 4, 2)


def test_block_allocator_fifo_and_trash_block(pkg):
    """The package's BlockAllocator against the reference's behaviour
    (cache_manager.py:13-42): ids 1..NB-1 in FIFO order, block 0 never handed
    out, released blocks appended at the tail, over-allocation refused with
    an AssertionError (the reference's assert) without taking any block."""
    from lean_infer_b200.cache import BlockAllocator, InsufficientBlocksError, blocks_for

    a = BlockAllocator(8)
    assert a.num_free == 7
    assert a.allocate(3) == [1, 2, 3]
    assert a.allocate(0) == []
    a.release([2, 1])
    assert a.allocate(4) == [4, 5, 6, 7]
    assert a.num_free == 2
    with pytest.raises(AssertionError):
        a.allocate(3)
    with pytest.raises(InsufficientBlocksError):
        a.allocate(3)
    assert a.num_free == 2
    assert a.allocate(2) == [2, 1]
    assert a.num_free == 0
    a.release([3])
    assert a.allocate(1) == [3]
    assert [blocks_for(n, 256) for n in (0, 1, 256, 257, 1024)] == [0, 1, 1, 2, 4]
