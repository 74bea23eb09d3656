"""The KV page allocator (velo_page_allocator_*, no GPU): the reference's own
allocator tests re-expressed (src/paged_attention.rs:237-317), and random
allocate / release sequences that must hand out the same page ids and the
same errors as the oracle's restatement of PagedAttentionBlockManager."""
import numpy as np
import pytest

import velo_cuda
import vo


def test_allocates_pages_from_a_fixed_budget():
    a = velo_cuda.PageAllocator(16, 4)
    pages = a.allocate(1, 24)
    assert len(pages) == 2
    assert a.free_pages() == 2
    assert a.mapped_pages(1) is not None and len(a.mapped_pages(1)) == 2


def test_release_returns_pages_to_pool():
    a = velo_cuda.PageAllocator(8, 2)
    a.allocate(2, 8)
    a.release(2)
    assert a.free_pages() == 2


def test_rejects_oversized_allocations():
    a = velo_cuda.PageAllocator(32, 1)
    with pytest.raises(velo_cuda.OutOfPages) as e:
        a.allocate(3, 64)
    assert (e.value.requested, e.value.available) == (2, 1)
    assert a.free_pages() == 1  # nothing taken


def test_mapped_pages_miss_and_release_error():
    a = velo_cuda.PageAllocator(16, 32)
    assert a.mapped_pages(1) is None
    with pytest.raises(velo_cuda.VeloError) as e:
        a.release(1)
    assert e.value.status == velo_cuda.ERR_UNKNOWN_HANDLE


def test_invalid_block_size():
    with pytest.raises(velo_cuda.VeloError) as e:
        velo_cuda.PageAllocator(0, 4)
    assert e.value.status == velo_cuda.ERR_INVALID_BLOCK_SIZE


def test_fifo_order_and_reallocation_keeps_old_pages_out():
    a = velo_cuda.PageAllocator(16, 6)
    assert list(a.allocate(7, 33)) == [0, 1, 2]
    assert list(a.allocate(8, 16)) == [3]
    a.release(7)  # 0, 1, 2 go to the back: free list 4 5 0 1 2
    assert list(a.allocate(9, 48)) == [4, 5, 0]
    # a second allocation for handle 8 replaces its mapping; page 3 is not returned
    assert list(a.allocate(8, 1)) == [1]
    assert a.free_pages() == 1
    a.release(8)
    assert a.free_pages() == 2
    assert list(a.allocate(10, 32)) == [2, 1]
    assert list(a.allocate(11, 0)) == []  # zero tokens: zero pages, still mapped
    assert a.mapped_pages(11) is not None and len(a.mapped_pages(11)) == 0


def test_pages_for_tokens_does_not_overflow():
    a = velo_cuda.PageAllocator(16, 1)
    big = (1 << 64) - 1
    assert a.pages_for_tokens(big) == big // 16 + 1


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_sequences_match_oracle(seed):
    g = np.random.default_rng(seed)
    bs, total = int(g.choice([8, 16, 32])), int(g.integers(1, 64))
    mine, ref = velo_cuda.PageAllocator(bs, total), vo.Allocator(bs, total)
    for _ in range(400):
        h = int(g.integers(0, 12))
        if g.random() < 0.6:
            n = int(g.integers(0, bs * 12))
            try:
                want = list(ref.allocate(h, n))
            except vo.OutOfPages as e:
                with pytest.raises(velo_cuda.OutOfPages) as got:
                    mine.allocate(h, n)
                assert (got.value.requested, got.value.available) == (e.requested, e.available)
            else:
                assert list(mine.allocate(h, n)) == want
        else:
            try:
                ref.release(h)
            except KeyError:
                with pytest.raises(velo_cuda.VeloError) as got:
                    mine.release(h)
                assert got.value.status == velo_cuda.ERR_UNKNOWN_HANDLE
            else:
                mine.release(h)
        assert mine.free_pages() == ref.free_pages()
