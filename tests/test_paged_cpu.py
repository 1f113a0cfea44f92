"""Host metadata of the paged KV cache against the reference's own unit tests
(src/inference/paged_attention.rs:535-730, restated case by case), plus the
copy-on-write page bookkeeping of PagedKv3Cache (no GPU needed)."""
import pytest

from ferrisres_b200.paged import (PAGE_POSITIONS, BlockAllocator, BlockTable,
                                  PagedAttentionManager, PagedKv3Cache, PrefixSharingManager,
                                  RequestState)
from ferrisres_b200._lib import OOMError


def test_block_allocator_basic():  # :535-549
    a = BlockAllocator(10, 16, 64)
    assert a.num_free() == 10
    b0 = a.allocate()
    assert b0 is not None and a.num_free() == 9
    assert a.allocate() is not None and a.num_free() == 8
    a.free(b0)
    assert a.num_free() == 9


def test_block_allocator_exhaustion():  # :551-560
    a = BlockAllocator(2, 16, 64)
    assert a.allocate() is not None and a.allocate() is not None
    assert a.allocate() is None


def test_block_allocator_ref_counting():  # :562-578
    a = BlockAllocator(4, 16, 64)
    b0 = a.allocate()
    assert a.ref_count(b0) == 1
    a.add_ref(b0)
    assert a.ref_count(b0) == 2
    a.free(b0)
    assert a.ref_count(b0) == 1 and a.num_free() == 3
    a.free(b0)
    assert a.ref_count(b0) == 0 and a.num_free() == 4


def test_block_table():  # :580-595
    t = BlockTable(16)
    assert t.num_blocks_needed() == 0
    t.append_block(0)
    t.append_block(1)
    t.add_tokens(25)
    assert t.num_blocks_needed() == 2 and t.num_tokens() == 25
    assert [t.block_for_position(p) for p in (0, 15, 16, 31)] == [0, 0, 1, 1]
    assert t.block_for_position(32) is None
    assert t.slot_in_block(5) == 5 and t.slot_in_block(16) == 0


def test_request_state():  # :597-604
    s = RequestState(42, 4, 16)
    assert s.request_id() == 42 and s.num_tokens() == 0 and s.num_layers() == 4
    assert s.layer_table(0).num_blocks_needed() == 0


def test_prefix_sharing():  # :606-630
    a = BlockAllocator(10, 16, 64)
    m = PrefixSharingManager(a, 16)
    m.register_prefix([1, 2, 3, 4], [[0], [1]])
    assert m.has_prefix([1, 2, 3, 4]) and not m.has_prefix([5, 6, 7])
    assert m.num_prefixes() == 1
    shared = m.lookup_prefix([1, 2, 3, 4])
    assert shared[0] == [0]
    assert a.ref_count(0) == 1 and a.ref_count(1) == 1
    assert m.lookup_prefix([9]) is None


def test_prefix_remove():  # :632-641
    m = PrefixSharingManager(BlockAllocator(10, 16, 64), 16)
    m.register_prefix([1, 2, 3], [[0]])
    m.remove_prefix([1, 2, 3])
    assert not m.has_prefix([1, 2, 3])


def test_paged_manager_create_and_free():  # :643-659
    m = PagedAttentionManager(4, 100, 16, 64)
    r = m.create_request_with_layers(32, 4)
    assert m.num_requests() == 1 and m.get_request(r).num_tokens() == 32
    assert m.num_free_blocks() == 92
    m.free_request(r)
    assert m.num_requests() == 0 and m.num_free_blocks() == 100


def test_paged_manager_fork():  # :661-680
    m = PagedAttentionManager(2, 100, 16, 64)
    p = m.create_request_with_layers(16, 2)
    assert m.num_free_blocks() == 98
    c = m.fork_request(p)
    assert m.num_requests() == 2 and m.num_free_blocks() == 98
    assert m.get_request(c).layer_table(1).table() == m.get_request(p).layer_table(1).table()
    m.free_request(p)
    assert m.num_free_blocks() == 98
    m.free_request(c)
    assert m.num_free_blocks() == 100
    assert m.fork_request(12345) is None


def test_utilization():  # :682-689
    m = PagedAttentionManager(2, 10, 16, 64)
    assert abs(m.utilization()) < 0.01
    m.create_request_with_layers(16, 2)
    assert abs(m.utilization() - 0.2) < 0.01


def test_memory_used_bytes_and_clear():  # :691-707
    a = BlockAllocator(10, 16, 64)
    assert a.memory_used_bytes() == 0
    a.allocate()
    assert a.memory_used_bytes() == 16 * 64 * 4 * 2
    t = BlockTable(16)
    t.append_block(0)
    t.add_tokens(10)
    t.clear()
    assert t.num_tokens() == 0 and t.num_blocks_allocated() == 0


def test_multiple_requests():  # :709-729
    m = PagedAttentionManager(2, 20, 16, 64)
    r1 = m.create_request_with_layers(16, 2)
    r2 = m.create_request_with_layers(32, 2)
    r3 = m.create_request_with_layers(8, 2)
    assert m.num_requests() == 3 and m.num_free_blocks() == 12
    m.free_request(r2)
    assert m.num_free_blocks() == 16
    m.free_request(r1)
    m.free_request(r3)
    assert m.num_free_blocks() == 20


def _host_only_cache(num_layers, num_pages):
    """PagedKv3Cache's bookkeeping without a device pool."""
    c = PagedKv3Cache.__new__(PagedKv3Cache)
    c.manager = PagedAttentionManager(num_layers, num_pages, PAGE_POSITIONS, 8 * 128)
    c.handle = None
    return c


def test_copy_on_write_bookkeeping():
    c = _host_only_cache(1, 8)
    a = c.manager.create_request(0)
    copies = []
    assert c._prepare(0, a, 40, copies) == 0 and not copies
    c._state(a).layer_table(0).add_tokens(40)
    assert len(c.block_table(a)) == 2
    b = c.fork_request(a)
    shared = c.block_table(a)
    assert c.block_table(b) == shared
    alloc = c.manager.allocator
    assert [alloc.ref_count(p) for p in shared] == [2, 2]
    # the child writes position 40: the partial page 1 is copied, page 0 stays shared
    assert c._prepare(0, b, 5, copies) == 40
    assert len(copies) == 1 and copies[0][0] == shared[1]
    tb = c.block_table(b)
    assert tb[0] == shared[0] and tb[1] == copies[0][1] != shared[1]
    assert alloc.ref_count(shared[0]) == 2 and alloc.ref_count(shared[1]) == 1
    # the parent now owns its partial page alone: no copy
    copies2 = []
    c._prepare(0, a, 30, copies2)
    assert not copies2 and c.block_table(a)[:2] == shared and len(c.block_table(a)) == 3
    # a full shared page is never copied: appends after a page boundary allocate
    d = c.manager.create_request(0)
    c._prepare(0, d, 32, [])
    c._state(d).layer_table(0).add_tokens(32)
    e = c.fork_request(d)
    cp = []
    c._prepare(0, e, 1, cp)
    assert not cp and c.block_table(e)[0] == c.block_table(d)[0]
    # exhaustion
    with pytest.raises(OOMError):
        c._prepare(0, e, 10 * PAGE_POSITIONS, [])
