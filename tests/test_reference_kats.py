"""The reference's own unit tests, ported one for one, run against both the
C++ host mirror (mitten_b200.host) and the oracle restatement
(oracle.host_ref).  These are the known-answer tests that pin page-id
behaviour:
  inference-engine/src/kv_pool.rs:104-161
  inference-engine/src/radix_cache.rs:305-424
"""
from __future__ import annotations

import uuid

import pytest

import oracle.host_ref as ref
from mitten_b200 import _lib, host

IMPLS = {
    "mirror": (host.KvCachePool, host.RadixCache),
    "oracle": (ref.KvCachePool, ref.RadixCache),
}
ERRORS = (_lib.MittenError, ref.RefError)


@pytest.fixture(params=sorted(IMPLS))
def impl(request):
    return IMPLS[request.param]


# ---------------------------------------------------------------- kv_pool.rs
def test_allocate_and_free(impl):  # kv_pool.rs:109-117
    pool = impl[0](16, 16)
    rid = uuid.uuid4()
    p1 = pool.allocate(rid)
    assert pool.free_pages() == 15
    pool.free(p1)
    assert pool.free_pages() == 16


def test_allocate_exhaustion(impl):  # kv_pool.rs:119-127
    pool = impl[0](2, 16)
    rid = uuid.uuid4()
    assert pool.allocate(rid) is not None
    assert pool.allocate(rid) is not None
    assert pool.allocate(rid) is None
    assert pool.free_pages() == 0


def test_required_bytes(impl):  # kv_pool.rs:129-136
    assert impl[0].required_bytes(1, 16, 1, 1, 1, 1) == 32
    assert impl[0].required_bytes(512, 16, 28, 4, 128, 2) == 2 * 512 * 16 * 28 * 4 * 128 * 2


def test_double_free_panics(impl):  # kv_pool.rs:138-150 (debug build)
    pool = impl[0](4, 16)
    rid = uuid.uuid4()
    p = pool.allocate(rid)
    pool.free(p)
    with pytest.raises(ERRORS):
        pool.free(p)
    assert pool.free_pages() == 4  # the failed free changed nothing


def test_lifo_order(impl):  # kv_pool.rs:19-20, 31, 46: stack initialised 0..n reversed
    pool = impl[0](8, 16)
    got = [pool.allocate(1) for _ in range(3)]
    assert got == [0, 1, 2]
    pool.free(1)
    assert pool.allocate(1) == 1
    assert pool.allocate(1) == 3


# ------------------------------------------------------------ radix_cache.rs
def test_empty_match(impl):  # radix_cache.rs:309-316
    cache = impl[1](4, 16)
    length, pages, nodes = cache.match_prefix([1, 2, 3])
    assert length == 0 and pages == [] and nodes == []


def test_insert_and_match_full(impl):  # radix_cache.rs:318-326
    cache = impl[1](4, 16)
    cache.insert_prefix([1, 2, 3, 4], [10])
    length, pages, nodes = cache.match_prefix([1, 2, 3, 4, 5])
    assert length == 4 and pages == [10] and len(nodes) == 1


def test_edge_split(impl):  # radix_cache.rs:328-344
    cache = impl[1](2, 16)
    cache.insert_prefix([1, 2, 3, 4], [10, 11])
    cache.insert_prefix([1, 2, 5, 6], [10, 12])
    l1, p1, _ = cache.match_prefix([1, 2, 3, 4])
    assert l1 == 4 and p1 == [10, 11]
    l2, p2, _ = cache.match_prefix([1, 2, 5, 6])
    assert l2 == 4 and p2 == [10, 12]


def test_lru_eviction(impl):  # radix_cache.rs:346-359
    cache = impl[1](2, 2)
    cache.insert_prefix([1, 2], [10])
    cache.insert_prefix([3, 4], [11])
    assert cache.total_cached_pages() == 2
    cache.insert_prefix([5, 6], [12])  # evicts [1, 2]
    assert cache.total_cached_pages() == 2
    length, _, _ = cache.match_prefix([1, 2])
    assert length == 0


def test_lock_prevents_eviction(impl):  # radix_cache.rs:361-378
    cache = impl[1](2, 1)
    cache.insert_prefix([1, 2], [10])
    _, _, nodes = cache.match_prefix([1, 2])
    cache.insert_prefix([3, 4], [11])
    assert cache.total_cached_pages() == 2  # overflowed: nothing evictable
    cache.unlock_nodes(nodes)
    freed = cache.evict_pages(1)
    assert len(freed) == 1


def test_insert_and_match_partial_edge(impl):  # radix_cache.rs:380-401
    cache = impl[1](4, 16)
    cache.insert_prefix([1, 2, 3, 4], [10])
    cache.insert_prefix([1, 2, 5, 6], [11])
    length, pages, _ = cache.match_prefix([1, 2, 3, 4])
    assert len(pages) == length // 4
    l2, p2, _ = cache.match_prefix([1, 2, 5, 6])
    assert len(p2) == l2 // 4


def test_promote_request(impl):  # radix_cache.rs:403-414
    cache = impl[1](8, 16)
    input_ids = list(range(1, 9))
    cache.promote_request(input_ids, 8, [42])
    length, pages, _ = cache.match_prefix(list(range(1, 9)))
    assert length == 8 and pages == [42]


def test_page_alignment(impl):  # radix_cache.rs:416-424
    cache = impl[1](4, 16)
    cache.insert_prefix([1, 2, 3, 4, 5, 6], [10])
    length, pages, _ = cache.match_prefix([1, 2, 3, 4, 5, 6])
    assert length == 4 and pages == [10]


def test_partial_edge_match_returns_zero_after_split(impl):
    # The comment at radix_cache.rs:392-396 states the expected value: a
    # 0-page [1,2] node stops the walk, so [1,2,3,4] matches nothing.
    cache = impl[1](4, 16)
    cache.insert_prefix([1, 2, 3, 4], [10])
    cache.insert_prefix([1, 2, 5, 6], [11])
    assert cache.match_prefix([1, 2, 3, 4])[0] == 0
