"""Host side of the paged K/V cache: the page allocator (no device work)."""

import pytest

from ultrametric.paged import PageAllocator


def test_allocator_assigns_pages_as_tokens_arrive():
    a = PageAllocator(num_pages=6, page_size=4)
    a.add(0)
    a.add(1)
    assert a.reserve(0, 5) == [0, 1]       # 5 tokens -> 2 pages
    assert a.reserve(1, 1) == [2]
    assert a.reserve(0, 3) == []           # 8 tokens fit in 2 pages
    assert a.reserve(0, 1) == [3]          # the 9th token opens a page
    assert a.pages[0] == [0, 1, 3] and a.length[0] == 9
    a.release(1)
    assert a.reserve(0, 4) == [2]          # freed page reused
    with pytest.raises(RuntimeError):
        a.reserve(0, 100)
    with pytest.raises(ValueError):
        a.add(0)
