"""The allocation-free flatten_sort_count entry point, called through the C ABI.

Callers that cannot allocate device memory where they route tokens (runtimes
with a fixed memory pool that forbid cudaMalloc after start-up, or C callers
without an allocator) use zs_flatten_sort_count_noalloc, whose scratch is a fixed array
inside the library.  Its results must equal those of the workspace-taking
zs_flatten_sort_count, call after call (the shared array keeps the previous
call's contents).  This file is collected last so that a failing run that
stops at the first failure has run every other test first.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _workspace_entry_point(Z, ids, E):
    n = ids.numel()
    sei = torch.empty(n, dtype=torch.long, device="cuda")
    ssi = torch.empty(n, dtype=torch.long, device="cuda")
    off = torch.empty(E, dtype=torch.long, device="cuda")
    ws = torch.empty(max(int(Z.lib().zs_flatten_sort_count_workspace(n, E)), 1), dtype=torch.uint8, device="cuda")
    Z.check(Z.lib().zs_flatten_sort_count(ids.data_ptr(), n, E, sei.data_ptr(), ssi.data_ptr(), off.data_ptr(),
                                          ws.data_ptr(), ws.numel(), Z.stream_of(ids)), "zs_flatten_sort_count")
    return sei, ssi, off


def _noalloc_entry_point(Z, ids, E):
    n = ids.numel()
    sei = torch.full((n,), -7, dtype=torch.long, device="cuda")
    ssi = torch.full((n,), -7, dtype=torch.long, device="cuda")
    off = torch.full((E,), -7, dtype=torch.long, device="cuda")
    rc = Z.lib().zs_flatten_sort_count_noalloc(ids.data_ptr(), n, E, sei.data_ptr(), ssi.data_ptr(), off.data_ptr(),
                                               Z.stream_of(ids))
    Z.check(rc, "zs_flatten_sort_count_noalloc")
    return sei, ssi, off


def test_noalloc_flatten_sort_count_matches_workspace_entry_point():
    from zs_b200 import _lib as Z

    g = torch.Generator(device="cuda").manual_seed(2024)
    cases = [(131072, 64), (49999, 128), (131072, 64)]   # consecutive calls reuse the shared scratch
    for n, E in cases:
        w = torch.softmax(torch.randn(E, device="cuda", generator=g) * 2, 0)
        ids = torch.multinomial(w, n, replacement=True, generator=g)
        ref = _workspace_entry_point(Z, ids, E)
        got = _noalloc_entry_point(Z, ids, E)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
    assert Z.device_error() == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    from zs_b200 import _lib as Z

    cap = Z.lib().zs_flatten_sort_count_noalloc_max_scratch_ints()
    assert cap == 1 << 18
    E = 1023                      # 1024 buckets per 4096-slot chunk -> 256 chunks fit
    n_ok = 256 * 4096
    n_bad = n_ok + 1
    dummy = torch.zeros(1, dtype=torch.long, device="cuda")
    rc = Z.lib().zs_flatten_sort_count_noalloc(dummy.data_ptr(), n_bad, E, dummy.data_ptr(), dummy.data_ptr(),
                                               dummy.data_ptr(), Z.stream_of(dummy))
    assert rc == 8  # ZS_ERR_SCRATCH_LIMIT
    assert b"scratch" in Z.lib().zs_error_string(rc)


def test_noalloc_at_its_limit_matches_workspace_entry_point():
    """The largest problem the fixed scratch accepts (256 chunks x 1024 buckets = all of
    it): the histogram scan no longer fits shared memory and runs in place in the fixed
    array; two calls in a row, each equal to the workspace entry point."""
    from zs_b200 import _lib as Z

    E, n = 1023, 256 * 4096
    assert Z.lib().zs_flatten_sort_count_workspace(n, E) // 4 == Z.lib().zs_flatten_sort_count_noalloc_max_scratch_ints()
    g = torch.Generator(device="cuda").manual_seed(7)
    for _ in range(2):
        w = torch.softmax(torch.randn(E, device="cuda", generator=g) * 3, 0)
        ids = torch.multinomial(w, n, replacement=True, generator=g)
        ref = _workspace_entry_point(Z, ids, E)
        got = _noalloc_entry_point(Z, ids, E)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
    assert Z.device_error() == 0
