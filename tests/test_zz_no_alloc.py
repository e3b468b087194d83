"""The allocation-free prefix sum, gsb_inclusive_scan_i32_noalloc.

It serves callers that may not allocate device memory where they need the scan
(a host application that owns all device memory, or an allocator's own
callbacks): its scratch is a static device array inside the library. This file
is collected last so that a run stopping at the first failure has run everything
else first; it also passes when run on its own in a fresh process.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _scan_with_caller_scratch(lib, x):
    n = x.numel()
    out = torch.empty(n, dtype=torch.int64, device=DEV)
    nbytes = lib.gsb_scan_scratch_bytes(n)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc = lib.gsb_inclusive_scan_i32(x.data_ptr(), out.data_ptr(), n, scratch.data_ptr(), nbytes,
                                    torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == 0, lib.gsb_last_error()
    return out


def _scan_noalloc(lib, x):
    out = torch.empty(x.numel(), dtype=torch.int64, device=DEV)
    rc = lib.gsb_inclusive_scan_i32_noalloc(x.data_ptr(), out.data_ptr(), x.numel(),
                                            torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == 0, lib.gsb_last_error()
    return out


def test_noalloc_scan_matches_caller_scratch_scan_twice():
    from gsplat_b200.cuda import _backend

    lib = _backend.lib()
    g = torch.Generator(device=DEV).manual_seed(0)
    # calls in a row; later ones are smaller, so stale tile sums from earlier
    # calls are still in the static scratch when they run. Sizes: several
    # thousand tiles, one value short of a 2048-value tile boundary, one past it.
    for n in (3_000_001, 40_000, 2 * 2048 - 1, 2048 + 1):
        x = torch.randint(0, 1000, (n,), device=DEV, dtype=torch.int32, generator=g)
        ref = _scan_with_caller_scratch(lib, x)
        got = _scan_noalloc(lib, x)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)  # integer scan: bit-exact
        # and against an independent prefix sum
        assert torch.equal(got, torch.cumsum(x.long(), 0))


def test_noalloc_scan_rejects_sizes_beyond_its_scratch():
    from gsplat_b200.cuda import _backend

    lib = _backend.lib()
    too_many = (1 << 27) + 1
    rc = lib.gsb_inclusive_scan_i32_noalloc(None, None, too_many, None)
    assert rc == -1
    assert b"exceeds the maximum" in lib.gsb_last_error()
