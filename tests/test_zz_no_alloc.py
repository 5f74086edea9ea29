"""opus_bucket_max_load_noalloc (static device scratch) against opus_bucket_max_load, through the C ABI.

Kept in its own file, collected last, so it runs both alone and after every
other test in the same process.
"""
import ctypes

import numpy as np
import pytest
import torch

from opus_b200 import _lib

DEV = "cuda"
NOALLOC_MAX_BUCKETS = 262144


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _packed(rng, numel, k):
    buckets = rng.integers(0, k, numel).astype(np.uint32)
    signs = rng.integers(0, 2, numel).astype(np.uint32) << np.uint32(31)
    return buckets, torch.from_numpy((buckets | signs).view(np.int32)).to(DEV)


def test_noalloc_rejects_k_beyond_static_scratch():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    rc = lib.opus_bucket_max_load_noalloc(null, 0, NOALLOC_MAX_BUCKETS + 1, null, null)
    assert rc == _lib.OPUS_ERR_INVALID and "static scratch" in _lib.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("numel,k", [(3072 * 768, 16384), (1_000_003, NOALLOC_MAX_BUCKETS), (77, 8)])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(numel, k):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(numel + k)
    for _ in range(2):  # the second call must start from zeroed counts
        buckets, packed = _packed(rng, numel, k)
        counts = torch.empty(k, dtype=torch.int32, device=DEV)
        out_ws = torch.empty(1, dtype=torch.int64, device=DEV)
        out_na = torch.full((1,), -7, dtype=torch.int64, device=DEV)
        assert lib.opus_bucket_max_load(_p(packed), numel, k, _p(counts), k, _p(out_ws), stream) == 0
        assert lib.opus_bucket_max_load_noalloc(_p(packed), numel, k, _p(out_na), stream) == 0
        torch.cuda.synchronize()
        want = int(np.bincount(buckets.astype(np.int64), minlength=k).max())
        assert int(out_na.item()) == int(out_ws.item()) == want


@pytest.mark.gpu
def test_noalloc_flags_bucket_outside_k():
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    bad = torch.tensor([1, 2, 40, 3], dtype=torch.int32, device=DEV)
    out = torch.empty(1, dtype=torch.int64, device=DEV)
    assert lib.opus_bucket_max_load_noalloc(_p(bad), 4, 16, _p(out), stream) == 0
    torch.cuda.synchronize()
    assert int(out.item()) == -1
    assert _lib.device_error() == 0  # the library's error word is left alone
    good = torch.tensor([1, 1, 3], dtype=torch.int32, device=DEV)
    assert lib.opus_bucket_max_load_noalloc(_p(good), 3, 16, _p(out), stream) == 0
    torch.cuda.synchronize()
    assert int(out.item()) == 2
