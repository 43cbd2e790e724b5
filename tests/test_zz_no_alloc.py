"""The allocation-free paged decode entry point (akt_decode_paged_noalloc).

It serves callers that cannot allocate device memory when they run the decode
-- plugin hosts that pass only input and output buffers, and runtimes that
forbid cudaMalloc after start-up -- by keeping the split-KV partials in a
fixed array inside the library.  These tests call it through the C ABI and
check its output against the workspace entry point (akt_decode_paged) on the
same inputs, within the suite's decode tolerance (max-abs 2e-3, no NaNs), on
two calls in a row, and check that an oversized call is rejected with a clear
error instead of running.  The file is collected last so that a failure here
comes after every other test has run; it also passes on its own.
"""
import ctypes
import os
import sys

import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from attention_kernel_triton_b200 import _lib  # noqa: E402
from attention_kernel_triton_b200 import workloads as W  # noqa: E402
from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import (  # noqa: E402
    _paged_args, decode_paged_into)

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def _noalloc(out, c, scale):
    a = _paged_args(c.q, c.cache, c.indptr, c.indices, c.last_page_len, out, scale)
    rc = _lib.lib().akt_decode_paged_noalloc(ctypes.byref(a), _lib.stream_ptr(out.device))
    return rc


@pytest.mark.parametrize("shape", [
    dict(B=16, Hq=32, Hkv=8, D=128, page_size=16),           # cfg3 head layout, 16 sequences
    dict(B=5, Hq=8, Hkv=2, D=64, page_size=64, min_len=1, max_len=3000),
])
def test_noalloc_matches_workspace_entry_point_on_two_calls(shape):
    torch.cuda.set_device(0)
    _lib.device_status(0, clear=True)
    c = W.make_paged(seed=77, device=DEV, **shape)
    B, Hq, _, D = c.q.shape
    scale = 1.0 / D ** 0.5
    ref = torch.empty((B, Hq, D), dtype=c.q.dtype, device=DEV)
    decode_paged_into(ref, c.q, c.cache, c.indptr, c.indices, c.last_page_len, scale)
    for _ in range(2):
        out = torch.full((B, Hq, D), float("nan"), dtype=c.q.dtype, device=DEV)
        _lib.check(_noalloc(out, c, scale))
        torch.cuda.synchronize()
        assert not torch.isnan(out).any()
        assert (out.float() - ref.float()).abs().max().item() <= TOL
    assert _lib.device_status(0) == 0


def test_noalloc_lengthens_chunks_when_the_default_split_does_not_fit():
    # 16 sequences of ~140K tokens (4.6 GB pool): the default split's partials need more
    # than the 16 MiB the library holds, so the entry point plans longer chunks until they
    # fit; the output must still match the workspace entry point, on two calls in a row
    torch.cuda.set_device(0)
    _lib.device_status(0, clear=True)
    c = W.make_paged(B=16, Hq=64, Hkv=8, D=64, page_size=16, min_len=130000, max_len=150000, seed=79,
                     device=DEV)
    B, Hq, _, D = c.q.shape
    scale = 1.0 / D ** 0.5
    ref = torch.empty((B, Hq, D), dtype=c.q.dtype, device=DEV)
    a = _paged_args(c.q, c.cache, c.indptr, c.indices, c.last_page_len, ref, scale)
    assert _lib.lib().akt_decode_paged_workspace_size(ctypes.byref(a)) > (16 << 20)
    decode_paged_into(ref, c.q, c.cache, c.indptr, c.indices, c.last_page_len, scale)
    for _ in range(2):
        out = torch.full((B, Hq, D), float("nan"), dtype=c.q.dtype, device=DEV)
        _lib.check(_noalloc(out, c, scale))
        torch.cuda.synchronize()
        assert not torch.isnan(out).any()
        assert (out.float() - ref.float()).abs().max().item() <= TOL
    assert _lib.device_status(0) == 0


def test_noalloc_rejects_calls_beyond_its_scratch():
    torch.cuda.set_device(0)
    c = W.make_paged(B=2, Hq=8, Hkv=2, D=128, page_size=16, lens=[40, 50], seed=78, device=DEV)
    out = torch.empty((2, 8, 128), dtype=c.q.dtype, device=DEV)
    a = _paged_args(c.q, c.cache, c.indptr, c.indices, c.last_page_len, out, 0.1)
    a.batch = 4_000_000  # more sequences than the fixed scratch can plan for; nothing is launched
    rc = _lib.lib().akt_decode_paged_noalloc(ctypes.byref(a), _lib.stream_ptr(out.device))
    assert rc == _lib.AKT_ERR_WORKSPACE
    assert b"at most" in _lib.lib().akt_last_error()
