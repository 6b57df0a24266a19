"""The allocation-free single-query attention entry point.

Callers that cannot allocate device memory where they run (FFI hosts without a
device allocator of their own, serving loops kept off the allocator) call
``vdit_attention_1q_noalloc``; its split-K partials live in a fixed device
array inside the library instead of a workspace.  This checks it through the
C ABI against ``vdit_attention_1q`` (caller workspace) on two calls in a row,
since every call reuses the same array, and that oversize requests are
refused.  The file sorts last so a run stopping at the first failure has run
everything else first; it also passes alone in a fresh process.
"""
import math

import pytest
import torch

from vdit import _lib
from vdit import fast_kernels as fk

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm())


def noalloc_1q(q, kv, heads, hd):
    """One call of vdit_attention_1q_noalloc on the current stream."""
    lib = _lib.load()
    d = heads * hd
    out = torch.empty(d, dtype=torch.bfloat16, device=kv.device)
    q = q.reshape(-1).to(torch.bfloat16).contiguous()
    rc = lib.vdit_attention_1q_noalloc(q.data_ptr(), kv[:, :d].data_ptr(), kv[:, d:].data_ptr(), kv.stride(0),
                                       kv.shape[0], heads, hd, float(1.0 / math.sqrt(hd)), out.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    return rc, out


@pytest.mark.parametrize("n,heads,hd", [(1, 12, 128), (16384, 12, 128), (5000, 16, 96), (70000, 2, 96)])
def test_noalloc_matches_workspace_entry_point(n, heads, hd):
    g = torch.Generator(device=DEV).manual_seed(n + heads)
    d = heads * hd
    q = torch.randn(d, device=DEV, generator=g)
    kv = torch.randn(n, 2 * d, device=DEV, generator=g).to(torch.bfloat16)
    ref = fk.attention_1q(q, kv, heads, hd)
    for _ in range(2):                       # the second call reuses the array the first one filled
        rc, out = noalloc_1q(q, kv, heads, hd)
        assert rc == 0, _lib.lib().vdit_error_string(rc)
        torch.cuda.synchronize()
        assert rel(out, ref) < 1e-2
    assert _lib.device_error() == 0


def test_noalloc_padded_kv_rows():
    """K/V rows with a stride beyond 2 * heads * head_dim (padded rows)."""
    heads, hd, n = 12, 128, 3000
    d = heads * hd
    g = torch.Generator(device=DEV).manual_seed(7)
    q = torch.randn(d, device=DEV, generator=g)
    kv = torch.randn(n, 2 * d + 64, device=DEV, generator=g).to(torch.bfloat16)[:, :2 * d]
    assert kv.stride(0) == 2 * d + 64
    ref = fk.attention_1q(q, kv, heads, hd)
    for _ in range(2):
        rc, out = noalloc_1q(q, kv, heads, hd)
        assert rc == 0
        torch.cuda.synchronize()
        assert rel(out, ref) < 1e-2


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_on_a_second_device():
    """Each GPU holds its own array and the library looks up its address per device: a
    call on cuda:1 after calls on cuda:0 matches the workspace entry point there."""
    heads, hd, n = 12, 128, 5000
    d = heads * hd
    for dev in ("cuda:0", "cuda:1", "cuda:0"):
        with torch.cuda.device(dev):
            g = torch.Generator(device=dev).manual_seed(11)
            q = torch.randn(d, device=dev, generator=g)
            kv = torch.randn(n, 2 * d, device=dev, generator=g).to(torch.bfloat16)
            ref = fk.attention_1q(q, kv, heads, hd)
            rc, out = noalloc_1q(q, kv, heads, hd)
            assert rc == 0
            torch.cuda.synchronize()
            assert rel(out, ref) < 1e-2
            assert _lib.device_error() == 0


def test_noalloc_refuses_sizes_beyond_its_scratch():
    heads, hd = 2048, 128                    # heads * splits * (hd + 2) floats > 1 MiB
    kv = torch.zeros(1, 2 * heads * hd, device=DEV, dtype=torch.bfloat16)
    rc, _ = noalloc_1q(torch.zeros(heads * hd, device=DEV), kv, heads, hd)
    assert rc == -7
    assert b"no-alloc" in _lib.lib().vdit_error_string(rc)
