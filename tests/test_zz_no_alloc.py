"""gfst_exact_topk_noalloc: the exact top-k without any device allocation.

Some callers cannot allocate device memory for a call: a host whose device
memory is reserved up front by its own pool allocator (a raw cudaMalloc goes
around the pool and fails once the pool holds the free memory), or a
latency-bound loop that cannot take the device-wide synchronisation cudaFree
implies.  For them the entry point takes its tournament workspace from a
static 1 MiB device array.  This test calls it through the C ABI, as such a
caller would, and checks it against gfst_exact_topk (same kernels, workspace
from the caller) on two calls in a row, one of which needs the scratch; the
results must be identical.  It also checks that a request whose workspace
does not fit is rejected before anything runs.

The file is named to be collected last, so a run that stops at the first
failure has run every other test first.
"""
import ctypes

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import _native as nat

pytestmark = pytest.mark.gpu

GFST_BF16 = 1
GFST_F32 = 0


def _bank(count, d, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    if dtype == torch.bfloat16:
        keys = (torch.randint(-16, 16, (count, d), generator=g) / 8.0).to(dtype)
        q = (torch.randint(-16, 16, (d,), generator=g) / 8.0).to(dtype)
    else:
        keys = torch.randn((count, d), generator=g)
        q = torch.randn((d,), generator=g)
    return keys.to(device).contiguous(), q.to(device).contiguous()


def _with_workspace(lib, keys, q, k, code, stream):
    count, d = keys.shape
    ws_bytes = int(lib.gfst_exact_topk_workspace_bytes(count, k))
    ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=keys.device)
    s = torch.empty((k,), dtype=torch.float32, device=keys.device)
    i = torch.empty((k,), dtype=torch.int64, device=keys.device)
    st = lib.gfst_exact_topk(keys.data_ptr(), q.data_ptr(), count, d, k, code, 1, s.data_ptr(), i.data_ptr(),
                             ws.data_ptr() if ws_bytes else None, ws_bytes, stream)
    assert st == 0, lib.gfst_last_error()
    return s, i


def _no_alloc(lib, keys, q, k, code, stream):
    count, d = keys.shape
    s = torch.empty((k,), dtype=torch.float32, device=keys.device)
    i = torch.empty((k,), dtype=torch.int64, device=keys.device)
    st = lib.gfst_exact_topk_noalloc(keys.data_ptr(), q.data_ptr(), count, d, k, code, 1, s.data_ptr(),
                                     i.data_ptr(), stream)
    assert st == 0, lib.gfst_last_error()
    return s, i


@pytest.mark.parametrize("dtype,code", [(torch.bfloat16, GFST_BF16), (torch.float32, GFST_F32)])
def test_no_alloc_matches_workspace_entry_point(cuda_device, dtype, code):
    lib = nat.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    cases = [(100000, 128, 64, 1), (20000, 64, 300, 2)]  # both need the scratch (more than 16,384 keys)
    with torch.cuda.device(cuda_device):
        for count, d, k, seed in cases:  # two calls in a row, the second over the first's scratch contents
            keys, q = _bank(count, d, dtype, seed, cuda_device)
            assert lib.gfst_exact_topk_workspace_bytes(count, k) > 0
            want_s, want_i = _with_workspace(lib, keys, q, k, code, stream)
            got_s, got_i = _no_alloc(lib, keys, q, k, code, stream)
            torch.cuda.synchronize(cuda_device)
            assert torch.equal(got_i, want_i)
            assert torch.equal(got_s, want_s)
            # and the answer is the top k: scores descending, ties by index
            s, i = got_s.cpu().numpy(), got_i.cpu().numpy()
            assert (np.diff(s) <= 0).all()
            assert all(i[j] < i[j + 1] for j in range(k - 1) if s[j] == s[j + 1])
        # a single-tile bank needs no scratch at all
        keys, q = _bank(5000, 64, dtype, 3, cuda_device)
        want_s, want_i = _with_workspace(lib, keys, q, 40, code, stream)
        got_s, got_i = _no_alloc(lib, keys, q, 40, code, stream)
        torch.cuda.synchronize(cuda_device)
        assert torch.equal(got_i, want_i) and torch.equal(got_s, want_s)
    assert lib.gfst_check_device_errors(1) == 0


def test_no_alloc_rejects_requests_beyond_its_scratch(cuda_device):
    lib = nat.load()
    out_s = torch.empty((8192,), dtype=torch.float32, device=cuda_device)
    out_i = torch.empty((8192,), dtype=torch.int64, device=cuda_device)
    keys = torch.empty((1,), dtype=torch.float32, device=cuda_device)
    # 2 * ceil(200000 / 16384) * 8192 keys of workspace: far above 1 MiB; rejected
    # before any launch (the key pointer is never read)
    st = lib.gfst_exact_topk_noalloc(keys.data_ptr(), keys.data_ptr(), 200000, 64, 8192, GFST_F32, 1,
                                     out_s.data_ptr(), out_i.data_ptr(), ctypes.c_void_p(0))
    assert st == 2  # GFST_ERR_SHAPE
    assert b"static scratch" in lib.gfst_last_error()
