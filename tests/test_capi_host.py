"""The C-ABI library loads without a GPU, exports every symbol declared in
include/gfst_b200.h, and rejects bad arguments on the host before touching
the device (no kernel is launched by these calls)."""
import re
from pathlib import Path

import pytest

from gfst_hmb_public_b200 import _native as nat

HEADER = Path(__file__).resolve().parents[1] / "include" / "gfst_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"GFST_API\s+[\w\s\*]+?\b(gfst_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = nat.load()
    names = declared()
    assert len(names) >= 8
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(nat.exported_symbols())


def test_status_strings_and_version():
    lib = nat.load()
    assert lib.gfst_status_string(0) == b"ok"
    assert lib.gfst_status_string(2) == b"unsupported shape"
    assert lib.gfst_abi_version() >> 16 == 1


def test_host_validation_rejects_without_launching():
    lib = nat.load()
    # r > 32
    assert lib.gfst_frame_update_qr(None, None, None, 1.0, None, 4, 64, 40, 0, 1e-8, 0, None) == 2
    assert b"r=40" in lib.gfst_last_error()
    # r > d
    assert lib.gfst_frame_update_qr(None, None, None, 1.0, None, 4, 4, 8, 0, 1e-8, 0, None) == 2
    # unknown sign mode
    assert lib.gfst_frame_update_qr(None, None, None, 1.0, None, 4, 64, 8, 0, 1e-8, 7, None) == 1
    # rank too large
    assert lib.gfst_frame_update_qr(None, None, None, 1.0, None, 4, 64, 8, 9, 1e-8, 0, None) == 2
    # null buffers with work to do
    assert lib.gfst_frame_update_qr(None, None, None, 1.0, None, 4, 64, 8, 0, 1e-8, 0, None) == 1
    # empty batch is a no-op
    assert lib.gfst_frame_update_qr(None, None, None, 1.0, None, 0, 64, 8, 0, 1e-8, 0, None) == 0
    # streaming alignment rule: d*m, r*m multiples of 4
    assert lib.gfst_frame_stream(None, None, None, 1.0, 4, 8, 6, 3, 1, 1e-8, 0, None, 0, None) in (1, 3)
    # commit: slot out of range, bad dtype
    assert lib.gfst_block_commit_mean(None, None, None, None, None, 2, 4, 4, 16, 64, 64, 1, None) == 1
    assert lib.gfst_block_topk(None, None, 1, 1, 4, 4, 64, 33, 0, None, None, None) == 2
    assert lib.gfst_block_topk(None, None, 1, 1, 4, 4, 64, 2, 5, None, None, None) == 7
    assert lib.gfst_exact_readout(None, None, None, None, 1, 1, 4, 16, 64, 64, 0, 1, None, None, None, None) == 2
    # local tracker: d % 4, nested dims not increasing, too many levels
    import ctypes
    dims = (ctypes.c_int32 * 2)(8, 16)
    bad = (ctypes.c_int32 * 2)(16, 8)
    rates = (ctypes.c_double * 3)(0.05, 0.1, 0.2)
    assert lib.gfst_local_tracker_stream(None, None, None, 2, 4, 66, 32, 2, dims, rates, 1e-6, 1e-6, 1e-8, 0,
                                         None, None) == 3
    assert lib.gfst_local_tracker_stream(None, None, None, 2, 4, 64, 32, 2, bad, rates, 1e-6, 1e-6, 1e-8, 0,
                                         None, None) == 2
    assert lib.gfst_local_tracker_stream(None, None, None, 2, 4, 64, 32, 5, dims, rates, 1e-6, 1e-6, 1e-8, 0,
                                         None, None) == 2
    assert lib.gfst_local_tracker_stream(None, None, None, 0, 4, 64, 32, 2, dims, rates, 1e-6, 1e-6, 1e-8, 0,
                                         None, None) == 0
    # streaming QR method: unknown code; CholeskyQR2 outside its classes (host
    # buffers stand in for device pointers: the call returns before any launch)
    buf = (ctypes.c_float * 4096)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.gfst_frame_stream_ex(None, None, None, 1.0, 4, 8, 64, 8, 4, 1e-8, 0, None, 0, 7, None) == 1
    assert lib.gfst_frame_stream_ex(p, p, p, 1.0, 4, 8, 64, 8, 4, 1e-8, 0, None, 0, 3, None) == 2
    assert b"CholeskyQR2" in lib.gfst_last_error()
    assert lib.gfst_frame_stream_ex(p, p, p, 1.0, 4, 8, 8, 8, 4, 1e-8, 0, None, 0, 2, None) == 2
    assert b"CholeskyQR2" in lib.gfst_last_error()
    # MPUC scan: widths not multiples of 4, stage too wide, no workspace (the
    # call returns before touching the device)
    from gfst_hmb_public_b200 import mpuc

    wts = mpuc._WeightsC(**{n: ctypes.cast(buf, ctypes.c_void_p).value for n, _ in mpuc.WEIGHT_FIELDS})
    wp = ctypes.addressof(wts)
    assert lib.gfst_mpuc_recurrent_scan(wp, 30, 16, 16, 64, 8, p, p, p, 2, 4, p, p, p, p, p, p, 4096, None) == 2
    assert lib.gfst_mpuc_recurrent_scan(wp, 8192, 16, 16, 64, 8, p, p, p, 2, 4, p, p, p, p, p, p, 4096, None) == 2
    assert lib.gfst_mpuc_recurrent_scan(None, 32, 16, 16, 64, 8, p, p, p, 2, 4, p, p, p, p, p, p, 4096, None) == 1
    assert lib.gfst_mpuc_recurrent_scan(wp, 32, 16, 16, 64, 8, p, p, p, 0, 4, p, p, p, p, p, p, 0, None) == 0
    # centroid cell write: L * W too large, too many cells, null buffers, empty
    assert lib.gfst_centroid_cell_commit(None, None, None, None, 4, 512, 4, 16, 32, 16, None, None, None, None,
                                         None, None) == 2
    assert lib.gfst_centroid_cell_commit(None, None, None, None, 4, 64, 2, 300, 32, 16, None, None, None, None,
                                         None, None) == 2
    assert lib.gfst_centroid_cell_commit(None, None, None, None, 4, 64, 2, 16, 32, 16, None, None, None, None,
                                         None, None) == 1
    assert lib.gfst_centroid_cell_commit(None, None, None, None, 0, 64, 2, 16, 32, 16, None, None, None, None,
                                         None, None) == 0
    # centroid readout: no params, K > 32, non-positive temperature, too many heads
    from gfst_hmb_public_b200.centroid import CentroidParams
    prm = CentroidParams().to_c()
    pp = ctypes.cast(ctypes.pointer(prm), ctypes.c_void_p)
    args = lambda K, H, params: (None,) * 13 + (1, 1, 4, 16, 32, H, 8, 4, 8, 2, K, params) + (None,) * 11  # noqa
    assert lib.gfst_centroid_readout(*args(4, 2, None)) == 1
    assert lib.gfst_centroid_readout(*args(33, 2, pp)) == 2
    assert lib.gfst_centroid_readout(*args(4, 9, pp)) == 2
    bad_t = CentroidParams(temperature=0.0).to_c()
    assert lib.gfst_centroid_readout(*args(4, 2, ctypes.cast(ctypes.pointer(bad_t), ctypes.c_void_p))) == 1


def test_segmented_and_block_score_host_rejects():
    import ctypes

    lib = nat.load()
    fake = ctypes.c_void_p(256)  # never dereferenced: every call below returns before any launch
    assert lib.gfst_segmented_max(None, None, 16385, 4, fake, None) == 2
    assert lib.gfst_segmented_max(None, None, 8, 16385, fake, None) == 2
    assert lib.gfst_segmented_max(None, None, -1, 4, fake, None) == 1
    assert lib.gfst_segmented_max(None, None, 8, 0, None, None) == 0
    assert lib.gfst_segmented_max(fake, fake, 8, 4, None, None) == 1
    assert lib.gfst_segmented_logsumexp_occurrence(fake, fake, fake, fake, 8, 4, fake, None, fake, None) == 1
    assert lib.gfst_segmented_logsumexp_occurrence(fake, fake, None, fake, 8, 4, fake, fake, fake, None) == 1
    assert lib.gfst_segmented_logsumexp_occurrence(None, None, None, None, 20000, 4, fake, fake, fake, None) == 2
    assert lib.gfst_exact_block_score(None, None, None, -1, 8, 8, 1, None, None) == 1
    assert lib.gfst_exact_block_score(None, None, None, 0, 8, 8, 1, None, None) == 0
    assert lib.gfst_exact_block_score(None, None, None, 4, 8, 8, 1, None, None) == 1
    assert lib.gfst_exact_block_score(fake, fake, fake, 4, 8, 8, 5, fake, None) == 7
    assert lib.gfst_heev(fake, 4, 65, 2, fake, fake, None, None) == 2
    assert lib.gfst_heev(fake, 4, 8, 1, fake, fake, None, None) == 7
    assert lib.gfst_heev(None, 0, 8, 2, None, None, None, None) == 0
    assert lib.gfst_heev(None, 2, 8, 2, None, None, None, None) == 1
    assert lib.gfst_exact_block_materialize(fake, 10, 4, -1, 2, fake, None) == 1
    assert lib.gfst_exact_block_materialize(fake, 10, 4, 5, 4, fake, None) == 1
    assert lib.gfst_exact_block_materialize(fake, 10, 4, 5, 11, fake, None) == 1
    assert lib.gfst_exact_block_materialize(None, 10, 4, 3, 3, None, None) == 0
    assert lib.gfst_debug_bounded_wait(0, None) == 1
    assert lib.gfst_debug_bounded_wait(3_000_000_000, None) == 1


def test_python_ops_reject_cpu_tensors():
    import torch

    from gfst_hmb_public_b200 import gfst, readout, retrieval

    with pytest.raises(RuntimeError):
        gfst.canonical_qr_batched(torch.randn(2, 8, 4))
    with pytest.raises(RuntimeError):
        retrieval.block_topk(torch.randn(1, 2, 8), torch.randn(1, 4, 8), 2)
    with pytest.raises(RuntimeError):
        readout.exact_readout(torch.randn(1, 2, 8), torch.randn(1, 2, 4, 8), None,
                              torch.zeros(1, 2, 2, dtype=torch.int32))
    with pytest.raises(RuntimeError):
        readout.segmented_logsumexp_occurrence(torch.randn(4), torch.zeros(4, dtype=torch.long),
                                               torch.zeros(4, dtype=torch.long), torch.zeros(4, dtype=torch.long),
                                               group_count=1)
    with pytest.raises(RuntimeError):
        readout.exact_block_score(torch.randn(8), torch.randn(3, 8), torch.randn(8, 8))
    from gfst_hmb_public_b200 import tracker

    with pytest.raises(RuntimeError):
        tracker.local_tracker_stream(torch.eye(8, 4)[None].contiguous(), torch.zeros(1, 1, 4, 4),
                                     torch.randn(1, 3, 8), flag_dims=(2, 4), forgetting_rates=(0.1, 0.2))
    with pytest.raises(RuntimeError):
        retrieval.BlockRetriever().search(state=object(), layer_idx=0, batch_idx=0, keys_tensor=torch.eye(4),
                                          query_tensor=torch.ones(4), top_k=2)
