"""The failure path of the in-kernel waits, exercised without a fault: a wait on
an mbarrier that nothing completes gives up after its cycle budget, the
sticky device error word reports GFST_ERR_TIMEOUT to the host, reading it
clears it, and the context keeps running kernels afterwards."""
import pytest
import torch

from gfst_hmb_public_b200 import _native, retrieval

pytestmark = pytest.mark.gpu

GFST_ERR_TIMEOUT = 6


def test_bounded_wait_gives_up_and_context_stays_usable(cuda_device):
    lib = _native.load()
    assert lib.gfst_check_device_errors(1) == 0
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    with torch.cuda.device(cuda_device):
        assert lib.gfst_debug_bounded_wait(2_000_000, stream) == 0  # about a millisecond
        assert lib.gfst_check_device_errors(0) == GFST_ERR_TIMEOUT
        assert lib.gfst_check_device_errors(1) == GFST_ERR_TIMEOUT  # read and clear
        assert lib.gfst_check_device_errors(0) == 0
    # a tensor-core retrieval launch after the probe still gives the right answer
    g = torch.Generator().manual_seed(4)
    Q = torch.randn((2, 64, 128), generator=g).to(torch.bfloat16)
    K = torch.randn((2, 300, 128), generator=g).to(torch.bfloat16)
    scores, idx = retrieval.block_topk(Q.to(cuda_device), K.to(cuda_device), 4)
    ref = torch.topk(Q.float() @ K.float().transpose(1, 2), 4, dim=-1)
    assert torch.allclose(scores.cpu(), ref.values, rtol=1e-5, atol=1e-4)
    assert lib.gfst_check_device_errors(1) == 0


def test_timeout_seen_right_after_a_side_stream_launch(cuda_device):
    """The probe runs on a non-blocking torch stream (as the step's kernels do);
    the check synchronises the device, so the status is visible at once, and
    the raising helper reports it."""
    lib = _native.load()
    assert lib.gfst_check_device_errors(1) == 0
    side = torch.cuda.Stream(cuda_device)
    with torch.cuda.device(cuda_device):
        assert lib.gfst_debug_bounded_wait(2_000_000, side.cuda_stream) == 0
        assert lib.gfst_check_device_errors(0) == GFST_ERR_TIMEOUT
        with pytest.raises(RuntimeError, match="timed out"):
            _native.check_device_errors()  # raises and clears
        _native.check_device_errors()     # nothing left


def test_step_check_errors_flag(cuda_device):
    """With check_errors=True a step raises when a failure was recorded before
    it completed; without a failure it runs normally."""
    from gfst_hmb_public_b200.step import StreamingStep

    S, d, r, L = 4, 64, 8, 16
    st = StreamingStep(S, d=d, r=r, block_len=L, n_slots=4, k=2, dtype=torch.float32, device=cuda_device,
                       check_errors=True)
    st.set_frames(torch.linalg.qr(torch.randn((S, d, r), device=cuda_device))[0])
    A = torch.randn((S, L, d, 1), device=cuda_device) / 8
    B = torch.randn((S, L, r, 1), device=cuda_device) / 8
    K, V, Q = (torch.randn((S, L, d), device=cuda_device) for _ in range(3))
    st.step(A, B, K, V, Q)
    lib = _native.load()
    with torch.cuda.device(cuda_device):
        assert lib.gfst_debug_bounded_wait(2_000_000, torch.cuda.current_stream().cuda_stream) == 0
    with pytest.raises(RuntimeError, match="timed out"):
        st.step(A, B, K, V, Q)
    st.step(A, B, K, V, Q)  # the report was cleared
