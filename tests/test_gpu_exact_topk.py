"""exact_topk / BlockRetriever.search for any top_k (gfst_exact_topk).

The reference's FaissGpuRetriever.exact_topk (retrieval.py:165-172) takes any
k <= count and ranks keys @ q in the keys' dtype; with bf16 keys the scores
are bf16, so equal scores are common and torch.topk orders them arbitrarily.

Bars: bf16 banks -- the returned scores equal the reference's bf16 scores
exactly and the chosen keys agree up to the order of equal scores (golden
vectors from the reference's own exact_topk); fp32 banks -- indices bit-exact
where the oracle's consecutive scores differ by more than 1e-3 relative, scores
within 1e-5; ties always resolve to the lower index.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import retrieval
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_bf16_banks_match_reference(cuda_device):
    z = np.load(GOLDEN / "retrieval_exact_topk_bf16.npz")
    for c in range(4):
        keys = torch.from_numpy(z[f"c{c}_keys"]).view(torch.bfloat16).to(cuda_device)
        q = torch.from_numpy(z[f"c{c}_query"]).view(torch.bfloat16).to(cuda_device)
        k = int(z[f"c{c}_k"])
        idx, sc = retrieval.BlockRetriever.exact_topk(keys, q, k)
        idx, sc = idx.cpu().numpy(), sc.cpu().numpy()
        assert idx.dtype == np.int64 and sc.dtype == np.float32 and idx.shape == (k,)
        assert go.same_topk_up_to_ties(idx, sc, z[f"c{c}_idx"], z[f"c{c}_scores"], z[f"c{c}_all_scores"])
        for j in range(1, k):
            if sc[j] == sc[j - 1]:
                assert idx[j] > idx[j - 1]


def test_fp32_bank_matches_reference_golden(cuda_device):
    z = np.load(GOLDEN / "retrieval_exact_topk.npz")
    keys = torch.from_numpy(z["keys"]).to(cuda_device)
    for qi in range(z["queries"].shape[0]):
        idx, sc = retrieval.exact_topk(keys, torch.from_numpy(z["queries"][qi]).to(cuda_device), 5)
        ref_s = z["top_scores"][qi]
        sep = np.ones(5, bool)
        gaps = np.abs(np.diff(ref_s)) > 1e-3 * np.maximum(np.abs(ref_s[:-1]), 1e-30)
        sep[1:] &= gaps
        sep[:-1] &= gaps
        assert np.array_equal(idx.cpu().numpy()[sep], z["top_idx"][qi][sep])
        np.testing.assert_allclose(sc.cpu().numpy(), ref_s, rtol=1e-5, atol=1e-5)
    si, ss = retrieval.exact_topk(torch.from_numpy(z["small_keys"]).to(cuda_device),
                                  torch.from_numpy(z["small_query"]).to(cuda_device), 3)
    assert si.tolist() == [0, 5, 2]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("count,d,k", [(1, 8, 1), (33, 64, 33), (16384, 32, 16384), (16385, 64, 100),
                                       (100000, 128, 97), (40000, 32, 8192), (70001, 16, 1)])
def test_any_k_against_oracle(cuda_device, dtype, count, d, k):
    g = torch.Generator().manual_seed(count + k)
    if dtype == torch.bfloat16:
        # multiples of 1/8: float32 sums are exact in any order, so the bf16
        # score of every key is unambiguous (and many scores tie)
        keys = (torch.randint(-16, 16, (count, d), generator=g) / 8.0).to(dtype)
        q = (torch.randint(-16, 16, (d,), generator=g) / 8.0).to(dtype)
    else:
        keys = torch.randn((count, d), generator=g)
        q = torch.randn((d,), generator=g)
    idx, sc = retrieval.exact_topk(keys.to(cuda_device), q.to(cuda_device), k)
    bf = dtype == torch.bfloat16
    ref_i, ref_s = go.exact_topk(keys.float().numpy(), q.float().numpy(), k, round_bf16=bf)
    idx, sc = idx.cpu().numpy(), sc.cpu().numpy()
    if bf:
        all_s = go.to_bf16_f32((keys.double() @ q.double()).float().numpy())
        assert go.same_topk_up_to_ties(idx, sc, ref_i, ref_s, all_s)
        assert np.array_equal(idx, ref_i)  # the oracle breaks ties the same way
    else:
        sep = np.ones(k, bool)
        if k > 1:
            gaps = np.abs(np.diff(ref_s)) > 1e-3 * np.maximum(np.abs(ref_s[:-1]), 1e-30)
            sep[1:] &= gaps
            sep[:-1] &= gaps
        assert np.array_equal(idx[sep], ref_i[sep])
        np.testing.assert_allclose(sc, ref_s, rtol=1e-5, atol=1e-4)


def test_special_values(cuda_device):
    keys = torch.zeros((10, 8), device=cuda_device)
    keys[0, 0] = float("nan")          # NaN score ranks last
    keys[1, 0] = float("inf")          # +inf first
    keys[2, 0] = -1.0                  # -0.0 x ... and +0 tie by index
    keys[3, 0] = float("-inf")         # -inf before NaN
    q = torch.zeros((8,), device=cuda_device)
    q[0] = 1.0
    idx, sc = retrieval.exact_topk(keys, q, 10)
    idx = idx.tolist()
    assert idx[0] == 1 and idx[-1] == 0 and idx[-2] == 3
    assert idx[1:7] == [4, 5, 6, 7, 8, 9] and idx[7] == 2
    assert torch.isnan(sc[-1]) and sc[0] == float("inf")


def test_search_any_k_and_limits(cuda_device):
    class State:
        state_version = 0

    keys = torch.randn((50, 16), device=cuda_device)
    q = torch.randn((16,), device=cuda_device)
    r = retrieval.BlockRetriever()
    idx, sc = r.search(state=State(), layer_idx=0, batch_idx=0, keys_tensor=keys, query_tensor=q, top_k=80)
    assert idx.shape == (50,) and sorted(idx.tolist()) == list(range(50))
    assert (sc[:-1] >= sc[1:]).all()
    with pytest.raises(RuntimeError):  # above 8192 for a bank of more than 16,384 keys
        retrieval.exact_topk(torch.randn((20000, 16), device=cuda_device), q, 9000)
