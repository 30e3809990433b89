"""Single-kernel cases for profiling (ncu) and quick timing.

    python -m gfst_hmb_public_b200.cases CASE [--streams S] [--repeat R] [--batch B]

Each case builds seeded inputs on cuda:0, launches its kernel ``repeat`` times
(the first launch is a warm-up) and prints one line with the CUDA-event time of
the last launch.  CASE is one of:

  frames      streaming pass of 64 tokens, 128x32 frames, rank-4 updates
  frames_mid  streaming pass of 64 tokens, 128x16 frames, rank-2 updates (default 256 streams)
  batched_qr  one update+QR launch over 65,536 frames of 64x8
  topk        tensor-core score + top-16 of 64 queries over 512 summaries per stream
  topk_long   tensor-core score + top-8 of 1024 queries over 8192 summaries per stream
  readout     exact-token readout of 64 queries x 16 blocks of 64 tokens per stream
  readout_i8  the same readout with the int8 first look (int8 key copies + side data)
  commit      one 64-token block commit per stream
  tracker     64 tokens of the local tracker (d=64, flag dims 8/16/32, nested levels + features)
  readout_long  exact-token readout of 1024 queries x 8 blocks of 128 tokens per stream out of 8192 blocks
  commit_eig  reference-faithful block commit (float64 eigen summary) of 64 x 64 projector sums
  block_tracker  one 64-token block of the block tracker (d=64, r=32: update + QR + projector sums)
  centroid_commit  centroid cell commit of 64-token blocks
  centroid_readout  centroid readout of 64 queries x 8 blocks per stream
  segmented   log-sum-exp collapse of one candidate list (--streams = elements, default 2048)
  block_score block token scores through a 128 x 128 bf16 projection (--streams = tokens, default 65536)
  heev        batched symmetric eigendecomposition of 64 x 64 float64 matrices (--streams = matrices, default 2048)
  open_block  open-block readout merge of 64 queries over a 64-token open block per stream (bf16, d=128)
  exact_topk  one query against a bf16 bank (--streams = keys, default 8192; top-16)
  mpuc_scan   MPUC recurrent scan of a d_model 2048 cell (fast 1024, mid 512, slow 512,
              bridge rank 128) over 256 tokens (--streams = sequences, default 8)
"""
from __future__ import annotations

import argparse
import math

import torch

from . import block_commit, centroid, gfst, memory, mpuc, readout, retrieval, tracker, workloads as wl


def _timed(fn, repeat: int, batch: int = 1) -> float:
    """CUDA-event time of the last of ``repeat`` rounds; a round is ``batch``
    back-to-back calls and the time is per call (batch > 1 hides the Python
    call overhead of microsecond kernels)."""
    ms = 0.0
    for _ in range(repeat):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(batch):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / batch
    return ms


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("case", choices=["frames", "frames_mid", "batched_qr", "topk", "topk_long", "readout", "readout_i8",
                                         "commit", "tracker",
                                         "readout_long", "commit_eig", "block_tracker", "centroid_commit",
                                         "centroid_readout", "segmented", "block_score", "heev", "open_block",
                                         "exact_topk", "mpuc_scan"])
    parser.add_argument("--streams", type=int, default=None)
    parser.add_argument("--repeat", type=int, default=2)
    parser.add_argument("--batch", type=int, default=1, help="calls per timed round (segmented, block_score)")
    parser.add_argument("--qr-method", default="auto", choices=["auto", "householder", "cholesky2", "cholesky2_split"],
                        help="QR of the frames cases")
    args = parser.parse_args()
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(20261201)
    bf = torch.bfloat16

    if args.case in ("frames", "frames_mid"):
        S = args.streams or (2048 if args.case == "frames" else 256)
        r, m = (32, 4) if args.case == "frames" else (16, 2)
        U = gfst.frame_update_qr(torch.randn((S, 128, r), generator=g, device=dev), sign_mode="r_diag_positive")
        A = torch.randn((S, 64, 128, m), generator=g, device=dev) / math.sqrt(128)
        B = torch.randn((S, 64, r, m), generator=g, device=dev) / math.sqrt(128)
        ms = _timed(lambda: gfst.stream_frames(U, A, B, sign_mode="r_diag_positive", qr_method=args.qr_method),
                    args.repeat)
        units = f"{S * 64 / ms / 1e3:.2f} M frame-tokens/s"
    elif args.case == "batched_qr":
        x = wl.batched_qr_inputs(65536, 64, 8, seed=20261202, device=dev)
        out = torch.empty_like(x)
        ms = _timed(lambda: gfst.frame_update_qr(x, sign_mode="r_diag_positive", out=out), args.repeat)
        units = f"{2 * x.numel() * 4 / ms / 1e6:.0f} GB/s"
    elif args.case in ("topk", "topk_long"):
        S, Nq, NB, k = (args.streams or 2048, 64, 512, 16) if args.case == "topk" else (args.streams or 64, 1024, 8192, 8)
        Q = torch.randn((S, Nq, 128), generator=g, device=dev).to(bf)
        K = torch.randn((S, NB, 128), generator=g, device=dev).to(bf)
        ms = _timed(lambda: retrieval.block_topk(Q, K, k), args.repeat)
        units = f"{2.0 * S * Nq * NB * 128 / ms / 1e9:.1f} TFLOP/s"
    elif args.case == "readout":
        S = args.streams or 1024
        pool = torch.randn((S, 512, 64, 128), generator=g, device=dev).to(bf)
        Q = torch.randn((S, 64, 128), generator=g, device=dev).to(bf)
        sel = torch.randint(0, 512, (S, 64, 16), generator=g, device=dev, dtype=torch.int32)
        ms = _timed(lambda: readout.exact_readout(Q, pool, pool, sel), args.repeat)
        units = f"{S * 64 * 16 * 64 * 128 * 2 / ms / 1e6:.0f} GB/s per-query bytes"
    elif args.case == "readout_i8":
        S = args.streams or 1024
        pool = torch.randn((S, 512, 64, 128), generator=g, device=dev).to(bf)
        pool8 = torch.empty((S, 512, 64, 128), dtype=torch.int8, device=dev)
        meta = torch.empty((S, 512, 64 + 4), dtype=torch.float32, device=dev)
        for b in range(512):
            memory.block_commit_i8(pool[:, b], pool8, meta, b)
        Q = torch.randn((S, 64, 128), generator=g, device=dev).to(bf)
        sel = torch.randint(0, 512, (S, 64, 16), generator=g, device=dev, dtype=torch.int32)
        ms = _timed(lambda: readout.exact_readout(Q, pool, pool, sel, k8=(pool8, meta)), args.repeat)
        units = f"{S * 64 * 16 * 64 * 128 * 2 / ms / 1e6:.0f} GB/s per-query bf16 bytes"
    elif args.case == "readout_long":
        S = args.streams or 16
        pool = torch.randn((S, 8192, 128, 128), generator=g, device=dev, dtype=bf)
        Q = torch.randn((S, 1024, 128), generator=g, device=dev).to(bf)
        sel = torch.randint(0, 8192, (S, 1024, 8), generator=g, device=dev, dtype=torch.int32)
        ms = _timed(lambda: readout.exact_readout(Q, pool, pool, sel), args.repeat)
        units = f"{S * 1024 * 8 * 128 * 128 * 2 / ms / 1e6:.0f} GB/s per-query bytes"
    elif args.case == "commit_eig":
        S = args.streams or 2048
        Uq = torch.linalg.qr(torch.randn((S, 64, 32), generator=g, device=dev))[0]
        ps = 64.0 * (Uq @ Uq.transpose(1, 2)) + 0.01 * torch.randn((S, 64, 64), generator=g, device=dev)
        rs = torch.randn((S, 64), generator=g, device=dev)
        ms = _timed(lambda: block_commit.gfst_block_commit(projector_sum=ps, reduced_sum=rs, token_count=64,
                                                          max_flag_dim=32, flag_dims=(8, 16, 32)), args.repeat)
        units = f"{S / ms / 1e3:.2f} M blocks/s"
    elif args.case == "block_tracker":
        S = args.streams or 2048
        bt = tracker.BlockTracker(S, reduced_dim=64, flag_dims=(8, 16, 32), block_len=1 << 30, device=dev)
        x = torch.randn((S, 64, 64), generator=g, device=dev)
        ms = _timed(lambda: tracker.block_tracker_stream(bt.largest_basis, bt.projector_sum, bt.reduced_sum, x,
                                                         rate=0.2), args.repeat)
        units = f"{S * 64 / ms / 1e3:.2f} M tokens/s"
    elif args.case in ("centroid_commit", "centroid_readout"):
        # streaming shapes: 64-token blocks, 16 cells, 2 memberships, key 32 /
        # value 16 per head, 4 heads, 128-dim token keys, top-16 blocks
        S, NB, L, W, C, dk, dv, H, dq, K, Nq = args.streams or 256, 512, 64, 2, 16, 32, 16, 4, 128, 16, 64
        ids = torch.randint(0, C, (S, NB, L, W), generator=g, device=dev, dtype=torch.int32)
        w = torch.rand((S, NB, L, W), generator=g, device=dev)
        w = w / w.sum(-1, keepdim=True)
        ck = torch.randn((S, NB, L, dk), generator=g, device=dev)
        cv = torch.randn((S, NB, L, dv), generator=g, device=dev)
        if args.case == "centroid_commit":
            ms = _timed(lambda: centroid.centroid_cell_commit(ids, w, ck, cv, C), args.repeat)
            units = f"{S * NB / ms / 1e3:.2f} M blocks/s"
        else:
            tid, twq, keys, vals, cnt = centroid.centroid_cell_commit(ids, w, ck, cv, C)
            del ck, cv, w, ids
            store = dict(token_keys=torch.randn((S, NB, L, dq), generator=g, device=dev),
                         token_features=torch.randn((S, NB, L, H, dv), generator=g, device=dev),
                         token_ids=torch.randint(0, 32000, (S, NB, L), generator=g, device=dev, dtype=torch.int32),
                         token_cell_ids=tid, token_cell_weights_q=twq, cell_keys=keys, cell_values_q=vals,
                         cell_counts=cnt)
            Q = torch.randn((S, Nq, dq), generator=g, device=dev)
            qh = torch.randn((S, Nq, H, dk), generator=g, device=dev)
            sel = torch.randint(0, NB, (S, Nq, K), generator=g, device=dev, dtype=torch.int32)
            sc = torch.randn((S, Nq, K), generator=g, device=dev)
            ms = _timed(lambda: centroid.centroid_readout(Q, qh, sel, sc, **store), args.repeat)
            per_q = K * L * (dq + H * dv) * 4
            units = f"{S * Nq / ms / 1e3:.2f} M queries/s, {S * Nq * per_q / ms / 1e6:.0f} GB/s of token rows"
    elif args.case == "segmented":
        n = args.streams or 2048
        scores = torch.randn((n,), generator=g, device=dev)
        inverse = torch.randint(0, max(1, n // 2), (n,), generator=g, device=dev)
        groups = int(inverse.max()) + 1
        blk = torch.randint(0, 512, (n,), generator=g, device=dev)
        ms = _timed(lambda: readout.segmented_logsumexp_occurrence(scores, inverse, blk, blk, group_count=groups),
                    args.repeat, args.batch)
        units = f"{n / ms / 1e3:.2f} M elements/s ({groups} groups)"
    elif args.case == "block_score":
        m = args.streams or 65536
        q = torch.randn((128,), generator=g, device=dev).to(bf)
        F = torch.randn((m, 128), generator=g, device=dev).to(bf)
        Wp = torch.randn((128, 128), generator=g, device=dev).to(bf)
        ms = _timed(lambda: readout.exact_block_score(q, F, Wp), args.repeat, args.batch)
        units = f"{2.0 * m * 128 * 128 / ms / 1e9:.2f} TFLOP/s, {m * 128 * 2 / ms / 1e6:.0f} GB/s of features"
    elif args.case == "heev":
        nb = args.streams or 2048
        x = torch.randn((nb, 64, 64), generator=g, device=dev, dtype=torch.float64)
        a = x + x.transpose(-1, -2)
        ms = _timed(lambda: block_commit.gfst_heev(a, check=False), args.repeat, args.batch)
        units = f"{nb / ms / 1e3:.2f} M matrices/s"
    elif args.case == "tracker":
        S = args.streams or 2048
        tr = tracker.LocalTracker(S, reduced_dim=64, flag_dims=(8, 16, 32), device=dev)
        x = torch.randn((S, 64, 64), generator=g, device=dev)
        ms = _timed(lambda: tr.step(x), args.repeat)
        units = f"{S * 64 / ms / 1e3:.2f} M tokens/s"
    elif args.case == "open_block":
        S = args.streams or 2048
        Q = torch.randn((S, 64, 128), generator=g, device=dev).to(bf)
        Ko = torch.randn((S, 64, 128), generator=g, device=dev).to(bf)
        Vo = torch.randn((S, 64, 128), generator=g, device=dev).to(bf)
        bt = torch.full((S, 64), -1, dtype=torch.int32, device=dev)
        bs = torch.full((S, 64), float("-inf"), device=dev)
        ov = torch.zeros((S, 64, 128), dtype=bf, device=dev)
        ms = _timed(lambda: readout.open_block_readout(Q, Ko, Vo, bt, bs, ov, open_base=512 * 64), args.repeat)
        units = f"{S * 64 * 128 * 2 * 2 / ms / 1e6:.0f} GB/s of queries and open keys"
    elif args.case == "exact_topk":
        n = args.streams or 8192
        keys = torch.randn((n, 128), generator=g, device=dev).to(bf)
        q = torch.randn((128,), generator=g, device=dev).to(bf)
        ms = _timed(lambda: retrieval.exact_topk(keys, q, 16), args.repeat, args.batch)
        units = f"{n * 128 * 2 / ms / 1e6:.0f} GB/s of keys"
    elif args.case == "mpuc_scan":
        B, T = args.streams or 8, 256
        cell = wl.mpuc_cell_weights(2048, seed=20261210, device=dev)
        ins = [torch.randn((B, T, n), generator=g, device=dev) for n in (cell.F, cell.M, cell.S)]
        ms = _timed(lambda: mpuc.recurrent_scan(cell, *ins), args.repeat)
        units = f"{ms * 1e3 / T:.2f} us per token, {B * T / ms / 1e3:.3f} M sequence-tokens/s"
    else:  # commit
        S = args.streams or 2048
        mem = memory.BlockMemory(S, 4, 64, 128, dtype=bf, device=dev)
        Kb = torch.randn((S, 64, 128), generator=g, device=dev).to(bf)
        ms = _timed(lambda: mem.commit(Kb, Kb), args.repeat)
        units = f"{S * 64 * 128 * 2 * 4 / ms / 1e6:.0f} GB/s"
    print(f"{args.case}: {ms:.4f} ms  {units}", flush=True)


if __name__ == "__main__":
    main()
