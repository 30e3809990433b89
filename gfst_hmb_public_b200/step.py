"""The streaming GFST-HMB step on one GPU: frames, block commit and sparse readout.

One step consumes one block of L tokens for every (batch, head) stream:

* frames   ``U <- QR(U + sum_i u_i v_i^T)`` for each of the L tokens, the frame
           held in registers across the block (gfst_frame_stream);
* readout  for each of the L queries: score every committed block summary
           (tcgen05 GEMM + top-k), then score the tokens of the k selected
           blocks and of the step's own block up to the query's position, and
           return the best token and its value row;
* commit   the block's keys and values go into the memory ring and its summary
           key (mean of the keys) into the summary table.

The frame update and the readout are independent within a step, so they run on
two CUDA streams: the frame kernel is FP32-ALU bound and the readout is HBM
bound, and the two overlap on the SMs.  The commit follows the readout on the
memory stream.  What a query at position p of the step's block sees is what the
reference's query of that token sees (pkhairkh/gfst-hmb-public): the committed
blocks (a block summary is appended after the retrieval of the block's last
token, modeling.py:3618-3632) and, since each token is appended to the exact
store before its own retrieval (modeling.py:3807 vs 3853), positions [0, p] of
its own block while p < L - 1 (modeling.py:2948-2963); at p = L - 1 the exact
store has already closed the block (state.py:749-815), so that query sees the
committed blocks only.

Reference loop being replaced (pkhairkh/gfst-hmb-public): the per-token
``for token: for batch:`` loop of GfstHmbSublayer (src/gfst_hmb_mpuc/modeling.py:
3943-3961) calling _update_local_bases (2299-2423), _update_block_memory
(3401-3571) and the retrieval/readout path (2714-2920, 984-1316).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat
from . import gfst, memory, readout, retrieval


@dataclass
class StepOutputs:
    """Per-query results of one step.  best_tok is the token index slot * L + p
    of the best token in the memory ring, or open_base + p for position p of
    the step's own block (open_base = n_slots * L; that block is committed to
    ``slot`` at the end of the step), or -1 when nothing was valid."""
    best_tok: torch.Tensor    # [S, L] int32
    best_score: torch.Tensor  # [S, L] float32
    value: torch.Tensor       # [S, L, dv] memory dtype
    top_idx: torch.Tensor     # [S, L, k] int32 selected block slots
    open_base: int = 0
    slot: int = -1


class StreamingStep:
    """Frames + block memory + readout for ``n_streams`` independent streams."""

    def __init__(self, n_streams: int, *, d: int, r: int, block_len: int, n_slots: int, k: int,
                 dtype: torch.dtype = torch.bfloat16, device="cuda", sign_mode="r_diag_positive",
                 eps_sign: float = 1e-8, check_errors: bool = False, int8_keys: bool | None = None):
        """check_errors: after every step, wait for it and raise RuntimeError if
        a kernel recorded a device-side failure (a bounded wait that gave up);
        a debugging aid -- it makes every step synchronous.
        int8_keys: keep int8 copies of the committed keys and read them out
        with the int8 first look (exact_readout's ``k8``: the same results from
        about half the bytes); default on for bf16 memories with d = 128 or
        256 and 16 | L <= 256."""
        self.n_streams, self.d, self.r, self.block_len, self.n_slots, self.k = n_streams, d, r, block_len, n_slots, k
        self.sign_mode = sign_mode
        self.eps_sign = eps_sign
        self.check_errors = check_errors
        self.device = torch.device(device)
        self.U = torch.zeros((n_streams, d, r), dtype=torch.float32, device=self.device)
        if int8_keys is None:
            int8_keys = dtype == torch.bfloat16 and d in (128, 256) and block_len % 16 == 0 and block_len <= 256
        self.memory = memory.BlockMemory(n_streams, n_slots, block_len, d, d, dtype=dtype, device=self.device,
                                         int8_keys=int8_keys)
        self.frames_stream = torch.cuda.Stream(self.device)
        self.memory_stream = torch.cuda.Stream(self.device)

    def set_frames(self, U0: torch.Tensor) -> None:
        self.U.copy_(U0)

    def reset(self) -> None:
        """Empty the memory ring (the frames are left as they are)."""
        self.memory.reset()

    @property
    def open_base(self) -> int:
        """Token index of position 0 of the step's own block in StepOutputs.best_tok."""
        return self.n_slots * self.block_len

    def _memory_work(self, K: torch.Tensor, V: torch.Tensor, Q: torch.Tensor) -> StepOutputs:
        """Top-k, readout, open block and commit of one block, enqueued on the
        current stream (the memory stream)."""
        n_valid = self.memory.n_valid
        if n_valid > 0:
            top_s, top_i = retrieval.block_topk(Q, self.memory.summary, self.k, n_blocks=n_valid)
            best_tok, best_score, value = readout.exact_readout(Q, self.memory.pool_K, self.memory.pool_V, top_i,
                                                                k8=self.memory.k8)
        else:
            S, L = Q.shape[0], Q.shape[1]
            top_i = torch.full((S, L, self.k), -1, dtype=torch.int32, device=self.device)
            best_tok = torch.full((S, L), -1, dtype=torch.int32, device=self.device)
            best_score = torch.full((S, L), float("-inf"), dtype=torch.float32, device=self.device)
            value = torch.zeros((S, L, V.shape[-1]), dtype=V.dtype, device=self.device)
        readout.open_block_readout(Q, K, V, best_tok, best_score, value, open_base=self.open_base)
        slot = self.memory.commit(K, V)
        return StepOutputs(best_tok, best_score, value, top_i, self.open_base, slot)

    def _join(self, cur, results) -> None:
        cur.wait_stream(self.frames_stream)
        cur.wait_stream(self.memory_stream)
        # tensors produced on side streams are consumed on the current stream
        # (under CUDA-graph capture the graph's private pool keeps them instead)
        if not torch.cuda.is_current_stream_capturing():
            self.U.record_stream(cur)
            for res in results:
                for t in (res.best_tok, res.best_score, res.value, res.top_idx):
                    t.record_stream(cur)
        if self.check_errors:
            nat.check_device_errors()

    def step(self, A: torch.Tensor, B: torch.Tensor, K: torch.Tensor, V: torch.Tensor, Q: torch.Tensor,
             *, out: StepOutputs | None = None) -> StepOutputs:
        """A [S, L, d, m], B [S, L, r, m] fp32 update factors; K, V, Q [S, L, d]
        in the memory dtype.  Work is enqueued on the caller's current stream's
        device; the call returns once it is enqueued (outputs are ready when the
        current stream reaches them)."""
        cur = torch.cuda.current_stream(self.device)
        self.frames_stream.wait_stream(cur)
        self.memory_stream.wait_stream(cur)
        with torch.cuda.stream(self.frames_stream):
            gfst.stream_frames(self.U, A, B, eps_sign=self.eps_sign, sign_mode=self.sign_mode)
        with torch.cuda.stream(self.memory_stream):
            result = self._memory_work(K, V, Q)
        self._join(cur, (result,))
        if out is not None:
            out.best_tok.copy_(result.best_tok)
            out.best_score.copy_(result.best_score)
            out.value.copy_(result.value)
            out.top_idx.copy_(result.top_idx)
            out.open_base, out.slot = result.open_base, result.slot
            return out
        return result

    def run(self, blocks, *, block_events=None) -> list:
        """Several consecutive blocks in one call: ``blocks`` is a sequence of
        (A, B, K, V, Q) tuples as ``step`` takes them; returns one StepOutputs
        per block, the same values consecutive ``step`` calls return.
        ``block_events``, if given, holds one (frames_event, memory_event) pair
        of CUDA events per block, recorded on the two streams after that
        block's work (block i is done when both have completed).

        The frames of a block depend only on the frames of the block before,
        and its top-k, readout and commit only on the memory the blocks before
        committed, so the two chains run on their own streams with no join
        between blocks: the frame kernel of block i+1 may run beside the
        readout of block i (on B200, 20 blocks of 64 tokens with 512-block
        rings: 4.55 against 4.79 ms per block at 2048 streams, 1.03 against
        1.18 ms at 256).  The current stream waits for both chains at the end."""
        blocks = [tuple(b) for b in blocks]
        cur = torch.cuda.current_stream(self.device)
        self.frames_stream.wait_stream(cur)
        self.memory_stream.wait_stream(cur)
        if block_events is not None and len(block_events) < len(blocks):
            raise ValueError("block_events: one (frames, memory) event pair per block")
        results = []
        for i, (A, B, K, V, Q) in enumerate(blocks):
            with torch.cuda.stream(self.frames_stream):
                gfst.stream_frames(self.U, A, B, eps_sign=self.eps_sign, sign_mode=self.sign_mode)
                if block_events is not None:
                    block_events[i][0].record(self.frames_stream)
            with torch.cuda.stream(self.memory_stream):
                results.append(self._memory_work(K, V, Q))
                if block_events is not None:
                    block_events[i][1].record(self.memory_stream)
        self._join(cur, results)
        return results


class StreamingPass:
    """A whole streaming pass captured once as a CUDA graph and replayed.

    The pass is: empty the memory ring, load the frames ``U0``, then
    ``StreamingStep.run`` over ``blocks`` (each an (A, B, K, V, Q) tuple of
    device tensors, as ``step`` takes them).  At small batches the
    pass is a chain of short kernels whose launch cost exceeds their run time;
    replaying the captured graph launches them all at once.  The input tensors
    (``U0`` and every block) are read in place on each replay: copy new data
    into them, not new tensors.  ``outputs[i]`` holds block i's StepOutputs
    after each replay (the same tensors every time).  The capture follows one
    eager pass (which allocates and configures every kernel); the step must
    not synchronise (``check_errors`` off).
    """

    def __init__(self, step: StreamingStep, U0: torch.Tensor, blocks):
        if step.check_errors:
            raise ValueError("StreamingPass: a step with check_errors=True synchronises and cannot be captured")
        self.step_obj = step
        self.U0 = U0
        self.blocks = [tuple(b) for b in blocks]
        dev = step.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._run()                       # eager: allocations, kernel attributes
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.outputs = self._run()

    def _run(self):
        st = self.step_obj
        st.reset()
        st.set_frames(self.U0)
        return st.run(self.blocks)

    def replay(self) -> list:
        """Run the pass again on the current stream; returns ``outputs``."""
        self.graph.replay()
        return self.outputs


class HostPipeline:
    """Runs a StreamingStep on inputs held in pinned host memory.

    The inputs of step i+1 are copied to the device on an upload stream while
    step i computes (two device input buffers), and each step's results are
    copied back to pinned host buffers on a download stream, so host<->device
    traffic overlaps the kernels.  This is the end-to-end path a host-side
    caller uses; every byte of every step crosses the bus.
    """

    def __init__(self, step: StreamingStep, example_inputs):
        dev = step.device
        self.step_obj = step
        self.buffers = [[torch.empty_like(t, device=dev) for t in example_inputs] for _ in range(2)]
        self.upload = torch.cuda.Stream(dev)
        self.download = torch.cuda.Stream(dev)
        self.ready = [torch.cuda.Event() for _ in range(2)]
        self.free = [torch.cuda.Event() for _ in range(2)]
        self.done = [torch.cuda.Event() for _ in range(2)]
        for e in self.free:
            e.record(torch.cuda.current_stream(dev))

    def _upload(self, i: int, host_inputs) -> None:
        b = i % 2
        self.upload.wait_event(self.free[b])
        with torch.cuda.stream(self.upload):
            for d, h in zip(self.buffers[b], host_inputs):
                d.copy_(h, non_blocking=True)
        self.ready[b].record(self.upload)

    def run(self, host_inputs_per_step, host_outputs_per_step) -> None:
        """host_inputs_per_step: sequence of (A, B, K, V, Q) pinned tensors;
        host_outputs_per_step: sequence of (best_tok, best_score, value) pinned
        tensors receiving each step's results.  Returns once all work is enqueued."""
        cur = torch.cuda.current_stream(self.step_obj.device)
        n = len(host_inputs_per_step)
        if n == 0:
            return
        self._upload(0, host_inputs_per_step[0])
        for i in range(n):
            if i + 1 < n:
                self._upload(i + 1, host_inputs_per_step[i + 1])
            b = i % 2
            cur.wait_event(self.ready[b])
            out = self.step_obj.step(*self.buffers[b])
            self.free[b].record(cur)
            self.done[b].record(cur)
            self.download.wait_event(self.done[b])
            with torch.cuda.stream(self.download):
                for h, d in zip(host_outputs_per_step[i], (out.best_tok, out.best_score, out.value)):
                    h.copy_(d, non_blocking=True)
                for t in (out.best_tok, out.best_score, out.value):
                    t.record_stream(self.download)
        cur.wait_stream(self.download)

    def drain(self) -> None:
        """Wait for every enqueued step and its copies; raise RuntimeError if a
        kernel recorded a device-side failure (its results are then invalid)."""
        torch.cuda.synchronize(self.step_obj.device)
        nat.check_device_errors()
