"""B200-native (sm_100a) GFST-HMB streaming hot path.

Hand-written CUDA kernels behind the C ABI of ``include/gfst_b200.h``
(``libgfst_b200.so``, loaded with ctypes), with Python operators that keep the
reference project's surface (pkhairkh/gfst-hmb-public):

* ``gfst``       frame update + Householder thin QR (canonical_qr_batched,
                 gfst_local_qr, update_basis_batched, stream_frames)
* ``memory``     block commit into the block memory pool (mean summary keys)
* ``retrieval``  coarse block retrieval (BlockRetriever.search / exact_topk)
* ``readout``    exact-token gather, score and argmax inside selected blocks
* ``step``       the fused streaming step (frames + commit + readout)
* ``sharding``   multi-GPU: stream sharding and block-range sharded retrieval
* ``workloads``  seeded synthetic inputs

Every op requires CUDA tensors; nothing falls back to the CPU.
"""

__version__ = "0.1.0"
