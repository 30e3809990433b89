"""CPU oracle for the GFST-HMB streaming hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference's algorithm for every step of
the hot path (pkhairkh/gfst-hmb-public; each function cites the file:line it
follows).  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / reference arm may import it, and only as the checker or the timed
CPU baseline -- never as a fallback for the product path.

Pinning: the restatement is checked against golden vectors produced by the
reference's own code (``tests/golden/make_golden.py`` imports the reference's
``gfst.py``, ``retrieval.py`` and diagnostics by file path and records their
outputs) and against the known-answer cases in the reference's tests.

Modules:
  gfst_oracle      numpy/torch-CPU restatement (QR + sign rules, frame update,
                   streaming trajectories, block commit, top-k, exact readout)
  householder.c    plain-C fixed-order Householder QR (fp32), an independent
                   second restatement of the QR (built by oracle/build.py)
"""
