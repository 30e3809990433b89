"""torchrun worker for tests/test_bench_host.py: every rank starts a child
process with bench.child_env, and the children form a gloo group of their own
on a fresh port, as bench.py's sub-result children do (with NCCL)."""
import datetime
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

import torch.distributed as dist  # noqa: E402

if len(sys.argv) > 1 and sys.argv[1] == "child":
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=30))
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0)

import bench  # noqa: E402

dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
rank, world = dist.get_rank(), dist.get_world_size()
box = [bench._free_port() if rank == 0 else 0]
dist.broadcast_object_list(box, src=0)
env = bench.child_env(rank, world, int(os.environ.get("LOCAL_RANK", rank)), int(box[0]))
assert not any(k.startswith("TORCHELASTIC_") for k in env)
rc = subprocess.run([sys.executable, __file__, "child"], env=env, timeout=90).returncode
flag = [rc]
out = [None] * world
dist.all_gather_object(out, flag)
dist.destroy_process_group()
sys.exit(0 if all(r == [0] for r in out) else 1)
