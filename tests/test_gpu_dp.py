"""Data parallelism on two GPUs: each rank runs its batch slice of ResNet-18
(7 images over 2 ranks: 4 + 3, an uneven split), rank 0 gathers the output
rows over NCCL (gawee_dp_gather_output, sized by gawee_dp_output_bytes), and
the gathered rows match the oracle's forward of the full batch at the
reference's ResNet tolerance."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle
from tests.helpers import compare

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, os.environ["GAWEE_ROOT"])
from datetime import timedelta
from gawee_b200 import dp, synth
from gawee_b200.runtime import Model
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
full = synth.resnet18(7, image=64)
args = full.make_args()
s0, s1 = dp.shard_range(7, world, rank)
shard = synth.resnet18(s1 - s0, image=64)
m = Model(shard.mlir, device=rank)
m.set_args(dp.shard_args(args, [True] + [False] * (len(args) - 1), world, rank))
uid = dp.share_nccl_id(Model.dp_unique_id() if rank == 0 else bytes(128), rank)
m.dp_init(world, rank, uid)
total = m.dp_output_bytes(0)
assert total == 7 * 1000 * 4, total
out = torch.empty((7, 1000), device=f"cuda:{rank}") if rank == 0 else None
stream = torch.cuda.current_stream().cuda_stream
m.forward(stream)
m.dp_gather_output(0, out.data_ptr() if rank == 0 else None, stream)
m.synchronize(stream)
if rank == 0:
    np.save(os.environ["GAWEE_OUT"], out.cpu().numpy())
    np.save(os.environ["GAWEE_OUT"] + ".args.npy", args[0])
m.close()
dist.barrier()
dist.destroy_process_group()
"""


def test_two_gpu_uneven_batch_sharding_matches_oracle(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from gawee_b200 import synth

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    out = str(tmp_path / "gathered.npy")
    env = dict(os.environ, GAWEE_ROOT=ROOT, GAWEE_OUT=out, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
               WORLD_SIZE="2", NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, str(script)], env=dict(env, RANK=str(r), LOCAL_RANK=str(r)))
             for r in range(2)]
    codes = [p.wait(timeout=600) for p in procs]
    assert codes == [0, 0]
    gathered = np.load(out)
    full = synth.resnet18(7, image=64)
    want = oracle.run(full.mlir, full.make_args())[0]
    compare(gathered, want, 1e-4, 1e-4, "gathered rows vs oracle")
