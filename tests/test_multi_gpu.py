"""Member sharding on real GPUs with NCCL (runs only when 2+ GPUs are visible):
two ranks each run the block-sparse attention for their members and all-gather
the per-member outputs; the gathered ensemble must equal a one-GPU run."""
import os
import socket
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = textwrap.dedent(r"""
    import datetime, os, sys
    import torch, torch.distributed as dist
    sys.path.insert(0, os.environ["ROOT"])
    import mosaic_b200 as M
    from mosaic_b200 import ensemble as E
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    members, N, Hq, Hk = 4, 3072, 8, 2
    g = torch.Generator().manual_seed(0)
    q = torch.randn(members, N, Hq, 64, generator=g).bfloat16()
    k = torch.randn(members, N, Hk, 64, generator=g).bfloat16()
    v = torch.randn(members, N, Hk, 64, generator=g).bfloat16()
    w = torch.sigmoid(torch.randn(3, members, N, Hq, 1, generator=g)).bfloat16()
    fn = lambda qq, kk, vv, ww: M.mosaic_attn_func(qq.to(dev), kk.to(dev), vv.to(dev), ww.to(dev), 1024, 64, 8, False)
    out = E.run_sharded(fn, [q, k, v, w], members, batch_dims=[0, 0, 0, 1])
    ref = fn(q, k, v, w)  # the whole ensemble on this GPU
    ok = torch.equal(out, ref)
    t = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(t)
    dist.destroy_process_group()
    print("OK" if int(t.item()) == world else "MISMATCH")
""")


def test_nccl_member_sharding_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, ROOT=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.count("OK") == 2, r.stdout
