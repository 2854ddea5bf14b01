"""Row-sharded GEMV on 2, 4 and 8 GPUs of one box (one process per GPU through torch.distributed.run): the fused P2P
all-gather and the NCCL exchange both reproduce the unsharded output bit for bit and stay within the rule of the C
oracle's exact reference on sampled rows of every rank's slice (tests/dist_worker.py)."""

import os
import re
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_sharded_gemv_matches_single_gpu_and_oracle(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "60", "540", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "dist_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    # the ranks print concurrently, so lines may interleave: find each rank's verdict anywhere in the output
    res = dict(re.findall(r"RESULT (\d+) (ok|FAIL)", r.stdout))
    assert res == {str(q): "ok" for q in range(world)}, r.stdout[-3000:]
