"""Expert parallelism across GPUs: the EP forward on 2 (or 4) ranks must equal
the single-GPU forward bit for bit, eagerly and from CUDA graphs.  Runs
tests/ep_worker.py under torch.distributed.run; needs at least two GPUs."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(n):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(n), "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "ep_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    print(r.stdout[-4000:], r.stderr[-4000:])
    return r.returncode


@pytest.mark.parametrize("n", [2, 4, 8])
def test_ep_forward_equals_single_gpu(cuda, n):
    if cuda.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    assert run_ranks(n) == 0
