"""Expert parallelism on real GPUs (needs >= 2 visible GPUs; NCCL over NVLink)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
WORKER = Path(__file__).resolve().parent / 'ep_gpu_worker.py'


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs at least two GPUs')
@pytest.mark.parametrize('world', [2, 4, 8])
def test_ep_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f'needs {world} GPUs')
    env = dict(os.environ, NCCL_NVLS_ENABLE='0')
    cmd = ['timeout', '-k', '30', '300', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           f'--nproc-per-node={world}', '--master-addr', '127.0.0.1', f'--master-port={_port()}', str(WORKER)]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
