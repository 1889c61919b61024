"""Launches tests/tp_gpu_worker.py on two GPUs (torch.distributed.run, one
process per GPU, rendezvous on 127.0.0.1) for the tensor-parallel GPU tests,
and returns rank 0's observations (the npz it writes)."""
import os
import signal
import socket
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_tp_worker(out, *args, timeout=900):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "tp_gpu_worker.py"), "--out", str(out), *args]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="4")
    p = subprocess.Popen(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, start_new_session=True)
    try:
        log, _ = p.communicate(timeout=timeout)
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGTERM)
        log, _ = p.communicate()
        pytest.fail("tensor-parallel worker timed out:\n" + log.decode(errors="replace")[-4000:])
    text = log.decode(errors="replace")
    assert p.returncode == 0, text[-4000:]
    print(text[-2000:])
    return dict(np.load(out))
