"""The decode projection chain split over two GPUs (tensor parallel, fused
collectives): attn_output and ffn_down store LL words into every rank's slot
and the chain's LL-reduce phases add them into the residual inside the same
launch. Tokens and logits must equal the launch-per-projection split decoder's
bit for bit. Run after the one-GPU chain test; skipped with fewer than two
GPUs."""
import os
import signal
import subprocess
import sys

import numpy as np
import pytest

from test_tp_gpu import HERE, QWEN_PROMPT, QWEN_STEPS, _free_port

pytestmark = [pytest.mark.gpu, pytest.mark.newest(2)]
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def chain2(tmp_path_factory):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path_factory.mktemp("tpchain") / "rank0.npz"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_gpu_worker.py"), "--out", str(out), "--chain",
           "--qwen-prompt", str(QWEN_PROMPT), "--qwen-steps", str(QWEN_STEPS)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="4")
    p = subprocess.Popen(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, start_new_session=True)
    try:
        log, _ = p.communicate(timeout=900)
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGTERM)
        log, _ = p.communicate()
        pytest.fail("tensor-parallel worker timed out:\n" + log.decode(errors="replace")[-4000:])
    text = log.decode(errors="replace")
    assert p.returncode == 0, text[-4000:]
    return dict(np.load(out))


@pytest.mark.parametrize("name", ["tiny", "qwen"])
def test_split_chain_bitwise_equal(chain2, name):
    assert np.array_equal(chain2[f"{name}_chain_tokens"], chain2[f"{name}_plain_tokens"])
    a, b = chain2[f"{name}_chain_logits"], chain2[f"{name}_plain_logits"]
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    print(f"{name}: 2 GPUs, chain {float(chain2[name + '_chain_ms']):.2f} ms, "
          f"per-projection launches {float(chain2[name + '_plain_ms']):.2f} ms")
