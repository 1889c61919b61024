"""The decode projection chain split over two GPUs (tensor parallel, fused
collectives): attn_output and ffn_down store LL words into every rank's slot
and the chain's LL-reduce phases add them into the residual inside the same
launch. Tokens and logits must equal the launch-per-projection split decoder's
bit for bit. Run after the one-GPU chain test; skipped with fewer than two
GPUs."""
import numpy as np
import pytest

from test_tp_gpu import QWEN_PROMPT, QWEN_STEPS
from tp_launch import run_tp_worker

pytestmark = [pytest.mark.gpu, pytest.mark.newest(2)]
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def chain2(tmp_path_factory):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    return run_tp_worker(tmp_path_factory.mktemp("tpchain") / "rank0.npz", "--chain", "--qwen-prompt",
                         str(QWEN_PROMPT), "--qwen-steps", str(QWEN_STEPS))


@pytest.mark.parametrize("name", ["tiny", "qwen"])
def test_split_chain_bitwise_equal(chain2, name):
    assert np.array_equal(chain2[f"{name}_chain_tokens"], chain2[f"{name}_plain_tokens"])
    a, b = chain2[f"{name}_chain_logits"], chain2[f"{name}_plain_logits"]
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    print(f"{name}: 2 GPUs, chain {float(chain2[name + '_chain_ms']):.2f} ms, "
          f"per-projection launches {float(chain2[name + '_plain_ms']):.2f} ms")
