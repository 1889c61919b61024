"""The tensor-parallel communicator on ONE GPU: the single-rank all-reduce,
argument checks of the sharded model, and failure detection.

Failure detection is tested without a GPU fault: rank 0 of a two-rank
communicator whose "peer" is a second buffer on the same device runs an
all-reduce that the peer never joins (nothing ever sets the peer's flag). The
kernel's wait runs out after the communicator's timeout, sets the error word
and returns; the host reads the error, later collectives on the broken
communicator return at once, and the context stays usable. Rank 1 never
launches anything: two ranks' waiting kernels are never run on one GPU."""
import time

import numpy as np
import pytest

import neon_cuda as N
import synth as S
from conftest import load_golden

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TINY = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4, name="tiny")


@pytest.fixture(scope="module", autouse=True)
def device():
    assert torch.cuda.is_available()
    N.init(0)
    torch.cuda.set_device(0)


@pytest.mark.parametrize("n,add", [(1, False), (4096, True), (1000003, True), (8192 * 256, False)])
def test_single_rank_allreduce_is_exact(n, add):
    c = N.Comm(0, 1, n)
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, generator=g).cuda()
    out = torch.randn(n, generator=g).cuda()
    want = (out + x) if add else x.clone()
    c.allreduce(x, out, add=add, stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    c.check()
    assert torch.equal(out, want)
    c.free()


def test_allreduce_rejects_oversize():
    c = N.Comm(0, 1, 64)
    x = torch.zeros(1024, device="cuda")
    with pytest.raises(N.NeonError, match="larger than the communicator"):
        c.allreduce(x, x, n=1024)
    c.free()


def test_model_with_single_rank_comm_matches_golden():
    g = load_golden("decode_tiny.npz")
    c = N.Comm(0, 1, N.model_comm_floats(TINY, 1))
    m = N.Model(TINY, S.model_tensors(TINY, seed=3), c)
    assert np.array_equal(m.generate(g["prompt"], 16), g["tokens"])
    m.free()
    c.free()


def _loopback_pair(floats):
    c0, c1 = N.Comm(0, 2, floats), N.Comm(1, 2, floats)
    N.Comm.connect_local([c0, c1])
    return c0, c1


def test_sharded_model_argument_checks():
    c0, c1 = _loopback_pair(N.model_comm_floats(TINY, 2))
    with pytest.raises(N.NeonError, match="divisible"):
        N.Model(TINY.with_(n_head=6, n_kv_head=3), (), c0)
    small0, small1 = _loopback_pair(64)
    with pytest.raises(N.NeonError, match="neon_cuda_model_comm_floats"):
        N.Model(TINY, (), small0)
    unconnected = N.Comm(0, 2, N.model_comm_floats(TINY, 2))
    with pytest.raises(N.NeonError, match="not connected"):
        N.Model(TINY, (), unconnected)
    for c in (c0, c1, small0, small1, unconnected):
        c.free()


def test_peer_that_never_joins_times_out_and_context_survives():
    c0, c1 = _loopback_pair(4096)
    c0.set_timeout(0.2)
    x = torch.ones(4096, device="cuda")
    out = torch.zeros(4096, device="cuda")
    t0 = time.perf_counter()
    c0.allreduce(x, out, stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    with pytest.raises(N.NeonError, match="gave up waiting"):
        c0.check()
    assert 0.15 <= waited < 5.0
    # a broken communicator skips its later collectives instead of waiting again
    t0 = time.perf_counter()
    for _ in range(10):
        c0.allreduce(x, out, stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.15
    # the context is intact: a matvec still runs and is right
    W = S.q8_0_weights(64, 256, seed=5)
    X = S.activations(1, 256, seed=6)
    Y = np.zeros((1, 64), np.float32)
    N.proj_all_positions(N.TensorInfo("w", [256, 64], N.GGML_Q8_0, W), X, 256, Y, 64, 1)
    assert np.isfinite(Y).all() and np.abs(Y).sum() > 0
    c0.free()
    c1.free()
