"""Launch overlap (neon_cuda_set_launch_overlap): one-position Q4_0 / Q8_0
launches sized to half the CTAs an SM holds. Only the grid and the ring depth
change -- every row is still one tile's dot product in the same order -- so
the outputs must equal the default sizing's bit for bit, on single matvecs
and through the decode step. Collected after the other GPU suites (a variant
not yet run on a GPU): with -x, a failure here stops nothing else."""
import numpy as np
import pytest

import neon_cuda as N
import synth as S

pytestmark = [pytest.mark.gpu, pytest.mark.newest]
torch = pytest.importorskip("torch")


@pytest.fixture(autouse=True)
def device():
    assert torch.cuda.is_available()
    N.init(0)
    yield
    N.set_launch_overlap(False)


def run(dt, X, rows):
    dx = torch.from_numpy(X.copy()).cuda()
    dy = torch.full((rows,), -3.0, device="cuda")
    dt.matvec(dx, dy)
    torch.cuda.synchronize()
    return dy.cpu().numpy()


@pytest.mark.parametrize("typ", [S.GGML_Q4_0, S.GGML_Q8_0], ids=lambda t: S.TYPE_NAMES[t])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336), (1000, 1024), (24, 28672)])
def test_matvec_bitwise_equal(typ, rows, cols):
    W = S.weights(typ, rows, cols, seed=rows + cols)
    X = S.activations(1, cols, seed=5)[0]
    dt = N.DeviceTensor(W, typ, rows, cols)
    N.set_launch_overlap(False)
    a = run(dt, X, rows)
    N.set_launch_overlap(True)
    b = run(dt, X, rows)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_decode_bitwise_equal():
    cfg = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=64, rope_base=1e4)
    tensors = list(S.model_tensors(cfg, seed=23))
    prompt = S.prompt_tokens(9, cfg.n_vocab, 24)
    out = []
    for on in (False, True):
        N.set_launch_overlap(on)
        m = N.Model(cfg, tensors)
        toks = m.generate(prompt, 8)
        m.set_length(0)
        logits = [m.forward(prompt)] + [m.forward([t]) for t in toks[:4]]
        m.free()
        out.append((toks, logits))
    assert np.array_equal(out[0][0], out[1][0])
    for a, b in zip(out[0][1], out[1][1]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
