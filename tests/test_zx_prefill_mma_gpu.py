"""Multi-position projections (prefill) on the tensor cores
(neon_cuda_set_prefill_mma, csrc/neon_prefill.cuh) against the oracle: Q4_0
BIT FOR BIT (each output is dot_q4_0_q8_0's block sequence with the integer
block sums from int8 MMA), Q8_0 within the per-row matvec bar (TF32 MMA with X
split in two TF32 terms). Also the decoder's prompt pass with the switch on.
Collected after the other GPU suites (the kernel is the newest): with -x, a
failure here stops nothing else."""
import numpy as np
import pytest

import neon_cuda as N
import oracle as O
import synth as S
from conftest import MATVEC_RTOL, MODEL_L2_RTOL, max_rel_err, rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.newest]
torch = pytest.importorskip("torch")


@pytest.fixture(autouse=True)
def mma_on():
    assert torch.cuda.is_available()
    N.init(0)
    N.set_prefill_mma(True)
    yield
    N.set_prefill_mma(True)  # the default


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("rows,cols,seq", [(70, 320, 9), (64, 128, 66), (1000, 4096, 2), (4096, 4096, 128),
                                           (256, 1024, 517), (33, 32, 5)])
def test_bit_exact_with_the_reference_arithmetic(rows, cols, seq):
    W = S.weights(S.GGML_Q4_0, rows, cols, seed=rows + seq)
    X = S.activations(seq, cols, seed=seq + 1)
    dt = N.DeviceTensor(W, S.GGML_Q4_0, rows, cols)
    dx = torch.from_numpy(X.copy()).cuda()
    dy = torch.full((seq * (rows + 3),), -5.0, device="cuda")
    dt.matvec(dx, dy, seq=seq, x_stride=cols, y_stride=rows + 3)
    torch.cuda.synchronize()
    Y = dy.cpu().numpy().reshape(seq, rows + 3)
    assert np.array_equal(bits(Y[:, :rows]), bits(O.proj_all_positions(S.GGML_Q4_0, W, rows, cols, X)))
    assert np.all(Y[:, rows:] == -5.0)


@pytest.mark.parametrize("rows,cols,seq", [(70, 160, 9), (1000, 4096, 66), (4096, 4096, 64), (33, 32, 3)])
def test_q8_0_within_the_matvec_bar(rows, cols, seq):
    W = S.weights(S.GGML_Q8_0, rows, cols, seed=rows + seq)
    X = S.activations(seq, cols, seed=seq + 2)
    dt = N.DeviceTensor(W, S.GGML_Q8_0, rows, cols)
    dx = torch.from_numpy(X.copy()).cuda()
    dy = torch.zeros(seq * rows, device="cuda")
    dt.matvec(dx, dy, seq=seq)
    torch.cuda.synchronize()
    got = dy.cpu().numpy().reshape(seq, rows)
    assert max_rel_err(got, O.proj_all_positions(S.GGML_Q8_0, W, rows, cols, X)) <= MATVEC_RTOL


def test_multi_targets_bit_exact():
    cols, seq = 1024, 40
    X = S.activations(seq, cols, seed=2)
    specs = [(512, 11), (128, 12), (128, 13)]
    targets, dts = [], []
    for rows, seed in specs:
        W = S.weights(S.GGML_Q4_0, rows, cols, seed=seed)
        targets.append((W, rows))
        dts.append(N.DeviceTensor(W, S.GGML_Q4_0, rows, cols))
    ys = [torch.zeros(seq * r, device="cuda") for r, _ in specs]
    N.matvec_multi([(dt, y, None) for dt, y in zip(dts, ys)], torch.from_numpy(X.copy()).cuda(), seq=seq)
    torch.cuda.synchronize()
    for (W, rows), y in zip(targets, ys):
        assert np.array_equal(bits(y.cpu().numpy().reshape(seq, rows)),
                              bits(O.proj_all_positions(S.GGML_Q4_0, W, rows, cols, X)))


def test_decoder_prompt_pass():
    cfg = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=160, rope_base=1e4)
    tensors = list(S.model_tensors(cfg, seed=9))
    prompt = S.prompt_tokens(130, cfg.n_vocab, 10)
    m = N.Model(cfg, tensors)
    o = O.Model(cfg, tensors, "port")
    want_toks, want_logits = o.generate_greedy(prompt, 6)
    assert np.array_equal(m.generate(prompt, 6), want_toks)
    m.set_length(0)
    assert rel_l2(m.forward(prompt), want_logits[0]) <= MODEL_L2_RTOL
    m.free()


def test_prompt_pass_matches_the_cuda_core_kernels():
    """A Q8_0-weight decoder (no activation quantisation on its path): the
    prompt pass on the tensor-core projections and attention against the
    CUDA-core kernels, logits within fp32 noise."""
    cfg = S.ModelConfig(1000, 256, 2, 4, 2, 64, 512, ctx_len=200, rope_base=1e4)
    tensors = list(S.model_tensors(cfg, seed=12, wtype=S.GGML_Q8_0))
    prompt = S.prompt_tokens(150, cfg.n_vocab, 13)
    m = N.Model(cfg, tensors)
    on = m.forward(prompt)
    N.set_prefill_mma(False)
    m.set_length(0)
    off = m.forward(prompt)
    m.free()
    assert rel_l2(on, off) <= 1e-4 and int(np.argmax(on)) == int(np.argmax(off))
