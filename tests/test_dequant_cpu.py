"""The block decoders of the dequantising kernel (F32, F16, BF16, Q4_1, Q5_0,
Q5_1, Q4_K, Q5_K, Q6_K), built for the host from the same source the sm_100a
kernels compile (neon_dequant.cuh: dq_sub is __host__ __device__), decode the
device layout -- the GGUF rows at a 16-byte pitch, float rows zero-padded to
32-value blocks -- to exactly the oracle's values (dequantize_row,
rawllm_forward.hpp:301-321, itself pinned bit-exact to the reference)."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

import oracle as O
import synth as S
from conftest import PKG, ROOT

DQ_TYPES = [t for t in S.ALL_TYPES if t not in (S.GGML_Q4_0, S.GGML_Q8_0)]


@pytest.fixture(scope="module")
def dq(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("dqhost") / "libdqhost.so")
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    subprocess.check_call([nvcc if os.path.exists(nvcc) else "nvcc", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
                           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(PKG, "csrc"),
                           os.path.join(ROOT, "tests", "cpp", "dq_host.cu"), "-o", so])
    L = C.CDLL(so)
    L.dq_host_decode_row.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_void_p]
    L.dq_host_geometry.argtypes = [C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.dq_host_code_dots.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    L.dq_host_row.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]
    L.dq_host_ring_plan.argtypes = [C.c_int, C.c_int, C.c_longlong, C.c_size_t, C.c_int, C.c_int, C.c_void_p]
    return L


def geometry(L, t):
    be, bb, cb = C.c_int(), C.c_int(), C.c_int()
    L.dq_host_geometry(t, C.byref(be), C.byref(bb), C.byref(cb))
    return be.value, bb.value, cb.value


def device_row(L, t, row, cols):
    """One GGUF row laid out as the upload stores it: zero-padded to whole
    32-value blocks (float types) and to a 16-byte pitch."""
    be, bb, _ = geometry(L, t)
    nu = (cols + 31) // 32
    pitch = (nu // (be // 32) * bb + 15) & ~15
    buf = np.zeros(pitch, np.uint8)
    buf[:row.size] = row
    return buf, nu


def same(a, b):
    ua, ub = a.view(np.uint32), b.view(np.uint32)
    return (ua == ub) | (np.isnan(a) & np.isnan(b))


@pytest.mark.parametrize("typ", DQ_TYPES, ids=lambda t: S.TYPE_NAMES[t])
def test_device_decoder_matches_oracle(dq, typ):
    for cols in (512, 4096):
        synth = S.weights(typ, 8, cols, seed=11)
        rand = np.random.default_rng(typ).integers(0, 256, synth.shape, dtype=np.uint8)  # NaN/Inf/subnormal scales
        for M in (synth, rand):
            for r in range(M.shape[0]):
                buf, nu = device_row(dq, typ, M[r], cols)
                out = np.empty(nu * 32, np.float32)
                assert dq.dq_host_decode_row(typ, buf.ctypes.data, nu, out.ctypes.data) == 0
                assert same(out[:cols], O.dequantize_row(typ, M[r], cols)).all(), (S.TYPE_NAMES[typ], cols, r)


@pytest.mark.parametrize("typ", [S.GGML_F32, S.GGML_F16, S.GGML_BF16], ids=lambda t: S.TYPE_NAMES[t])
def test_ragged_float_rows_pad_with_zeros(dq, typ):
    cols = 45  # block size 1: any input dim is a valid float tensor
    W = S.weights(typ, 3, cols, seed=2)
    for r in range(3):
        buf, nu = device_row(dq, typ, W[r], cols)
        out = np.empty(nu * 32, np.float32)
        dq.dq_host_decode_row(typ, buf.ctypes.data, nu, out.ctypes.data)
        assert same(out[:cols], O.dequantize_row(typ, W[r], cols)).all()
        assert not out[cols:].any()


def test_chunks_stay_16_byte_aligned(dq):
    # every chunk of CB blocks starts on a 16-byte boundary of a row (the
    # 128-bit loads), and a chunk is 32 (or 64 for super-blocks) sub-blocks
    for t in DQ_TYPES:
        be, bb, cb = geometry(dq, t)
        assert (cb * bb) % 16 == 0 and cb * (be // 32) in (32, 64), S.TYPE_NAMES[t]
        assert bb == S.BLOCK_BYTES[t] * (32 if S.BLOCK_ELEMS[t] == 1 else 1)
    assert geometry(dq, S.GGML_Q4_0) == (0, 0, 0)


BLOCK_TYPES = [t for t in DQ_TYPES if t not in (S.GGML_F32, S.GGML_F16, S.GGML_BF16)]


@pytest.mark.parametrize("typ", BLOCK_TYPES, ids=lambda t: S.TYPE_NAMES[t])
def test_code_dot_products(dq, typ):
    """The kernel's per-sub-block dot, a*sum((code - OFF)*x) + b*sum(x) on
    packed pairs, against the exact dot of the oracle's weights with x: the
    same sum in another order (bound: a few fp32 ulps of sum |w*x|)."""
    cols = 2048
    W = S.weights(typ, 16, cols, seed=21)
    x = S.activations(1, cols, seed=22)[0]
    for r in range(W.shape[0]):
        buf, nu = device_row(dq, typ, W[r], cols)
        got = np.empty(nu, np.float32)
        assert dq.dq_host_code_dots(typ, buf.ctypes.data, nu, x.ctypes.data, got.ctypes.data) == 0
        w = O.dequantize_row(typ, W[r], cols).astype(np.float64).reshape(nu, 32)
        xx = x.astype(np.float64).reshape(nu, 32)
        exact = (w * xx).sum(axis=1)
        scale = (np.abs(w) * np.abs(xx)).sum(axis=1) + np.abs(w).max() * np.abs(xx).sum(axis=1)
        assert np.all(np.abs(got - exact) <= 2e-6 * scale), (S.TYPE_NAMES[typ], r)


@pytest.mark.parametrize("typ", S.ALL_TYPES, ids=lambda t: S.TYPE_NAMES[t])
def test_host_row_decoder(dq, typ):
    """neon::dq_row_host, which decodes non-F32 norm weights at load time,
    on host rows at every byte offset mod 16 (unaligned blocks): the oracle's
    values bit for bit, random bytes included; a ragged block row refused."""
    be = S.BLOCK_ELEMS[typ]
    n = 512
    rows = [S.weights(typ, 1, n, seed=31).reshape(-1),
            np.random.default_rng(typ + 7).integers(0, 256, S.weights(typ, 1, n, seed=31).size, dtype=np.uint8)]
    for row in rows:
        want = O.dequantize_row(typ, row, n)
        for off in range(16):
            buf = np.zeros(row.size + 16, np.uint8)
            buf[off:off + row.size] = row
            out = np.empty(n, np.float32)
            assert dq.dq_host_row(typ, buf.ctypes.data + off, n, out.ctypes.data) == 0
            assert same(out, want).all(), (S.TYPE_NAMES[typ], off)
    if be > 1:
        out = np.empty(n, np.float32)
        assert dq.dq_host_row(typ, rows[0].ctypes.data, n - 16, out.ctypes.data) == -1


RING_SHAPES = [(4096, 4096), (1000, 2048), (14336, 4096), (4096, 14336), (24, 28672), (77, 1013), (8, 32),
               (3, 256), (28672, 8192), (8192, 28672), (1024, 3072), (151936, 1024)]


@pytest.mark.parametrize("typ", DQ_TYPES, ids=lambda t: S.TYPE_NAMES[t])
def test_ring_plan_copies(dq, typ):
    """The bulk-copy ring kernel (matvec_dq_ring_kernel) on its own tile plan
    (neon::plan_dq_ring), its copy warp and compute warps emulated: every
    cp.async.bulk starts and ends on a 16-byte boundary on both sides, stays
    inside the tensor's rows x pitch bytes and its stage, fits one mbarrier
    phase's byte count; every block of every row is decoded exactly once, from
    bytes the copy delivered."""
    be, bb, _ = geometry(dq, typ)
    subs = be // 32
    for rows, cols in RING_SHAPES:
        if S.BLOCK_ELEMS[typ] > 1 and cols % S.BLOCK_ELEMS[typ]:
            continue
        nu = (cols + 31) // 32
        nblk = nu // subs
        pitch = (nblk * bb + 15) & ~15
        for sms in (148, 132):
            out = (C.c_int * 5)()
            dq.dq_host_ring_plan(typ, nblk, pitch, rows, sms, 40 * 1024, out)
            rpw, kcb, nch, rs, stage = list(out)
            RC = 8 * rpw
            xb = (nu * 36 * 4 + 127) & ~127
            if xb + stage > 220 * 1024:
                continue  # the launcher keeps the register-buffer kernel
            assert rs % 16 == 0 and stage % 128 == 0 and RC * rs <= stage and 1 <= kcb and nch >= 1
            assert (nch == 1) == (kcb >= nblk) and (nch > 1 or rs == pitch)
            seen = np.zeros(nblk, np.int64)
            for row0 in range(0, rows, RC) if rows <= 4096 else (0, ((rows - 1) // RC) * RC):
                nrows = min(RC, rows - row0)
                for chunk in range(nch):
                    if nch == 1:
                        copies = [(row0 * pitch, 0, nrows * pitch)]
                        cbytes = pitch
                    else:
                        off = chunk * rs
                        cbytes = min(rs, pitch - off)
                        assert cbytes > 0
                        copies = [((row0 + r) * pitch + off, r * rs, cbytes) for r in range(nrows)]
                    assert sum(c[2] for c in copies) < (1 << 20)
                    for src, dst, n in copies:
                        assert src % 16 == 0 and dst % 16 == 0 and n % 16 == 0
                        assert src + n <= rows * pitch and dst + n <= stage
                    k0 = chunk * kcb
                    nblk_c = min(kcb, nblk - k0)
                    assert nblk_c > 0 and k0 * bb % 16 == 0
                    # compute warps: blocks [0, nblk_c) of each row of the item
                    assert nblk_c * bb <= cbytes
                    if row0 == 0:
                        seen[k0:k0 + nblk_c] += 1
                    if typ in (S.GGML_F32, S.GGML_F16, S.GGML_BF16):
                        words = nblk_c * bb // 16
                        vpw = 4 if typ == S.GGML_F32 else 8
                        assert (nblk_c * bb) % 16 == 0 and k0 * 32 + vpw * words <= nu * 32
            assert np.all(seen == 1), (S.TYPE_NAMES[typ], rows, cols)
