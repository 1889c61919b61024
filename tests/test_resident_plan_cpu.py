"""The resident one-position kernel's launch arithmetic (csrc/neon_resident.cuh,
built for the host): plans, shared-memory layout, the span pieces every CTA
copies and the reads of its dot products, emulated at the benchmark shapes,
the decode shapes of the three benchmark models (one GPU and tensor-parallel
shards) and ragged multi-target calls.

For every CTA: each cp.async.bulk starts, ends and lands on a 16-byte
boundary, reads only the uploaded planes (payload rows x nb x P bytes; fp16
scales rows x nb plus the 16-byte tail), writes only its area of shared
memory, and the launch's bytes fit one mbarrier phase; every payload and scale
value a row's dot product reads was copied from that row and block; rows per
CTA stay within the kernel's register tiles and even (pair epilogues never
straddle two CTAs); two launches' CTAs fit one SM's shared memory."""
import ctypes as C
import os
import subprocess

import pytest

from conftest import PKG, ROOT

Q4_0, Q8_0 = 2, 8
SMEM_PER_SM = 228 * 1024
STATIC_SMEM = 3 * 1024  # the kernel's static shared memory, bounded (ptxas: under 2.1 KB)
MBAR_TX_MAX = (1 << 20) - 1


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("reshost") / "libreshost.so")
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    subprocess.check_call([nvcc if os.path.exists(nvcc) else "nvcc", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"),
                           "-I", os.path.join(PKG, "csrc"), os.path.join(ROOT, "tests", "cpp", "resident_host.cu"),
                           "-o", so])
    L = C.CDLL(so)
    L.resident_host_plan.argtypes = [C.c_int] * 6 + [C.c_void_p]
    L.resident_host_layout.argtypes = [C.c_int] * 4 + [C.c_void_p]
    L.resident_host_starts.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    L.resident_host_starts.restype = C.c_longlong
    L.resident_host_pieces.argtypes = [C.c_void_p, C.c_void_p] + [C.c_int] * 5 + [C.c_void_p] * 3
    return L


def starts(L, rows):
    n = len(rows)
    r = (C.c_longlong * n)(*rows)
    t = (C.c_int * n)()
    v = L.resident_host_starts(r, n, t)
    return list(t), int(v)


def plan(L, typ, nb, vrows, k, sms=148):
    out = (C.c_int * 5)()
    L.resident_host_plan(typ, nb, vrows, sms, k, SMEM_PER_SM, out)
    return dict(zip(("ok", "tpg", "rpc", "grid", "smem"), out))


def layout(L, typ, nb, rpc, tpg):
    out = (C.c_int * 6)()
    L.resident_host_layout(typ, nb, rpc, tpg, out)
    return dict(zip(("pay", "sc", "bar", "total", "x", "max_rows"), out))


def pieces(L, tile0, rows, v0, nloc, nb, P):
    n = len(rows)
    seg = (C.c_int * (5 * 8))()
    cp = (C.c_longlong * (6 * 8))()
    b = C.c_uint()
    k = L.resident_host_pieces((C.c_int * n)(*tile0), (C.c_int * n)(*rows), n, v0, nloc, nb, P, seg, cp,
                               C.byref(b))
    segs = [dict(zip(("lr0", "n", "span", "row0", "sb"), seg[5 * i:5 * i + 5])) for i in range(k)]
    copies = [dict(zip(("pay_src", "pay_dst", "pay_bytes", "sc_src", "sc_dst", "sc_bytes"), cp[6 * i:6 * i + 6]))
              for i in range(k)]
    return segs, copies, b.value


def check_launch(L, typ, rows, cols, k, sms=148):
    """Emulate every CTA of one launch over targets of `rows` x `cols`;
    returns the plan (ok False: the launcher takes the streaming kernel)."""
    P = 16 if typ == Q4_0 else 32
    nb = cols // 32
    tile0, vrows = starts(L, rows)
    assert all(t % 2 == 0 for t in tile0)
    p = plan(L, typ, nb, vrows, k, sms)
    if not p["ok"]:
        return p
    lay = layout(L, typ, nb, p["rpc"], p["tpg"])
    rpc, grid = p["rpc"], p["grid"]
    assert rpc % 2 == 0 and 2 <= rpc <= lay["max_rows"]
    assert (grid - 1) * rpc < vrows <= grid * rpc
    assert p["smem"] == lay["total"] and lay["total"] + STATIC_SMEM <= 227 * 1024
    per_sm = -(-grid // sms)
    assert 2 * per_sm * (lay["total"] + 1024 + 2048) <= SMEM_PER_SM, "two launches must fit one SM"
    assert lay["x"] <= lay["pay"] and lay["pay"] % 128 == 0 and lay["sc"] % 128 == 0 and lay["bar"] % 8 == 0
    pay_area = lay["sc"] - lay["pay"]
    sc_area_halfs = (lay["bar"] - lay["sc"]) // 2
    for cta in range(grid):
        v0 = cta * rpc
        nloc = min(rpc, vrows - v0)
        assert nloc > 0
        segs, copies, nbytes = pieces(L, tile0, rows, v0, nloc, nb, P)
        assert nbytes <= MBAR_TX_MAX
        assert nbytes == sum(c["pay_bytes"] + c["sc_bytes"] for c in copies)
        covered = set()
        for s, c in zip(segs, copies):
            r = rows[s["span"]]
            assert 0 <= s["row0"] and s["row0"] + s["n"] <= r
            assert s["lr0"] == tile0[s["span"]] + s["row0"] - v0
            # payload copy
            for v in (c["pay_src"], c["pay_dst"], c["pay_bytes"]):
                assert v % 16 == 0
            assert c["pay_src"] + c["pay_bytes"] <= r * nb * P
            assert c["pay_dst"] >= 0 and c["pay_dst"] + c["pay_bytes"] <= pay_area
            # scale window
            assert (2 * c["sc_src"]) % 16 == 0 and (2 * c["sc_dst"]) % 16 == 0 and c["sc_bytes"] % 16 == 0
            assert c["sc_src"] >= 0 and 2 * c["sc_src"] + c["sc_bytes"] <= r * nb * 2 + 16
            assert c["sc_dst"] >= 0 and 2 * c["sc_dst"] + c["sc_bytes"] <= 2 * sc_area_halfs
            # every read of the piece's rows lands on the copied value of that row and block
            for lr in sorted({s["lr0"], s["lr0"] + s["n"] - 1}):
                row = s["row0"] + lr - s["lr0"]
                for b in sorted({0, nb // 2, nb - 1}):
                    pay_idx = (lr * nb + b) * P
                    assert c["pay_dst"] <= pay_idx and pay_idx + P <= c["pay_dst"] + c["pay_bytes"]
                    assert c["pay_src"] + (pay_idx - c["pay_dst"]) == (row * nb + b) * P
                    sc_idx = s["sb"] + lr * nb + b
                    assert c["sc_dst"] <= sc_idx < c["sc_dst"] + c["sc_bytes"] // 2
                    assert c["sc_src"] + (sc_idx - c["sc_dst"]) == row * nb + b
            covered.update(range(s["lr0"], s["lr0"] + s["n"]))
        # local rows of no span are span padding (one row before a span that starts odd)
        for lr in set(range(nloc)) - covered:
            v = v0 + lr
            assert any(v + 1 == t for t in tile0), "an uncovered row must be the padding before a span"
            assert (lr * nb + nb) * P <= pay_area and nb <= sc_area_halfs  # its (unused) reads stay in bounds
    return p


def model_shapes(n_embd, q_dim, kv_dim, n_ff, world):
    """(rows list, cols) of a decode step's one-position launches on one rank."""
    q, kv, ff = q_dim // world, kv_dim // world, n_ff // world
    return [((q, kv, kv), n_embd), ((n_embd,), q), ((2 * ff,), n_embd), ((n_embd,), ff)]


MODELS = {
    "qwen3_0_6b": (1024, 2048, 1024, 3072),
    "phi4_mini": (3072, 3072, 1024, 8192),
    "llama3_70b": (8192, 8192, 1024, 28672),
}


@pytest.mark.parametrize("k", [1, 2, 4])
@pytest.mark.parametrize("typ", [Q4_0, Q8_0])
def test_benchmark_shapes(lib, typ, k):
    for rows, cols in [((4096,), 4096), ((14336,), 4096), ((4096,), 14336), ((28672,), 8192), ((8192,), 28672)]:
        check_launch(lib, typ, list(rows), cols, k)
    # the headline matvec takes the resident kernel at the default setting
    if typ == Q4_0:
        assert check_launch(lib, typ, [4096], 4096, 1)["ok"]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("model", sorted(MODELS))
def test_decode_shapes(lib, model, world):
    n_embd, q_dim, kv_dim, n_ff = MODELS[model]
    for rows, cols in model_shapes(n_embd, q_dim, kv_dim, n_ff, world):
        for k in (1, 2, 4):
            check_launch(lib, Q4_0, list(rows), cols, k)
    # the small model's projections are all resident
    if model == "qwen3_0_6b" and world == 1:
        for rows, cols in model_shapes(n_embd, q_dim, kv_dim, n_ff, world):
            assert check_launch(lib, Q4_0, list(rows), cols, 1)["ok"], (rows, cols)


@pytest.mark.parametrize("typ", [Q4_0, Q8_0])
@pytest.mark.parametrize("rows,cols", [((33, 65, 7), 800), ((1,), 32), ((5, 3, 1), 32), ((2048, 2049), 288),
                                       ((3,), 64), ((129,), 8192), ((301,), 800), ((77,), 1152),
                                       ((257, 130), 4096), ((7, 9, 11, 13, 15, 17, 19, 21), 224)])
def test_ragged_targets(lib, typ, rows, cols):
    for k in (1, 2, 4):
        for sms in (148, 132, 8):
            check_launch(lib, typ, list(rows), cols, k, sms)
