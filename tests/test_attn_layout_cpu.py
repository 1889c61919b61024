"""The decode attention's shared-memory layout (csrc/neon_attn_layout.h, built
for the host) at every ring depth the host may pick, with the kernel's copies
and writes emulated: at the configurations' shapes (and a 16K context) the
regions do not overlap, the ring holds its V tiles and, after the V pass, the
per-part and per-cluster partials that overlay it; every 16-byte copy of a V
row lands 16-byte aligned inside its slot and reads a cache row below the
capacity, as does every float4 read of a K row; the total fits the launch's
shared memory."""
import ctypes as C
import os
import subprocess

import pytest

from conftest import PKG, ROOT

SUB, MAX_SLOTS, SMEM_MAX, THREADS = 64, 8, 200 * 1024, 256


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("attnhost") / "libattnhost.so")
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    subprocess.check_call([nvcc if os.path.exists(nvcc) else "nvcc", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC", "-I", os.path.join(PKG, "csrc"),
                           os.path.join(ROOT, "tests", "cpp", "attn_host.cu"), "-o", so])
    L = C.CDLL(so)
    L.attn_host_layout.argtypes = [C.c_int] * 5 + [C.c_void_p]
    return L


# (name, n_head, n_kv_head, head_dim, ctx_len): the benchmark models' attention shapes
SHAPES = [("llama70b", 64, 8, 128, 2432), ("qwen3", 16, 8, 128, 385), ("phi4", 24, 8, 128, 1152),
          ("tiny", 4, 2, 64, 64), ("tiny-long", 8, 1, 64, 1100), ("wide", 6, 2, 64, 300), ("ctx16k", 64, 8, 128, 16384)]


@pytest.mark.parametrize("name,n_head,n_kv,hd,ctx", SHAPES, ids=[s[0] for s in SHAPES])
def test_layout_and_copies(lib, name, n_head, n_kv, hd, ctx):
    group = n_head // n_kv
    kv_dim = n_kv * hd
    cs = 16 if ctx > 1024 else 8
    chunk_max = -(-ctx // cs)
    items = -(-chunk_max // SUB)  # V tiles of the longest share: the ring's items
    pitch = hd + 16
    nd4 = hd // 4
    parts = THREADS // nd4
    for slots in range(2, max(2, min(MAX_SLOTS, items)) + 1):
        out = (C.c_int * 8)()
        lib.attn_host_layout(group, hd, chunk_max, cs, slots, out)
        q, sc, ring, co, csum, cmax, bar, total = list(out)
        if slots > 2 and total * 4 > SMEM_MAX:
            continue  # attn_pick_slots never takes this depth
        assert total * 4 <= 220 * 1024
        assert q == 0 and sc >= q + group * hd and ring >= sc + group * chunk_max
        assert csum - ring >= max(slots * SUB * pitch, parts * group * hd, cs * group * hd) and co == ring
        assert cmax >= csum + cs * 8 and bar >= cmax + cs * 8 and total == bar + 2 * slots
        assert all(v % 4 == 0 for v in (sc, ring, csum, cmax, bar)) and (bar * 4) % 8 == 0
        # the kernel's accesses at the longest share: V tile t -> slot t % slots as 16-byte
        # copies (row r, float4 column c at ring + slot*SUB*pitch + r*pitch + 4c); K rows read
        # straight from the cache in float4 columns
        L = ctx
        chunk = -(-L // cs)
        for rank in (0, cs - 1):
            s0 = min(L, rank * chunk)
            n = min(L, s0 + chunk) - s0
            n_sub = -(-n // SUB)
            for t in range(n_sub):
                rows = min(SUB, n - t * SUB)
                for r in (0, rows - 1):
                    pos = s0 + t * SUB + r
                    assert pos < ctx
                    for c in (0, nd4 - 1):
                        dst = ring + (t % slots) * SUB * pitch + r * pitch + 4 * c
                        assert (dst * 4) % 16 == 0 and dst + 4 <= ring + slots * SUB * pitch <= csum
                        for kvh in (0, n_kv - 1):
                            src = pos * kv_dim + kvh * hd + 4 * c
                            assert (src * 4) % 16 == 0 and src + 4 <= ctx * kv_dim
                    # its score goes to sc[gq * chunk_max + j0 + r], below the next region
                    assert t * SUB + r < chunk_max
