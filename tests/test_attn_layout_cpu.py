"""The decode attention's shared-memory layout (csrc/neon_attn_layout.h, built
for the host) at every ring depth the host may pick, with the kernel's copies
and writes emulated: at the configurations' shapes (and a 16K context) the
regions do not overlap, the ring holds its K and V tiles and, after the V
pass, the per-part and per-cluster partials that overlay it; every TMA box
lands 128-byte aligned inside its slot and starts at a cache row below the
capacity and a 16-byte-aligned column; the mbarriers are 8-byte aligned; the
total fits the launch's shared memory."""
import ctypes as C
import os
import subprocess

import pytest

from conftest import PKG, ROOT

SUB, BOX, MAX_SLOTS, SMEM_MAX, THREADS = 64, 16, 8, 200 * 1024, 256


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
    items = 2 * (-(-chunk_max // SUB))  # K then V tiles of the longest share: the ring's items
    pitch = hd
    parts = THREADS // (hd // 4)
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
        assert all(v % 4 == 0 for v in (sc, csum, cmax, bar)) and (bar * 4) % 8 == 0 and (ring * 4) % 128 == 0
        # the kernel's TMA copies at the longest share: item t (K tiles, then V tiles) -> slot
        # t % slots, box b of BOX rows at ring + slot*SUB*hd + b*BOX*hd, from cache row
        # s0 + j0 + b*BOX, column kvh*hd; rows past the cache's end arrive as zeros
        L = ctx
        chunk = -(-L // cs)
        for rank in (0, cs - 1):
            s0 = min(L, rank * chunk)
            n = min(L, s0 + chunk) - s0
            n_sub = -(-n // SUB)
            for t in range(2 * n_sub):
                sub = t - n_sub if t >= n_sub else t
                rows = min(SUB, n - sub * SUB)
                boxes = -(-rows // BOX)
                assert boxes * BOX * hd * 4 < (1 << 20)  # one mbarrier phase's byte count
                for b in range(boxes):
                    dst = ring + (t % slots) * SUB * pitch + b * BOX * pitch
                    assert (dst * 4) % 128 == 0 and dst + BOX * pitch <= ring + slots * SUB * pitch <= csum
                    y = s0 + sub * SUB + b * BOX
                    assert 0 <= y < ctx
                    for kvh in (0, n_kv - 1):
                        x = kvh * hd
                        assert (x * 4) % 16 == 0 and x + hd <= kv_dim
                # its scores go to sc[gq * chunk_max + j0 + r], r < rows, below the next region
                if t < n_sub:
                    assert sub * SUB + rows <= chunk_max
