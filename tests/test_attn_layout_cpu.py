"""The decode attention's cluster split and shared-memory layout
(csrc/neon_attn_layout.h, built for the host), with the kernel's copies,
rounds and exchanges emulated at every context length the benchmark models
and a 16K context reach, for cluster caps of 16 and 8 and several row
settings: the CTAs' shares cover [0, L) once with at most cs CTAs; every TMA
box (K rounds, then V rounds, item t in slot t % 2; one round-sized box per
dim block, or 32-row boxes for the item with the new row) starts at a cache row
below ctx_len, a 128-byte-aligned column and a 1024-byte-aligned offset
inside its slot; the K box with the new row is issued once, by the last
active CTA, after the dependency wait; the scores fit their region;
the maxima exchange fits the CTA's threads; the warps' p*v sums overlay
slot 0 only when they fit it; the partial-product region holds the CTA's o
for CTA 0 to read; the total fits the launch's shared memory."""
import ctypes as C
import os
import subprocess

import pytest

from conftest import PKG, ROOT

BOX, MIN_SCORES, SMEM_MAX, THREADS, WARPS = 32, 256, 200 * 1024, 256, 8


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("attnhost") / "libattnhost.so")
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    subprocess.check_call([nvcc if os.path.exists(nvcc) else "nvcc", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC", "-I", os.path.join(PKG, "csrc"),
                           os.path.join(ROOT, "tests", "cpp", "attn_host.cu"), "-o", so])
    L = C.CDLL(so)
    L.attn_host_layout.argtypes = [C.c_int] * 6 + [C.c_void_p]
    L.attn_host_plan.argtypes = [C.c_int] * 5 + [C.c_void_p]
    L.attn_host_rows.argtypes = [C.c_int] * 3
    return L


# (name, n_head, n_kv_head, head_dim, ctx_len): the benchmark models' attention shapes
SHAPES = [("llama70b", 64, 8, 128, 2432), ("qwen3", 16, 8, 128, 385), ("phi4", 24, 8, 128, 1152),
          ("tiny", 4, 2, 64, 64), ("tiny-long", 8, 1, 64, 1100), ("wide", 6, 2, 64, 300),
          ("hd256", 16, 2, 256, 4096), ("ctx16k", 64, 8, 128, 16384)]
ROWS = [(32, 128), (32, 32), (64, 64), (256, 1024)]  # (min_rows, share_rows)


def contexts(ctx):
    ls = set(range(1, min(ctx, 300) + 1)) | {ctx, ctx - 1, ctx // 2, ctx // 3 + 1}
    ls |= set(range(BOX - 1, ctx + 1, max(1, ctx // 97)))
    return sorted(l for l in ls if 1 <= l <= ctx)


@pytest.mark.parametrize("min_rows,share_rows", ROWS, ids=[f"{a}-{b}" for a, b in ROWS])
@pytest.mark.parametrize("name,n_head,n_kv,hd,ctx", SHAPES, ids=[s[0] for s in SHAPES])
def test_split_layout_and_copies(lib, name, n_head, n_kv, hd, ctx, min_rows, share_rows):
    group = n_head // n_kv
    bw = 32
    nbk = hd // bw
    for cs_max in (16, 8):
        plan = (C.c_int * 5)()
        assert lib.attn_host_plan(ctx, group, hd, cs_max, share_rows, plan)
        gp, cs, rr, score_rows, smem = list(plan)
        assert gp in (1, 2, 4, 8) and gp >= group and cs in (1, 2, 4, 8, 16) and cs <= cs_max
        up = lambda v: -(-v // BOX) * BOX
        share = up(-(-ctx // cs))
        assert share <= share_rows or cs == cs_max  # the smallest cluster for the share
        assert cs == 1 or up(-(-ctx // (cs // 2))) > share_rows
        assert rr % BOX == 0 and BOX <= rr <= share and score_rows >= max(share, MIN_SCORES)
        assert smem <= SMEM_MAX
        if smem > 112 * 1024:  # one CTA per SM only where no round size fits two
            small = (C.c_int * 12)()
            lib.attn_host_layout(hd, gp, bw, BOX, score_rows, cs, small)
            assert small[11] * 4 > 112 * 1024
        out = (C.c_int * 12)()
        lib.attn_host_layout(hd, gp, bw, rr, score_rows, cs, out)
        k, v, ps, sc, q, red, wm, wl, cmax, lsum, bar, total = list(out)
        assert smem == 4 * total
        assert k == 0 and v == rr * hd and (v * 4) % 1024 == 0 and ps == v + rr * hd
        assert sc >= ps + nbk * rr * gp and q >= sc + score_rows * gp and sc % 4 == 0 and q % 4 == 0
        end_q = q + gp * hd
        red_n = WARPS * gp * hd
        assert (red == k and red_n <= rr * hd) or (red >= end_q and red % 4 == 0)
        assert wm >= (red + red_n if red != k else end_q) and wl >= wm + WARPS * gp
        assert cmax >= wl + WARPS * gp and lsum >= cmax + cs * gp and bar >= lsum + gp and (bar * 4) % 8 == 0
        assert total == bar + 10  # five mbarriers
        assert gp * hd <= 8 * 256  # the kernel's output elements per thread: 8
        assert nbk * rr * gp >= gp * hd  # ps holds the CTA's o [gp][hd] at the end
        for world in (1, 2, 8):
            if n_kv % world:
                continue
            kv_dim = n_kv // world * hd
            for L in contexts(ctx):
                pos = L - 1
                rows = lib.attn_host_rows(L, cs, min(min_rows, score_rows))
                assert rows % BOX == 0 and rows <= score_rows
                n_act = -(-L // rows)
                assert 1 <= n_act <= cs and n_act * gp <= THREADS  # the maxima exchange
                covered = post = 0
                for rank in range(cs):
                    s0 = rank * rows
                    if s0 >= L:
                        continue
                    n = min(rows, L - s0)
                    assert s0 == covered
                    covered += n
                    nr = -(-n // rr)
                    for t in range(2 * nr):  # items: K rounds, then V rounds; item t in slot t % 2
                        r0 = (t % nr) * rr
                        nrb = -(-min(rr, n - r0) // BOX)
                        base = v if t % 2 else k
                        if pos >= s0 + r0 + nrb * BOX:  # no new row: one round-sized box per dim block
                            assert rr <= 256 and nbk * rr * bw * 4 < (1 << 20)
                            assert 0 <= s0 + r0 < ctx and s0 + r0 + rr - 1 >= s0 + min(rr, n - r0) - 1
                            for nb in range(nbk):
                                dst = base + nb * rr * bw
                                assert (dst * 4) % 1024 == 0 and dst + rr * bw <= base + rr * hd
                            continue
                        assert rank == n_act - 1 and t % nr == nr - 1  # the last CTA's last round
                        assert nrb * nbk * bw * BOX * 4 < (1 << 20)  # one mbarrier phase's byte count
                        for rb in range(nrb):
                            y = s0 + r0 + rb * BOX
                            assert 0 <= y <= pos < ctx
                            if pos < y + BOX and t < nr:  # the K box with the new row: after the wait
                                post += 1
                            for nb in range(nbk):
                                dst = base + (nb * rr + rb * BOX) * bw
                                assert (dst * 4) % 1024 == 0 and dst + BOX * bw <= base + rr * hd
                                for kvh in (0, kv_dim // hd - 1):
                                    x = kvh * hd + nb * bw
                                    assert (x * 4) % 128 == 0 and x + bw <= kv_dim
                assert covered == L and post == 1
