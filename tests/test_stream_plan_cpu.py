"""The one-position Q4_0 / Q8_0 kernel's tile plans (plan_stream_tiles,
csrc/neon_kernels.cuh, built for the host), with its copy warp and its dot
products emulated on each: the built-in planner's shapes at the benchmark and
model sizes, and every shape neon_cuda_set_stream_tiles can force. Every
cp.async.bulk starts, ends and lands on a 16-byte boundary, reads only the
uploaded planes (payload rows x nb x P bytes; fp16 scales rows x nb plus the
16-byte tail), writes only its stage, and fits one mbarrier phase's byte
count; every scale and payload byte a row's dot product reads was copied;
a shape that does not fit shared memory is reported as such (the launcher
refuses it)."""
import ctypes as C
import os
import subprocess

import pytest

from conftest import PKG, ROOT

Q4_0, Q8_0 = 2, 8
STAGE_TARGET, MAX_SMEM, MAX_STAGES = 80 * 1024, 220 * 1024, 3  # the streaming kernel's stage target


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("streamhost") / "libstreamhost.so")
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    subprocess.check_call([nvcc if os.path.exists(nvcc) else "nvcc", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"),
                           "-I", os.path.join(PKG, "csrc"), os.path.join(ROOT, "tests", "cpp", "stream_host.cu"),
                           "-o", so])
    L = C.CDLL(so)
    L.stream_host_plan.argtypes = [C.c_int, C.c_int, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.c_void_p]
    return L


def plan(L, typ, nb, rows, rc=0, kc=0, sms=148):
    out = (C.c_int * 8)()
    L.stream_host_plan(typ, nb, rows, sms, STAGE_TARGET, MAX_SMEM, rc, kc, out)
    return dict(zip(("rc", "kc", "nch", "stages", "stage_bytes", "smem", "sph", "x_bytes"), out))


def emulate(p, typ, rows, nb):
    """The copy warp's copies and the compute warps' reads of every item of a
    tensor of `rows` x `nb` blocks (first, second and last tiles, every chunk)."""
    P = 16 if typ == Q4_0 else 32
    RC, KC, nch, SPH = p["rc"], p["kc"], p["nch"], p["sph"]
    pay_end, sc_end = rows * nb * P, rows * nb * 2 + 16  # the planes as uploaded
    sc_base = RC * KC * P                                 # the stage's scale area
    assert sc_base % 16 == 0 and (SPH * 2) % 16 == 0 and p["stage_bytes"] % 128 == 0
    n_tiles = (rows + RC - 1) // RC
    for tile in sorted({0, min(1, n_tiles - 1), n_tiles - 1}):
        row0 = tile * RC
        nrows = min(RC, rows - row0)
        for chunk in range(nch):
            k0 = chunk * KC
            kc = min(KC, nb - k0)
            assert kc > 0
            copies = []  # (plane, src byte offset, stage byte offset, bytes)
            if nch == 1:
                e = row0 * nb
                off = e & 7
                copies.append(("pay", e * P, 0, nrows * nb * P))
                copies.append(("sc", (e - off) * 2, sc_base, 2 * ((off + nrows * nb + 7) & ~7)))
            else:
                for r in range(nrows):
                    e = (row0 + r) * nb + k0
                    off = e & 7
                    copies.append(("pay", e * P, r * KC * P, kc * P))
                    copies.append(("sc", (e - off) * 2, sc_base + r * SPH * 2, 2 * ((off + kc + 7) & ~7)))
            assert sum(c[3] for c in copies) < (1 << 20)
            for plane, src, dst, n in copies:
                assert src % 16 == 0 and dst % 16 == 0 and n % 16 == 0, (plane, src, dst, n)
                assert src + n <= (pay_end if plane == "pay" else sc_end), (plane, src, n)
                assert dst + n <= p["stage_bytes"], (plane, dst, n, p["stage_bytes"])
            # the dot products: row r's blocks bi < kc, scale sbase + bi and payload r*KC*P + bi*P
            for r in range(nrows):
                if nch == 1:
                    sbase = ((row0 * nb) & 7) + r * nb
                    window = (0, ((row0 * nb) & 7) + nrows * nb)
                else:
                    sbase = r * SPH + (((row0 + r) * nb + k0) & 7)
                    window = (r * SPH, r * SPH + (((row0 + r) * nb + k0) & 7) + kc)
                assert window[0] <= sbase and sbase + kc <= window[1]
                assert r * KC * P + kc * P <= RC * KC * P


SHAPES = [(Q4_0, 4096, 4096), (Q4_0, 28672, 8192), (Q4_0, 8192, 28672), (Q4_0, 10240, 8192), (Q4_0, 1024, 3072),
          (Q4_0, 6144, 1024), (Q4_0, 1000, 2048), (Q4_0, 3, 256), (Q8_0, 4096, 4096), (Q8_0, 14336, 4096),
          (Q8_0, 4096, 14336), (Q8_0, 151936, 1024), (Q8_0, 128256, 8192), (Q8_0, 300, 14336)]


@pytest.mark.parametrize("typ,rows,cols", SHAPES)
def test_built_in_plans(lib, typ, rows, cols):
    nb = cols // 32
    p = plan(lib, typ, nb, rows)
    assert p["smem"] <= MAX_SMEM and 1 <= p["stages"] <= MAX_STAGES
    assert p["smem"] == p["x_bytes"] + p["stages"] * p["stage_bytes"] + 2 * MAX_STAGES * 8
    emulate(p, typ, rows, nb)


@pytest.mark.parametrize("typ,rows,cols", SHAPES)
def test_every_forced_shape(lib, typ, rows, cols):
    nb = cols // 32
    for rc in (2, 4, 8, 16, 32):
        for kc in sorted({0, 8, 24, 40, 64, 100, 224, nb // 2, nb // 4, max(1, nb // 8), nb, nb + 5}):
            p = plan(lib, typ, nb, rows, rc, kc)
            assert p["rc"] == rc and (p["kc"] == nb if kc <= 0 or kc >= nb else p["kc"] == kc)
            assert p["nch"] == -(-nb // p["kc"])
            if p["smem"] > MAX_SMEM:
                continue  # refused by the launcher before any launch
            emulate(p, typ, rows, nb)
