"""The index arithmetic of the register-tiled fp32 prompt attention
(attn_prefill_f32_kernel in csrc/neon_decode.cu), emulated on the CPU for
several prompt shapes, positions and head dims: grid (query heads, 64-position
tiles), 256 threads as a 16 x 16 grid (ty, tx) owning rows 4ty.. of the tile,
keys 4tx.. of each 64-key tile and output dims (hd/16)tx..; the key tiles
cover [0, base + t0 + nq). Checked: every (position, key <= position) pair of
a live row is scored exactly once per pass and no key past a row's position
is admitted; every output element of every live row is written exactly once
and no element of a dead row is; every global load (Q, K, V rows, float4
along the head dim) and store stays inside its buffer and is 16-byte
aligned; every shared-memory access stays inside its region (112 KB at
head_dim 128: two CTAs per SM)."""
import numpy as np
import pytest

ROWS, KEYS, THREADS = 64, 64, 256


def smem_floats(hd):
    return hd * ROWS + hd * KEYS + KEYS * hd + KEYS * ROWS


# (seq, base, n_head, n_kv, hd, ctx): prompt chunks as forward_device issues them
CASES = [(256, 0, 4, 2, 64, 300), (1, 37, 8, 1, 128, 64), (70, 130, 6, 2, 64, 300), (256, 1792, 64, 8, 128, 2432),
         (33, 0, 16, 8, 128, 40)]


@pytest.mark.parametrize("seq,base,n_head,n_kv,hd,ctx", CASES)
def test_prefill_attention_tiling(seq, base, n_head, n_kv, hd, ctx):
    assert base + seq <= ctx
    group, dpt = n_head // n_kv, hd // 16
    q_dim, kv_dim = n_head * hd, n_kv * hd
    assert smem_floats(128) * 4 == 112 * 1024 and 2 * (smem_floats(128) * 4 + 1024) <= 228 * 1024
    tid = np.arange(THREADS)
    tx, ty = tid & 15, tid >> 4
    for h in sorted({0, n_head - 1}):  # the other heads differ by an offset only
        kvh = h // group
        for by in range(-(-seq // ROWS)):
            t0 = by * ROWS
            nq = min(ROWS, seq - t0)
            kend = base + t0 + nq
            ntiles = -(-kend // KEYS)
            assert kend <= ctx
            # Q staging: i -> (r, d4), loads of live rows only, transposed stores into qt [hd][64]
            i = np.arange(ROWS * (hd // 4))
            r, d4 = i % ROWS, i // ROWS
            live_q = r < nq
            src = (t0 + r[live_q]) * q_dim + h * hd + 4 * d4[live_q]
            assert src.min() >= 0 and (src + 3).max() < seq * q_dim and np.all(src % 4 == 0)
            assert (4 * d4 + 3).max() * ROWS + r.max() < hd * ROWS
            # K / V staging per tile: loads only below kend, stores inside kt / vs
            for t in range(ntiles):
                key = t * KEYS + (i % KEYS)
                ok = key < kend
                k_src = key[ok] * kv_dim + kvh * hd + 4 * (i // KEYS)[ok]
                assert (k_src + 3).max() < ctx * kv_dim and np.all(k_src % 4 == 0)
                rv, dv = i // (hd // 4), i % (hd // 4)
                assert (rv * hd + 4 * dv + 3).max() < KEYS * hd
            # pass structure: each thread's rows and keys, the causal mask
            scored = np.zeros((ROWS, kend), np.int32)
            for t in range(ntiles):
                for j in range(4):
                    for ii in range(4):
                        rows = 4 * ty + ii
                        keys = t * KEYS + 4 * tx + j
                        live = rows < nq
                        on = live & (keys <= base + t0 + rows)
                        assert np.all(keys[on] < kend)
                        np.add.at(scored, (rows[on], keys[on]), 1)
                        # p stored transposed at pt[(4tx + j) * 64 + 4ty ..]: inside [64 keys][64 rows]
                        assert ((4 * tx + j) * ROWS + 4 * ty + 3).max() < KEYS * ROWS
            for rr in range(nq):
                want = np.zeros(kend, np.int32)
                want[:base + t0 + rr + 1] = 1
                assert np.array_equal(scored[rr], want), (h, t0, rr)
            assert not scored[nq:].any()
            # outputs: rows 4ty+i (live), dims dpt*tx .. +dpt, float4 stores
            written = np.zeros((ROWS, hd), np.int32)
            for ii in range(4):
                rows = 4 * ty + ii
                live = rows < nq
                if not live.any():
                    continue
                for c in range(0, dpt, 4):
                    dst = (t0 + rows[live]) * q_dim + h * hd + dpt * tx[live] + c
                    assert (dst + 3).max() < seq * q_dim and np.all(dst % 4 == 0)
                    for e in range(4):
                        np.add.at(written, (rows[live], dpt * tx[live] + c + e), 1)
            assert np.all(written[:nq] == 1) and not written[nq:].any()
