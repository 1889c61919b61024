"""The index arithmetic of the tensor-core prefill kernels
(csrc/neon_prefill.cuh: matvec_mma_q4_0_kernel, and below matvec_mma_q8_0_kernel),
emulated on the CPU: the
staging of weights and activations into shared memory, every lane's MMA
fragments (PTX ISA layouts of mma.m16n8k32 .s8: A rows g / g+8 with values
4t..4t+3 and 16+4t..; B values 4t.. / 16+4t.. of column g; D rows g / g+8,
columns 2t, 2t+1), the integer products, and the scale pair each lane applies.
Every lane's block step must see exactly the reference's isum of its (row,
position, block) and the scales d_w[row, block], d_x[position, block]: then
its fma sequence is dot_q4_0_q8_0's, and the outputs are the reference's
bit for bit."""
import numpy as np
import pytest

import oracle as O
import synth as S

ROWS_T, POS_T, KB, WARPS = 64, 64, 4, 4
WP, XP = KB + 1, 2 * KB + 1  # staged pitches in 16-byte words


def vsub4(u, v):
    """__vsub4: per-byte subtraction, wrapping."""
    out = np.zeros_like(u)
    for i in range(4):
        sh = np.uint32(8 * i)
        out |= (((u >> sh) - (np.uint32(v) >> sh)) & np.uint32(0xFF)) << sh
    return out


def s8(word, i):
    return ((word >> np.uint32(8 * i)) & np.uint32(0xFF)).astype(np.uint8).view(np.int8).astype(np.int64)


def emulate(W, rows, cols, X):
    seq, nb = X.shape[0], cols // 32
    d, q = O.quantize_rows_q8_0(X)  # the device quantiser is bit-exact with this
    blocks = W.reshape(rows, nb, 18)
    payload = np.ascontiguousarray(blocks[:, :, 2:]).reshape(rows, nb, 16)
    wscale = blocks[:, :, :2].copy().view(np.float16).astype(np.float32).reshape(rows, nb)
    # expected per (row, pos, block): the exact integer sum and the scale pair
    qw = np.concatenate([(payload & 0xF).astype(np.int64) - 8, (payload >> 4).astype(np.int64) - 8], axis=2)
    isum = np.einsum("rbk,pbk->rpb", qw, q.reshape(seq, nb, 32).astype(np.int64))
    seen = np.zeros((rows, seq, nb), bool)
    lanes = np.arange(32)
    g, t = lanes // 4, lanes % 4
    for tile in range((rows + ROWS_T - 1) // ROWS_T):
        row0 = tile * ROWS_T
        for p0 in range(0, seq, POS_T):
            for c in range((nb + KB - 1) // KB):
                b0 = c * KB
                # the staged chunk, by the kernel's load/store indices
                sw = np.zeros((ROWS_T * WP, 16), np.uint8)
                swd = np.zeros(ROWS_T * KB, np.float32)
                sx = np.zeros((POS_T * XP, 16), np.uint8)
                sxd = np.zeros(POS_T * KB, np.float32)
                for tid in range(128):
                    for i in range(2):
                        idx = tid + 128 * i
                        row, kb = idx // KB, idx % KB
                        gr, gb = row0 + row, b0 + kb
                        if gr < rows and gb < nb:
                            sw[row * WP + kb] = payload[gr, gb]
                            swd[idx] = wscale[gr, gb]
                        gp = p0 + idx // KB
                        if gp < seq and gb < nb:
                            sxd[idx] = d[gp, gb]
                    for i in range(4):
                        idx = tid + 128 * i
                        pos, piece = idx // (2 * KB), idx % (2 * KB)
                        gp, gb = p0 + pos, b0 + piece // 2
                        if gp < seq and gb < nb:
                            sx[pos * XP + piece] = q[gp, gb * 32 + (piece & 1) * 16:gb * 32 + (piece & 1) * 16 + 16].view(np.uint8)
                w32 = sw.view(np.uint32).reshape(ROWS_T * WP, 4)
                x32 = sx.view(np.uint32).reshape(POS_T * XP, 4)
                for kb in range(min(KB, nb - b0)):
                    for w in range(WARPS):
                        wr = 16 * w
                        ug, ug8 = w32[(wr + g) * WP + kb, t], w32[(wr + g + 8) * WP + kb, t]
                        a = [vsub4(ug & np.uint32(0x0F0F0F0F), 0x08080808),
                             vsub4(ug8 & np.uint32(0x0F0F0F0F), 0x08080808),
                             vsub4((ug >> np.uint32(4)) & np.uint32(0x0F0F0F0F), 0x08080808),
                             vsub4((ug8 >> np.uint32(4)) & np.uint32(0x0F0F0F0F), 0x08080808)]
                        wdg, wdg8 = swd[(wr + g) * KB + kb], swd[(wr + g + 8) * KB + kb]
                        for j in range(8):
                            b0w = x32[(8 * j + g) * XP + 2 * kb, t]
                            b1w = x32[(8 * j + g) * XP + 2 * kb + 1, t]  # bytes 16+4t: word 4+t of the block
                            A = np.zeros((16, 32), np.int64)
                            B = np.zeros((32, 8), np.int64)
                            for l in range(32):
                                for i in range(4):
                                    A[g[l], 4 * t[l] + i] = s8(a[0][l], i)
                                    A[g[l] + 8, 4 * t[l] + i] = s8(a[1][l], i)
                                    A[g[l], 16 + 4 * t[l] + i] = s8(a[2][l], i)
                                    A[g[l] + 8, 16 + 4 * t[l] + i] = s8(a[3][l], i)
                                    B[4 * t[l] + i, g[l]] = s8(b0w[l], i)
                                    B[16 + 4 * t[l] + i, g[l]] = s8(b1w[l], i)
                            D = A @ B
                            for l in range(32):
                                xd0 = sxd[(8 * j + 2 * t[l]) * KB + kb]
                                xd1 = sxd[(8 * j + 2 * t[l] + 1) * KB + kb]
                                for e, (dr, dc, wsc, xsc) in enumerate(((0, 0, wdg[l], xd0), (0, 1, wdg[l], xd1),
                                                                         (8, 0, wdg8[l], xd0), (8, 1, wdg8[l], xd1))):
                                    r = row0 + wr + g[l] + dr
                                    p = p0 + 8 * j + 2 * t[l] + dc
                                    if r < rows and p < seq:
                                        b = b0 + kb
                                        assert D[g[l] + dr, 2 * t[l] + dc] == isum[r, p, b], (r, p, b)
                                        assert wsc == wscale[r, b] and xsc == d[p, b], (r, p, b)
                                        assert not seen[r, p, b]
                                        seen[r, p, b] = True
    assert seen.all(), "some (row, position, block) never reached an accumulator"


@pytest.mark.parametrize("rows,cols,seq", [(70, 320, 9), (64, 128, 66)])
def test_prefill_mma_fragments_reach_every_block_once(rows, cols, seq):
    W = S.weights(S.GGML_Q4_0, rows, cols, seed=rows + seq)
    X = S.activations(seq, cols, seed=seq)
    emulate(W, rows, cols, X)


KB8, WP8, XP8 = 2, 5, 17  # the Q8_0 kernel: blocks per chunk, staged pitches (uint4 / float4)


def emulate_q8(W, rows, cols, X):
    """matvec_mma_q8_0_kernel's staging and m16n8k8 TF32 fragments (A rows g /
    g+8, values t and t+4 of each 8-value step; B values t, t+4 of column g; D
    rows g / g+8, columns 2t, 2t+1): every lane's block step must sum exactly
    q[row, block, :] . x[pos, block, :] and scale it by d_w[row, block]."""
    seq, nb = X.shape[0], cols // 32
    blocks = W.reshape(rows, nb, 34)
    q = np.ascontiguousarray(blocks[:, :, 2:]).view(np.int8).reshape(rows, nb, 32).astype(np.float64)
    wscale = blocks[:, :, :2].copy().view(np.float16).astype(np.float32).reshape(rows, nb)
    xb = X.reshape(seq, nb, 32).astype(np.float64)
    want = np.einsum("rbk,pbk->rpb", q, xb)
    seen = np.zeros((rows, seq, nb), bool)
    lanes = np.arange(32)
    g, t = lanes // 4, lanes % 4
    for tile in range((rows + ROWS_T - 1) // ROWS_T):
        row0 = tile * ROWS_T
        for p0 in range(0, seq, POS_T):
            for c in range((nb + KB8 - 1) // KB8):
                b0 = c * KB8
                sw = np.zeros((ROWS_T * WP8, 16), np.uint8)
                swd = np.zeros(ROWS_T * KB8, np.float32)
                sx = np.zeros((POS_T * XP8, 4), np.float32)
                for tid in range(128):
                    for i in range(2):
                        idx = tid + 128 * i
                        row, piece = idx // (2 * KB8), idx % (2 * KB8)
                        gr, gb = row0 + row, b0 + piece // 2
                        if gr < rows and gb < nb:
                            sw[row * WP8 + piece] = blocks[gr, gb, 2 + (piece & 1) * 16:2 + (piece & 1) * 16 + 16]
                    row, kb = tid // KB8, tid % KB8
                    if row0 + row < rows and b0 + kb < nb:
                        swd[tid] = wscale[row0 + row, b0 + kb]
                    for i in range(8):
                        idx = tid + 128 * i
                        pos, piece = idx // (8 * KB8), idx % (8 * KB8)
                        gp, gb = p0 + pos, b0 + piece // 8
                        if gp < seq and gb < nb:
                            sx[pos * XP8 + piece] = X[gp, gb * 32 + (piece & 7) * 4:gb * 32 + (piece & 7) * 4 + 4]
                sq = sw.view(np.int8).reshape(ROWS_T * WP8 * 16)
                sxf = sx.reshape(-1)
                for kb in range(min(KB8, nb - b0)):
                    for w in range(WARPS):
                        wr = 16 * w
                        for j in range(8):
                            D = np.zeros((16, 8))
                            for ks in range(4):
                                A = np.zeros((16, 8))
                                B = np.zeros((8, 8))
                                for l in range(32):
                                    qg = ((wr + g[l]) * WP8 + 2 * kb) * 16
                                    qg8 = ((wr + g[l] + 8) * WP8 + 2 * kb) * 16
                                    xs = ((8 * j + g[l]) * XP8 + 8 * kb) * 4
                                    A[g[l], t[l]] = sq[qg + 8 * ks + t[l]]
                                    A[g[l] + 8, t[l]] = sq[qg8 + 8 * ks + t[l]]
                                    A[g[l], t[l] + 4] = sq[qg + 8 * ks + t[l] + 4]
                                    A[g[l] + 8, t[l] + 4] = sq[qg8 + 8 * ks + t[l] + 4]
                                    B[t[l], g[l]] = sxf[xs + 8 * ks + t[l]]
                                    B[t[l] + 4, g[l]] = sxf[xs + 8 * ks + t[l] + 4]
                                D += A @ B
                            for l in range(32):
                                dg, dg8 = swd[(wr + g[l]) * KB8 + kb], swd[(wr + g[l] + 8) * KB8 + kb]
                                for dr, dc, sc in ((0, 0, dg), (0, 1, dg), (8, 0, dg8), (8, 1, dg8)):
                                    r, p = row0 + wr + g[l] + dr, p0 + 8 * j + 2 * t[l] + dc
                                    if r < rows and p < seq:
                                        b = b0 + kb
                                        assert abs(D[g[l] + dr, 2 * t[l] + dc] - want[r, p, b]) <= 1e-9 * (1 + abs(want[r, p, b]))
                                        assert sc == wscale[r, b] and not seen[r, p, b]
                                        seen[r, p, b] = True
    assert seen.all()


@pytest.mark.parametrize("rows,cols,seq", [(70, 160, 9), (64, 64, 66)])
def test_prefill_mma_q8_0_fragments(rows, cols, seq):
    W = S.weights(S.GGML_Q8_0, rows, cols, seed=rows + seq)
    X = S.activations(seq, cols, seed=seq)
    emulate_q8(W, rows, cols, X)


def test_mma_float_bias_is_exact():
    """The Q4_0 prefill kernel seeds its int32 MMA accumulator with 0x4B400000
    and reads D as a float: 1.5 * 2^23 + isum exactly, so D - 12582912.0f is
    (float)isum for every block sum a Q4_0 x Q8_0 block can give
    (|isum| <= 32 * 8 * 127 < 2^22) -- checked over the whole range."""
    isum = np.arange(-32 * 8 * 127, 32 * 8 * 127 + 1, dtype=np.int64)
    d = (isum + 0x4B400000).astype(np.int32)
    f = d.view(np.float32) - np.float32(12582912.0)
    assert np.array_equal(f, isum.astype(np.float32))
    assert 32 * 8 * 127 < 2 ** 22


def test_tf32_split_carries_fp32():
    """x_hi + x_lo, each rounded to TF32 (10 mantissa bits, nearest, ties away
    as cvt.rna), reproduces x to within 2^-21 relative: the Q8_0 kernel's
    products q*x_hi + q*x_lo are fp32-accurate."""
    x = np.random.default_rng(1).standard_normal(200000).astype(np.float32)

    def tf32(v):
        u = v.view(np.uint32).astype(np.uint64)
        u = (u + 0x1000) & ~np.uint64(0x1FFF)  # round half away on the 13 dropped bits, clear them
        return u.astype(np.uint32).view(np.float32)

    hi = tf32(x)
    lo = tf32((x - hi).astype(np.float32))
    rel = np.abs((hi.astype(np.float64) + lo) - x) / np.abs(x)
    assert rel.max() <= 2.0 ** -21


def fast_expf(x):
    """engine::fast_expf (rawllm_common.hpp:88-100), as oracle_fast_expf restates it."""
    L = O.lib()
    import ctypes as C
    L.oracle_fast_expf.argtypes = [C.c_float]
    L.oracle_fast_expf.restype = C.c_float
    return np.array([L.oracle_fast_expf(float(v)) for v in np.ravel(x)], np.float64).reshape(np.shape(x))


def emulate_attention(q, K, V, base, hd, group, scale):
    """attn_prefill_mma_kernel's lanes (products in float64, no TF32 error):
    pass 1 row maxima of the masked scaled scores, pass 2 p, sums and P.V, by
    the kernel's fragment mapping of mma.m16n8k8 (A rows g / g+8, values t and
    t+4; B values t / t+4 of column g; C rows g / g+8, columns 2t, 2t+1)."""
    seq, q_dim = q.shape
    n_head = q_dim // hd
    out = np.zeros((seq, q_dim))
    lanes = np.arange(32)
    g, tq = lanes // 4, lanes % 4
    for h in range(n_head):
        kvh = h // group
        for t0 in range(0, seq, 64):
            nq = min(64, seq - t0)
            kend = base + t0 + nq
            Qs = np.zeros((64, hd))
            Qs[:nq] = q[t0:t0 + nq, h * hd:(h + 1) * hd]
            for w in range(4):
                r0, r1 = w * 16 + g, w * 16 + g + 8
                ok0, ok1 = t0 + r0 < seq, t0 + r1 < seq
                pos0, pos1 = base + t0 + r0, base + t0 + r1
                tiles = []
                for kt in range((kend + 63) // 64):
                    Ks = np.zeros((64, hd))
                    Vs = np.zeros((64, hd))
                    keys = np.arange(kt * 64, kt * 64 + 64)
                    valid = keys < kend
                    Ks[valid] = K[keys[valid], kvh * hd:(kvh + 1) * hd]
                    Vs[valid] = V[keys[valid], kvh * hd:(kvh + 1) * hd]
                    # scores: sc[lane][j][e] from the fragments
                    sc = np.zeros((32, 8, 4))
                    for ks in range(hd // 8):
                        A = np.zeros((16, 8))
                        for l in range(32):
                            A[g[l], tq[l]] = Qs[r0[l], 8 * ks + tq[l]]
                            A[g[l] + 8, tq[l]] = Qs[r1[l], 8 * ks + tq[l]]
                            A[g[l], tq[l] + 4] = Qs[r0[l], 8 * ks + tq[l] + 4]
                            A[g[l] + 8, tq[l] + 4] = Qs[r1[l], 8 * ks + tq[l] + 4]
                        for j in range(8):
                            B = np.zeros((8, 8))
                            for l in range(32):
                                B[tq[l], g[l]] = Ks[8 * j + g[l], 8 * ks + tq[l]]
                                B[tq[l] + 4, g[l]] = Ks[8 * j + g[l], 8 * ks + tq[l] + 4]
                            C = A @ B
                            sc[:, j, 0] += C[g, 2 * tq]
                            sc[:, j, 1] += C[g, 2 * tq + 1]
                            sc[:, j, 2] += C[g + 8, 2 * tq]
                            sc[:, j, 3] += C[g + 8, 2 * tq + 1]
                    tiles.append((kt, sc * scale, Vs))
                # pass 1
                m0 = np.full(32, -np.inf)
                m1 = np.full(32, -np.inf)
                for kt, sc, _ in tiles:
                    for j in range(8):
                        for e in range(4):
                            key = kt * 64 + 8 * j + 2 * tq + (e & 1)
                            if e < 2:
                                on = ok0 & (key <= pos0)
                                m0 = np.where(on, np.maximum(m0, sc[:, j, e]), m0)
                            else:
                                on = ok1 & (key <= pos1)
                                m1 = np.where(on, np.maximum(m1, sc[:, j, e]), m1)
                for o in (1, 2):  # the shuffle over the 4 lanes of a row
                    m0 = np.maximum(m0, m0[lanes ^ o])
                    m1 = np.maximum(m1, m1[lanes ^ o])
                # pass 2
                acc = np.zeros((32, hd // 8, 4))
                l0 = np.zeros(32)
                l1 = np.zeros(32)
                for kt, sc, Vs in tiles:
                    Ps = np.zeros((64, 64))
                    for j in range(8):
                        for e in range(4):
                            col = 8 * j + 2 * tq + (e & 1)
                            key = kt * 64 + col
                            on = (ok0 & (key <= pos0)) if e < 2 else (ok1 & (key <= pos1))
                            m = m0 if e < 2 else m1
                            p = np.where(on, fast_expf(np.where(on, sc[:, j, e] - m, 0.0)), 0.0)
                            if e < 2:
                                l0 += p
                            else:
                                l1 += p
                            Ps[np.where(e < 2, r0, r1), col] = p
                    for ks in range(8):
                        A = np.zeros((16, 8))
                        for l in range(32):
                            A[g[l], tq[l]] = Ps[r0[l], 8 * ks + tq[l]]
                            A[g[l] + 8, tq[l]] = Ps[r1[l], 8 * ks + tq[l]]
                            A[g[l], tq[l] + 4] = Ps[r0[l], 8 * ks + tq[l] + 4]
                            A[g[l] + 8, tq[l] + 4] = Ps[r1[l], 8 * ks + tq[l] + 4]
                        for n in range(hd // 8):
                            B = np.zeros((8, 8))
                            for l in range(32):
                                B[tq[l], g[l]] = Vs[8 * ks + tq[l], 8 * n + g[l]]
                                B[tq[l] + 4, g[l]] = Vs[8 * ks + tq[l] + 4, 8 * n + g[l]]
                            C = A @ B
                            acc[:, n, 0] += C[g, 2 * tq]
                            acc[:, n, 1] += C[g, 2 * tq + 1]
                            acc[:, n, 2] += C[g + 8, 2 * tq]
                            acc[:, n, 3] += C[g + 8, 2 * tq + 1]
                for o in (1, 2):
                    l0 = l0 + l0[lanes ^ o]
                    l1 = l1 + l1[lanes ^ o]
                for l in range(32):
                    for n in range(hd // 8):
                        d = 8 * n + 2 * tq[l]
                        if ok0[l]:
                            out[t0 + r0[l], h * hd + d:h * hd + d + 2] = acc[l, n, 0:2] / l0[l]
                        if ok1[l]:
                            out[t0 + r1[l], h * hd + d:h * hd + d + 2] = acc[l, n, 2:4] / l1[l]
    return out


def test_prefill_attention_fragments():
    """The emulated kernel equals a direct causal GQA attention with the
    reference's softmax (fast_expf of s minus each position's maximum)."""
    rng = np.random.default_rng(5)
    seq, base, hd, n_head, n_kv = 70, 5, 16, 2, 1
    scale = 1.0 / np.sqrt(hd)
    q = rng.standard_normal((seq, n_head * hd))
    K = rng.standard_normal((base + seq, n_kv * hd))
    V = rng.standard_normal((base + seq, n_kv * hd))
    got = emulate_attention(q, K, V, base, hd, n_head // n_kv, scale)
    want = np.zeros_like(got)
    for t in range(seq):
        for h in range(n_head):
            kvh = h // (n_head // n_kv)
            s = K[:base + t + 1, kvh * hd:(kvh + 1) * hd] @ q[t, h * hd:(h + 1) * hd] * scale
            p = fast_expf(s - s.max())
            want[t, h * hd:(h + 1) * hd] = (p / p.sum()) @ V[:base + t + 1, kvh * hd:(kvh + 1) * hd]
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-12)
