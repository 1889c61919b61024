"""The index arithmetic of the tensor-core prefill kernel
(csrc/neon_prefill.cuh, matvec_mma_q4_0_kernel), emulated on the CPU: the
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
