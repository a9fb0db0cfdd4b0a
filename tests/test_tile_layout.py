"""The grouped-ring tile layout of the PQ codes and the stripe arithmetic the ADC
scan relies on, restated in numpy (CPU only).

The scan kernel (csrc/pq.cu, pq_stagger_kernel) reads lane j's 16 steps from half
tile H with MPL 16-byte loads at byte offset H*64*MPL + (8u + j)*16 and indexes the
bytes statically.  A stripe may start on any multiple of 8 rows.  These tests check
that such a load yields, at step i and sub-quantizer byte s, the code byte of the
vector and block the lane works on at that step.  They also check that the combined
main + delta stream (gring_mix_kernel, mix_stripes) holds every main and delta row
exactly once, where the scan's position classification expects it.
"""
import numpy as np


def gring_tiles(count):
    return (count + 7) // 16 + 3


def gring_layout(codes, M):
    """Tiles of one list, as gring_layout_kernel writes them."""
    count = codes.shape[0]
    mpl = M // 8
    total = gring_tiles(count) * 128 * mpl
    e = np.arange(total)
    T = e // (128 * mpl)
    r = e % (128 * mpl)
    u, jj = r // 128, (r % 128) // 16
    b = 16 * u + r % 16
    i, s = b // mpl, b % mpl
    g = 16 * T + i - jj
    g8 = np.floor_divide(g, 8)
    blk = g - 8 * g8
    v = 8 * g8 + jj
    ok = (v >= 0) & (v < count)
    out = np.zeros(total, np.uint8)
    out[ok] = codes[v[ok], mpl * blk[ok] + s[ok]]
    return out


def lane_load(buf, H, j, mpl):
    """Bytes [step i][s] of lane j's 16 steps from half tile H (load_tile)."""
    w = np.zeros((16, mpl), np.int64)
    for i in range(16):
        for s in range(mpl):
            byte = i * mpl + s
            off = H * 64 * mpl + (8 * (byte // 16) + j) * 16 + byte % 16
            w[i, s] = buf[off] if off < buf.size else -1
    return w


def test_half_tile_stripe_starts_read_the_lane_steps():
    rng = np.random.default_rng(7)
    for M in (16, 32, 48):
        mpl = M // 8
        for count in (1, 9, 40, 257, 600):
            codes = rng.integers(0, 256, size=(count, M), dtype=np.uint8)
            buf = gring_layout(codes, M)
            for a in range(0, count, 8):                 # every stripe start a multiple of 8
                for x0 in (0, 16, 32):
                    H = a // 8 + 2 * (x0 // 16)
                    if H > 2 * gring_tiles(count) - 2:      # the kernel clamps its loads here
                        continue
                    for j in range(8):
                        w = lane_load(buf, H, j, mpl)
                        for i in range(16):
                            g = a + x0 + i - j          # global step of lane j
                            blk, v = g % 8, 8 * (g // 8) + j
                            for s in range(mpl):
                                want = codes[v, mpl * blk + s] if 0 <= v < count else 0
                                assert w[i, s] == want, (M, count, a, x0, j, i, s)


def mix_stripes(cm, cd, rings=32):
    sm, sd = -(-cm // rings), -(-cd // rings)
    return sm, sd, (sm + sd + 7) // 8 * 8


def test_combined_stream_holds_each_row_once():
    for cm, cd in ((0, 5), (7, 0), (1526, 15), (9400, 153), (100, 2), (31, 33), (4096, 700)):
        sm, sd, S = mix_stripes(cm, cd)
        assert S % 8 == 0 and S >= sm + sd
        seen_m = np.zeros(cm, np.int32)
        seen_d = np.zeros(cd, np.int32)
        for p in range(32 * S):
            r, x = divmod(p, S)
            if x < sm:
                mi = r * sm + x
                if mi < cm:
                    seen_m[mi] += 1
            elif x < sm + sd:
                di = r * sd + x - sm
                if di < cd:
                    seen_d[di] += 1
        assert (seen_m == 1).all() and (seen_d == 1).all(), (cm, cd)
        # the scan's per-warp delta range: stripe r holds min(Sd, max(0, cd - r*Sd)) delta rows
        assert sum(min(sd, max(0, cd - r * sd)) for r in range(32)) == cd
