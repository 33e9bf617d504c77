"""Index arithmetic of the device kernels, restated in Python and checked
exhaustively on small shapes (no GPU): every element is visited once and no
access leaves its buffer."""
import itertools


def ring_positions(H, W, ph, pw):
    """zero_ring_blocks (conv_tc.cu): ring index -> (hp, wp) of the padded plane."""
    Hp, Wp = H + 2 * ph, W + 2 * pw
    band = ph * Wp
    out = []
    for i0 in range(Hp * Wp - H * W):
        i = i0
        if i < band:
            hp, wp = i // Wp, i % Wp
        elif i < 2 * band:
            i -= band
            hp, wp = H + ph + i // Wp, i % Wp
        else:
            i -= 2 * band
            k = i % (2 * pw)
            hp, wp = ph + i // (2 * pw), (k if k < pw else W + k)
        out.append((hp, wp))
    return out, Hp, Wp


def test_zero_ring_enumerates_exactly_the_padding():
    for H, W, ph, pw in itertools.product((1, 5, 9), (1, 4, 7), (0, 1, 3), (0, 1, 2)):
        pos, Hp, Wp = ring_positions(H, W, ph, pw)
        want = {(a, b) for a in range(Hp) for b in range(Wp)
                if a < ph or a >= H + ph or b < pw or b >= W + pw}
        assert len(pos) == len(set(pos)) and set(pos) == want


def test_input_limb_rows_swizzle():
    """x_limbs_block (conv_tc.cu): thread t covers pixel group pg and channel
    quad cc4; its hi / lo words land in 32 distinct banks per warp store and
    phase 2 reads logical 16-byte chunk ch at physical chunk ch ^ (pg & 7)."""
    cover = set()
    for t in range(256):
        cover.add(((t & 7) + 8 * (t >> 7), (t >> 3) & 15))
    assert len(cover) == 256

    def hi_w(pg, c):
        return 4 * ((c >> 2) ^ (pg & 7)) + (c & 3)

    def lo_w(pg, c):
        return 4 * ((4 + (c >> 2)) ^ (pg & 7)) + (c & 3)

    for pg in range(16):
        words = [hi_w(pg, c) for c in range(16)] + [lo_w(pg, c) for c in range(16)]
        assert sorted(words) == list(range(32))
        for ch in range(8):
            phys = [4 * (ch ^ (pg & 7)) + w for w in range(4)]
            src = [hi_w(pg, 4 * ch + w) for w in range(4)] if ch < 4 else \
                [lo_w(pg, 4 * (ch - 4) + w) for w in range(4)]
            assert phys == src
    for w in range(8):
        for fn in (hi_w, lo_w):
            banks = {fn((t & 7) + 8 * (t >> 7), (t >> 3) & 15) % 32 for t in range(32 * w, 32 * w + 32)}
            assert len(banks) == 32


def test_stacked_weight_layout_covers_every_k_step_once():
    """w_stack_blocks / conv_stk_kernel (conv_tc.cu): K step kb = tap*Cg + g
    lives in pair kb // 2 at byte offset 64 * (kb % 2); the MMA for sub-block u
    reads bytes [64h + 32u, 64h + 32u + 32) of the pair's rows."""
    for taps, Cg in itertools.product((1, 2, 3, 9), (1, 2, 4)):
        nkb = taps * Cg
        npairs = (nkb + 1) // 2
        seen = set()
        for tap in range(taps):
            for g in range(Cg):
                kb = tap * Cg + g
                pair, half = kb >> 1, kb & 1
                assert pair < npairs
                for u in range(2):
                    lo = 64 * half + 32 * u
                    seen.add((pair, lo))
                    assert 0 <= lo and lo + 32 <= 128
        assert len(seen) == 2 * nkb


def test_stacked_limb_recombination_is_exact():
    """HH = acc1 - 128 S_hi and MID = acc1' + acc2 - 128 S_lo in 32-bit two's
    complement equal the direct limb products for extreme codes."""
    import random
    rnd = random.Random(5)

    def limbs(q):
        return q >> 8, q & 255

    for K in (1, 7, 64, 4096):
        a = [rnd.choice((-32767, 32767, -1, 0, 1, rnd.randint(-32767, 32767))) for _ in range(K)]
        b = [rnd.choice((-32767, 32767, -1, 0, 1, rnd.randint(-32767, 32767))) for _ in range(K)]
        ah, al = zip(*map(limbs, a))
        bh, bl = zip(*map(limbs, b))
        wrap = lambda v: (v + 2 ** 31) % 2 ** 32 - 2 ** 31  # noqa: E731
        acc1_f = wrap(sum(x * (y + 128) for x, y in zip(ah, bh)))
        acc1_m = wrap(sum(x * y for x, y in zip(ah, bl)))
        acc2_f = wrap(sum(x * (y + 128) for x, y in zip(al, bh)))
        acc2_m = wrap(sum(x * y for x, y in zip(al, bl)))
        s_hi, s_lo = wrap(sum(ah)), wrap(sum(al))
        hh = wrap(acc1_f - 128 * s_hi)
        mid = wrap(acc1_m + acc2_f - 128 * s_lo)
        ll = acc2_m
        assert 65536 * hh + 256 * mid + ll == sum(x * y for x, y in zip(a, b))
