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


def _ceil_div(a, b):
    return (a + b - 1) // b


def test_conv_prep_block_split_covers_each_job_once():
    """conv_prep_kernel (conv_tc.cu): blocks [0, wgrid) prepare the weight,
    [wgrid, wgrid + zgrid) zero the padding ring, the rest quantise the input.
    Restates the host grid sizes and the kernel's split: every x block maps to
    one (image, pixel run, channel group), every w_limbs block to one (filter,
    group, tap run) whose 64 x nt items each hit one (channel, tap) slot, and
    the grid-strided ring and stacked-tile loops visit every item once."""
    WQ_TAPS, XQ_W, STK_N = 32, 128, 144
    for N, C, H, W, F, k, pad, stk in [(2, 64, 7, 9, 64, 3, 1, True), (1, 200, 5, 5, 96, 3, 1, False),
                                       (3, 70, 4, 6, 256, 5, 2, False), (2, 64, 9, 9, 48, 1, 0, True)]:
        taps = k * k
        Cg = _ceil_div(C, 64)
        Hp, Wp = H + 2 * pad, W + 2 * pad
        npairs = _ceil_div(taps * Cg, 2)
        ring = Hp * Wp - H * W
        zblocks = max(1, min(_ceil_div(N * ring * Cg * 8, 256), 8 * 148)) if pad else 0
        runs = _ceil_div(H * W, XQ_W)
        xblocks = N * runs * Cg
        wblocks = _ceil_div(npairs * STK_N * 8, 256) if stk else F * Cg * _ceil_div(taps, WQ_TAPS)
        grid = wblocks + zblocks + xblocks
        seen_x, seen_w, seen_z, seen_s = set(), set(), [], []
        for blk in range(grid):
            b = blk
            if b < wblocks:
                if stk:
                    seen_s += [b * 256 + t + s * wblocks * 256 for t in range(256)
                               for s in range(_ceil_div(npairs * STK_N * 8, wblocks * 256))
                               if b * 256 + t + s * wblocks * 256 < npairs * STK_N * 8]
                else:
                    r = _ceil_div(taps, WQ_TAPS)
                    run, g, f = b % r, (b // r) % Cg, b // (r * Cg)
                    nt = min(WQ_TAPS, taps - run * WQ_TAPS)
                    items = [(it // nt, it - (it // nt) * nt) for it in range(64 * nt)]
                    assert sorted(items) == [(cc, t) for cc in range(64) for t in range(nt)]
                    seen_w.add((f, g, run))
                continue
            b -= wblocks
            if b < zblocks:
                total = N * ring * Cg * 8
                it = b * 256
                while it < total:
                    seen_z += [i for i in range(it, min(it + 256, total))]
                    it += zblocks * 256
                continue
            b -= zblocks
            seen_x.add((b // Cg // runs, (b // Cg) % runs, b % Cg))
        assert len(seen_x) == xblocks == N * runs * Cg
        if stk:
            assert sorted(seen_s) == list(range(npairs * STK_N * 8))
        else:
            assert len(seen_w) == wblocks
        if pad:
            assert sorted(seen_z) == list(range(N * ring * Cg * 8))


def test_depthwise_partials_cover_input_and_filters():
    """depthwise_scaled_launch (conv.cu): nparts blocks of depthwise_amax_kernel
    take chunks [b*cx, (b+1)*cx) of the input and [b*cw, (b+1)*cw) of the
    filters, clipped to the ends; chunks are whole 16-byte vectors, cover each
    element once, and nparts never exceeds the 512 partial words per operand
    that the workspace holds."""
    for nx, nw, esize in [(64 * 512 * 49, 512 * 9, 2), (7, 3, 2), (1000003, 25, 4), (16 * 1024 * 1024, 7 * 7 * 64, 2)]:
        vec = 16 // esize
        nparts = max(1, min(512, _ceil_div(nx * esize, 4 * 1024)))
        cx = _ceil_div(_ceil_div(nx, nparts), vec) * vec
        cw = _ceil_div(_ceil_div(nw, nparts), vec) * vec
        assert nparts <= 512 and cx % vec == 0 and cw % vec == 0
        for n, c in ((nx, cx), (nw, cw)):
            spans = [(min(n, b * c), min(n, (b + 1) * c)) for b in range(nparts)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(nparts - 1))
