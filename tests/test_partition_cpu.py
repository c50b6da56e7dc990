"""The page pass's work partition (``grid_size``, ``grid_of`` / ``part_begin`` in
turbopolar_b200/csrc/tp_attention.cu), restated and checked on CPU for the bounds the kernels
rely on: every CTA's unit range spans at most two (KV head, query chunk) segments (its partials
fill two workspace slots), and the CTAs sharing one segment fit the split combine's contributor
table -- at most the SM count for one wave, at most three when a large batch needs more waves.
"""

SMS = 148          # B200
MAX_CONTRIB = 192  # kMaxContrib


def grid_size(segs, sms=SMS):
    return sms if segs <= sms else sms * ((segs + sms - 1) // sms)


def ranges(segs, n_pages, sms=SMS):
    uph = 2 * n_pages
    U = segs * uph
    C = min(U, grid_size(segs, sms))
    k, r = U // C, U - (U // C) * C
    begin = [c * k + (c * r) // C for c in range(C + 1)]
    return uph, begin


def test_partition_bounds():
    for segs in list(range(1, 700, 3)) + [148, 149, 192, 200, 296, 297, 444, 445]:
        for n_pages in (1, 2, 3, 5, 64, 512):
            uph, begin = ranges(segs, n_pages)
            C = len(begin) - 1
            assert begin[0] == 0 and begin[-1] == segs * uph
            assert all(begin[c + 1] > begin[c] for c in range(C))  # no CTA without units
            for c in range(C):
                assert (begin[c + 1] - 1) // uph - begin[c] // uph + 1 <= 2, (segs, n_pages, c)
            per_seg = [0] * segs
            for c in range(C):
                for s in range(begin[c] // uph, (begin[c + 1] - 1) // uph + 1):
                    per_seg[s] += 1
            limit = 3 if segs > SMS else min(C, MAX_CONTRIB)
            assert max(per_seg) <= limit, (segs, n_pages, max(per_seg))


def test_large_batches_fill_whole_waves():
    # 40 sequences x 8 KV heads: 320 segments on 148 SMs -> 3 waves of 148 CTAs, balanced.
    assert grid_size(320) == 3 * 148
    uph, begin = ranges(320, 64)
    sizes = {begin[c + 1] - begin[c] for c in range(len(begin) - 1)}
    assert max(sizes) - min(sizes) <= 1
