"""The page pass's work partitions (``make_part``, ``grid_of`` / ``part_begin``, ``grid_size`` in
turbopolar_b200/csrc/tp_attention.cu), restated and checked on CPU for the bounds the kernels
rely on.

* Flat partition (no more (KV head, query chunk) segments than SMs): one CTA per SM, the units
  of all segments cut into contiguous ranges; every range spans at most two segments (its
  partials fill two workspace slots) and the CTAs sharing one segment fit the split combine's
  contributor table.
* More segments than SMs (large batches), when the CTAs own nearly equal numbers of segments
  (the largest share at most 1.25x the mean): the whole-segment partition, one CTA per SM owning
  the segments [floor(c*V/G), floor((c+1)*V/G)); every segment has exactly one owner (its one
  records are its CTA's compute warps' partials) and every CTA owns at least one.  Inside a CTA,
  warp w streams units w, w + 7, ... of the CTA's segments laid end to end.
* Otherwise, whole waves of the flat partition: every CTA holds between half a segment and one,
  a segment spreads over at most three CTAs.
"""

SMS = 148          # B200
MAX_CONTRIB = 192  # kMaxContrib
CONSUMERS = 7


def part_begin(c, U, C):
    k, r = U // C, U - (U // C) * C
    return c * k + (c * r) // C


def grid_size(segs, sms=SMS):
    """(grid, whole-segment partition) for `segs` segments."""
    if segs <= sms:
        return sms, False
    waves = (segs + sms - 1) // sms
    return (sms, True) if 4 * waves * sms <= 5 * segs else (waves * sms, False)


def test_partition_choice():
    assert grid_size(144) == (148, False)
    assert grid_size(152) == (296, False)       # 19 x 8 KV heads: two waves
    assert grid_size(296) == (148, True)        # two segments per CTA, balanced
    assert grid_size(320) == (444, False)       # 40 x 8: owners would hold 2 or 3 segments
    assert grid_size(512) == (148, True)
    assert grid_size(1024) == (148, True)
    for segs in range(149, 5000):
        grid, owner = grid_size(segs)
        assert owner == (segs > grid)


def test_multi_wave_flat_partition_bounds():
    for segs in [s for s in range(149, 900, 7) if not grid_size(s)[1]] + [152, 192, 200, 320]:
        grid, owner = grid_size(segs)
        assert not owner and grid >= segs
        for n_pages in (1, 2, 3, 64):
            uph = 2 * n_pages
            U = segs * uph
            C = min(U, grid)
            begin = [part_begin(c, U, C) for c in range(C + 1)]
            per_seg = [0] * segs
            for c in range(C):
                first, last = begin[c] // uph, (begin[c + 1] - 1) // uph
                assert begin[c + 1] > begin[c] and last - first + 1 <= 2
                for s_ in range(first, last + 1):
                    per_seg[s_] += 1
            assert max(per_seg) <= 3, (segs, n_pages)


def test_flat_partition_bounds():
    for segs in list(range(1, SMS + 1, 3)) + [SMS]:
        for n_pages in (1, 2, 3, 5, 64, 512):
            uph = 2 * n_pages
            U = segs * uph
            C = min(U, SMS)
            begin = [part_begin(c, U, C) for c in range(C + 1)]
            assert begin[0] == 0 and begin[-1] == U
            assert all(begin[c + 1] > begin[c] for c in range(C))
            per_seg = [0] * segs
            for c in range(C):
                first, last = begin[c] // uph, (begin[c + 1] - 1) // uph
                assert last - first + 1 <= 2, (segs, n_pages, c)
                for s in range(first, last + 1):
                    per_seg[s] += 1
            assert max(per_seg) <= min(C, MAX_CONTRIB)


def test_whole_segment_partition_bounds():
    for segs in [s for s in range(149, 5000, 13) if grid_size(s)[1]] + [296, 512, 1024, 4096]:
        owners = [0] * segs
        for c in range(SMS):
            s0, s1 = part_begin(c, segs, SMS), part_begin(c + 1, segs, SMS)
            assert s1 - s0 >= 1
            for s in range(s0, s1):
                owners[s] += 1
        assert all(o == 1 for o in owners)
        # Balance: the CTAs own floor(V/G) or ceil(V/G) segments.
        sizes = {part_begin(c + 1, segs, SMS) - part_begin(c, segs, SMS) for c in range(SMS)}
        assert max(sizes) - min(sizes) <= 1


def test_whole_segment_unit_order_and_records():
    """Warp w takes CTA units w, w + 7, ... of the CTA's segments laid end to end (unit_at and the
    compute warp's loop); together the warps take every unit once, and each warp's units of one
    segment are consecutive in its order, so it leaves one record per segment (empty for a
    segment it has no unit of)."""
    for n_pages in (1, 2, 3, 4, 9, 64):
        uph = 2 * n_pages
        for nseg in (1, 2, 7):
            n = nseg * uph
            seen = set()
            for w in range(CONSUMERS):
                units = [(k // uph, k % uph) for k in range(w, n, CONSUMERS)]
                nu = (n - 1 - w) // CONSUMERS + 1 if n > w else 0
                assert len(units) == nu
                segs = [sl for sl, _ in units]
                assert segs == sorted(segs)  # one run per segment
                seen.update(units)
            assert seen == {(sl, j) for sl in range(nseg) for j in range(uph)}


SEG_RECS = 56  # kSegRecs: records of all heads that segment_combine_kernel stages in one chunk
MAX_HEADS = 8  # kMaxHeads: query heads of one segment


def test_segment_combine_records_fit_one_chunk():
    """segment_combine_kernel (plain attention over more segments than SMs) stages the records
    of every head of a segment at once: seven per segment with whole segments (one per compute
    warp), at most three with whole waves; times at most eight heads, within its 56 records."""
    for segs in list(range(149, 3000, 11)) + [152, 192, 200, 296, 320, 512, 1024]:
        grid, owner = grid_size(segs)
        if owner:
            n_max = CONSUMERS
        else:
            n_max = 0
            for n_pages in (1, 2, 3, 64):
                uph = 2 * n_pages
                U = segs * uph
                C = min(U, grid)
                begin = [part_begin(c, U, C) for c in range(C + 1)]
                per_seg = [0] * segs
                for c in range(C):
                    for s_ in range(begin[c] // uph, (begin[c + 1] - 1) // uph + 1):
                        per_seg[s_] += 1
                n_max = max(n_max, max(per_seg))
        assert n_max * MAX_HEADS <= SEG_RECS, (segs, n_max)
