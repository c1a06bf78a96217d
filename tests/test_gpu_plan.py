"""The decode plan (metagross_b200/csrc/mg_plan.cu): the split of a step's
pages over the SMs.  Each case builds a plan on the GPU, checks it word for
word against a plain-Python restatement of the same partition, and checks
the invariants the attention kernel relies on: every unit (committed page or
staged tail) of every sequence is covered exactly once, a cut sequence's
pieces own distinct contiguous partial slots, and no CTA holds more segments
than fit the flat record array (batch + grid records)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAGIC = 0x6D67706C


def _C():
    from metagross_b200 import _C

    return _C


INLINE = 4
PIDS = 128  # page ids of each CTA's first segment kept in the plan
TAIL_UNITS = 2  # a staged tail weighs two units in the partition


def layout(batch, grid):
    off_counts = 16
    off_offs = off_counts + grid
    off_recs = (off_offs + grid + 7) // 8 * 8
    off_pids = off_recs + grid * INLINE * 8
    off_flat = off_pids + grid * PIDS
    off_empty = off_flat + (batch + grid) * 8
    return off_counts, off_offs, off_recs, off_pids, off_flat, off_empty


def plan_ref(lens, P, max_blocks, has_staging, G):
    """Plain-Python statement of the partition (mirrors mg_plan.cu)."""
    B = len(lens)
    off_counts, off_offs, off_recs, off_pids, off_flat, off_empty = layout(B, G)
    lens = [l if (0 <= l and l // P <= max_blocks) else 0 for l in lens]
    units = [l // P + (TAIL_UNITS if has_staging and l % P else 0) for l in lens]
    pre = np.concatenate([[0], np.cumsum(units)]).astype(np.int64)
    W = int(pre[-1])
    counts = [0] * G
    recs = {}
    empties = [b for b in range(B) if units[b] == 0]
    nonempty = B - len(empties)
    chunk = W > 0 and nonempty <= G

    def tail_of(b):
        return lens[b] % P if has_staging else 0

    if chunk:
        lo, hi = (W + G - 1) // G, max(max(units), (W + G - 1) // G)
        while lo < hi:
            mid = lo + (hi - lo) // 2
            if sum((u + mid - 1) // mid for u in units) <= G:
                hi = mid
            else:
                lo = mid + 1
        S = lo
        # the longest chunk within 5/4 of, or 16 units above, the even share
        chunk = S * min(W, G) * 4 <= W * 5 or (S - 16) * min(W, G) <= W
    used = 0
    if chunk:
        k = [(u + S - 1) // S for u in units]
        kpre = np.concatenate([[0], np.cumsum(k)])
        spl = [kk if kk > 1 else 0 for kk in k]
        ppre = np.concatenate([[0], np.cumsum(spl)])
        used = int(kpre[-1])
        for b in range(B):
            u, np_b, tb = units[b], lens[b] // P, tail_of(b)
            for j in range(k[b]):
                ulo, uhi = j * u // k[b], (j + 1) * u // k[b]
                c = int(kpre[b]) + j
                recs[(c, 0)] = (b, ulo, max(0, min(uhi, np_b) - ulo), tb if (uhi == u and tb > 0) else 0,
                                int(ppre[b]) + j if k[b] > 1 else -1, int(ppre[b]), k[b], 0)
                counts[c] = 1
    elif W > 0:
        GR = min(W, G)
        used = GR

        def cta_of_unit(u):
            l, h = 0, GR - 1
            while l < h:
                mid = (l + h + 1) // 2
                if mid * W // GR <= u:
                    l = mid
                else:
                    h = mid - 1
            return l

        pieces = [cta_of_unit(pre[b + 1] - 1) - cta_of_unit(pre[b]) + 1 if units[b] else 0 for b in range(B)]
        ppre = np.concatenate([[0], np.cumsum([p if p > 1 else 0 for p in pieces])])
        for c in range(GR):
            u0, u1 = c * W // GR, (c + 1) * W // GR
            b = max(i for i in range(B) if pre[i] <= u0)
            kk = 0
            while b < B and pre[b] < u1:
                ub, ue = int(pre[b]), int(pre[b + 1])
                if ue > ub:
                    lo_, hi_ = max(u0, ub) - ub, min(u1, ue) - ub
                    np_b, tb = lens[b] // P, tail_of(b)
                    whole = lo_ == 0 and hi_ == ue - ub
                    recs[(c, kk)] = (b, lo_, max(0, min(hi_, np_b) - lo_), tb if (hi_ == ue - ub and tb > 0) else 0,
                                     -1 if whole else int(ppre[b]) + (c - cta_of_unit(ub)), int(ppre[b]), pieces[b], 0)
                    kk += 1
                b += 1
            counts[c] = kk
    return dict(off_offs=off_offs, off_recs=off_recs, off_pids=off_pids, off_flat=off_flat, off_empty=off_empty,
                counts=counts, recs=recs, empties=empties, mode=1 if chunk else 2, W=W, used=used)


def build_plan(lens, P=16, max_blocks=None, has_staging=True):
    C = _C()
    B = len(lens)
    max_blocks = max_blocks or max(1, max(lens) // P + 1)
    k_pool = torch.zeros(1, P, 1, 64, dtype=torch.int8, device="cuda")
    bt = torch.randint(0, 1 << 20, (B, max_blocks), generator=torch.Generator().manual_seed(B),
                       dtype=torch.int32).cuda()
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    plan = torch.zeros(C.decode_plan_bytes(B), dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.decode_plan(k_pool, bt, sl, has_staging, plan, status)
    words = plan.view(torch.int32).cpu().numpy()
    return words, int(status.item()), max_blocks, bt.cpu().numpy()


def check(words, ref, lens, P, has_staging, G, bt=None):
    B = len(lens)
    assert words[0] == MAGIC and words[1] == B and words[2] == G
    assert words[4] == len(ref["empties"]) and words[5] == ref["mode"] and words[6] == ref["W"]
    assert words[7] == ref["used"] and words[8] == int(has_staging)
    counts = words[16:16 + G]
    assert counts.tolist() == ref["counts"]
    offs = words[ref["off_offs"]:ref["off_offs"] + G]
    np.testing.assert_array_equal(offs[:ref["used"]], np.concatenate([[0], np.cumsum(counts)])[:ref["used"]])
    assert int(counts.sum()) <= B + G
    for (c, k), rec in ref["recs"].items():
        o = ref["off_flat"] + (int(offs[c]) + k) * 8
        assert tuple(words[o:o + 8].tolist()) == rec, (c, k)
        if k < INLINE:
            o = ref["off_recs"] + (c * INLINE + k) * 8
            assert tuple(words[o:o + 8].tolist()) == rec, (c, k, "inline")
    assert sorted(words[ref["off_empty"]:ref["off_empty"] + len(ref["empties"])].tolist()) == ref["empties"]
    # page ids of each CTA's first segment, copied from the block table
    if bt is not None:
        for c in range(G):
            want = np.zeros(PIDS, dtype=np.int64)
            if counts[c] > 0:
                b, lo, npg = ref["recs"][(c, 0)][:3]
                n = min(npg, PIDS)
                want[:n] = bt[b, lo:lo + n]
            np.testing.assert_array_equal(words[ref["off_pids"] + c * PIDS:ref["off_pids"] + (c + 1) * PIDS], want)
    # invariants: every unit covered once, partial slots distinct per sequence
    cover = {b: [] for b in range(B)}
    slots = set()
    for c in range(G):
        for k in range(counts[c]):
            o = ref["off_flat"] + (int(offs[c]) + k) * 8
            b, lo, npg, tail, pslot, pbase, ncov, _ = words[o:o + 8].tolist()
            cover[b].append((lo, npg, tail, pslot))
            if pslot >= 0:
                assert pbase <= pslot < pbase + ncov
                assert pslot not in slots
                slots.add(pslot)
    for b in range(B):
        np_b = lens[b] // P
        tb = lens[b] % P if has_staging else 0
        pages = sorted(p for lo, npg, _, _ in cover[b] for p in range(lo, lo + npg))
        assert pages == list(range(np_b)), b
        assert sum(t for _, _, t, _ in cover[b]) == tb, b
        if cover[b]:
            assert (len(cover[b]) == 1) == all(ps < 0 for *_, ps in cover[b])


def _grid():
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("case", ["uniform32", "ragged64", "one_long", "tiny_many", "with_empty", "staging_off",
                                  "more_than_sms", "all_empty", "skewed_fewer_than_sms"])
def test_plan_matches_restatement(case):
    G = _grid()
    g = np.random.default_rng(sum(map(ord, case)))
    has_staging = True
    if case == "uniform32":
        lens = [1017] * 32
    elif case == "ragged64":
        lens = g.integers(128, 2049, 64).tolist()
    elif case == "one_long":
        lens = [16 * 5000 + 7]
    elif case == "tiny_many":
        lens = g.integers(1, 40, 300).tolist()
    elif case == "with_empty":
        lens = [0, 35, 0, 1024, 3, 0, 16]
    elif case == "staging_off":
        lens = g.integers(0, 600, 40).tolist()
        has_staging = False
    elif case == "more_than_sms":
        lens = g.lognormal(np.log(2048), 0.8, 1024).clip(1, 32768).astype(int).tolist()
    elif case == "skewed_fewer_than_sms":
        # fewer sequences than SMs, heavy-tailed: the longest chunk would be over twice the even share
        lens = g.lognormal(np.log(2048), 1.0, 128).clip(1, 32768).astype(int).tolist()
        lens[5] = 32768
    else:
        lens = [0, 0, 0]
    words, status, max_blocks, bt = build_plan(lens, has_staging=has_staging)
    assert status == 0
    ref = plan_ref(lens, 16, max_blocks, has_staging, G)
    check(words, ref, lens, 16, has_staging, G, bt)
    if case == "skewed_fewer_than_sms":
        assert ref["mode"] == 2  # stream-K although every sequence would fit on its own SMs


def test_plan_flags_bad_lengths():
    G = _grid()
    lens = [40, -3, 16 * 100]  # max_blocks 4: the last is too long, -3 negative
    words, status, max_blocks, bt = build_plan(lens, max_blocks=4)
    assert status & 0x80
    ref = plan_ref(lens, 16, 4, True, G)
    check(words, ref, [40, 0, 0], 16, True, G, bt)
