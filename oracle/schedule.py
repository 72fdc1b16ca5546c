"""Oracle (test infrastructure only): restatement of the split-KV work partition.

Nothing in the product imports this module. The product computes the same partition on the
device (scheduler kernel, ``tq_mla_kernels.cu``); tests compare the metadata bit for bit.

The reference specifies only that the launch grid does not depend on the data and that split-K
uses a fixed split (``docs/TEST-PLAN.md:205-207``); the partition itself is builder-defined:
  - a unit is one query token; its pages are ``ceil(n / 64)`` for ``n`` visible keys;
  - units are laid end to end in a virtual page space: a unit with pages occupies
    ``SEGMENT_COST_PAGES`` (the start-up cost of a segment: query load, pipeline refill,
    epilogue) followed by its pages; with ``C`` CTA pairs and ``W`` virtual pages in total,
    pair ``c`` takes ``[c*q, min((c+1)*q, W))`` with ``q = ceil(W / C)`` and processes the
    pages of each unit that fall in that range;
  - a unit whose pages fall in more than one pair is split; its partial results go to
    consecutive workspace slots starting at ``split_off[u]`` (an exclusive scan over split
    units), in pair order, and a combine kernel merges them;
  - units with no visible key get zeros and lse = -inf.
The device constant ``kSegmentCostPages`` (``tq_mla_layout.h``) equals ``SEGMENT_COST_PAGES``.
"""

import numpy as np

PAGE_ROWS = 64


def unit_pages(n_visible):
    n = np.maximum(np.asarray(n_visible, dtype=np.int64), 0)
    return (n + PAGE_ROWS - 1) // PAGE_ROWS


SEGMENT_COST_PAGES = 8


def partition(n_visible, clusters: int):
    """Return a dict of int64 arrays mirroring the device metadata."""
    pages = unit_pages(n_visible)
    t = len(pages)
    live = pages > 0
    vlen = np.where(live, pages + SEGMENT_COST_PAGES, 0)
    vstart = np.zeros(t, dtype=np.int64)
    if t:
        vstart[1:] = np.cumsum(vlen)[:-1]
    gstart = vstart + np.where(live, SEGMENT_COST_PAGES, 0)  # virtual start of the pages
    total = int(vlen.sum())
    quota = -(-total // clusters) if total else 0
    first = np.full(t, -1, dtype=np.int64)
    nsplit = np.zeros(t, dtype=np.int64)
    if quota:
        first[live] = gstart[live] // quota
        last = (gstart + pages - 1) // quota
        nsplit[live] = last[live] - first[live] + 1
    split_counts = np.where(nsplit >= 2, nsplit, 0)
    split_off = np.zeros(t, dtype=np.int64)
    if t:
        split_off[1:] = np.cumsum(split_counts)[:-1]
    begin_unit = np.full(clusters, -1, dtype=np.int64)
    for u in np.flatnonzero(live):
        c_lo = -(-int(vstart[u]) // quota)
        c_hi = (int(gstart[u]) + int(pages[u]) - 1) // quota
        for c in range(c_lo, c_hi + 1):
            begin_unit[c] = u
    combine_units = np.flatnonzero(nsplit >= 2)
    empty_units = np.flatnonzero(~live)
    return {
        "pages": pages, "gstart": gstart, "total": total, "quota": quota,
        "first_cluster": first, "nsplit": nsplit, "split_off": split_off,
        "begin_unit": begin_unit, "combine_units": combine_units, "empty_units": empty_units,
        "slots": int(split_counts.sum()),
    }


def segments(meta, c):
    """The ``(unit, first_page, n_pages, slot)`` segments pair ``c`` processes, in order."""
    total, quota = meta["total"], meta["quota"]
    out = []
    if not quota or c * quota >= total or meta["begin_unit"][c] < 0:
        return out
    g, g_end = c * quota, min((c + 1) * quota, total)
    u = int(meta["begin_unit"][c])
    t = len(meta["pages"])
    while g < g_end and u < t:
        pages = int(meta["pages"][u])
        a = int(meta["gstart"][u])
        if pages <= 0 or g >= a + pages:
            u += 1
            continue
        g = max(g, a)  # the unit's start-up cost carries no pages
        if g >= g_end:
            break
        n = min(a + pages, g_end) - g
        slot = -1
        if meta["nsplit"][u] >= 2:
            slot = int(meta["split_off"][u] + c - meta["first_cluster"][u])
        out.append((u, g - a, n, slot))
        g += n
        u += 1
    return out
