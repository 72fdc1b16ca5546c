"""Oracle (test infrastructure only): restatement of the split-KV work partition.

Nothing in the product imports this module. The product computes the same partition on the
device (scheduler kernel, ``tq_mla_kernels.cu``); tests compare the metadata bit for bit.

The reference specifies only that the launch grid does not depend on the data and that split-K
uses a fixed split (``docs/TEST-PLAN.md:205-207``); the partition itself is builder-defined:
  - a unit is one query token; its pages are ``ceil(n / 64)`` for ``n`` visible keys;
  - the units' pages are laid end to end (global page index ``G``); with ``C`` CTA pairs and
    ``W`` total pages, pair ``c`` takes the global range ``[c*q, min((c+1)*q, W))`` with
    ``q = ceil(W / C)``;
  - a unit touched by more than one pair is split; its partial results go to consecutive
    workspace slots starting at ``split_off[u]`` (an exclusive scan over split units), in pair
    order, and a combine kernel merges them;
  - units with no visible key are written (zeros, lse = -inf) by the combine kernel.
"""

import numpy as np

PAGE_ROWS = 64


def unit_pages(n_visible):
    n = np.maximum(np.asarray(n_visible, dtype=np.int64), 0)
    return (n + PAGE_ROWS - 1) // PAGE_ROWS


def partition(n_visible, clusters: int):
    """Return a dict of int64 arrays mirroring the device metadata."""
    pages = unit_pages(n_visible)
    t = len(pages)
    gstart = np.zeros(t, dtype=np.int64)
    if t:
        gstart[1:] = np.cumsum(pages)[:-1]
    total = int(pages.sum())
    quota = -(-total // clusters) if total else 0
    first = np.full(t, -1, dtype=np.int64)
    nsplit = np.zeros(t, dtype=np.int64)
    live = pages > 0
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
        c_lo = -(-int(gstart[u]) // quota)
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
    if not quota or c * quota >= total:
        return out
    g, g_end = c * quota, min((c + 1) * quota, total)
    u = int(meta["begin_unit"][c])
    p = g - int(meta["gstart"][u])
    while g < g_end:
        n = min(int(meta["pages"][u]) - p, g_end - g)
        slot = -1
        if meta["nsplit"][u] >= 2:
            slot = int(meta["split_off"][u] + c - meta["first_cluster"][u])
        out.append((u, p, n, slot))
        g += n
        u += 1
        while u < len(meta["pages"]) and meta["pages"][u] == 0:
            u += 1
        p = 0
    return out
