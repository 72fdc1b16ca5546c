"""Oracle (test infrastructure only): NumPy restatement of the shared Philox4x32-10 test stream.

Nothing in the product imports this module. Tests, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` use it as the checker for the product's C++/CUDA Philox.

Algorithm restated from the reference:
  - round function and key schedule: ``reference/src/tq_reference/philox.py:54-70`` and
    ``crates/tq-testkit/src/philox.rs:57-70``;
  - word mapping ``(seed, stream, i)`` -> lane ``i % 4`` of the block with key
    ``[seed lo, seed hi]`` and counter ``[(i//4) lo, (i//4) hi, stream lo, stream hi]``:
    ``reference/contracts/philox.md:63-75``, ``reference/src/tq_reference/philox.py:81-103``;
  - uniform map ``(w >> 8) * 2**-24``: ``reference/src/tq_reference/philox.py:106-115``.

Parity is pinned against the reference's Random123 known-answer fixtures
(``tests/fixtures/philox-v1/{blocks,streams,uniform}.tsv``), committed under ``tests/golden``.
"""

import numpy as np

M0 = 0xD2511F53
M1 = 0xCD9E8D57
W0 = 0x9E3779B9
W1 = 0xBB67AE85
MASK32 = 0xFFFFFFFF
U64_MAX = (1 << 64) - 1


def _ten_rounds(c0, c1, c2, c3, k0: int, k1: int):
    """Ten Philox rounds over uint32 arrays. Keys are Python ints bumped per round mod 2**32."""
    for r in range(10):
        p0 = c0.astype(np.uint64) * np.uint64(M0)
        p1 = c2.astype(np.uint64) * np.uint64(M1)
        rk0 = np.uint32((k0 + r * W0) & MASK32)
        rk1 = np.uint32((k1 + r * W1) & MASK32)
        hi0 = (p0 >> np.uint64(32)).astype(np.uint32)
        hi1 = (p1 >> np.uint64(32)).astype(np.uint32)
        c0, c1, c2, c3 = hi1 ^ c1 ^ rk0, p1.astype(np.uint32), hi0 ^ c3 ^ rk1, p0.astype(np.uint32)
    return c0, c1, c2, c3


def block(counter, key):
    """One Philox4x32-10 block: ``counter`` four u32 words, ``key`` two u32 words -> four words."""
    c = [np.array([int(x) & MASK32], dtype=np.uint32) for x in counter]
    out = _ten_rounds(c[0], c[1], c[2], c[3], int(key[0]) & MASK32, int(key[1]) & MASK32)
    return np.concatenate(out).astype(np.uint32)


def words(seed: int, stream: int, start: int, count: int) -> np.ndarray:
    """``count`` words of stream ``stream`` starting at word offset ``start``."""
    for name, v in (("seed", seed), ("stream", stream), ("start", start), ("count", count)):
        if not 0 <= int(v) <= U64_MAX:
            raise ValueError(f"{name} must be in [0, 2**64)")
    if count == 0:
        return np.zeros(0, dtype=np.uint32)
    if start + count - 1 > U64_MAX:
        raise ValueError("word range exceeds u64")
    first = start // 4
    nblocks = (start + count - 1) // 4 - first + 1
    group = np.uint64(first) + np.arange(nblocks, dtype=np.uint64)
    c0 = (group & np.uint64(MASK32)).astype(np.uint32)
    c1 = (group >> np.uint64(32)).astype(np.uint32)
    c2 = np.full(nblocks, stream & MASK32, dtype=np.uint32)
    c3 = np.full(nblocks, stream >> 32, dtype=np.uint32)
    lanes = np.stack(_ten_rounds(c0, c1, c2, c3, seed & MASK32, seed >> 32), axis=-1).reshape(-1)
    off = start - first * 4
    return np.ascontiguousarray(lanes[off : off + count])


def uniform_f32(w: np.ndarray) -> np.ndarray:
    """Exact float32 ``(w >> 8) * 2**-24`` in ``[0, 1)``."""
    w = np.asarray(w, dtype=np.uint32)
    return (np.right_shift(w, np.uint32(8)).astype(np.float32) * np.float32(2.0**-24)).astype(
        np.float32
    )
