"""Philox4x32-10 stream: oracle and product (C ABI) against the reference's Random123 KATs.

Mirrors reference/tests/test_philox_acceptance.py (blocks, streams, uniform mapping,
partition/overlap invariance, exhaustion) on tests/golden/philox-v1/*.tsv.
"""

import ctypes
import hashlib

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import philox as op
from tq_mla import _abi, inputs

FIX = GOLDEN / "philox-v1"
MAX64 = (1 << 64) - 1


def _rows(name):
    return [line.split() for line in (FIX / name).read_text().splitlines() if line[0] != "#"]


BLOCKS = [tuple(int(v, 16) for v in r) for r in _rows("blocks.tsv")]
STREAMS = [(*[int(v, 16) for v in r[:3]], int(r[3]), tuple(int(v, 16) for v in r[4:]))
           for r in _rows("streams.tsv")]
UNIFORMS = [tuple(int(v, 16) for v in r) for r in _rows("uniform.tsv")]


def test_fixture_files_match_their_pinned_digests():
    for line in (FIX / "SHA256SUMS").read_text().splitlines():
        digest, name = line.split()
        assert hashlib.sha256((FIX / name).read_bytes()).hexdigest() == digest
    assert len(BLOCKS) == 199 and len(STREAMS) == 160 and len(UNIFORMS) == 96


def _lib_block(counter, key):
    c = (ctypes.c_uint32 * 4)(*counter)
    k = (ctypes.c_uint32 * 2)(*key)
    o = (ctypes.c_uint32 * 4)()
    _abi.lib.tq_philox_block(c, k, o)
    return tuple(o)


@pytest.mark.parametrize("row", BLOCKS[:3] + BLOCKS[3::17])
def test_official_and_sweep_blocks(row):
    counter, key, expected = row[:4], row[4:6], row[6:]
    assert tuple(int(x) for x in op.block(counter, key)) == expected
    assert _lib_block(counter, key) == expected


def test_all_blocks_product():
    for row in BLOCKS:
        assert _lib_block(row[:4], row[4:6]) == row[6:]


def test_all_streams_oracle_and_product():
    for seed, stream, start, count, expected in STREAMS:
        assert tuple(int(x) for x in op.words(seed, stream, start, count)) == expected
        assert tuple(int(x) for x in inputs.philox_words(seed, stream, start, count)) == expected


def test_uniform_bits_oracle_and_product():
    for word, bits in UNIFORMS:
        ours = np.float32(_abi.lib.tq_philox_uniform_f32(word)).view(np.uint32)
        assert int(ours) == bits
        assert int(op.uniform_f32(np.array([word], np.uint32)).view(np.uint32)[0]) == bits


@pytest.mark.parametrize("seed", [0, 1, 0x0123456789ABCDEF, 1 << 63, MAX64])
@pytest.mark.parametrize("start", [0, 1, 3, 5, (1 << 32) - 2])
def test_partition_and_overlap_invariance(seed, start):
    whole = inputs.philox_words(seed, 7, start, 37)
    parts = np.concatenate([inputs.philox_words(seed, 7, start + a, b - a)
                            for a, b in ((0, 5), (5, 6), (6, 30), (30, 37))])
    np.testing.assert_array_equal(whole, parts)
    np.testing.assert_array_equal(whole, op.words(seed, 7, start, 37))


def test_exhausted_range_is_rejected_without_writing():
    out = np.full(4, 0xDEADBEEF, dtype=np.uint32)
    st = _abi.lib.tq_philox_words(0, 0, MAX64 - 1, out.ctypes.data_as(
        ctypes.POINTER(ctypes.c_uint32)), 3)
    assert st == 105
    assert (out == 0xDEADBEEF).all()
    # The last legal word is reachable; an empty request is valid at every start.
    assert _abi.lib.tq_philox_words(0, 0, MAX64, out.ctypes.data_as(
        ctypes.POINTER(ctypes.c_uint32)), 1) == 0
    assert _abi.lib.tq_philox_words(0, 0, MAX64, None, 0) == 0
    with pytest.raises(ValueError):
        op.words(0, 0, MAX64 - 1, 3)
