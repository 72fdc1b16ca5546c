"""CPU legs of the benchmark: inputs rebuilt by the oracle alone, no product library loaded."""

import json
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT
from oracle import generate as ogen
from tq_mla import inputs


@pytest.mark.parametrize("name", ["cpu", "decode", "decode_fp8", "prefill", "longctx", "mtp",
                                  "sparse", "sparse_fp8"])
def test_oracle_workload_metadata_matches_the_product(name):
    """The oracle's restated workload table gives the product's metadata bit for bit."""
    a, b = ogen.config(name), inputs.config(name)
    assert (a.name, a.seed, a.heads, a.width, a.scale) == (b.name, b.seed, b.heads, b.width,
                                                           b.scale)
    for x, y in ((a.kv_len, b.kv_len), (a.q_per_seq, b.q_per_seq), (a.prefix, b.prefix),
                 (a.page_table, b.extra["page_table"]), (a.q_pos(), b.q_pos()),
                 (a.seq_id(), b.seq_id()), (a.tok_off, b.tok_off_global),
                 (a.token_start, b.token_global)):
        np.testing.assert_array_equal(x, y)
    assert a.pool_pages == b.pool_pages


def test_sharded_batches_keep_the_first_sequences():
    """A job of N x 64 decode sequences starts with the one-GPU batch's lengths."""
    one, eight = ogen.config("decode"), ogen.config("decode", batch=512)
    np.testing.assert_array_equal(one.kv_len, eight.kv_len[:64])
    np.testing.assert_array_equal(one.tok_off, eight.tok_off[:64])


def test_reference_arm_loads_no_product_library():
    """``bench.py --impl reference`` runs the oracle restatement without libtq_mla.so."""
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--config', 'cpu', '--steps', '2',"
        " '--warmup', '1']\n"
        "runpy.run_path('bench.py', run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "assert 'libtq_mla' not in maps, 'product library mapped'\n"
        "assert 'tq_mla._abi' not in sys.modules\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 1
    assert line["value"] > 0 and line["cpu_baseline"]["kind"] == "port"
    assert line["config"]["workload"] == "cpu_decode_h16"
