"""The native benchmark binary (tq_bench): built in-tree, linked to the in-tree library only, and
drawing the same host metadata (lengths, block tables, token-balanced shards) as the Python host
mirror, bit for bit. Its GPU run is covered by tests/test_gpu_native_bench.py."""

import json
import subprocess

import numpy as np
import pytest

from tq_mla import build, inputs


def _meta(*args):
    r = subprocess.run([str(build.BENCH), "--dump-meta", *args], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout)


def test_binary_links_the_in_tree_library():
    build.build_bench()
    r = subprocess.run(["ldd", str(build.BENCH)], capture_output=True, text=True, timeout=60)
    line = [x for x in r.stdout.splitlines() if "libtq_mla.so" in x]
    assert line and str(build.PKG) in line[0], r.stdout
    assert "libtorch" not in r.stdout and "libpython" not in r.stdout


@pytest.mark.parametrize("name,world,strong", [
    ("cpu", 1, False), ("decode", 1, False), ("prefill", 1, False), ("longctx", 1, False),
    ("mtp", 1, False), ("decode", 8, False), ("mtp", 2, True), ("mtp", 8, True)])
def test_metadata_matches_the_host_mirror(name, world, strong):
    build.build_bench()
    batch = None if (world == 1 or strong or name == "cpu") else \
        {"decode": 64, "mtp": 512}[name] * world
    full = inputs.config(name, batch=batch)
    for rank in sorted({0, world - 1}):
        w = full if world == 1 else inputs.shard(full, world, rank)
        args = ["--config", name, "--world", str(world), "--rank", str(rank)]
        m = _meta(*args, *(["--strong"] if strong else []))
        assert m["name"] == w.name and m["heads"] == w.heads and m["width"] == w.width
        assert np.float32(m["scale"]) == np.float32(w.scale)
        assert m["pool_pages"] == w.pool_pages
        for key, ref in (("kv_len", w.kv_len), ("q_per_seq", w.q_per_seq),
                         ("prefix", w.prefix), ("token_global", w.token_global),
                         ("tok_off_global", w.tok_off_global)):
            np.testing.assert_array_equal(np.array(m[key]), ref, err_msg=(name, key))
        table = np.array(m["page_table"]).reshape(len(w.kv_len), -1)
        np.testing.assert_array_equal(table, w.extra["page_table"])
