"""GPU run of the native benchmark binary: its output equals the Python front end's launch bit
for bit and matches the oracle; its JSON carries the timing protocol's statistics."""

import json
import subprocess

import numpy as np
import pytest
import torch

from conftest import assert_parity
import gpu_helpers as gh
from tq_mla import build, inputs, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["cpu", "decode"])
def test_native_bench_output_matches_oracle_and_python(cuda_device, tmp_path, name):
    build.build_bench()
    dump = tmp_path / "out.bin"
    r = subprocess.run([str(build.BENCH), "--config", name, "--steps", "20", "--warmup", "3",
                        "--runs", "50", "--steps-per-run", "2", "--graph", "--dump-out",
                        str(dump)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["device_error_flags"] == 0 and line["e2e"]["results_equal_resident_run"]
    st = line["step_stats"]
    assert st["runs"] == 50 and st["ms_p10"] <= st["ms_median"] <= st["ms_p90"]
    assert line["graph_stats"]["runs"] == 50 and line["kernel_ms_per_launch"] > 0
    w = inputs.config(name)
    b = inputs.materialize(w, cuda_device)
    out, lse = ops.mla_decode(b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len,
                              scale=w.scale, query_counts=b.query_counts)
    torch.cuda.synchronize()
    raw = np.fromfile(dump, dtype=np.uint8)
    n_out = out.numel() * 2
    nat_out = torch.from_numpy(raw[:n_out].copy()).view(torch.bfloat16).view(out.shape)
    nat_lse = torch.from_numpy(raw[n_out:].copy()).view(torch.float32).view(lse.shape)
    assert torch.equal(nat_out, out.cpu()) and torch.equal(nat_lse, lse.cpu())
    order, ref_out, ref_lse = gh.oracle_tokens(b, w, range(w.tokens))
    assert_parity(nat_out[order].double().numpy(), nat_lse[order].double().numpy(), ref_out,
                  ref_lse, label=f"native {name}")
