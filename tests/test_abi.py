"""The C ABI: the in-tree library loads without a GPU, exports every entry point that
include/tq_mla.h declares, and its structs have the layout a C compiler gives the header."""

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT
from tq_mla import _abi

HEADER = ROOT / "include" / "tq_mla.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tq_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 16
    for name in names:
        assert hasattr(_abi.lib, name), name
        assert name in _abi.PROTOTYPES, name
    assert _abi.lib.tq_mla_version().startswith(b"tq_mla")
    assert _abi.lib.tq_mla_status_string(12) == b"Alias"


def test_library_is_the_in_tree_build():
    assert _abi.LIB_PATH.parent == ROOT / "tensorquay-engine_b200" / "tq_mla"
    assert _abi.LIB_PATH.exists()


STRUCTS = {
    "TqTensorSpec": (_abi.TqTensorSpec, ["shape", "strides_bytes", "rank", "dtype",
                                          "device_address", "buffer_bytes"]),
    "TqMlaSpec": (_abi.TqMlaSpec, ["q", "kv", "page_table", "seq_id", "q_pos", "kv_len", "out",
                                   "lse", "kv_format", "softmax_scale"]),
    "TqMlaParams": (_abi.TqMlaParams, ["spec", "tokens", "heads", "row_stride",
                                       "max_queries_per_sequence", "should_launch", "idx",
                                       "k_len", "topk", "sparse", "digest"]),
    "TqCombineParams": (_abi.TqCombineParams, ["parts", "part_out", "out_stride_head",
                                               "out_dtype"]),
    "TqWorkspaceLayout": (_abi.TqWorkspaceLayout, ["total_bytes", "part_out", "sparse_rows",
                                                   "sparse_count", "pairs"]),
    "TqContractError": (_abi.TqContractError, ["field", "kind"]),
    "TqCommId": (_abi.TqCommId, ["internal"]),
    "TqContextMergeParams": (_abi.TqContextMergeParams, ["tokens", "gather_out_bytes", "out",
                                                         "out_stride_head", "out_dtype"]),
    "TqKvWriteSpec": (_abi.TqKvWriteSpec, ["src", "kv", "page_table", "seq_id", "pos",
                                           "kv_format", "norm_weight", "norm_eps"]),
    "TqPrologueSpec": (_abi.TqPrologueSpec, ["x", "w_qa", "w_uk", "kv", "q", "heads", "nope_dim",
                                             "rope_dim", "kv_format", "q_eps", "kv_eps",
                                             "rope_theta"]),
}


def test_struct_layout_matches_a_c_compiler(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(){"]
    for cname, (_, fields) in STRUCTS.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f in fields:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    try:
        subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    except FileNotFoundError:
        pytest.fail("gcc is required for the ABI layout check")
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                        check=True).stdout.splitlines())
    for cname, (cls, fields) in STRUCTS.items():
        assert int(got[cname]) == ctypes.sizeof(cls), cname
        for f in fields:
            assert int(got[f"{cname}.{f}"]) == getattr(cls, f).offset, (cname, f)
