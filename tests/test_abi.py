"""The C ABI library: it loads without a GPU, exports every entry point that
include/graphkv_b200.h declares, and the ctypes structs match the C layout."""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

from graphkv_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "graphkv_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int32_t|size_t|const char\*)\s+(gkv_\w+)\(", text, re.M)))


def test_header_declares_the_bound_functions():
    assert declared_functions() == sorted(L._PROTOTYPES)


@pytest.mark.skipif(not os.path.exists(L.LIB_PATH), reason="library not built")
def test_library_exports_every_declared_symbol():
    lib = L.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.gkv_abi_version() == 1
    assert lib.gkv_select_workspace_bytes(1000) >= 1000


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc missing")
def test_struct_layout_matches_c(tmp_path):
    src = tmp_path / "layout.c"
    fields = {
        "gkv_tensor_spec": ["bits", "group_size", "scale_dtype", "reserved"],
        "gkv_plan": ["idx_retained", "spec", "hadamard_divisor", "retained_k", "codes", "scales", "zero_points"],
        "gkv_layer_in": ["k", "v", "k_stride", "v_stride", "heads"],
        "gkv_select_policy": ["seq_len", "keep_cold", "n_cold", "reserved"],
    }
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for st, fs in fields.items():
        lines.append(f'printf("{st} %zu\\n", sizeof({st}));')
        for f in fs:
            lines.append(f'printf("{st}.{f} %zu\\n", offsetof({st}, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split("\n")
               if line)
    py = {"gkv_tensor_spec": L.TensorSpec, "gkv_plan": L.Plan, "gkv_layer_in": L.LayerIn,
          "gkv_select_policy": L.SelectPolicy}
    for st, fs in fields.items():
        assert int(got[st]) == ctypes.sizeof(py[st]), st
        for f in fs:
            assert int(got[f"{st}.{f}"]) == getattr(py[st], f).offset, f"{st}.{f}"
