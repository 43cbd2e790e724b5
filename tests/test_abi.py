"""The C ABI: the library loads without a GPU, exports every function declared
in include/*.h, and the ctypes argument structs match the C layout that gcc
computes from the header (sizes and field offsets)."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

from attention_kernel_triton_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(akt_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # the binding declares exactly the header's functions
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(akt_\w+)\b", out))
    assert names <= exported


def test_abi_version_and_error_string():
    L = _lib.lib()
    assert L.akt_abi_version() == 1
    assert isinstance(L.akt_last_error(), bytes)


STRUCTS = {
    "akt_prefill_args": _lib.PrefillArgs,
    "akt_decode_dense_args": _lib.DecodeDenseArgs,
    "akt_decode_paged_args": _lib.DecodePagedArgs,
    "akt_sparse_dense_args": _lib.SparseDenseArgs,
    "akt_sparse_paged_args": _lib.SparsePagedArgs,
    "akt_mask_to_index_args": _lib.MaskToIndexArgs,
    "akt_index_to_mask_args": _lib.IndexToMaskArgs,
    "akt_append_paged_args": _lib.AppendPagedArgs,
    "akt_peer_exchange": _lib.PeerExchange,
}


def test_ctypes_structs_match_c_layout(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "akt.h"', "int main(void){"]
    for cname, py in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    seen = 0
    for line in out:
        if not line:
            continue
        cname, field, val = line.split()
        py = STRUCTS[cname]
        if field == "size":
            assert ctypes.sizeof(py) == int(val), cname
        else:
            assert getattr(py, field).offset == int(val), (cname, field)
        seen += 1
    assert seen == sum(len(s._fields_) + 1 for s in STRUCTS.values())


def test_invalid_arguments_are_rejected_without_a_gpu():
    L = _lib.lib()
    a = _lib.DecodePagedArgs()
    a.batch, a.num_qo_heads, a.num_kv_heads, a.head_dim, a.page_size = 1, 3, 2, 128, 16
    assert L.akt_decode_paged(ctypes.byref(a), None, 0, None) == _lib.AKT_ERR_INVALID
    assert b"multiple" in L.akt_last_error()
    a.num_qo_heads, a.head_dim = 4, 96
    assert L.akt_decode_paged(ctypes.byref(a), None, 0, None) == _lib.AKT_ERR_UNSUPPORTED
    with pytest.raises(_lib.UnsupportedLayout):
        _lib.check(_lib.AKT_ERR_UNSUPPORTED)
