"""The C-ABI surface, checked without a GPU: the product library loads and
exports every function that include/*.h declares, and the Python mirror
agrees with the headers on the op ids, the magic and the struct layout.
No compute call is made here."""
import ctypes as C
import os
import re

import pytest

import ppdl

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def _declared():
    names = []
    pat = re.compile(r"PPDL(?:_OPS)?_API\s+[\w\s\*]*?\b(ppdl_\w+)\s*\(")
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += [m.group(1) for m in pat.finditer(src)]
    return names


def test_headers_declare_functions():
    names = _declared()
    assert "ppdl_op_launch" in names and "ppdl_op_supported" in names


@pytest.mark.parametrize("name", _declared())
def test_library_exports_declared_symbol(name):
    lib = ppdl.lib()
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_op_ids_match_header():
    src = open(os.path.join(ROOT, "include", "ppdl_ops.h")).read()
    ids = dict(re.findall(r"#define PPDL_OP_(\w+)\s+(\d+)", src))
    assert int(ids["MASKBOX"]) == ppdl.OP_MASKBOX == 1
    assert int(ids["MSDEF"]) == ppdl.OP_MSDEF == 2
    assert int(ids["WG4_INPUT"]) == ppdl.OP_WG4_INPUT == 10
    assert int(ids["WG4_OUTPUT"]) == ppdl.OP_WG4_OUTPUT == 11
    assert int(ids["WG4_MADD"]) == ppdl.OP_WG4_MADD == 12
    assert int(ids["TOPK"]) == ppdl.OP_TOPK == 13
    assert "0x5050444C" in src and ppdl.PPDL_MAGIC == 0x5050444C


def test_desc_layout():
    # ppdl_tensor = pointer + 4 x int64; desc = dst + 4 src + 16 int32
    assert C.sizeof(ppdl.Tensor) == 40
    assert C.sizeof(ppdl.OpDesc) == 5 * 40 + 64
