"""The Python bindings (pocketforge_b200/_lib.py) against the C ABI header
(include/pf_b200.h), no GPU: every bound function has the header's number of
parameters, a pointer where the header has one, and the header's integer or
float width elsewhere, and the header's return type."""
import ctypes as C
import os
import re

import pytest

from pocketforge_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "pf_b200.h")

SCALARS = {"int32_t": C.c_int32, "uint32_t": C.c_uint32, "int64_t": C.c_int64, "float": C.c_float,
           "size_t": C.c_size_t, "pf_status": C.c_int32}


def declarations():
    text = re.sub(r"/\*.*?\*/", " ", open(HEADER).read(), flags=re.S)
    out = {}
    for ret, name, params in re.findall(r"PF_API\s+([\w\s\*]+?)\s*\b(pf_\w+)\s*\(([^)]*)\)\s*;", text):
        ps = [p.strip() for p in params.split(",")]
        out[name] = (ret.strip(), [] if ps == ["void"] or ps == [""] else ps)
    return out


def kind(ctype):
    if ctype in (C.c_void_p, C.c_char_p) or (isinstance(ctype, type) and issubclass(ctype, C._Pointer)):
        return "pointer"
    return ctype


def expected(decl_type):
    if "*" in decl_type:
        return "pointer"
    base = decl_type.replace("const", "").split()[0]
    return SCALARS[base]


def test_bound_functions_match_the_header():
    L = _lib.lib()
    decls = declarations()
    assert len(decls) >= 50
    checked = 0
    for name, (ret, params) in sorted(decls.items()):
        fn = getattr(L, name)
        if fn.argtypes is None:  # not bound from Python
            continue
        checked += 1
        assert len(fn.argtypes) == len(params), (name, params)
        for i, (p, t) in enumerate(zip(params, fn.argtypes)):
            want = expected(p.rsplit(" ", 1)[0] if not p.endswith("*") else p)
            assert kind(t) == want, (name, i, p, t)
        if ret == "void":
            assert fn.restype is None, name
        elif "*" in ret:
            assert kind(fn.restype) == "pointer", name
        else:
            assert fn.restype == SCALARS[ret], (name, ret, fn.restype)
    assert checked >= 40


@pytest.mark.parametrize("name", ["pf_gemm_packed", "pf_sample_rows", "pf_engine_create"])
def test_parser_reads_known_declarations(name):
    ret, params = declarations()[name]
    assert ret == "pf_status" and len(params) >= 3
