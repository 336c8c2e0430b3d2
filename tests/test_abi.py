"""The C ABI library: it loads, exports every symbol the header declares, its
ctypes structures match the C layout, and argument errors come back as status
codes with messages (no GPU needed for any of this)."""
from __future__ import annotations

import ctypes
import re
import shutil
import subprocess

import pytest

from conftest import ROOT
from projectgorgon_b200 import _abi

HEADER = ROOT / "include" / "gorgon_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"GORGON_API\s+[\w\s\*]+?\b(gorgon_\w+)\s*\(", text)))


def test_library_loads_and_reports_version():
    lib = _abi.lib()
    assert lib.gorgon_abi_version() == 1


def test_every_declared_symbol_is_exported_and_bound():
    syms = declared_symbols()
    assert len(syms) >= 9
    lib = _abi.lib()
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_abi.SIGNATURES)
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True,
                             text=True, check=True).stdout
        exported = set(re.findall(r"\bT (gorgon_\w+)", out))
        assert exported == set(syms)


STRUCTS = {
    "gorgon_tree_attn_params": _abi.TreeAttnParams,
    "gorgon_verify_params": _abi.VerifyParams,
    "gorgon_kv_trim_params": _abi.KvTrimParams,
}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_ctypes_layout_matches_c_header(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "gorgon_b200.h"', "int main(void){"]
    for cname, cls in STRUCTS.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.split() for l in out if l)
    for cname, cls in STRUCTS.items():
        assert int(got[cname]) == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(cls, fname).offset, (cname, fname)


def _err(rc):
    return rc, _abi.lib().gorgon_last_error().decode()


def test_attention_argument_errors_are_status_codes():
    lib = _abi.lib()
    rc, msg = _err(lib.gorgon_tree_attn(None, None, 0, None))
    assert rc == _abi.GORGON_ERR_INVALID and "null" in msg
    p = _abi.TreeAttnParams()
    p.dtype = 7
    assert _err(lib.gorgon_tree_attn(p, None, 0, None))[0] == _abi.GORGON_ERR_INVALID
    p.dtype = _abi.BF16
    p.batch, p.heads_q, p.heads_kv, p.n_tree, p.kv_len, p.head_dim = 1, 6, 4, 3, 8, 64
    rc, msg = _err(lib.gorgon_tree_attn(p, None, 0, None))
    assert rc == _abi.GORGON_ERR_INVALID and "multiple" in msg
    p.heads_q = 8
    p.kv_len = 2
    rc, msg = _err(lib.gorgon_tree_attn(p, None, 0, None))
    assert rc == _abi.GORGON_ERR_INVALID and "kv_len" in msg
    p.kv_len, p.head_dim = 8, 512
    assert _err(lib.gorgon_tree_attn(p, None, 0, None))[0] == _abi.GORGON_ERR_UNSUPPORTED
    assert lib.gorgon_tree_attn_workspace_size(None) == 0


def test_verify_and_trim_argument_errors():
    lib = _abi.lib()
    v = _abi.VerifyParams()
    v.batch, v.rows, v.vocab, v.n, v.prompt_len = 1, 4, 10, 0, 1
    assert _err(lib.gorgon_verify(v, None, 0, None))[0] == _abi.GORGON_ERR_UNSUPPORTED
    v.n, v.prompt_len = 3, 0
    assert _err(lib.gorgon_verify(v, None, 0, None))[0] == _abi.GORGON_ERR_INVALID
    v.prompt_len = 1
    rc, msg = _err(lib.gorgon_verify(v, None, 0, None))
    assert rc == _abi.GORGON_ERR_INVALID and "null" in msg
    t = _abi.KvTrimParams()
    t.elem_bytes, t.layers, t.batch, t.heads, t.seq_capacity, t.head_dim = 3, 1, 1, 1, 4, 8
    assert _err(lib.gorgon_kv_trim(t, None))[0] == _abi.GORGON_ERR_INVALID
    t.elem_bytes, t.max_len = 2, 300
    assert _err(lib.gorgon_kv_trim(t, None))[0] == _abi.GORGON_ERR_UNSUPPORTED
    assert _err(lib.gorgon_tree_mask(None, 1, -1, 0, -1, None, None))[0] == _abi.GORGON_ERR_INVALID


def test_empty_problems_are_no_ops():
    lib = _abi.lib()
    assert lib.gorgon_tree_mask(None, 0, 5, 0, -1, None, None) == 0
    t = _abi.KvTrimParams()
    t.elem_bytes = 2
    assert lib.gorgon_kv_trim(t, None) == 0


def test_wait_limit_setter_round_trips():
    """gorgon_set_wait_limit_ns returns the previous bound; ns <= 0 changes nothing."""
    first = _abi.set_wait_limit_ns(123456)
    try:
        assert first > 0
        assert _abi.set_wait_limit_ns(0) == 123456
        assert _abi.set_wait_limit_ns(-5) == 123456
    finally:
        _abi.set_wait_limit_ns(first)
    assert _abi.set_wait_limit_ns(0) == first
