"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU needed)."""
import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT
from minimaxh3_b200 import _lib


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"MH3_API\s+[\w\s\*]+?\b(mh3_\w+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert {"mh3_fp8_attention_fwd", "mh3_quantize_qkv", "mh3_quantize_rows"} <= names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in sorted(_declared()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert _declared() == set(_lib.EXPORTED)


def test_host_only_calls():
    lib = _lib.load()
    assert lib.mh3_abi_version() == 7
    assert lib.mh3_qkv_workspace_bytes(1, 40, 32760, 128) == 2 * 40 * 128 * 128 * 4
    assert lib.mh3_qkv_workspace_bytes(0, 1, 1, 128) == 0


def test_invalid_arguments_are_rejected_without_gpu():
    lib = _lib.load()
    a = _lib.AttnArgs()
    a.head_dim = 96
    rc = lib.mh3_fp8_attention_fwd(a, None)
    assert rc == _lib.MH3_ERR_INVALID
    assert b"head_dim" in lib.mh3_last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, "attn")
    assert lib.mh3_fp8_attention_fwd(None, None) == _lib.MH3_ERR_INVALID
    q = _lib.QkvQuantArgs()
    q.head_dim = 128
    assert lib.mh3_quantize_qkv(q, None) == _lib.MH3_ERR_INVALID
    assert lib.mh3_quantize_rows(None, 8, 0, 4, 12, None, None, None) == _lib.MH3_ERR_INVALID
    # mh3_key_bias: null output, empty sizes, rows shorter than a whole 128-key tile
    assert lib.mh3_key_bias(None, 0, None, 0, 2, 300, None, 384, None, None) == _lib.MH3_ERR_INVALID
    assert lib.mh3_key_bias(None, 0, None, 0, 0, 300, 16, 384, None, None) == _lib.MH3_ERR_INVALID
    assert lib.mh3_key_bias(None, 0, None, 0, 2, 300, 16, 300, None, None) == _lib.MH3_ERR_INVALID
    assert b"ceil(seqlen_k/128)*128" in lib.mh3_last_error()


def test_struct_sizes_match_c_layout():
    # AttnArgs: 8 int32, then pointer/int64 fields; see include/mh3_b200.h.
    assert ctypes.sizeof(_lib.AttnArgs) % 8 == 0
    assert _lib.AttnArgs.q8.offset == 32
    assert _lib.AttnArgs.logit_scale_log2.offset + 8 == _lib.AttnArgs.cu_seqlens_q.offset
    assert _lib.QkvQuantArgs.q.offset == 24
    assert _lib.QkvQuantArgs.v_out_dtype.offset == _lib.QkvQuantArgs.q_premul.offset + 4


def test_struct_offsets_match_gcc(tmp_path):
    """Compile a C probe against the header and compare every field offset."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "mh3_b200.h"', "int main(void){"]
    structs = (("mh3_attn_args", _lib.AttnArgs), ("mh3_qkv_quant_args", _lib.QkvQuantArgs),
               ("mh3_gemm_args", _lib.GemmArgs))
    for cname, cls in structs:
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0;}")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {}
    for line in out:
        if line:
            parts = line.split()
            got[(parts[0], parts[1])] = int(parts[2])
    for cname, cls in structs:
        assert got[(cname, "size")] == ctypes.sizeof(cls)
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, (cname, fname)
