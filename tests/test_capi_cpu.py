"""The C ABI: libmie.so loads, exports every entry point include/mie.h
declares, and the ctypes mirrors match the C struct layouts (sizes and field
offsets as gcc lays them out).  No kernel is launched."""

import ctypes
import os
import re
import subprocess
import sys

import pytest

from moe_engine import capi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "mie.h")

STRUCTS = {
    "mie_moe_args": capi.MoeArgs,
    "mie_attn_args": capi.AttnArgs,
    "mie_qkv_args": capi.QkvArgs,
    "mie_proj_args": capi.ProjArgs,
    "mie_lmhead_args": capi.LmHeadArgs,
    "mie_layer_desc": capi.LayerDesc,
    "mie_step_desc": capi.StepDesc,
    "mie_prefill_attn_args": capi.PrefillAttnArgs,
    "mie_peer_reduce_args": capi.PeerReduceArgs,
}


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(mie_\w+)\s*\(", text, re.M)))


def c_field_names(struct_name):
    text = open(HEADER).read()
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (struct_name, struct_name), text, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return re.findall(r"(\w+)\s*(?:\[[^\]]*\])?\s*;", body)


@pytest.fixture(scope="module")
def lib():
    if not capi.library_available():
        from moe_engine.build import build

        build()
    return capi.load()


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 13
    for n in names:
        assert hasattr(lib, n), n
        assert n in capi.SYMBOLS, n
    assert set(capi.SYMBOLS) == set(names)


def test_status_strings_and_version(lib):
    assert lib.mie_version() >= 1
    for code in range(6):
        assert lib.mie_status_string(code)
    assert b"unknown" in lib.mie_status_string(99)


def test_null_arguments_rejected_without_a_gpu(lib):
    # Validation happens on the host before any CUDA call.
    for name in ("mie_moe_decode", "mie_attn_decode", "mie_qkv_rope_store", "mie_proj_residual",
                 "mie_lmhead_argmax", "mie_decode_step", "mie_decode_head", "mie_moe_route"):
        assert getattr(lib, name)(None, None) == capi.MIE_ERR_INVALID
    assert lib.mie_decode_layer(None, 0, None) == capi.MIE_ERR_INVALID
    a = capi.MoeArgs()
    a.dtype = 7
    assert lib.mie_moe_decode(ctypes.byref(a), None) == capi.MIE_ERR_UNSUPPORTED
    at = capi.AttnArgs()
    at.head_dim = 48
    assert lib.mie_attn_decode(ctypes.byref(at), None) == capi.MIE_ERR_UNSUPPORTED


def test_ctypes_structs_match_c_layout(tmp_path):
    """Compile a probe against include/mie.h with gcc and compare layouts."""
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){"]
    for cname, cls in STRUCTS.items():
        fields = c_field_names(cname)
        py = [f[0] for f in cls._fields_]
        assert [f.rstrip("_") for f in py] == fields, cname
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f in fields:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    c_layout = dict(l.split() for l in out if l.strip())
    for cname, cls in STRUCTS.items():
        assert int(c_layout[cname]) == ctypes.sizeof(cls), cname
        for pyname, _ in cls._fields_:
            cf = pyname.rstrip("_")
            assert int(c_layout[f"{cname}.{cf}"]) == getattr(cls, pyname).offset, f"{cname}.{cf}"


def test_product_fails_loudly_without_library(monkeypatch):
    monkeypatch.setattr(capi, "LIB_PATH", "/nonexistent/libmie.so")
    monkeypatch.setattr(capi, "_lib", None)
    with pytest.raises(RuntimeError, match="libmie.so not found"):
        capi.load()
