"""The C ABI without a GPU: the library loads, exports every function that
``include/moe_b200.h`` declares, its structs agree with the ctypes mirror, and
argument validation answers with the documented status codes."""
import ctypes
import os
import re
import subprocess

import pytest

from moe_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(REPO, "include", f) for f in sorted(os.listdir(os.path.join(REPO, "include")))
           if f.endswith(".h")]


def declared_functions():
    names = []
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(moe_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "moe_fp8_forward" in names and "moe_fp8_workspace_size" in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_declared_symbol(name):
    lib = _lib.load()
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert name in _lib.SYMBOLS, f"{name} has no ctypes signature in moe_b200/_lib.py"


def test_struct_layout_matches_header(tmp_path):
    """Compile the header with the host C compiler and compare sizeof/offsetof
    with the ctypes mirror used by the Python layer."""
    fields = {"MoeFwdArgs": _lib.MoeFwdArgs, "MoeWorkspaceLayout": _lib.MoeWorkspaceLayout}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "moe_b200.h"', 'int main(){']
    for sname, cls in fields.items():
        lines.append(f'printf("{sname} %zu\\n", sizeof({sname}));')
        for f, _ in cls._fields_:
            lines.append(f'printf("{sname}.{f} %zu\\n", offsetof({sname}, {f}));')
    lines.append("return 0;}")
    c = tmp_path / "probe.c"
    c.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(REPO, "include"), str(c), "-o", str(exe)],
                   check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                 check=True).stdout.splitlines())
    for sname, cls in fields.items():
        assert int(got[sname]) == ctypes.sizeof(cls), sname
        for f, _ in cls._fields_:
            assert int(got[f"{sname}.{f}"]) == getattr(cls, f).offset, f"{sname}.{f}"


def _args(**kw):
    a = _lib.MoeFwdArgs()
    d = dict(T=64, H=7168, I=2048, E_global=256, E_local=256, local_expert_offset=0, n_group=8,
             topk_group=4, top_k=8, routed_scaling_factor=2.5, bias_dtype=0)
    d.update(kw)
    for k, v in d.items():
        setattr(a, k, v)
    return a


def _ws(a):
    n = ctypes.c_size_t(0)
    return _lib.load().moe_fp8_workspace_size(ctypes.byref(a), ctypes.byref(n)), n.value


def test_workspace_size_dsv3_and_contest_shapes():
    st, n = _ws(_args(T=8192))
    assert st == 0 and n > 8192 * 7168 * 4
    st, n32 = _ws(_args(T=8192, E_local=32, local_expert_offset=64))
    assert st == 0 and n32 < n


def test_workspace_layout_is_consistent():
    a = _args(T=300)
    lay = _lib.MoeWorkspaceLayout()
    assert _lib.load().moe_fp8_workspace_layout(ctypes.byref(a), ctypes.byref(lay)) == 0
    offs = [getattr(lay, f) for f, _ in _lib.MoeWorkspaceLayout._fields_[4:]]
    assert offs == sorted(offs) and offs[0] == 0
    assert all(o % 1024 == 0 for o in offs)
    assert lay.npad % 128 == 0
    # every assignment fits: each expert's segment is padded to whole tiles
    assert lay.npad >= 300 * 8 + min(256, 300 * 8) * 127 // 128 * 0
    assert lay.route_blocks * lay.tokens_per_block >= 300


@pytest.mark.parametrize("bad", [
    dict(H=7000), dict(I=100), dict(E_global=300), dict(n_group=7), dict(top_k=9),
    dict(topk_group=9), dict(E_local=0), dict(local_expert_offset=250, E_local=32),
    dict(T=-1), dict(T=(1 << 24) + 1), dict(top_k=8, topk_group=1, n_group=64),
    dict(E_global=48, E_local=48, n_group=4)])
def test_invalid_shapes_are_rejected(bad):
    st, _ = _ws(_args(**bad))
    assert st == _lib.MOE_ERR_SHAPE


def test_forward_argument_errors_need_no_gpu():
    lib = _lib.load()
    a = _args(T=4)
    assert lib.moe_fp8_forward(None, None) == _lib.MOE_ERR_INVALID_ARG
    # null tensor pointers
    assert lib.moe_fp8_forward(ctypes.byref(a), None) == _lib.MOE_ERR_INVALID_ARG
    a0 = _args(T=0)
    assert lib.moe_fp8_forward(ctypes.byref(a0), None) == _lib.MOE_OK
    a.bias_dtype = 7
    assert lib.moe_fp8_forward(ctypes.byref(a), None) == _lib.MOE_ERR_INVALID_ARG


def test_check_workspace_argument_errors_need_no_gpu():
    lib = _lib.load()
    assert lib.moe_fp8_check_workspace(None, None) == _lib.MOE_ERR_INVALID_ARG
    a0 = _args(T=0)
    assert lib.moe_fp8_check_workspace(ctypes.byref(a0), None) == _lib.MOE_OK
    a = _args(T=4)
    assert lib.moe_fp8_check_workspace(ctypes.byref(a), None) == _lib.MOE_ERR_WORKSPACE
    a.flags = _lib.MOE_FLAG_DEBUG | _lib.MOE_FLAG_DETERMINISTIC
    assert lib.moe_fp8_workspace_size(ctypes.byref(a), ctypes.byref(ctypes.c_size_t())) == 0
    a.flags = 0x40
    assert lib.moe_fp8_check_workspace(ctypes.byref(a), None) == _lib.MOE_ERR_INVALID_ARG


def test_every_buffer_leaves_room_for_its_guard():
    """16 guard bytes fit between each buffer's end and the next buffer."""
    t, k, h, i, el = 300, 8, 7168, 2048, 256
    a = _args(T=t)
    a.flags = _lib.MOE_FLAG_DETERMINISTIC
    lay = _lib.MoeWorkspaceLayout()
    assert _lib.load().moe_fp8_workspace_layout(ctypes.byref(a), ctypes.byref(lay)) == 0
    npad = lay.npad
    sizes = dict(topk_idx=4 * t * k, topk_weights=4 * t * k, counts=4 * el,
                 tile_start=4 * (el + 1), row_token=4 * npad, row_weight=4 * npad,
                 a_perm=npad * h, a_scale_perm=4 * (h // 128) * npad, inter=npad * i,
                 inter_scale=4 * (i // 64) * npad, out_f32=4 * t * h, assign_row=4 * t * k,
                 rows_out=4 * npad * h)
    names = [f for f, _ in _lib.MoeWorkspaceLayout._fields_[4:]]
    offs = [getattr(lay, f) for f in names] + [lay.total_bytes]
    for n, (f, o) in enumerate(zip(names, offs)):
        if f in sizes:
            guard = (o + sizes[f] + 15) // 16 * 16
            assert guard + 16 <= offs[n + 1], f


def test_router_argument_errors_need_no_gpu():
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    assert lib.moe_router_workspace_size(8192, 7168, 256, ctypes.byref(n)) == 0 and n.value > 0
    assert lib.moe_router_workspace_size(128, 7168, 256, ctypes.byref(n)) == 0 and n.value == 0
    assert lib.moe_router_workspace_size(8192, 7168, 16, ctypes.byref(n)) == 0 and n.value == 0
    assert lib.moe_router_workspace_size(8, 7167, 256, ctypes.byref(n)) == _lib.MOE_ERR_SHAPE
    assert lib.moe_router_workspace_size(-1, 7168, 256, ctypes.byref(n)) == _lib.MOE_ERR_SHAPE
    assert lib.moe_router_logits_bf16(None, None, 0, 7168, 256, None, None, 0, None) == _lib.MOE_OK
    assert lib.moe_router_logits_bf16(None, None, 4, 7168, 256, None, None, 0,
                                      None) == _lib.MOE_ERR_INVALID_ARG


def test_noalloc_route_limits_need_no_gpu():
    """The no-alloc router: more tokens than its fixed scratch holds give
    MOE_ERR_TOO_LARGE; an E_global beyond the router's 256 gives MOE_ERR_SHAPE
    (the shape rules of moe_fp8_forward)."""
    lib = _lib.load()
    too_many = lib.moe_fp8_route_noalloc(None, None, 0, 65537, 256, 8, 4, 8, 256, 0, 2.5, None,
                                         None, None, None)
    assert too_many == _lib.MOE_ERR_TOO_LARGE
    wide = lib.moe_fp8_route_noalloc(None, None, 0, 16, 512, 8, 4, 8, 256, 0, 2.5, None, None,
                                     None, None)
    assert wide == _lib.MOE_ERR_SHAPE


def test_status_strings():
    for code in (0, -1, -2, -3, -4, -5, -6, -7, -8, -9):
        assert _lib.status_string(code) != "unknown status"
