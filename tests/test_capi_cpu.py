"""CPU checks of the C ABI boundary: the library loads, exports every entry point
include/fa_b200.h declares, its argument structs match the ctypes mirrors byte for
byte, and the host-side validation answers without a GPU."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from tilelang_fa_v100 import _ext

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fa_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(fa_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("fa_fwd", "fa_bwd", "fa_paged_prefill", "fa_decode", "fa_bwd_workspace_size",
                 "fa_decode_workspace_size", "fa_status_string"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _ext.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _ext.SIGNATURES, "ctypes signature missing for " + name


def _c_layout(struct_name, fields):
    body = "\n".join('  printf("%%s %%zu\\n", "%s", offsetof(%s, %s));' % (f, struct_name, f)
                     for f in fields)
    prog = """#include <stdio.h>
#include <stddef.h>
#include "fa_b200.h"
int main(void) {
  printf("sizeof %%zu\\n", sizeof(%s));
%s
  return 0;
}
""" % (struct_name, body)
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "l.c")
        exe = os.path.join(d, "l")
        open(c, "w").write(prog)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    return dict((a, int(b)) for a, b in (ln.split() for ln in out.strip().splitlines()))


@pytest.mark.parametrize("cname,cls", [("fa_fwd_args_t", _ext.FwdArgs),
                                       ("fa_bwd_args_t", _ext.BwdArgs),
                                       ("fa_varlen_fwd_args_t", _ext.VarlenFwdArgs),
                                       ("fa_varlen_bwd_args_t", _ext.VarlenBwdArgs),
                                       ("fa_paged_args_t", _ext.PagedArgs),
                                       ("fa_decode_args_t", _ext.DecodeArgs),
                                       ("fa_kv_write_args_t", _ext.KvWriteArgs)])
def test_struct_layout_matches_c(cname, cls):
    fields = [f for f, _ in cls._fields_]
    lay = _c_layout(cname, fields)
    assert lay["sizeof"] == ctypes.sizeof(cls)
    for f in fields:
        assert lay[f] == getattr(cls, f).offset, f


def test_status_strings_and_version():
    lib = _ext.load()
    assert b"sm_100a" in lib.fa_version()
    for s in range(-7, 1):
        assert lib.fa_status_string(s)
    assert lib.fa_launch_count() >= 0


def test_null_arguments_rejected_on_host():
    lib = _ext.load()
    a = _ext.FwdArgs()
    assert lib.fa_fwd(ctypes.byref(a), None) == _ext.FA_ERR_INVALID_ARG
    assert lib.fa_fwd(None, None) == _ext.FA_ERR_INVALID_ARG
    p = _ext.PagedArgs()
    assert lib.fa_paged_prefill(ctypes.byref(p), None) == _ext.FA_ERR_INVALID_ARG
    d = _ext.DecodeArgs()
    assert lib.fa_decode(ctypes.byref(d), None, 0, None) == _ext.FA_ERR_INVALID_ARG
    b = _ext.BwdArgs()
    assert lib.fa_bwd(ctypes.byref(b), None, 0, None) == _ext.FA_ERR_INVALID_ARG
    w = _ext.KvWriteArgs()
    assert lib.fa_kv_cache_write(ctypes.byref(w), None) == _ext.FA_ERR_INVALID_ARG
    assert lib.fa_kv_cache_write(None, None) == _ext.FA_ERR_INVALID_ARG
    w.num_tokens, w.num_kv_heads, w.head_dim, w.page_size, w.num_pages = 4, 8, 128, 16, 10
    assert lib.fa_kv_cache_write(ctypes.byref(w), None) == _ext.FA_ERR_INVALID_ARG  # null tensors


def test_unsupported_head_dim_rejected_on_host():
    lib = _ext.load()
    a = _ext.FwdArgs(1, 1, 1, 1, 1)
    a.batch, a.seqlen_q, a.seqlen_k, a.num_heads, a.num_heads_k = 1, 8, 8, 2, 2
    for d in (16, 48, 80, 192, 512):  # dense head dims are 32 / 64 / 96 / 128 / 256
        a.head_dim, a.dtype = d, 0
        assert lib.fa_fwd(ctypes.byref(a), None) == _ext.FA_ERR_UNSUPPORTED
    a.head_dim, a.num_heads_k = 64, 3  # H % Hk != 0
    assert lib.fa_fwd(ctypes.byref(a), None) == _ext.FA_ERR_INVALID_ARG


def test_decode_workspace_size_is_host_computed():
    lib = _ext.load()
    d = _ext.DecodeArgs()
    d.batch, d.num_heads, d.num_kv_heads, d.head_dim = 256, 32, 8, 128
    d.page_size, d.num_pages, d.max_blocks, d.dtype = 16, 70000, 512, 1
    n = lib.fa_decode_workspace_size(ctypes.byref(d))
    assert n > 256 * 32 * 128 * 4  # several splits of fp32 partial outputs
    d.num_splits = 1
    assert lib.fa_decode_workspace_size(ctypes.byref(d)) == 0


def test_varlen_entry_points_validate_on_host():
    lib = _ext.load()
    assert lib.fa_varlen_fwd(None, None) == _ext.FA_ERR_INVALID_ARG
    a = _ext.VarlenFwdArgs()
    assert lib.fa_varlen_fwd(ctypes.byref(a), None) == _ext.FA_ERR_INVALID_ARG  # null tensors
    a.q = a.k = a.v = a.out = a.lse = a.cu_seqlens_q = a.cu_seqlens_k = 16
    a.batch, a.total_q, a.total_k, a.max_seqlen_q, a.max_seqlen_k = 2, 10, 12, 6, 7
    a.num_heads, a.num_heads_k, a.dtype = 4, 2, 1
    for d in (32, 96, 512):  # varlen head dims are 64 / 128 / 256
        a.head_dim = d
        assert lib.fa_varlen_fwd(ctypes.byref(a), None) == _ext.FA_ERR_UNSUPPORTED
    a.head_dim, a.num_heads_k = 64, 3  # H % Hk != 0
    assert lib.fa_varlen_fwd(ctypes.byref(a), None) == _ext.FA_ERR_INVALID_ARG
    a.num_heads_k, a.softmax_scale, a.softcap = 2, 0.125, -1.0
    assert lib.fa_varlen_fwd(ctypes.byref(a), None) == _ext.FA_ERR_INVALID_ARG
    a.softcap = 0.0
    a.q_stride[0], a.q_stride[1] = 4 * 64 + 4, 64  # token stride not a multiple of 8
    assert lib.fa_varlen_fwd(ctypes.byref(a), None) == _ext.FA_ERR_ALIGNMENT
    b = _ext.VarlenBwdArgs()
    assert lib.fa_varlen_bwd(ctypes.byref(b), None, 0, None) == _ext.FA_ERR_INVALID_ARG
    # workspace: the dense backward's for batch x max_seqlen_q rows
    b.batch, b.total_q, b.total_k, b.max_seqlen_q, b.max_seqlen_k = 3, 300, 400, 200, 250
    b.num_heads, b.num_heads_k, b.head_dim = 4, 2, 128
    d = _ext.BwdArgs()
    d.batch, d.seqlen_q, d.seqlen_k, d.num_heads, d.num_heads_k, d.head_dim = 3, 200, 250, 4, 2, 128
    assert lib.fa_varlen_bwd_workspace_size(ctypes.byref(b)) == lib.fa_bwd_workspace_size(ctypes.byref(d))
