"""The C-ABI library loads without a GPU and exports every symbol the header declares."""

import ctypes
import re
from pathlib import Path

import pytest

from anchorkv_b200 import _lib
from anchorkv_b200 import pool as P

ROOT = Path(__file__).resolve().parents[1]
HEADER = (ROOT / "include" / "anchorkv_b200.h").read_text()
DECLARED = sorted(set(re.findall(r"\b(akv_\w+)\s*\(", HEADER)))


def test_header_declares_the_boundary():
    assert {"akv_quantize", "akv_dequantize", "akv_pack_pages", "akv_repack_pages", "akv_unpack_pages",
            "akv_decode_partials", "akv_merge", "akv_packed_attention"} <= set(DECLARED)


@pytest.mark.parametrize("name", DECLARED)
def test_library_exports_declared_symbol(name):
    lib = _lib.load()
    assert isinstance(getattr(lib, name), ctypes._CFuncPtr)
    assert name in _lib.PROTOTYPES, "every declared entry point has a ctypes prototype"


def test_host_helpers_need_no_gpu():
    lib = _lib.load()
    assert lib.akv_abi_version() == 5
    assert _lib.status_string(_lib.ERR_INVALID).startswith("invalid")
    for dim in (64, 128):
        for group in (32, 64, 128, 16 * dim):
            for bits, mode in P.BITS_TO_MODE.items():
                assert lib.akv_record_bytes(dim, group, mode) == P.record_bytes(dim, group, bits)
    assert lib.akv_record_bytes(128, 2048, _lib.MODE_SKIP) == 0
    assert lib.akv_record_bytes(128, 3, _lib.MODE_INT4) == -1


def test_invalid_arguments_are_rejected_before_any_launch():
    """Null pointers and unsupported geometry return a status; nothing is launched,
    so this runs without a GPU."""
    lib = _lib.load()
    assert lib.akv_quantize(None, 0, 10, 16, 8, 0, None, None, None) == _lib.ERR_INVALID
    assert lib.akv_decode_partials(None, 0, None, 0, None, 0, None, 0, 0, 1, 1, 1, 128, 64, 1.0, 1,
                                   None, 0, None, None) == _lib.ERR_INVALID
    with pytest.raises(ValueError):
        _lib.call("akv_merge", None, 1, 1, 128, None, 0, 0, None, None, None)
    with pytest.raises(ValueError):
        _lib.call("akv_merge_states", None, 2, 1, 1, 128, None, 0, 0, None)


def test_allocation_free_entry_reports_the_workspace_entrys_status():
    """akv_packed_attention_static returns the plan's own status (unsupported
    head_dim, inconsistent heads) as akv_packed_attention does; both checks
    come before any CUDA call, so this runs without a GPU.  The non-null
    pointers are never dereferenced."""
    lib = _lib.load()
    fake = ctypes.c_void_p(0x1000)

    def static(batch, q_heads, kv_heads, head_dim):
        return lib.akv_packed_attention_static(fake, 1 << 20, fake, 64, None, 64, fake, 0, head_dim, batch,
                                               q_heads, kv_heads, head_dim, 16 * head_dim, 1.0, 4, fake, 0,
                                               head_dim, None, None)

    assert static(1, 16, 8, 96) == _lib.ERR_UNSUPPORTED
    assert static(1, 12, 8, 128) == _lib.ERR_INVALID  # 12 query heads over 8 KV heads
    assert lib.akv_workspace_bytes(1, 16, 8, 96, 64, 4) == -1


def test_every_entry_point_checks_its_arguments_before_a_launch():
    """Each call below fails its host-side checks (or is an empty request, which
    returns before any launch); none reaches the CUDA runtime, so this runs
    without a GPU.  Pointers are never dereferenced: 0x1000 stands for an
    aligned buffer, 0x1004 / 0x1008 for misaligned ones."""
    lib = _lib.load()
    vp = ctypes.c_void_p
    ok, inval, unsup = _lib.OK, _lib.ERR_INVALID, _lib.ERR_UNSUPPORTED
    a, a4, a8 = vp(0x1000), vp(0x1004), vp(0x1008)
    tensor, page = _lib.SEM_TENSOR, _lib.SEM_PAGE
    f16 = _lib.DTYPE_F16
    assert lib.akv_status_string(99).decode() == "unknown status"

    # akv_quantize(src, src_dtype, numel, group, bits, semantics, payload, scales, stream)
    assert lib.akv_quantize(a, f16, 64, 16, 5, tensor, a, a, None) == inval          # bits
    assert lib.akv_quantize(a, f16, 64, 15, 4, tensor, a, a, None) == inval          # odd INT4 group
    assert lib.akv_quantize(a, f16, 64, 16, 8, 7, a, a, None) == inval               # semantics
    assert lib.akv_quantize(a, f16, 0, 16, 8, tensor, a, a, None) == inval           # empty
    assert lib.akv_quantize(a, f16, 64, 0, 8, tensor, a, a, None) == inval           # group
    assert lib.akv_quantize(a, 9, 64, 16, 8, tensor, a, a, None) == inval            # source dtype
    assert lib.akv_quantize(a, 9, 60, 12, 8, page, a, a, None) == inval              # (the flat path too)
    # akv_dequantize(payload, scales, numel, group, bits, out, out_dtype, stream)
    assert lib.akv_dequantize(a, a, 64, 16, 8, None, f16, None) == inval
    assert lib.akv_dequantize(a, a, 64, 16, 2, a, f16, None) == inval
    assert lib.akv_dequantize(a, a, 64, 16, 8, a, 9, None) == inval
    assert lib.akv_dequantize(a, a, 60, 12, 8, a, 9, None) == inval

    # akv_pack_pages(src_k, src_v, outer_stride, head_stride, blocks_per_row, n_pages, dst_desc,
    #                arena, arena_bytes, heads, head_dim, group, semantics, dev_status, stream)
    def pack(src=a, outer=8192, head=4096, bpr=4, n=1, heads=2, dim=128, group=2048, sem=tensor):
        return lib.akv_pack_pages(src, a, outer, head, bpr, n, a, a, 1 << 20, heads, dim, group, sem, None, None)

    assert pack(dim=96) == unsup and pack(group=48) == unsup and pack(dim=64, group=2048) == unsup
    assert pack(heads=0) == inval and pack(src=a8) == inval and pack(outer=8196) == inval
    assert pack(bpr=0) == inval and pack(n=-1) == inval and pack(sem=5) == inval
    assert pack(n=0) == ok  # nothing to pack: no launch
    # akv_repack_pages(src_desc, dst_desc, n_pages, arena, arena_bytes, heads, head_dim, group,
    #                  semantics, dev_status, stream)
    assert lib.akv_repack_pages(a, a, -1, a, 1 << 20, 2, 128, 64, page, None, None) == inval
    assert lib.akv_repack_pages(a, a, 1, a8, 1 << 20, 2, 128, 64, page, None, None) == inval
    assert lib.akv_repack_pages(a, a, 1, a, 1 << 20, 2, 128, 64, 3, None, None) == inval
    assert lib.akv_repack_pages(a, a, 1, a, 1 << 20, 2, 64, 2048, page, None, None) == unsup
    assert lib.akv_repack_pages(a, a, 0, a, 1 << 20, 2, 128, 64, page, None, None) == ok
    # akv_unpack_pages(desc, n_pages, arena, arena_bytes, heads, head_dim, group, out_k, out_v,
    #                  out_dtype, dev_status, stream)
    assert lib.akv_unpack_pages(a, 1, a, 1 << 20, 2, 128, 64, a, a, 7, None, None) == inval
    assert lib.akv_unpack_pages(a, 1, a, 1 << 20, 2, 128, 64, a8, a, f16, None, None) == inval
    assert lib.akv_unpack_pages(None, 1, a, 1 << 20, 2, 128, 64, a, a, f16, None, None) == inval
    assert lib.akv_unpack_pages(a, 0, a, 1 << 20, 2, 128, 64, a, a, f16, None, None) == ok

    # akv_append_rows(src_k, src_v, batch_stride, head_stride, token_stride, batch, rows, first_row,
    #                 table, table_stride, page, new_desc, arena, arena_bytes, heads, head_dim, status, stream)
    def append(src=a, strides=(4096, 2048, 128), batch=2, rows=1, first=0, stride=8, page_=0, dim=128):
        return lib.akv_append_rows(src, a, *strides, batch, rows, first, a, stride, page_, None, a, 1 << 20, 2,
                                   dim, None, None)

    assert append(dim=32) == unsup
    assert append(rows=0) == inval and append(first=12, rows=5) == inval and append(first=-1) == inval
    assert append(stride=3, page_=3) == inval and append(page_=-1) == inval and append(batch=0) == inval
    assert append(src=a4) == inval and append(strides=(4096, 2048, 130)) == inval

    # workspace, exchange and merge geometry
    assert lib.akv_workspace_bytes(0, 16, 8, 128, 64, 4) == -1
    assert lib.akv_workspace_bytes(1, 16, 8, 128, -1, 4) == -1
    assert lib.akv_exchange_bytes(9, 1, 32, 128) == -1 and lib.akv_exchange_bytes(0, 1, 32, 128) == -1
    assert lib.akv_exchange_bytes(2, 1, 32, 96) == -1
    assert lib.akv_exchange_bytes(2, 1, 32, 128) == 2 * 2 * 4 * 32 * 130 * 8  # 4 part-states per row
    assert lib.akv_exchange_bytes(2, 4, 32, 64) == 2 * 2 * 1 * 128 * 66 * 8   # one per row past 64 rows
    peers = (vp * 2)(0x1000, 0x2000)
    bad_peers = (vp * 2)(0x1000, 0x2008)

    def exchange(epoch=1, rank=0, world=2, dim=128, buffers=peers):
        return lib.akv_merge_exchange(a, 1, 32, dim, buffers, rank, world, epoch, a, 0, dim, None, None)

    assert exchange(epoch=0) == inval and exchange(rank=2) == inval and exchange(rank=-1) == inval
    assert exchange(world=9) == inval and exchange(dim=96) == unsup and exchange(buffers=bad_peers) == inval
    assert lib.akv_merge(a, 1, 16, 96, a, 0, 96, None, None, None) == unsup
    assert lib.akv_merge(a, 0, 16, 128, a, 0, 128, None, None, None) == inval
    assert lib.akv_merge(a, 1, 16, 128, None, 0, 128, None, None, None) == inval
    assert lib.akv_merge_states(a, 0, 1, 16, 128, a, 0, 128, None) == inval
    assert lib.akv_merge_states(a, 2, 1, 16, 96, a, 0, 96, None) == unsup

    # allocation helpers
    handle = ctypes.create_string_buffer(64)
    out = vp()
    assert lib.akv_ipc_alloc(0, ctypes.byref(out), handle) == inval
    assert lib.akv_ipc_alloc(64, None, handle) == inval
    assert lib.akv_ipc_open(None, ctypes.byref(out)) == inval
    assert lib.akv_ipc_close(None) == inval and lib.akv_ipc_free(None) == inval
    assert lib.akv_status_alloc(None, None) == inval and lib.akv_status_free(None) == inval


C_CALLER = r"""
#include "anchorkv_b200.h"
#include <stdio.h>
int main(void) {
  /* host-only calls: no GPU needed */
  long long int4_record = (long long)akv_record_bytes(128, 2048, AKV_MODE_INT4);
  int empty = akv_quantize(0, AKV_DTYPE_F16, 0, 16, 8, AKV_SEM_TENSOR, 0, 0, 0);
  printf("%d %lld %d %lld\n", akv_abi_version(), int4_record, empty, (long long)akv_static_scratch_bytes());
  return 0;
}
"""


@pytest.mark.parametrize("compiler,flags", [("gcc", ["-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror"]),
                                            ("g++", ["-std=c++17", "-Wall", "-Wextra", "-Werror", "-x", "c++"])])
def test_header_serves_c_and_cxx_callers(tmp_path, compiler, flags):
    """A C or C++ program includes the header, links the library and calls it,
    with no Python in between (the binding a C or C++ host would add)."""
    import shutil
    import subprocess

    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} is not installed")
    src, exe = tmp_path / "caller.c", tmp_path / "caller"
    src.write_text(C_CALLER)
    libdir = _lib.LIB_PATH.parent
    subprocess.run([compiler, *flags, "-I", str(ROOT / "include"), str(src), "-L", str(libdir), "-lanchorkv_b200",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    lib = _lib.load()
    assert out == [str(lib.akv_abi_version()), str(P.record_bytes(128, 2048, 4)), str(_lib.ERR_INVALID),
                   str(lib.akv_static_scratch_bytes())]
