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
