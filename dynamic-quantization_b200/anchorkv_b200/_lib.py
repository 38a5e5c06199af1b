"""ctypes binding of libanchorkv_b200.so (the C ABI in include/anchorkv_b200.h).

The library is built in-tree (``dynamic-quantization_b200/build.py``) and
loaded once per process.  There is no fallback: if the library or a CUDA device
is missing, every compute entry point raises :class:`NativeUnavailableError`.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libanchorkv_b200.so"

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_SCRATCH = 0, 1, 2, 3, 4
DEV_BAD_DESCRIPTOR, DEV_TIMEOUT = 1, 2
MODE_SKIP, MODE_INT4, MODE_INT8, MODE_FP16 = 0, 1, 2, 3
SEM_TENSOR, SEM_PAGE = 0, 1
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2

_c_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

# name -> (restype, argtypes); the order follows the header.
PROTOTYPES = {
    "akv_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "akv_abi_version": (ctypes.c_int, []),
    "akv_status_alloc": (ctypes.c_int, [ctypes.POINTER(_c_p), ctypes.POINTER(_c_p)]),
    "akv_status_free": (ctypes.c_int, [_c_p]),
    "akv_record_bytes": (_i64, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "akv_quantize": (ctypes.c_int, [_c_p, ctypes.c_int, _i64, _i64, ctypes.c_int, ctypes.c_int,
                                    _c_p, _c_p, _c_p]),
    "akv_dequantize": (ctypes.c_int, [_c_p, _c_p, _i64, _i64, ctypes.c_int, _c_p, ctypes.c_int, _c_p]),
    "akv_pack_pages": (ctypes.c_int, [_c_p, _c_p, _i64, _i64, _i64, _i64, _c_p, _c_p, _i64,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _c_p, _c_p]),
    "akv_repack_pages": (ctypes.c_int, [_c_p, _c_p, _i64, _c_p, _i64, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, _c_p, _c_p]),
    "akv_unpack_pages": (ctypes.c_int, [_c_p, _i64, _c_p, _i64, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, _c_p, _c_p, ctypes.c_int, _c_p, _c_p]),
    "akv_append_rows": (ctypes.c_int, [_c_p, _c_p, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       _c_p, _i64, ctypes.c_int, _c_p, _c_p, _i64, ctypes.c_int, ctypes.c_int,
                                       _c_p, _c_p]),
    "akv_workspace_bytes": (_i64, [ctypes.c_int] * 6),
    "akv_decode_partials": (ctypes.c_int, [_c_p, _i64, _c_p, _i64, _c_p, _i32, _c_p, _i64, _i64,
                                           _i32, _i32, _i32, _i32, _i32, _f32, _i32, _c_p, _i64, _c_p,
                                           _c_p]),
    "akv_exchange_bytes": (_i64, [_i32, _i32, _i32, _i32]),
    "akv_merge_exchange": (ctypes.c_int, [_c_p, _i32, _i32, _i32, _c_p, _i32, _i32, ctypes.c_uint32, _c_p, _i64,
                                          _i64, _c_p, _c_p]),
    "akv_ipc_alloc": (ctypes.c_int, [_i64, ctypes.POINTER(_c_p), _c_p]),
    "akv_ipc_open": (ctypes.c_int, [_c_p, ctypes.POINTER(_c_p)]),
    "akv_ipc_close": (ctypes.c_int, [_c_p]),
    "akv_ipc_free": (ctypes.c_int, [_c_p]),
    "akv_merge": (ctypes.c_int, [_c_p, _i32, _i32, _i32, _c_p, _i64, _i64, _c_p, _c_p, _c_p]),
    "akv_merge_states": (ctypes.c_int, [_c_p, _i32, _i32, _i32, _i32, _c_p, _i64, _i64, _c_p]),
    "akv_packed_attention": (ctypes.c_int, [_c_p, _i64, _c_p, _i64, _c_p, _i32, _c_p, _i64, _i64,
                                            _i32, _i32, _i32, _i32, _i32, _f32, _i32, _c_p, _i64,
                                            _i64, _c_p, _i64, _c_p, _c_p]),
    "akv_packed_attention_static": (ctypes.c_int, [_c_p, _i64, _c_p, _i64, _c_p, _i32, _c_p, _i64, _i64,
                                                   _i32, _i32, _i32, _i32, _i32, _f32, _i32, _c_p, _i64,
                                                   _i64, _c_p, _c_p]),
    "akv_static_scratch_bytes": (_i64, []),
}


class NativeUnavailableError(RuntimeError):
    """The CUDA library or a CUDA device is missing; there is no CPU fallback."""


class KernelError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


_lock = threading.Lock()
_lib = None


def load(path: Path | str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and return the library with its prototypes set."""
    global _lib
    lib = _lib
    if lib is not None:  # loaded: no lock on the per-call path
        return lib
    with _lock:
        if _lib is None:
            p = Path(path)
            if not p.exists():
                raise NativeUnavailableError(
                    f"{p} is missing; build it with `python dynamic-quantization_b200/build.py`")
            lib = ctypes.CDLL(str(p))
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def status_string(status: int) -> str:
    return load().akv_status_string(status).decode()


def call(name: str, *args) -> None:
    """Call an entry point that returns a status; raise on failure.

    Invalid arguments map to ValueError (the reference's convention for bad
    geometry), everything else to KernelError."""
    status = getattr(load(), name)(*args)
    if status == OK:
        return
    msg = f"{name}: {status_string(status)}"
    if status in (ERR_INVALID, ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise KernelError(msg)


def require_cuda(tensor, what: str = "tensor") -> None:
    if not getattr(tensor, "is_cuda", False):
        raise ValueError(f"{what} must be a CUDA tensor: anchorkv_b200 runs its data plane on the GPU only")


def stream_of(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


DEV_BITS = {DEV_BAD_DESCRIPTOR: "a page descriptor outside the arena or misaligned (page skipped)",
            DEV_TIMEOUT: "a bounded wait that gave up (a bulk copy or a peer's exchange flag)"}


class StatusWord:
    """The int32 word a device's kernels OR their AKV_DEV_* error bits into.

    It lives in mapped pinned host memory (akv_status_alloc): kernels write it
    through its device address (:meth:`data_ptr`), the host reads it through
    its host address with no copy and no synchronisation, so every API call
    can check it before launching.  A kernel's bits are visible once it has
    finished."""

    def __init__(self, index: int):
        import torch

        host, dev = ctypes.c_void_p(), ctypes.c_void_p()
        with torch.cuda.device(index):
            call("akv_status_alloc", ctypes.byref(host), ctypes.byref(dev))
        self.index = index
        self._dev = dev.value
        self._word = ctypes.c_int32.from_address(host.value)

    def data_ptr(self) -> int:
        return self._dev

    @property
    def value(self) -> int:
        return self._word.value

    def clear(self) -> None:
        self._word.value = 0


def describe_status(bits: int) -> str:
    parts = [text for bit, text in DEV_BITS.items() if bits & bit]
    return "; ".join(parts) or f"unknown device status bits {bits:#x}"


_status = {}


def status_word(device) -> StatusWord:
    """The device's status word (one per device, created on first use)."""
    word = _status.get(device)  # fast path: the device object seen before
    if word is not None:
        return word
    import torch

    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in _status:
        _status[key] = StatusWord(key)
    if dev.index is not None:  # "cuda" without an index follows the current device: not cached by name
        _status[device] = _status[key]
    return _status[key]


def raise_pending(device) -> None:
    """Raise :class:`KernelError` if a kernel that has finished on ``device``
    reported an error (and clear the word, so the call after this one runs).

    The reference signals bad input with exceptions from host code; here the
    page table and exchange flags are read on the device, so their errors
    surface on the next API call instead of as silent zeros."""
    word = status_word(device)
    bits = word.value
    if bits:
        word.clear()
        raise KernelError(f"an earlier kernel on cuda:{word.index} reported: {describe_status(bits)}")


def status_ptr(device) -> int:
    """Device address of ``device``'s status word for a launch, after raising
    any error a finished kernel already reported there (:func:`raise_pending`)."""
    word = status_word(device)
    if word.value:
        raise_pending(device)
    return word.data_ptr()


def take_device_status(device=None) -> int:
    """Synchronise, return and clear the device error bits (0 = no error)."""
    import torch

    dev = device if device is not None else torch.cuda.current_device()
    word = status_word(dev)
    torch.cuda.synchronize(word.index)
    value = word.value
    word.clear()
    return value
