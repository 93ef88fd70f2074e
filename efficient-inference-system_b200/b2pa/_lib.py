"""ctypes binding of libb2pa.so (the C ABI declared in include/b2pa.h).

The library is loaded from the package's in-tree ``lib/`` directory.  There is
no fallback: if the shared object is missing or fails to load, every entry
point raises ``RuntimeError`` telling the caller to build it.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent.parent / "lib" / "libb2pa.so"

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

STATUS_NAMES = {
    0: "B2PA_OK",
    -1: "B2PA_ERR_INVALID_ARGUMENT",
    -2: "B2PA_ERR_UNSUPPORTED",
    -3: "B2PA_ERR_BAD_BLOCK_ID",
    -4: "B2PA_ERR_WORKSPACE",
    -5: "B2PA_ERR_CUDA",
    -6: "B2PA_ERR_DEVICE_TIMEOUT",
}
STATUS_CODES = {name: code for code, name in STATUS_NAMES.items()}

# Every symbol include/b2pa.h declares, with its ctypes signature.
_I64P = ctypes.POINTER(ctypes.c_int64)
_VP = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
SIGNATURES: dict[str, tuple] = {
    "b2pa_abi_version": (_I, []),
    "b2pa_last_error_string": (ctypes.c_char_p, []),
    "b2pa_status_read": (_I, [_VP, ctypes.POINTER(ctypes.c_int32), _VP]),
    "b2pa_status_clear": (_I, [_VP, _VP]),
    "b2pa_kv_append": (_I, [_VP, _I64P, _VP, _I64P, _VP, _VP, _I64P, _I64, _VP, _I64, _I, _VP, _VP,
                            _I, _I, _I, _I, _I, _I, _VP, _VP]),
    "b2pa_paged_decode_workspace_size": (ctypes.c_size_t, [_I, _I, _I, _I, _I, _I]),
    "b2pa_paged_decode": (_I, [_VP, _I64P, _VP, _VP, _I64P, _I64, _VP, _I64, _I, _VP, _VP, _VP, _I64P,
                               _I, _I, _I, _I, ctypes.c_float, _I, _VP, ctypes.c_size_t, _VP, _VP]),
    "b2pa_paged_decode_append": (_I, [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _VP, _I64P, _I64, _VP, _I64, _I,
                                      _VP, _VP, _VP, _VP, _VP, _VP, _I64P, _I, _I, _I, _I, ctypes.c_float, _I,
                                      _VP, ctypes.c_size_t, _VP, _VP]),
    "b2pa_paged_decode_noalloc": (_I, [_VP, _I64P, _VP, _VP, _I64P, _I64, _VP, _I64, _I, _VP, _VP, _VP, _I64P,
                                       _I, _I, _I, _I, ctypes.c_float, _I, _VP, _VP]),
    "b2pa_paged_prefill_workspace_size": (ctypes.c_size_t, [_I, _I, _I, _I, _I, _I, _I]),
    "b2pa_paged_prefill": (_I, [_VP, _I64P, _VP, _VP, _I64P, _I64, _VP, _I64, _I, _VP, _VP, _VP, _I64P,
                                _I, _I, _I, _I, _I, ctypes.c_float, _I, _VP, ctypes.c_size_t, _VP, _VP]),
    "b2pa_paged_prefill_append": (_I, [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _VP, _I64P, _I64, _VP, _I64, _I,
                                       _VP, _VP, _VP, _VP, _VP, _VP, _I64P, _I, _I, _I, _I, _I, ctypes.c_float,
                                       _I, _VP, ctypes.c_size_t, _VP, _VP]),
    "b2pa_zero_blocks": (_I, [_VP, _VP, _I64P, _I64, _VP, _I, _I, _I, _I, _I, _VP, _VP]),
    "b2pa_patch_table": (_I, [_VP, _I64, _VP, _I, _VP, _VP]),
    "b2pa_selftest_wait_timeout": (_I, [_VP, _VP, _VP]),
    "b2pa_rows_linear": (_I, [_VP, _I64, _I, _I, _VP, _VP, ctypes.c_float, _VP, _VP, _I, _I, _VP, _I64, _I,
                              _VP, _VP]),
    "b2pa_rows_embed": (_I, [_VP, _VP, _I, _VP, _I64, _VP, _I64, _I, _VP, _I64, _VP, _VP]),
    "b2pa_rows_argmax": (_I, [_VP, _I64, _I, _I, _VP, _VP, _VP]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads libb2pa.so once and binds every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("B2PA_LIB", str(LIB_PATH)))
        if not path.exists():
            raise RuntimeError(
                f"libb2pa.so not found at {path}; build it with `python -m b2pa.build` "
                "(or __graft_entry__.build()). There is no CPU fallback.")
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return load().b2pa_last_error_string().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: {STATUS_NAMES.get(rc, rc)}: {last_error()}")


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return DTYPE_F32
    if dtype == torch.bfloat16:
        return DTYPE_BF16
    if dtype == torch.float16:
        return DTYPE_F16
    raise TypeError(f"b2pa supports float32, bfloat16 and float16, not {dtype}")


def strides4(t: torch.Tensor):
    if t.dim() != 4:
        raise ValueError(f"expected a 4-d tensor, got shape {tuple(t.shape)}")
    return (ctypes.c_int64 * 4)(*t.stride())


def stream_handle(device: torch.device) -> int:
    """The raw cudaStream_t of the current stream of ``device``."""
    return torch._C._cuda_getCurrentRawStream(device.index if device.index is not None else torch.cuda.current_device())


# ------------------------------------------------------------ per-device state
_status: dict[int, torch.Tensor] = {}
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def status_buffer(device: torch.device) -> torch.Tensor:
    """The device status word kernels on this device report into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _status.get(idx)
    if buf is None:
        buf = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = buf
    return buf


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A cached byte buffer of at least ``nbytes`` for the current stream.

    One buffer per (device, stream): kernels on one stream run in order, so
    reusing the buffer across calls on that stream is safe.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch._C._cuda_getCurrentRawStream(idx))
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(int(nbytes * 1.25), 1 << 20)
        buf = torch.empty(size, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[key] = buf
    return buf


def read_status(device: torch.device) -> int:
    """Synchronising read of the device status word (0 = no fault seen)."""
    buf = status_buffer(device)
    host = ctypes.c_int32(0)
    check(load().b2pa_status_read(buf.data_ptr(), ctypes.byref(host), stream_handle(device)), "b2pa_status_read")
    return int(host.value)


def clear_status(device: torch.device) -> None:
    buf = status_buffer(device)
    check(load().b2pa_status_clear(buf.data_ptr(), stream_handle(device)), "b2pa_status_clear")


def raise_on_device_status(device: torch.device, what: str = "b2pa kernels") -> None:
    code = read_status(device)
    if code != 0:
        clear_status(device)
        raise RuntimeError(f"{what} reported {STATUS_NAMES.get(code, code)} on {device}")
