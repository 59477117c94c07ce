"""ctypes binding of libhisparse.so, whose C ABI is declared in include/hisparse.h.

The shared library is built in-tree (nano-hisparse_b200/libhisparse.so) by
``make -C nano-hisparse_b200/csrc`` or ``__graft_entry__.build()``. There is no
fallback: importing an operator without the library raises immediately.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent.parent / "libhisparse.so"
ABI_VERSION = 1

HS_OK, HS_ERR_INVALID_ARGUMENT, HS_ERR_UNSUPPORTED, HS_ERR_WORKSPACE, HS_ERR_CUDA, \
    HS_ERR_NOT_MAPPED = range(6)
HS_FLOAT32, HS_FLOAT16, HS_BFLOAT16, HS_INT32, HS_INT64 = range(5)
DEVICE_FLAGS = {
    1: "a row index beyond the pool or host store was skipped",
    2: "ceil(length / page_size) exceeded the table capacity",
    4: "an LRU entry outside [0, hot_rows) was found; tables left unchanged",
    8: "more misses than hot rows; tables left unchanged",
    16: "a bounded wait for an asynchronous copy ran out; results are invalid",
    32: "a batched metadata pointer was not 16-byte aligned; the request was skipped",
}

_DTYPES = {torch.float32: HS_FLOAT32, torch.float16: HS_FLOAT16, torch.bfloat16: HS_BFLOAT16}

_P, _I64, _INT, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
_SIGNATURES = {
    "hs_version": ([], _INT),
    "hs_status_string": ([_INT], ctypes.c_char_p),
    "hs_last_error": ([], ctypes.c_char_p),
    "hs_host_device_pointer": ([_P, ctypes.POINTER(_P)], _INT),
    "hs_quest_workspace_bytes": ([_INT, _I64], _SZ),
    "hs_quest_select": ([_P, _INT, _P, _P, _INT, _INT, _INT, _INT, _I64, _I64, _INT, _INT,
                         _INT, _P, _I64, _P, _P, _SZ, _P, _P], _INT),
    "hs_quest_select_batched": ([_INT, _P, _I64, _INT, _P, _P, _INT, _P, _INT, _INT, _INT, _I64,
                                 _INT, _INT, _INT, _P, _I64, _P, _P, _SZ, _P, _P], _INT),
    "hs_quest_partial_scores_batched": ([_INT, _P, _I64, _INT, _P, _P, _INT, _P, _INT, _INT,
                                         _INT, _I64, _INT, _P, _P, _P], _INT),
    "hs_quest_select_partials": ([_INT, _P, _INT, _P, _INT, _I64, _INT, _INT, _INT, _P, _I64,
                                  _P, _P, _SZ, _P, _P], _INT),
    "hs_resolve_workspace_bytes": ([_INT, _I64, _I64], _SZ),
    "hs_resolve_rows": ([_P, _INT, _I64, _P, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _INT, _P,
                         _P, _P, _P, _P, _I64, _I64, _P, _P, _SZ, _P, _P], _INT),
    "hs_resolve_rows_batched": ([_INT, _P, _I64, _P, _P, _I64, _P, _I64, _P, _P, _I64, _P, _INT,
                                 _P, _P, _P, _P, _P, _P, _SZ, _P, _P], _INT),
    "hs_gather_rows": ([_P, _I64, _P, _I64, _P, _P, _I64, _I64, _INT, _I64, _P, _P], _INT),
    "hs_attend_workspace_bytes": ([_INT, _INT, _INT, _INT, _I64], _SZ),
    "hs_attend_rows": ([_INT, _P, _I64, _INT, _P, _I64, _INT, _P, _I64, _I64, _I64, _P, _I64,
                        _INT, _INT, _INT, _INT, _P, _SZ, _P, _P], _INT),
    "hs_attend_rows_phase": ([_INT, _P, _I64, _INT, _P, _I64, _INT, _P, _I64, _I64, _P, _INT,
                              _INT, _INT, _INT, _INT, _INT, _INT, _INT, _P, _SZ, _P, _P], _INT),
    "hs_attend_merge": ([_INT, _INT, _P, _I64, _INT, _INT, _INT, _INT, _I64, _P, _SZ, _P, _P],
                        _INT),
    "hs_append_rows": ([_INT, _P, _P, _I64, _INT, _P, _P, _P, _P, _I64, _P, _P, _I64, _P, _P,
                        _P, _INT, _INT, _INT, _P, _P], _INT),
    "hs_attend_rows_static": ([_INT, _P, _I64, _INT, _P, _I64, _INT, _P, _I64, _I64, _I64, _P,
                               _I64, _INT, _INT, _INT, _INT, _P, _P], _INT),
}

_lib = None
_lock = threading.Lock()


def load():
    """Load libhisparse.so once and bind every entry point of the header."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `make -C nano-hisparse_b200/csrc` "
                "(the sm_100a kernels have no fallback)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (argtypes, restype) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes, fn.restype = argtypes, restype
        if lib.hs_version() != ABI_VERSION:
            raise ImportError(f"libhisparse ABI {lib.hs_version()} != expected {ABI_VERSION}")
        _lib = lib
    return _lib


def check(status: int):
    """Raise the exception matching an hs_status (ValueError for bad arguments)."""
    if status == HS_OK:
        return
    message = load().hs_last_error().decode(errors="replace")
    if status in (HS_ERR_INVALID_ARGUMENT, HS_ERR_UNSUPPORTED, HS_ERR_WORKSPACE):
        raise ValueError(message)
    raise RuntimeError(message)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"unsupported element type {dtype}") from None


def stream_of(device) -> int:
    """cudaStream_t of torch's current stream on `device`."""
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and (not isinstance(t, torch.Tensor) or t.device.type != "cuda"):
            raise ValueError("hisparse_b200 operators take CUDA tensors; there is no CPU path")


def ptr(t):
    return None if t is None else t.data_ptr()


_status_words: dict = {}


def status_word(device) -> torch.Tensor:
    """Per-device int32 word into which kernels OR the HS_DEV_* flags."""
    device = torch.device(device)
    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _status_words.get(index)
    if word is None:
        # a normal (non-inference) tensor, so that it can be cleared anywhere
        with torch.inference_mode(False):
            word = torch.zeros(1, dtype=torch.int32, device=f"cuda:{index}")
        _status_words[index] = word
    return word


def device_flags(device, reset=True) -> list[str]:
    """Reads (synchronously) and optionally clears the device status word;
    returns the flag descriptions. Diagnostic only, never on the decode path."""
    word = status_word(device)
    value = int(word.item())
    if reset:
        with torch.no_grad():
            word.zero_()
    return [text for bit, text in DEVICE_FLAGS.items() if value & bit]


def workspace(nbytes: int, device, zeroed: bool = False) -> torch.Tensor | None:
    """Scratch from the caching allocator (stream-ordered, graph-safe)."""
    if nbytes == 0:
        return None
    if zeroed:
        return torch.zeros(nbytes, dtype=torch.uint8, device=device)
    return torch.empty(nbytes, dtype=torch.uint8, device=device)
