"""ctypes binding of libopus_b200.so (the C ABI declared in include/opus_b200.h).

The library is built in-tree (``python -m opus_b200.csrc.build``).  Loading
fails loudly when it is missing: the selection path has no host fallback.
"""
from __future__ import annotations

import ctypes
import re
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libopus_b200.so")
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "opus_b200.h"

OPUS_OK = 0
OPUS_ERR_INVALID = 1
OPUS_ERR_CUDA = 2
OPUS_ERR_UNSUPPORTED = 3
OPUS_ERR_DEVICE = 4

DTYPE_BF16 = 0
DTYPE_F32 = 1

_c_int, _c_i64, _c_f32, _c_f64, _c_p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_double, ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/opus_b200.h
SIGNATURES: dict[str, tuple] = {
    "opus_abi_version": (_c_int, []),
    "opus_last_error": (ctypes.c_char_p, []),
    "opus_device_error": (_c_int, [ctypes.POINTER(_c_int)]),
    "opus_selftest_stalled_wait": (_c_int, [_c_p]),
    "opus_pack_hash_sign": (_c_int, [_c_p, _c_p, _c_i64, _c_i64, _c_p, _c_p]),
    "opus_bucket_max_load": (_c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_p]),
    "opus_bucket_max_load_noalloc": (_c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_p]),
    "opus_sketch_table_entries": (_c_i64, [_c_int, _c_int]),
    "opus_build_sketch_table": (_c_int, [_c_p, _c_p, _c_p, _c_f32, _c_int, _c_int, _c_p, _c_i64, _c_p]),
    "opus_sketch_gemm": (_c_int, [_c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p, _c_i64, _c_i64, _c_int,
                                  _c_int, _c_p, _c_int, _c_f32, _c_p]),
    "opus_ghost_gram": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f32, _c_p, _c_int,
                                 _c_p]),
    "opus_per_sample_grad": (_c_int, [_c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p, _c_p, _c_int, _c_p]),
    "opus_sketch_dense": (_c_int, [_c_p, _c_int, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_int, _c_p,
                                   _c_int, _c_p]),
    "opus_desketch": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_f32, _c_int, _c_int, _c_i64, _c_f32, _c_p, _c_p]),
    "opus_ghost_score": (_c_int, [_c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p, _c_f32, _c_p, _c_int,
                                  _c_p]),
    "opus_sketch_dot": (_c_int, [_c_p, _c_p, _c_int, _c_i64, _c_f32, _c_p, _c_int, _c_p]),
    "opus_sketch_dot_layers": (_c_int, [_c_p, _c_i64, _c_p, _c_p, _c_int, _c_int, _c_i64, _c_p, _c_int, _c_p]),
    "opus_sketch_gram": (_c_int, [_c_p, _c_int, _c_p, _c_int, _c_i64, _c_f32, _c_p, _c_int, _c_p]),
    "opus_boltzmann_select": (_c_int, [_c_p, _c_p, _c_int, _c_int, _c_f64, _c_p, _c_p, _c_p]),
    "opus_greedy_select": (_c_int, [_c_p, _c_p, _c_int, _c_int, _c_p, _c_p]),
    "opus_boltzmann_select_blocks": (_c_int, [_c_p, _c_p, _c_int, _c_int, _c_int, _c_f64, _c_p, _c_p, _c_p]),
    "opus_greedy_select_blocks": (_c_int, [_c_p, _c_p, _c_int, _c_int, _c_int, _c_p, _c_p]),
    "opus_split_bf16": (_c_int, [_c_p, _c_i64, _c_p, _c_p, _c_p]),
    "opus_gemm_bf16": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_f32, _c_p, _c_int, _c_int, _c_p]),
    "opus_muon_S_workspace_bytes": (_c_i64, [_c_int, _c_int]),
    "opus_muon_S": (_c_int, [_c_p, _c_int, _c_int, _c_int, _c_p, _c_i64, _c_p, _c_p]),
    "opus_kernel_launches": (_c_i64, []),
    "opus_adam_diag": (_c_int, [_c_p, _c_f32, _c_i64, _c_p, _c_p]),
    "opus_sketch_dense_rows": (_c_int, [_c_p, _c_int, _c_i64, _c_p, _c_i64, _c_int, _c_p, _c_int, _c_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_timer = None  # the active KernelTimer, if any

# entry points that launch no kernel of their own or only query state
_UNTIMED = {"opus_abi_version", "opus_last_error", "opus_device_error", "opus_sketch_table_entries",
            "opus_muon_S_workspace_bytes", "opus_kernel_launches"}


class KernelTimer:
    """Device time of every library entry point called while it is active.

    Each call is bracketed by two CUDA events recorded on the current stream
    (the stream the front end launches on), so the figures are the calls'
    own device durations, taken live inside whatever region is being timed.
    summary() synchronises and returns {entry point: (calls, total ms)}.
    """

    def __init__(self):
        self.records: list = []

    def __enter__(self):
        global _timer
        self._prev, _timer = _timer, self
        return self

    def __exit__(self, *exc):
        global _timer
        _timer = self._prev
        return False

    def summary(self) -> dict:
        import torch

        torch.cuda.synchronize()
        out: dict = {}
        for name, s, e in self.records:
            n, ms = out.get(name, (0, 0.0))
            out[name] = (n + 1, ms + s.elapsed_time(e))
        return out


class _TimedLib:
    """The loaded library with each entry point wrapped in a pair of CUDA events."""

    def __init__(self, lib, timer):
        self._lib, self._t = lib, timer

    def __getattr__(self, name):
        fn = getattr(self._lib, name)
        if not name.startswith("opus_") or name in _UNTIMED:
            return fn
        import torch

        def call(*args):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            rc = fn(*args)
            e.record()
            self._t.records.append((name, s, e))
            return rc
        return call


def header_symbols() -> list[str]:
    """Every entry point declared with OPUS_API in include/opus_b200.h."""
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"OPUS_API\s+[\w\s\*]+?\b(opus_\w+)\s*\(", text)))


def load() -> ctypes.CDLL:
    """Load (once) and return the library with argument types declared (timed under a KernelTimer)."""
    lib = _load()
    return lib if _timer is None else _TimedLib(lib, _timer)


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is not built; run `python -m opus_b200.csrc.build` "
                "(the OPUS selection path has no fallback without its CUDA kernels)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().opus_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Map a non-zero status to the exception type the reference raises."""
    if rc == OPUS_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == OPUS_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


def device_error() -> int:
    """Synchronise the current device and return (and clear) its error word."""
    code = _c_int(0)
    rc = load().opus_device_error(ctypes.byref(code))
    if rc not in (OPUS_OK, OPUS_ERR_DEVICE):
        check(rc, "opus_device_error")
    return int(code.value)
