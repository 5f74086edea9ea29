"""The C ABI library loads and exports what include/opus_b200.h declares (no GPU needed)."""
import ctypes
import subprocess

import pytest

from opus_b200 import _lib


def test_library_loads_and_reports_version():
    lib = _lib.load()
    assert lib.opus_abi_version() == 3
    assert _lib.last_error() == "" or isinstance(_lib.last_error(), str)


def test_every_header_symbol_is_exported():
    declared = _lib.header_symbols()
    assert len(declared) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in declared if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    lib = _lib.load()
    for s in declared:
        assert getattr(lib, s) is not None


def test_binding_table_matches_header():
    assert sorted(_lib.SIGNATURES) == _lib.header_symbols()


def test_no_internal_symbols_leak():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    names = [line.split()[-1] for line in out.splitlines() if line.strip()]
    assert all(n.startswith("opus_") for n in names if n.startswith("opus") or "opus" in n)


def _null():
    return ctypes.c_void_p(0)


def test_argument_validation_without_device():
    """Entry points reject bad arguments before touching the device (status codes, message set)."""
    lib = _lib.load()
    rc = lib.opus_sketch_gemm(_null(), _null(), _lib.DTYPE_F32, 1, 1, 8, 8, _null(), 0, 16, 4, 1, _null(), 0,
                              1.0, _null())
    assert rc == _lib.OPUS_ERR_UNSUPPORTED and "bf16" in _lib.last_error()
    rc = lib.opus_sketch_gemm(_null(), _null(), _lib.DTYPE_BF16, -1, 1, 8, 8, _null(), 0, 16, 4, 1, _null(), 0,
                              1.0, _null())
    assert rc == _lib.OPUS_ERR_INVALID
    with pytest.raises(ValueError):
        _lib.check(rc, "opus_sketch_gemm")
    rc = lib.opus_boltzmann_select(_null(), _null(), 0, 1, 1.0, _null(), _null(), _null())
    assert rc == _lib.OPUS_ERR_UNSUPPORTED
    rc = lib.opus_boltzmann_select(_null(), _null(), 10, 11, 1.0, _null(), _null(), _null())
    assert rc == _lib.OPUS_ERR_INVALID
    rc = lib.opus_boltzmann_select(_null(), _null(), 8193, 1, 1.0, _null(), _null(), _null())
    assert rc == _lib.OPUS_ERR_UNSUPPORTED and "8192" in _lib.last_error()  # one CTA holds at most 8192
    rc = lib.opus_boltzmann_select_blocks(_null(), _null(), 12, 5, 2, 1.0, _null(), _null(), _null())
    assert rc == _lib.OPUS_ERR_INVALID  # the block must divide n
    rc = lib.opus_greedy_select(_null(), _null(), 4 * 8192 + 1, 1, _null(), _null())
    assert rc == _lib.OPUS_ERR_UNSUPPORTED
    rc = lib.opus_ghost_score(_null(), _null(), _lib.DTYPE_BF16, 1, 1, 12, 8, _null(), 1.0, _null(), 0, _null())
    assert rc == _lib.OPUS_ERR_INVALID  # NULL pointers
    assert lib.opus_sketch_table_entries(128, 256) == 16384
    assert lib.opus_sketch_table_entries(129, 256) == 2 * 16384
    assert lib.opus_sketch_table_entries(0, 256) == 0
    rc = lib.opus_build_sketch_table(_null(), _null(), _null(), 1e-8, 128, 256, _null(), 10, _null())
    assert rc == _lib.OPUS_ERR_INVALID
    with pytest.raises(RuntimeError):
        _lib.check(_lib.OPUS_ERR_CUDA, "x")


def test_ops_refuse_cpu_tensors():
    import torch

    from opus_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.sketch_dot(torch.zeros(2, 4), torch.zeros(4))
