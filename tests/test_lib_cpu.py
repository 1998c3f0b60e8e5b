"""CPU checks of the C ABI library: it loads and exports every declared symbol."""
import ctypes
import subprocess

from androidllm_b200 import _lib


def test_header_symbols_all_exported():
    declared = _lib.header_symbols()
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    # every declared symbol has a ctypes signature in the binding
    assert set(declared) == set(_lib.SIGNATURES)


def test_abi_version_and_error_string():
    assert _lib.lib.alm_abi_version() == 100
    assert isinstance(_lib.lib.alm_last_error(), bytes)


def test_null_arguments_are_rejected_without_touching_a_device():
    # argument validation happens before any CUDA call
    assert _lib.lib.alm_ctx_create(0, None) == 1
    assert b"null" in _lib.lib.alm_last_error()
    assert _lib.lib.alm_qweight_upload(None, None, None, 4, 64, 16, 64, 64, None) == 1
    assert _lib.lib.alm_spec_begin(None, 0, 0) == 1
    h = ctypes.c_void_p()
    assert _lib.lib.alm_kv_read(None, 0, 0, 1, None, None) == 1
    assert h.value is None
