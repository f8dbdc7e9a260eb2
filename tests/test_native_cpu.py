"""CPU-side checks of the C ABI: the library builds for sm_100a, loads, and
exports every entry point declared in include/adallm_b200.h.  No kernel runs."""
import ctypes
import subprocess

import pytest

from adallm_b200 import _native as N
from adallm_b200 import build as B


@pytest.fixture(scope="module")
def built():
    return B.build()


def test_library_exports_every_declared_symbol(built):
    declared = N.declared_symbols()
    assert len(declared) >= 10
    h = ctypes.CDLL(built)
    for name in declared:
        assert hasattr(h, name), f"{name} declared in include/adallm_b200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    ada = {s for s in exported if s.startswith("ada_")}
    assert ada == set(declared), f"exported but undeclared: {sorted(ada - set(declared))}"


def test_binding_signatures_cover_header(built):
    assert set(N._SIGS) == set(N.declared_symbols())


def test_status_strings_and_version(built):
    lib = N.lib()
    assert lib.ada_abi_version() >= 1
    assert lib.ada_status_string(0) == b"ok"
    assert b"workspace" in lib.ada_status_string(N.ADA_ERR_WORKSPACE)


def test_argument_errors_are_reported_before_any_launch(built):
    lib = N.lib()
    # head_dim 64 is not implemented -> UNSUPPORTED, without touching the (null) pointers' memory
    st = lib.ada_fp8_paged_decode(16, 0, 0, 0, 16, 16, 0, 0, 0, 4, 16, 4, 4, 16, 1, 8, 2, 64, 16, 1.0, 1.0, 1.0, 0,
                                  16, 0, 16, 1 << 20, None)
    assert st == N.ADA_ERR_UNSUPPORTED
    st = lib.ada_rmsnorm(None, 0, None, 0, None, 0, None, None, 0, 4, 128, 1e-6, 0, 0, None)
    assert st == N.ADA_ERR_INVALID_ARG
    # unknown attention launch flags are rejected
    st = lib.ada_fp8_paged_decode_quant_ex(16, 0, 0, 0, 16, 16, 0, 0, 0, 4, 16, 4, 4, 16, 1, 32, 8, 128, 16, 1.0,
                                           1.0, 1.0, 0, None, 0, 4, 16, 16, None, 16, 16, 1 << 20, 2, None)
    assert st == N.ADA_ERR_INVALID_ARG
    with pytest.raises(ValueError):
        N.check(N.ADA_ERR_ALIGNMENT, "x")
    with pytest.raises(RuntimeError, match="no fallback"):
        N.check(N.ADA_ERR_LAUNCH, "x")
