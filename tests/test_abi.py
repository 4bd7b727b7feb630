"""CPU checks of the C-ABI boundary: the library loads, exports every entry point the header
declares, and its structures have the header's layout. No compute call (there is no GPU here)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from tricast_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tricast_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(tc_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    names = declared_functions()
    assert {"tc_cast", "tc_quantize", "tc_gemm", "tc_error_stats", "tc_last_error"} <= set(names)
    for name in names:
        assert hasattr(lib, name), name


def test_python_binding_covers_header():
    assert set(declared_functions()) <= set(N.EXPORTS)


def test_struct_layouts_match_c(tmp_path):
    src = tmp_path / "sizes.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "tricast_b200.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(tc_format), '
                   'sizeof(tc_quant_spec), sizeof(tc_quant_out), sizeof(tc_operand), sizeof(tc_mma_spec), '
                   'offsetof(tc_quant_spec, mse_search), offsetof(tc_operand, alpha), '
                   'offsetof(tc_mma_spec, out_dtype));return 0;}\n')
    exe = tmp_path / "sizes"
    try:
        subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    except (OSError, subprocess.CalledProcessError):
        pytest.skip("no C compiler")
    want = list(map(int, subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()))
    got = [ctypes.sizeof(N.TcFormat), ctypes.sizeof(N.TcQuantSpec), ctypes.sizeof(N.TcQuantOut),
           ctypes.sizeof(N.TcOperand), ctypes.sizeof(N.TcMmaSpec), N.TcQuantSpec.mse_search.offset,
           N.TcOperand.alpha.offset, N.TcMmaSpec.out_dtype.offset]
    assert got == want


def test_version_and_error_string():
    lib = N.lib()
    assert b"sm_100a" in lib.tc_version()
    assert lib.tc_last_error() == b""


def test_invalid_arguments_fail_without_gpu():
    """Argument validation happens before any device work, so it is testable here."""
    lib = N.lib()
    fmt = N.tc_format("fp8_e4m3")
    assert lib.tc_cast(None, None, None, 4, fmt, 0, 1, 32, None) == N.TC_INVALID_ARGUMENT
    assert b"null" in lib.tc_last_error()
    e8 = N.tc_format("e8m0")
    assert lib.tc_cast(ctypes.c_void_p(16), ctypes.c_void_p(16), None, 4, e8, 5, 1, 32, None) == N.TC_INVALID_ARGUMENT
    assert b"power-of-two" in lib.tc_last_error()
