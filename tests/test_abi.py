"""The C ABI library: loads, exports every declared symbol, host-side checks (no GPU)."""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np
import pytest

import qraf_b200
from conftest import ROOT


def declared_functions():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(qraf_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(qraf_b200.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_row_bytes():
    assert qraf_b200.row_bytes(qraf_b200.Q8_0, 4096) == 4608
    assert qraf_b200.row_bytes(qraf_b200.Q4_0, 4096) == 2304
    assert qraf_b200.row_bytes(qraf_b200.Q4_0, 28672) == 16128
    assert qraf_b200.row_bytes(qraf_b200.Q8_0, 33) == 72          # ragged last block keeps a full block
    assert qraf_b200.row_bytes(qraf_b200.Q4_0, 50, 7) == 8 * 5    # odd block: 2 + 7 // 2 bytes
    assert qraf_b200.row_bytes(30, 64) == 0


def test_fill_normal_matches_reference_idiom():
    import oracle

    if oracle.reference_available():
        ref = oracle.Reference()
        for seed, mean, std in [(42, 0.0, 0.02), (43, 0.0, 1.0), (7, 1.5, 3.0)]:
            a = qraf_b200.fill_normal(seed, mean, std, 10001)
            assert np.array_equal(a, ref.fill_normal(seed, mean, std, 10001))
    # Pinned independently of the reference build: the config digests were made
    # from the reference's generator, and test_oracle checks them via this one.


def test_host_argument_checks_without_gpu():
    lib = qraf_b200.lib
    w = qraf_b200.qraf_weight_t()
    assert lib.qraf_cuda_weight_wrap(None, 100, 30, 32, 1, 32, C.byref(w)) == qraf_b200.ERR_UNSUPPORTED
    assert lib.qraf_cuda_weight_wrap(None, 100, 10, 0, 1, 32, C.byref(w)) == qraf_b200.ERR_INVALID
    assert lib.qraf_cuda_weight_wrap(None, 35, 10, 32, 1, 32, C.byref(w)) == qraf_b200.ERR_INVALID
    assert "need 36" in qraf_b200.last_error()
    assert lib.qraf_cuda_quantize(30, None, 8, 32, None, None) == qraf_b200.ERR_UNSUPPORTED


def test_host_entry_unknown_dtype_zero_fills_like_the_reference():
    # backend.cpp:195-198: an unknown quantized dtype leaves y zeroed.  No GPU is touched.
    y = np.full(5, 7.0, dtype=np.float32)
    x = np.ones(32, dtype=np.float32)
    w = np.zeros(100, dtype=np.uint8)
    qraf_b200.dispatch_matvec_q(w, w.size, 30, 32, 5, 32, x, y)
    assert np.all(y == 0.0)


def test_product_has_no_cpu_fallback():
    # The package must not import the oracle or contain a host compute path.
    pkg = os.path.join(ROOT, "qraf_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
                text = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in text and "from oracle" not in text, f
                assert "qraf_oracle" not in text, f


@pytest.mark.parametrize("lang,std", [("c", "c99"), ("c++", "c++17")])
def test_header_is_plain_c_abi(lang, std, tmp_path):
    """include/*.h compiles as C99 and as C++17, and a C program that calls an
    entry point links against the library (plain pointers and sizes, extern "C")."""
    import shutil
    import subprocess

    cc = shutil.which("gcc" if lang == "c" else "g++")
    if cc is None:
        pytest.skip("no host compiler")
    src = tmp_path / ("t.c" if lang == "c" else "t.cpp")
    src.write_text('#include "qraf_cuda.h"\n#include <stdio.h>\n'
                   'int main(void) { printf("%llu\\n", (unsigned long long)qraf_row_bytes(QRAF_DTYPE_Q4_0, 32, 4096));'
                   ' return 0; }\n')
    exe = tmp_path / "t"
    libdir = os.path.dirname(qraf_b200.LIB_PATH)
    out = subprocess.run([cc, f"-std={std}", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                          "-L", libdir, "-lqraf_cuda", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == "2304", (run.stdout, run.stderr)
