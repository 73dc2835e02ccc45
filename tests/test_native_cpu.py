"""Native CPU tests: the C header compiled as C99 against the built library, and the
library's host-only decisions (admission, band watchdog) driven with fakes in C++.
Both are compiled here with the system compilers and run without a GPU."""
import shutil
import subprocess

import pytest

from conftest import ROOT

NATIVE = ROOT / "tests" / "native"
LIBDIR = ROOT / "scunet-rs_b200"


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, **kw)
    assert r.returncode == 0, f"{' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}"
    return r.stdout


@pytest.mark.skipif(shutil.which("cc") is None, reason="no C compiler")
def test_c_abi_from_c99(scb, tmp_path):
    scb.build.build()
    exe = tmp_path / "abi_smoke"
    _run(["cc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{ROOT / 'include'}",
          str(NATIVE / "abi_smoke.c"), str(LIBDIR / "libscunet_b200.so"), f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)])
    out = _run([str(exe)])
    assert "abi ok" in out


@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_host_logic(tmp_path):
    exe = tmp_path / "host_logic"
    _run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", f"-I{LIBDIR / 'csrc'}",
          str(NATIVE / "host_logic_test.cpp"), "-o", str(exe)])
    assert "host logic ok" in _run([str(exe)])
