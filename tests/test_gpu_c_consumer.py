"""A C99 program as the engine's consumer of libmiag (tests/c/moe_forwarder.c):
it includes only include/miag/miag.h, loads the experts through the
reference loader port and runs the INTEGRATION.md moe() forwarder token by
token, against the reference's own moe() built from source (oracle/_ref)."""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import warnings

import pytest

from conftest import ROOT
from motoria_b200 import build

pytestmark = pytest.mark.gpu
REF_LIB = ROOT / "oracle" / "_ref" / "libmia_ref.so"


def compile_consumer(out_dir):
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.fail("no C compiler")
    lib_dir = ROOT / "motoria_b200" / "lib"
    exe = out_dir / "moe_forwarder"
    cmd = [cc, "-std=c99", "-O2", "-Wall", "-Wextra", "-pedantic", f"-I{ROOT / 'include'}",
           str(ROOT / "tests" / "c" / "moe_forwarder.c"), "-o", str(exe),
           f"-L{lib_dir}", "-lmiag", f"-L{REF_LIB.parent}", "-lmia_ref",
           f"-Wl,-rpath,{lib_dir}:{REF_LIB.parent}", "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c99_engine_forwarder_matches_the_reference_moe(torch_cuda, tmp_path):
    build.build()
    if not REF_LIB.exists():
        msg = "NOT CHECKED: oracle/_ref/libmia_ref.so (the reference build) is absent"
        warnings.warn(msg)
        print(msg, file=sys.stderr)
        pytest.skip(msg)
    exe = compile_consumer(tmp_path)
    r = subprocess.run([str(exe), "6"], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ))
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ok" in r.stdout
