"""miag_moe's host-side transfer pieces, on the CPU: the threads that copy a
pageable caller buffer through the pinned staging buffer, and the split of a
large batch into pieces (motoria_b200/csrc/host_copy.h, compiled with g++)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


def test_copy_threads_and_piece_split(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not found")
    exe = tmp_path / "host_copy_test"
    subprocess.run([gxx, "-O2", "-std=c++17", "-pthread", "-Wall", "-Werror",
                    str(HERE / "c" / "host_copy_test.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip() == "ok"
