"""Builds libmiag.so (the sm_100a CUDA library behind include/miag/miag.h).

    python -m motoria_b200.build

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only (no fast-math:
the kernels rely on IEEE division, square root and rounding), links them into
``motoria_b200/lib/libmiag.so`` with the CUDA runtime linked statically, and
skips the work when the library is newer than every source.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OBJ_DIR = PKG / "_build"
LIB = PKG / "lib" / "libmiag.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-Xptxas", "-warn-spills",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: libmiag needs the CUDA toolkit to build")
    return exe


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    srcs = sources()
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.rglob("*.h"))
    if not force and not _stale(LIB, srcs + headers + [Path(__file__)]):
        return LIB
    OBJ_DIR.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    exe = nvcc()

    def compile_one(src: Path) -> Path:
        obj = OBJ_DIR / (src.stem + ".o")
        cmd = [exe, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr)
        return obj

    workers = max(1, min(len(srcs), os.cpu_count() or 1))
    with cf.ThreadPoolExecutor(workers) as ex:
        objs = list(ex.map(compile_one, srcs))
    cmd = [exe, "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
           "-o", str(LIB), *map(str, objs), "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link of libmiag.so failed:\n{r.stderr}")
    return LIB


ENGINE = PKG / "engine"


def reference_tree() -> Path | None:
    """The motorIa source tree the engine applications build from:
    $MIA_REFERENCE, else the reference_path of BASELINE.json beside the
    package; None when neither names a tree."""
    import json

    cand = os.environ.get("MIA_REFERENCE")
    if not cand:
        try:
            cand = json.loads((PKG.parent / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if cand and (Path(cand) / "src" / "app" / "serve.c").exists():
        return Path(cand)
    return None


def build_engine() -> Path | None:
    """The engine's applications (mia, mia-serve, mia-dump) with the model
    layer on the GPU (engine/mia_model_gpu.c over libmiag), built from the
    reference tree where one exists (engine/Makefile); returns their
    directory, or None without a tree (they may have been built elsewhere)."""
    build()
    tree = reference_tree()
    if tree is None:
        return None
    r = subprocess.run(["make", "-s", "-C", str(ENGINE), f"REF={tree}"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"engine build failed:\n{r.stdout}\n{r.stderr}")
    return ENGINE / "_bin"


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
