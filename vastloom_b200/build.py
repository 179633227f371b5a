"""In-tree build of the vlb200 CUDA library (sm_100a) and of the codebook data file.

    python -m vastloom_b200.build            # library + codebooks
    python -m vastloom_b200.build --check    # also print ptxas register/spill lines

The library is linked with nvcc directly (no torch extension), so the product is a plain C-ABI
shared object: vastloom_b200/libvlb200.so.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libvlb200.so"
DATA = PKG / "data"
GRIDS = DATA / "iq_grids.bin"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["vlb_kernels.cu", "vlb_decode.cu", "vlb_prefill.cu", "vlb_ep.cu", "vlb_abi.cu", "vlb_noalloc.cu", "vlb_ep_driver.cu"]


def reference_root() -> Path:
    """The vastloom reference source tree the build-time tools read: $VLB_REFERENCE, else a
    `reference` directory beside this repository. It is only needed here, in the build container;
    the GPU box runs on the files built from it."""
    env = os.environ.get("VLB_REFERENCE")
    return Path(env) if env else ROOT.parent / "reference"


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the vlb200 library needs the CUDA 12.9 toolchain")


def _run(cmd: list[str], cwd: Path | None = None) -> str:
    proc = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose_ptxas: bool = False) -> str:
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps.append(ROOT / "include" / "vlb200.h")
    if not force and not verbose_ptxas and not _stale(LIB, deps):
        return ""
    objs = []
    out = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    # the translation units compile in parallel (the expert kernels' format instances dominate)
    procs = []
    for s in SOURCES:
        obj = build_dir / (Path(s).stem + ".o")
        cmd = [_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
               "-I", str(ROOT / "include"), "-c", str(CSRC / s), "-o", str(obj)]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
        objs.append(str(obj))
    for cmd, proc in procs:
        so, se = proc.communicate()
        if proc.returncode != 0:
            raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{so}\n{se}")
        out.append(so + se)
    tmp = LIB.with_suffix(".so.tmp")
    _run([_nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart"])
    os.replace(tmp, LIB)
    return "".join(out)


def build_codebooks(reference: Path | None = None, force: bool = False) -> bool:
    """Writes data/iq_grids.bin from the reference tree's codebook data files.

    Returns False (and leaves any existing file alone) when the reference tree is absent, as on
    the GPU box, which uses the file built here."""
    ref = Path(reference) if reference else reference_root()
    inc = ref / "src" / "inference"
    if not (inc / "iq2xxs_grid.inc").exists():
        return GRIDS.exists()
    if GRIDS.exists() and not force:
        return True
    DATA.mkdir(exist_ok=True)
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    exe = build_dir / "gen_codebooks"
    _run(["g++", "-std=c++17", "-O1", "-I", str(inc), str(CSRC / "gen_codebooks.cpp"), "-o", str(exe)])
    _run([str(exe), str(GRIDS)])
    return True


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--check", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args(argv)
    log = build_library(force=a.force, verbose_ptxas=a.check)
    if a.check:
        print(log)
    ok = build_codebooks(force=a.force)
    print(f"library: {LIB} ({LIB.stat().st_size} bytes); codebooks: {'ok' if ok else 'missing'}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
