"""Build libpdx_moe.so in-tree with nvcc for sm_100a (B200).

    python -m pdscope_b200.build            # build if sources changed
    python -m pdscope_b200.build --force    # rebuild

The library is a single nvcc translation unit (csrc/pdx_moe.cu includes the
kernel files); it links the CUDA runtime statically and needs no libcuda at
link time (cuTensorMapEncodeTiled is resolved through the runtime's driver
entry-point query).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libpdx_moe.so"
STAMP = PKG / ".libpdx_moe.sha256"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-shared",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def _nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the pdx_moe CUDA library cannot be built")
    return cand


def source_digest():
    h = hashlib.sha256()
    files = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "pdx_moe.h"]
    for f in files:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    digest = source_digest()
    if not force and LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == digest:
        return LIB
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-o", str(LIB) + ".tmp",
           str(CSRC / "pdx_moe.cu")]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    (PKG / "build.log").write_text(" ".join(cmd) + "\n" + log)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed building libpdx_moe.so:\n" + log[-6000:])
    if verbose:
        print(log)
    os.replace(str(LIB) + ".tmp", LIB)
    STAMP.write_text(digest + "\n")
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
