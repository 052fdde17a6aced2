"""Build recipe for libpu_attn.so (sm_100a) — plain nvcc, in-tree output.

    python pallas-unbound_b200/build.py [--force] [--verbose]

Compiles csrc/pu_attn.cu for `-gencode arch=compute_100a,code=sm_100a` and
links a shared library into pallas_flash/_native/.  The CUDA runtime is
linked statically and libcuda is reached through the runtime's driver entry
point, so the library loads on hosts without a GPU driver (symbol checks).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = PKG_ROOT.parent / "include"
OUT_DIR = PKG_ROOT / "pallas_flash" / "_native"
LIB_NAME = "libpu_attn.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-warn-spills",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def source_hash() -> str:
    h = hashlib.sha256()
    for p in sources():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def lib_path() -> Path:
    return OUT_DIR / LIB_NAME


def is_current() -> bool:
    stamp = OUT_DIR / (LIB_NAME + ".hash")
    return lib_path().exists() and stamp.exists() and stamp.read_text().strip() == source_hash()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library unless an up-to-date build exists; return its path."""
    if not force and is_current():
        return lib_path()
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    tmp = OUT_DIR / (LIB_NAME + ".tmp")
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        *NVCC_FLAGS,
        "-shared",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
        str(CSRC / "pu_attn.cu"),
        "-o",
        str(tmp),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or "spill" in res.stderr.lower():
        sys.stderr.write(res.stderr)
    os.replace(tmp, lib_path())
    (OUT_DIR / (LIB_NAME + ".hash")).write_text(source_hash() + "\n")
    return lib_path()


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
