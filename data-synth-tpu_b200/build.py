"""Build ``qk_b200/libqk_b200.so`` from ``csrc/*.cu`` with nvcc for sm_100a.

    python data-synth-tpu_b200/build.py [--force]

The library is built in-tree (next to the Python package) so it ships with the
repository snapshot; it is rebuilt only when a source or header is newer than it.
"""

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
LIB = HERE / "qk_b200" / "libqk_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--threads", "0"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolchain is required")
    return path


def sources():
    return sorted(CSRC.glob("*.cu"))


def stale():
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in deps)


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", "-shared", "-o", str(LIB)]
    cmd += [str(s) for s in sources()]
    if verbose:
        print(" ".join(cmd), flush=True)
    env = dict(os.environ)
    result = subprocess.run(cmd, cwd=objdir, env=env, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError(f"nvcc failed with exit code {result.returncode}")
    return LIB


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=True))
