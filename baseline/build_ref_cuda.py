"""Build the reference's own CUDA extension as a reported baseline.

The reference (freezeng123456/JunQi) ships a CUDA implementation of this
path, the ``junqi_cuda`` pybind11 module (``src/env/cuda``).  This script
builds it for sm_100a without its CMake project -- nvcc on its sources with
relocatable device code, one device link, one host link -- and installs it,
together with the reference's Python packages (``junqi_core``,
``junqi_rl``), under ``baseline/_ref`` (git-ignored; it travels to the GPU
box with the working tree).  ``bench.py --impl reference-cuda`` then times
the reference's ``GpuRollout`` per-ply chain with it.

Run where the reference checkout exists::

    python baseline/build_ref_cuda.py <reference checkout>

Nothing is written into the reference checkout: sources are compiled from
a copy under a temporary directory.  The one source change the build needs
on CUDA 12.9 is dropping the
``#undef __noinline__`` block of ``rollout_history.cu``, which otherwise
breaks the CUDA headers included after it; it is made in the copy.
"""
from __future__ import annotations

import shutil
import subprocess
import sys
import sysconfig
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NVCC = "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
KERNELS = ["tables.cu", "game_state.cu", "observation.cu", "belief.cu", "combat_memory.cu", "rollout_history.cu"]


def run(cmd, **kw):
    print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True, **kw)


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: python baseline/build_ref_cuda.py <reference checkout>")
    ref = Path(sys.argv[1]).resolve()
    import pybind11
    OUT.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        # 1. the reference's Python packages, installed from a copy (setuptools writes into the source tree)
        src = tmp / "ref"
        shutil.copytree(ref, src, ignore=shutil.ignore_patterns(".git", "build", "*.so", "assets", "replays"))
        run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
             "--find-links", "/opt/wheelhouse", "--target", OUT, "--upgrade", src])
        # 2. the CUDA extension
        cu = src / "src" / "env" / "cuda"
        rh = cu / "src" / "rollout_history.cu"
        text = rh.read_text()
        patched = text.replace("#ifdef __noinline__\n#undef __noinline__\n#endif\n", "")
        if patched == text:
            raise SystemExit("rollout_history.cu: the expected #undef __noinline__ block was not found")
        rh.write_text(patched)
        inc = ["-I", cu / "include", "-I", cu / "src", "-I", pybind11.get_include(),
               "-I", sysconfig.get_paths()["include"]]
        objs = []
        for k in KERNELS:
            o = tmp / (k + ".o")
            run([NVCC, *ARCH, "-O3", "-DNDEBUG", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", *inc, "-c",
                 cu / "src" / k, "-o", o])
            objs.append(o)
        b = tmp / "bindings.o"
        run([NVCC, *ARCH, "-O3", "-DNDEBUG", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler",
             "-fvisibility=hidden", *inc, "-c", cu / "src" / "bindings.cpp", "-o", b])
        dl = tmp / "dlink.o"
        run([NVCC, *ARCH, "-dlink", "-Xcompiler", "-fPIC", *objs, "-o", dl])
        so = OUT / "junqi_rl" / ("junqi_cuda" + sysconfig.get_config_var("EXT_SUFFIX"))
        run(["g++", "-shared", "-o", so, *objs, b, dl, "-L/usr/local/cuda/lib64", "-lcudart", "-lcuda",
             "-lcudadevrt"])
    print("built", so)


if __name__ == "__main__":
    main()
