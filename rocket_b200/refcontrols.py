"""Reference-arm kernel controls: the reference's SIMT kernels, compiled unchanged, timed
on the same B200 as this framework's kernels (`kbench --impl reference`).

    python -m rocket_b200.refcontrols build [--src <reference checkout>]

copies the reference engine's kernel sources (engines/glm5-moe-nvfp4-2b/src/kernels.{cu,h},
their header and bench/kda_step_dropin.cuh) into baseline/_ref/controls_src/ as shipped
and compiles them with baseline/controls.cu (a forwarding shim) into
baseline/_ref/controls.so for sm_100a.  baseline/_ref is outside the package and git-ignored:
the framework never imports it.  `load()` returns the ctypes library or None.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OUT_DIR = os.path.join(ROOT, "baseline", "_ref")
SO = os.path.join(OUT_DIR, "controls.so")
ENGINE = os.path.join("engines", "glm5-moe-nvfp4-2b")
FILES = [os.path.join("src", "kernels.cu"), os.path.join("src", "kernels.h"),
         os.path.join("bench", "kda_step_dropin.cuh")]


def build(src: str) -> str:
    """Copy the reference kernel sources as shipped and compile the control library."""
    dst = os.path.join(OUT_DIR, "controls_src")
    for f in FILES:
        os.makedirs(os.path.dirname(os.path.join(dst, f)), exist_ok=True)
        shutil.copyfile(os.path.join(src, ENGINE, f), os.path.join(dst, f))
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-I", os.path.join(dst, "src"),
           os.path.join(dst, "src", "kernels.cu"), os.path.join(ROOT, "baseline", "controls.cu"),
           "-lcublas", "-o", SO]
    subprocess.run(cmd, check=True)
    return SO


def load():
    if not os.path.exists(SO):
        return None
    lib = ctypes.CDLL(SO)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.ctl_rmsnorm.argtypes = [P, P, P, I, I, F, P]
    lib.ctl_moe_router.argtypes = [P, P, P, P, I, I, I, I, F, P]
    lib.ctl_nvfp4_quantize_rows.argtypes = [P, P, P, P, P, P, I, I, P]
    lib.ctl_kda_step.argtypes = [P, P, P, P, P, P, P, I, I, I, I, P]
    for f in (lib.ctl_rmsnorm, lib.ctl_moe_router, lib.ctl_nvfp4_quantize_rows, lib.ctl_kda_step):
        f.restype = I
    return lib


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("cmd", choices=["build"])
    ap.add_argument("--src", default=os.environ.get("ROCKET_REFERENCE_SRC"), required="ROCKET_REFERENCE_SRC" not in os.environ,
                    help="the reference checkout (or ROCKET_REFERENCE_SRC)")
    a = ap.parse_args()
    print(build(a.src))
    sys.exit(0)
