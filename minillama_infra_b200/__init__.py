"""B200 (sm_100a) INT8 group-64 linear path of MiniLlama-Infra.

The compute lives in hand-written CUDA behind a C ABI (include/mli_gemv.h,
lib/libmli_gemv.so) plus a drop-in shim with the reference's own launcher
signatures (lib/libmli_dropin.so).  This package holds the build recipe, the
ctypes binding, torch-tensor wrappers named like the reference launchers
(``ops``), seeded synthetic workloads (``synth``) and the row-sharded
multi-GPU classifier (``shard``).
"""
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8) -> None:
    """Compile every CUDA source for sm_100a into lib/ (in-tree)."""
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", PKG_DIR], check=True)
