"""Compile the reference's C++ store from its own source into oracle/_ref/ (test oracle and
timed CPU baseline only; never part of the product).

The reference JIT-builds code/lema/csrc/store.cpp with torch's extension builder and OpenMP
(code/lema/cache.py:69-95). This recipe compiles that same single file, where it lies under
the read-only reference checkout, with the same flags, into oracle/_ref/lema_store_ref.so.
The system g++ is used because the environment's default CXX wrapper cannot link -fopenmp.
Run in the build container (where the reference exists); the GPU box loads the prebuilt
.so through `oracle.ref_store()`. The checkout is the argument, else LEMA_REFERENCE_ROOT,
else the build container's conventional location (`reference_root()`).

    python -m oracle.build_ref [REFERENCE_ROOT]
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "lema_store_ref"
_CONVENTIONAL_ROOT = "/root/reference"


def reference_root() -> Path:
    """The read-only reference checkout: LEMA_REFERENCE_ROOT, else the conventional location."""
    return Path(os.environ.get("LEMA_REFERENCE_ROOT", _CONVENTIONAL_ROOT))


def build(reference_root_dir: str | Path | None = None) -> Path | None:
    root = Path(reference_root_dir) if reference_root_dir is not None else reference_root()
    src = root / "code" / "lema" / "csrc" / "store.cpp"
    if not src.exists():
        return None
    OUT.mkdir(parents=True, exist_ok=True)
    target = OUT / f"{NAME}.so"
    if target.exists() and target.stat().st_mtime >= src.stat().st_mtime:
        return target
    env_keep = {k: os.environ.get(k) for k in ("CXX", "CC")}
    os.environ["CXX"] = "/usr/bin/g++"
    os.environ["CC"] = "/usr/bin/gcc"
    try:
        from torch.utils.cpp_extension import load
        load(name=NAME, sources=[str(src)], build_directory=str(OUT),
             extra_cflags=["-O3", "-funroll-loops", "-fopenmp"], extra_ldflags=["-fopenmp"],
             verbose=False)
    finally:
        for k, v in env_keep.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return target if target.exists() else None


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None))
