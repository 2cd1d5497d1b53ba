"""Build FlashAttnTile's CUDA C++ paged-decode baseline into ``oracle/_ref/`` -- test infrastructure.

The reference ships one hand-written CUDA decode kernel (``csrc/paged_decode.cu``
with its pybind module ``csrc/bindings.cpp``, loaded by ``flashattn_tile/native.py``).
This recipe compiles those two files, where they lie in a reference checkout
(nothing is copied), for sm_100a with the reference's own nvcc flags
(``-O3 --use_fast_math``, ``native.py:39-47``) into ``oracle/_ref/flashattn_native*.so``.
It is used only as a same-box comparator (timing) and as a second parity check
in the GPU tests; this library never loads it.

    python -m oracle.build_ref_native [reference checkout]

The checkout defaults to ``../reference`` beside this repository; without one
the build is skipped (machines that only run tests use the prebuilt module).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
OUT = ROOT / "oracle" / "_ref"


def reference_root(arg: str | None = None) -> Path | None:
    cand = Path(arg) if arg else ROOT.parent / "reference"
    return cand if (cand / "csrc" / "paged_decode.cu").is_file() else None


def built_module() -> Path | None:
    hits = sorted(OUT.glob("flashattn_native*.so"))
    return hits[0] if hits else None


def build(ref: str | None = None, verbose: bool = False) -> Path | None:
    src = reference_root(ref)
    if src is None:
        return built_module()
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load

    load(name="flashattn_native", sources=[str(src / "csrc" / "paged_decode.cu"), str(src / "csrc" / "bindings.cpp")],
         build_directory=str(OUT), extra_cflags=["-O3"],
         extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a"],
         verbose=verbose)
    return built_module()


def load_module():
    """Import the prebuilt module (no compilation); None when it was never built."""
    import importlib.util

    path = built_module()
    if path is None:
        return None
    import torch  # noqa: F401  (the extension links against torch's libraries)

    spec = importlib.util.spec_from_file_location("flashattn_native", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
