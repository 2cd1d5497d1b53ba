"""The C-ABI library: it loads without a GPU and exports every symbol the header declares.

No test here launches device work: the calls below fail host-side validation
before any CUDA call is made.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def _declared_functions() -> set[str]:
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(fat_\w+)\s*\(", text))
    return names


def test_library_builds_and_loads():
    from flashattntile_b200 import _lib

    lib = _lib.load()
    assert lib.fat_version().decode().startswith("flashattn_tile_b200")
    assert lib.fat_last_error() is not None


def test_every_declared_symbol_is_exported_and_bound():
    from flashattntile_b200 import _lib

    declared = _declared_functions()
    assert {"fat_paged_decode", "fat_prefill_varlen", "fat_gather_paged"} <= declared
    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in sorted(declared):
        assert hasattr(raw, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in _lib.py"


def test_host_side_validation_errors_without_gpu():
    from flashattntile_b200 import _lib

    lib = _lib.load()
    # num_heads not divisible by num_kv_heads: rejected before any CUDA call.
    rc = lib.fat_paged_decode(None, 0, 0, None, None, 0, 0, 0, 1, None, 0, 1, None, None, None, 0, None, 0, 0,
                              2, 3, 2, 128, 16, 0, 0, 0, 0.1, 1, None, 0, None, None)
    assert rc == _lib.FAT_ERR_INVALID_ARGUMENT
    assert b"divisible" in lib.fat_last_error()
    # split_k hint outside 1..64
    rc = lib.fat_paged_decode(None, 0, 0, None, None, 0, 0, 0, 1, None, 0, 1, None, None, None, 0, None, 0, 0,
                              2, 4, 2, 128, 16, 0, 0, 0, 0.1, 0, None, 0, None, None)
    assert rc == _lib.FAT_ERR_INVALID_ARGUMENT and b"split_k" in lib.fat_last_error()
    # unsupported page size / dtype
    rc = lib.fat_paged_decode(None, 0, 0, None, None, 0, 0, 0, 1, None, 0, 1, None, None, None, 0, None, 0, 0,
                              2, 4, 2, 128, 24, 0, 0, 0, 0.1, 1, None, 0, None, None)
    assert rc == _lib.FAT_ERR_UNSUPPORTED and b"page_size" in lib.fat_last_error()
    rc = lib.fat_prefill_varlen(None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, None, None, 1, 1, 1, 4, 2, 64, 1, 1,
                                1, 0.1, 2, 2, None, None)
    assert rc == _lib.FAT_ERR_UNSUPPORTED and b"fp16 or bf16" in lib.fat_last_error()
    # process-wide switches: values outside their range are refused
    assert lib.fat_set_prefill_schedule(2) == -2 and b"schedule" in lib.fat_last_error()


def test_status_codes_map_to_python_exceptions():
    from flashattntile_b200 import _lib

    _lib.load()
    with pytest.raises(ValueError):
        _lib.check(_lib.FAT_ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.FAT_ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.FAT_ERR_CUDA, "x")
    _lib.check(_lib.FAT_OK, "x")


def test_every_decode_entry_forwards_its_scratch_arguments():
    """With every other pointer present (16-byte aligned dummies, never dereferenced
    because validation fails first), a NULL or too-small scratch must be rejected
    by each decode entry point -- proof that the entry forwards what it was given."""
    import ctypes

    from flashattntile_b200 import _lib

    lib = _lib.load()
    buf = (ctypes.c_uint8 * 4096)()
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    q = k = v = out = base
    table = lens = base + 1024
    lse = base + 2048
    common = (q, 128 * 4, 128, k, v, 16 * 2 * 128, 2 * 128, 128, 4, table, 2, 2, lens, None, None, 0, out, 4 * 128,
              128)
    tail_dims = (2, 4, 2, 128, 16, 0, 0, 0, 0.1, 1)
    for ws, nbytes, want in ((None, 0, _lib.FAT_ERR_INVALID_ARGUMENT), (base, 16, _lib.FAT_ERR_WORKSPACE)):
        rc = lib.fat_paged_decode(*common, *tail_dims, ws, nbytes, None, None)
        assert rc == want, (rc, lib.fat_last_error())
        rc = lib.fat_paged_decode_lse(*common, lse, 4, *tail_dims, ws, nbytes, None, None)
        assert rc == want, (rc, lib.fat_last_error())


def test_decode_loop_has_no_cpu_path():
    import torch

    from flashattntile_b200.decode_loop import DecodeLoop
    from flashattntile_b200.paging import PagedKVCache

    k = torch.zeros(4, 16, 2, 64, dtype=torch.float16)
    cache = PagedKVCache(k, k.clone(), torch.zeros(1, 4, dtype=torch.int32), torch.zeros(1, dtype=torch.int32), 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        DecodeLoop(cache, num_heads=4)


def test_decode_call_struct_matches_the_header():
    """The ctypes mirror of ``fat_decode_call`` has the C struct's size and field offsets."""
    import shutil
    import subprocess
    import tempfile

    from flashattntile_b200 import _lib

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    fields = [name for name, _ in _lib.DecodeCall._fields_]
    root = Path(__file__).resolve().parents[1]
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"flashattn_tile_b200.h\"\nint main(void) {\n"
    src += '  printf("%zu\\n", sizeof(fat_decode_call));\n'
    for f in fields:
        src += f'  printf("%zu\\n", offsetof(fat_decode_call, {f}));\n'
    src += "  return 0;\n}\n"
    with tempfile.TemporaryDirectory() as d:
        c, exe = Path(d) / "layout.c", Path(d) / "layout"
        c.write_text(src)
        subprocess.run([gcc, "-I", str(root / "include"), str(c), "-o", str(exe)], check=True)
        values = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    import ctypes

    assert values[0] == ctypes.sizeof(_lib.DecodeCall)
    assert values[1:] == [getattr(_lib.DecodeCall, f).offset for f in fields]
