"""The C-ABI library loads and exports every symbol include/b2dec.h declares (no GPU)."""
import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    src = (ROOT / "include" / "b2dec.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(pkg):
    from importlib import import_module
    build = import_module("aricode-ml_b200.build")
    lib = ctypes.CDLL(str(build.build()))
    names = declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert missing == []


def test_create_without_gpu_fails_cleanly(pkg):
    """No device: creation returns an error code (never aborts the process)."""
    import torch
    if torch.cuda.is_available():
        return
    rt = pkg.runtime
    ctx = ctypes.c_void_p()
    rc = rt.lib().b2_create_synthetic(b"{}", 0, 0.02, 0, ctypes.byref(ctx))
    assert rc < 0 and not ctx
