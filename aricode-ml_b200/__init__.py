"""B200-native decode path for aricode-ml decoders (int8 GEMV, KV-cache attention,
norms, activations, greedy argmax) behind the reference's packer surface.

The directory name carries a hyphen, so import it with
``importlib.import_module("aricode-ml_b200")``; the package also registers itself
as ``aricode_ml_b200`` for ordinary ``import`` statements afterwards.
"""
import sys as _sys

_sys.modules.setdefault("aricode_ml_b200", _sys.modules[__name__])

from . import arch, blob, pack, runtime, synth  # noqa: E402,F401

__all__ = ["arch", "blob", "pack", "runtime", "synth"]
