"""vkflame_b200 — B200-native quantised-linear hot path of vkflame.

Python front-end over the C ABI of ``lib/libvkflame_rt.so`` (see
``include/vkflame_rt.h``), mirroring the reference's loader
(python/vkflame/__init__.py:19-42): find the runtime library, call
``vkflame_init()``, fail loudly if it cannot.  There is no CPU fallback:
without the built library or a B200 the import of :mod:`vkflame_b200.rt`
raises.
"""
from pathlib import Path

__version__ = "0.1.0"

PKG_DIR = Path(__file__).resolve().parent
LIB_DIR = PKG_DIR / "lib"
CSRC_DIR = PKG_DIR / "csrc"

LIBS = {
    "rt": LIB_DIR / "libvkflame_rt.so",
    "hip": LIB_DIR / "libamdhip64.so.6",
    "hipblas": LIB_DIR / "libhipblas.so.2",
    "hipblaslt": LIB_DIR / "libhipblaslt.so.0",
    "rocblas": LIB_DIR / "librocblas.so.4",
}
