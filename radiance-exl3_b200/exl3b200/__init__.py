"""exl3b200 -- the host-side mirror of radiance-exl3's EXL3 routed-expert plugin interface for the B200 library.

The product is the C-ABI library lib/libexl3b200.so (a radiance kernel plugin: include/exl3b200.h). This package
drives it the way the engine does (rad.py), builds seeded cases of the ops (cases.py) and exposes the routed-MoE
layer built from the library's entry points (layer.py). There is no fallback: a missing or unbuilt library is an
error, never a silent CPU path.
"""
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
LIB_PATH = ROOT / "lib" / "libexl3b200.so"


def library_path():
    if not LIB_PATH.exists():
        raise FileNotFoundError(
            f"{LIB_PATH} is not built: run `make -C {ROOT / 'csrc'}` (or __graft_entry__.build()); "
            "there is no CPU fallback for the EXL3 B200 ops")
    return LIB_PATH


def load_plugin():
    from .rad import Plugin
    return Plugin(library_path())
