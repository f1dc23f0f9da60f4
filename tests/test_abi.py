"""The C-ABI libraries load and export every function their headers declare
(no GPU needed: nothing is called)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import vkflame_b200 as V

ROOT = Path(__file__).resolve().parents[1]
HEADERS = {
    "rt": "vkflame_rt.h",
    "hip": "vkflame_hip.h",
    "hipblas": "vkflame_hipblas.h",
    "hipblaslt": "vkflame_hipblaslt.h",
    "rocblas": "vkflame_rocblas.h",
}
DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", re.M)


def declared(header: str) -> set:
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"#define[^\n]*", "", text)
    names = set(DECL.findall(text))
    return {n for n in names if n not in {"if", "return", "sizeof", "typedef"} and not n.startswith("VKF_STATIC")}


def exported(lib: Path) -> set:
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if ln.strip()}


@pytest.mark.parametrize("key", list(HEADERS))
def test_library_exports_header(key):
    hdr = ROOT / "include" / HEADERS[key]
    if not hdr.exists():
        pytest.skip(f"{hdr.name} not part of this build yet")
    lib = V.LIBS[key]
    assert lib.exists(), f"{lib} not built"
    ctypes.CDLL(str(lib))  # loads (resolves its own dependencies)
    missing = {n for n in declared(HEADERS[key]) if not n.startswith("vkf_")} - exported(lib)
    assert not missing, f"{lib.name} lacks {sorted(missing)}"


def test_python_signatures_cover_header():
    from vkflame_b200 import rt
    assert declared("vkflame_rt.h") - {n for n in declared("vkflame_rt.h") if n.startswith("vkf_")} <= set(
        rt.declared_symbols())
