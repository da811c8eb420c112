"""The C-ABI library loads and exports every symbol include/*.h declares
(no device work: this runs on machines without a GPU)."""
import ctypes
import glob
import os
import re

import ferrite_b200 as fb
from conftest import ROOT


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        names.update(re.findall(r"\b(fb_[a-z0-9_]+)\s*\(", txt))
    return names


def test_library_exports_all_declared_symbols():
    lib = fb.lib()
    decl = declared_symbols()
    assert decl, "no declarations found"
    missing = [n for n in sorted(decl) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(fb.EXPORTED) == decl


def test_abi_version_and_error_path():
    lib = fb.lib()
    assert lib.fb_abi_version() == 1
    # invalid arguments are rejected on the host with a message, no device work
    rc = lib.fb_qtensor_info(None, None, None, None, None)
    assert rc == -1
    assert b"null" in lib.fb_last_error()


def test_library_links_no_torch():
    # the product library depends on the CUDA runtime only (no torch symbols)
    import subprocess
    out = subprocess.run(["ldd", fb.LIB_PATH], capture_output=True, text=True).stdout
    assert "torch" not in out and "c10" not in out
