"""CPU checks of the C-ABI boundary: the library loads and exports every declared symbol."""
import os
import re
import subprocess

import pytest

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "vitfp4.h")).read()
    return re.findall(r"VF4_API\s+[\w\s\*]+?\b(vf4_\w+)\s*\(", src)


def test_header_declares_entry_points():
    names = _declared()
    for must in ("vf4_cast_nvfp4", "vf4_gemm_nvfp4", "vf4_amax", "vf4_to_blocked", "vf4_pack_e2m1",
                 "vf4_last_error_string"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from vitfp4 import _lib
    path = _lib.library_path()
    if not os.path.exists(path):
        pytest.skip("libvitfp4.so not built (run __graft_entry__.build())")
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (vf4_\w+)", out))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing
    lib = _lib.lib()  # loads and binds argtypes for every signature
    assert lib.vf4_version() >= 100
    assert set(_lib.SIGNATURES) <= exported


def test_python_binding_covers_header():
    from vitfp4 import _lib
    assert set(_declared()) <= set(_lib.SIGNATURES)
