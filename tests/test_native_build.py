"""The native extension shares the process's C++ runtime (CPU check of the built module)."""

import shutil
import subprocess

import pytest


def _so():
    from difflet_b200 import _native

    p = _native._so_path(False)
    if p is None:
        pytest.skip("extension not built")
    return p


def test_extension_links_the_shared_cpp_runtime():
    """libstdc++ must come from libstdc++.so.6 (the copy torch uses), not be linked in
    statically: a second copy of the C++ runtime has its own iostream / locale state, and an
    error message that formats a number then dereferences a null facet instead of raising."""
    if shutil.which("readelf") is None or shutil.which("nm") is None:
        pytest.skip("binutils not installed")
    so = str(_so())
    dyn = subprocess.run(["readelf", "-d", so], capture_output=True, text=True, check=True).stdout
    assert "[libstdc++.so.6]" in dyn
    syms = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    runtime = [ln for ln in syms.splitlines() if "_ZNSt6locale" in ln or "_ZNSt8ios_base" in ln]
    assert not runtime, runtime[:5]
