"""Build-level checks of the native extension (CPU; skipped when it is not built)."""
import subprocess
from pathlib import Path

import pytest

PKG = Path(__file__).resolve().parents[1] / "mini_megatron_b200"


def _so():
    found = sorted(PKG.glob("_C*.so"))
    if not found:
        pytest.skip("extension not built")
    return found[0]


def test_extension_uses_the_shared_cxx_runtime():
    # A static copy of libstdc++ inside the extension breaks TORCH_CHECK message formatting.
    out = subprocess.run(["ldd", str(_so())], capture_output=True, text=True).stdout
    assert "libstdc++.so.6" in out, out


def test_extension_is_built_for_sm100a_only():
    out = subprocess.run(["cuobjdump", "--list-elf", str(_so())], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = {line.split(".")[-2] for line in out.stdout.splitlines() if ".cubin" in line}
    assert arches and all(a.startswith("sm_100a") for a in arches), out.stdout
