"""The C-ABI library loads and exports every entry point include/*.h declares."""
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent

# Entry points of the reference headers this library replaces
# (DANCE include/gpu_vamana_builder.h:30-81).
REFERENCE_SYMBOLS = [
    "gpu_vamana_build", "gpu_vamana_build_float", "gpu_vamana_vnew2_build", "gpu_vamana_vnew2_build_float",
    "gpu_vamana_vnew2_build_device", "gpu_vamana_vnew2_build_device_float", "gpu_vamana_get_last_medoid",
    "gpu_vamana_get_last_stats", "gpu_vamana_vnew2_get_last_medoid", "gpu_vamana_vnew2_get_last_stats",
    # DANCE include/gpu_vamana_filtered.h:79-123
    "gpu_vamana_filtered_build_uint8", "gpu_vamana_filtered_build_float", "gpu_vamana_filtered_get_last_stats",
]


CPP_HEADERS = {"gpu_merge.h"}  # C++ (namespace diskann) declarations, bound through their C forms


def declared_symbols(cpp=False):
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        if (h.name in CPP_HEADERS) != cpp:
            continue
        for m in re.finditer(r"DANCE_API\s+[\w\s\*]+?\b(\w+)\s*\(", h.read_text()):
            names.add(m.group(1))
    return sorted(names)


def exported_symbols(lib_path):
    out = subprocess.run(["nm", "-DC", "--defined-only", str(lib_path)], capture_output=True, text=True,
                         check=True).stdout
    names = set()
    for line in out.splitlines():
        if " T " not in line:
            continue
        sym = line.split(" T ", 1)[1]
        names.add(sym.split("(")[0].split("::")[-1])
    return names


def test_headers_declare_reference_abi():
    decl = set(declared_symbols())
    missing = [s for s in REFERENCE_SYMBOLS if s not in decl]
    assert not missing, f"reference entry points not declared: {missing}"


def test_library_exports_every_declared_symbol(dance_lib):
    from dance_b200 import LIB_PATH, SIGNATURES
    exported = exported_symbols(LIB_PATH)
    decl = declared_symbols()
    assert decl, "no DANCE_API declarations found"
    missing = [s for s in decl + declared_symbols(cpp=True) if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    # the Python binding declares exactly the header surface
    assert sorted(SIGNATURES) == decl


def test_library_loads_without_gpu(dance_lib):
    # Loading and pure-host calls must work without a device.
    from dance_b200 import default_params
    p = default_params()
    assert p.iters == 4 and abs(p.alpha - 1.2) < 1e-7 and p.final_min_degree == 64
    assert p.medoid_candidates == 1024 and p.medoid_samples == 4096 and p.init_random_seeds == 8
    assert dance_lib.dance_kernel_launch_count() == 0


def test_invalid_arguments_rejected_before_any_device_work(dance_lib):
    import numpy as np
    from dance_b200 import vamana
    from dance_b200 import DanceError
    x = np.zeros((10, 8), np.uint8)
    for bad in [dict(R=0, L=8, C=8, STEPS=4), dict(R=8, L=8, C=4, STEPS=4), dict(R=8, L=0, C=8, STEPS=4)]:
        with pytest.raises(DanceError):
            vamana.gpu_vamana_vnew2_build(x, **bad)
    assert "invalid parameters" in dance_lib.dance_last_error().decode()


def test_sm100a_only_build_recipe():
    from dance_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
