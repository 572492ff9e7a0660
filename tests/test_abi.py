"""The C ABI boundary, on the CPU: the library loads, and it exports every function its public headers declare."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:P2CU_API\s+|P2_API\s+)?[A-Za-z_][\w\s\*]*?\b((?:p2|p2cu)_\w+)\s*\(", text, re.M):
            if "typedef" in text[max(0, m.start() - 20):m.start()]:
                continue
            names.add(m.group(1))
    return names


def test_headers_declare_the_entry_points():
    names = declared_functions()
    for required in ("p2cu_sgemm_fvb", "p2cu_sgemm_fvb_q8a", "p2cu_quant_rows", "p2cu_sgemm"):
        assert required in names


def test_library_exports_every_declared_function(pkg):
    lib = pkg.lib()   # raises if the library is missing: there is no CPU fallback
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"declared in include/*.h but not exported: {missing}"


def test_python_signatures_cover_the_exports(pkg):
    for name in pkg.SIGNATURES:
        assert hasattr(pkg.lib(), name)


def test_oracle_is_not_linked_by_the_product():
    """The product library must not depend on the test-side checkers."""
    so = (ROOT / "phonon-2-c_b200" / "libphonon2_b200.so").read_bytes()
    assert b"liboracle" not in so and b"orc_" not in so and b"libphonon2_ref" not in so


def test_probes_library_exports_its_header_and_stays_out_of_the_product():
    """The test-only probes library (hardware rates, the packed-arithmetic check) loads without a GPU, exports every
    function probes.h declares, and none of them is in the product library."""
    import ctypes
    header = (ROOT / "phonon-2-c_b200" / "csrc" / "probes.h").read_text()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    names = set(re.findall(r"^\s*P2PROBE_API\s+[\w\s\*]*?\b(p2cu_\w+)\s*\(", header, re.M))
    assert "p2cu_probe_packed_math" in names and "p2cu_probe_int8_mma" in names
    probes = ctypes.CDLL(str(ROOT / "phonon-2-c_b200" / "libphonon2_probes.so"))
    assert not [n for n in sorted(names) if not hasattr(probes, n)]
    product = ctypes.CDLL(str(ROOT / "phonon-2-c_b200" / "libphonon2_b200.so"))
    assert not [n for n in sorted(names) if hasattr(product, n)]
