"""The drop-in claim at link level: phonon-2-c's remaining sources, with blas.c, encoder.c and decoder.c taken out of
its library, resolve every symbol against libphonon2_b200.so. CPU only (compile and link, nothing runs); skipped
where the reference sources or the built library are absent."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "phonon-2-c_b200" / "libphonon2_b200.so"
REF = Path(os.environ.get("P2_REFERENCE_SRC", "/root/reference/csrc"))
KEEP = ["threadpool", "tensor_ops", "mel", "weights", "tokens", "wav", "resample", "segment", "engine", "json"]
# With the log-mel front end on the device too, mel.c leaves the reference's library as well.
KEEP_NO_MEL = [k for k in KEEP if k != "mel"]


@pytest.mark.skipif(not (REF / "engine.c").exists() or not LIB.exists() or shutil.which("gcc") is None,
                    reason="needs the reference sources, the built library and gcc")
@pytest.mark.parametrize("keep", [KEEP, KEEP_NO_MEL], ids=["mel-on-host", "mel-on-device"])
def test_reference_engine_links_against_library(tmp_path, keep):
    objs = []
    for name in keep:
        o = tmp_path / f"{name}.o"
        subprocess.run(["gcc", "-O1", "-std=c11", "-pthread", "-fPIC", "-D_GNU_SOURCE", "-w", f"-I{REF}", "-c",
                        str(REF / f"{name}.c"), "-o", str(o)], check=True)
        objs.append(str(o))
    # the engine library
    r = subprocess.run(["gcc", "-shared", "-o", str(tmp_path / "libphonon2_engine.so"), *objs,
                        f"-L{LIB.parent}", "-lphonon2_b200", "-Wl,--no-undefined", "-lm", "-lpthread"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    # and the command-line program on top of it
    main_o = tmp_path / "main.o"
    subprocess.run(["gcc", "-O1", "-std=c11", "-pthread", "-D_GNU_SOURCE", "-w", f"-I{REF}", "-c",
                    str(REF / "main.c"), "-o", str(main_o)], check=True)
    r = subprocess.run(["gcc", "-o", str(tmp_path / "phonon2"), str(main_o), *objs, f"-L{LIB.parent}",
                        "-lphonon2_b200", "-lm", "-lpthread"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
