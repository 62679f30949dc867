"""The C ABI from plain C (C11, no C++ in the caller): tests/c/host_abi.c is compiled against
include/vcsrmc.h, linked with libvcsrmc.so and run on the host entry points."""
import ctypes
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "vcsr_mc_b200")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_plain_c_program_uses_the_library(tmp_path):
    exe = str(tmp_path / "host_abi")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "host_abi.c"), "-o", exe, "-L", LIBDIR, "-lvcsrmc",
                    "-Wl,-rpath," + LIBDIR], check=True, capture_output=True, text=True)
    mtx = tmp_path / "a.mtx"
    mtx.write_text("%%MatrixMarket matrix coordinate real general\n% demo\n5 7 6\n1 1 2.5\n1 6 -1\n2 3 4\n"
                   "3 7 0.5\n5 2 1\n5 5 -3\n")
    out = subprocess.run([exe, str(mtx), str(tmp_path / "a.csr")], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    fields = dict(kv.split("=") for kv in out.stdout.split())
    assert (fields["M"], fields["N"], fields["nnz"], fields["cache"]) == ("5", "7", "6", "same")
    assert fields["filled"] == "6" and int(fields["items"]) >= 1


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_ctypes_structs_match_the_header(tmp_path):
    """The ctypes mirrors of the ABI's structs have the header's size and field offsets."""
    from vcsr_mc_b200 import _lib

    structs = {"vcsrmc_device_info": _lib.DeviceInfo, "vcsrmc_upload_options": _lib.UploadOptions}
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "vcsrmc.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'    printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'    printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["    return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = str(tmp_path / "layout")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o", exe],
                   check=True, capture_output=True, text=True)
    out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {(a, b): int(c) for a, b, c in (ln.split() for ln in out if ln)}
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
