"""The ROWS plan's work units and the BAND plan's view, built on the host, checked on the CPU:
tests/cpp/layout_check.cpp is linked against the library's own objects (the host functions
build_row_view, pack_units, build_band_view and choose_band of plan_rows.cu / plan_band.cu,
with libvcsrmc.so's csr_to_vcsr_mc making the formats) and states their rules
as properties of the output (see its header). No GPU is used: the program calls host code only."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "vcsr_mc_b200", "csrc")
OBJS = [os.path.join(ROOT, "vcsr_mc_b200", "_build", "cuda", n) for n in ("plan_rows.o", "plan_band.o")]
CUDA = "/usr/local/cuda"


@pytest.mark.skipif(shutil.which("g++") is None or not all(os.path.exists(o) for o in OBJS)
                    or not os.path.exists(os.path.join(CUDA, "lib64", "libcudart_static.a")),
                    reason="needs g++, the CUDA static runtime and the built objects (make -C vcsr_mc_b200/csrc)")
def test_host_layout_builders(tmp_path):
    exe = str(tmp_path / "layout_check")
    build = subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
                            "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "cpp", "layout_check.cpp"),
                            *OBJS, "-L", os.path.join(ROOT, "vcsr_mc_b200"), "-lvcsrmc",
                            "-Wl,-rpath," + os.path.join(ROOT, "vcsr_mc_b200"), "-L", os.path.join(CUDA, "lib64"),
                            "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-o", exe], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-2000:]
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.startswith("OK"), out.stdout[-2000:]
    fields = dict(kv.split("=") for kv in out.stdout.split()[1:])
    assert int(fields["row_views"]) > 0
    assert int(fields["densest_tile"]) > 256  # tiles beyond the producers' register window are covered
    assert int(fields["stencil_band"]) == 62  # the 100^3 stencil's windows fill 64-column tiles exactly
