"""The spmm_vcsr driver (the reference's command-line surface) on the GPU: every algorithm must pass
the reference's own acceptance check (src/main.cpp:257-291) against its fp64 CPU result."""
import csv
import io
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVER = os.path.join(ROOT, "vcsr_mc_b200", "spmm_vcsr")


def run_driver(*args):
    out = subprocess.run([DRIVER, *args, "--csv", "--check", "cpu"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    return list(csv.DictReader(io.StringIO(out.stdout)))


@pytest.mark.parametrize("extra", [[], ["--plan", "segment"], ["--plan", "rows", "--b16"], ["--plan", "band", "--b16"],
                                   ["--plan", "hybrid", "--b16"], ["--reorder", "rcm"],
                                   ["--bdist", "wide", "--segw", "32", "--tileK", "128"],
                                   ["--flush-l2", "--peak-gbs", "6545.3"]],
                         ids=["reference-call", "segment", "rows-b16", "band-b16", "hybrid-b16", "rcm", "wide-s32-t128",
                              "flush-roofline"])
def test_driver_all_algorithms_pass(extra):
    rows = run_driver("--gen", "c1", "--algo", "all", "--repeat", "2", "--warmup", "1", *extra)
    algos = {r["algo"]: r for r in rows}
    assert {"vcsr_mc", "vcsr_mc_fp32", "cusparse", "cusparse_fp16"} <= set(algos)
    for name, r in algos.items():
        assert r["validation"] == "pass", (name, r)
        assert float(r["gflops"]) > 0
        assert float(r["gbps_alg"]) > 0
        assert (r["roofline_frac"] != "") == ("--peak-gbs" in extra)


def test_driver_mtx_input(tmp_path):
    path = tmp_path / "a.mtx"
    path.write_text("%%MatrixMarket matrix coordinate real symmetric\n4 4 5\n1 1 2\n2 1 -1\n3 3 4\n4 2 1.5\n4 4 3\n")
    rows = run_driver("--mtx", str(path), "--algo", "vcsr_mc,vcsr_mc_fp32", "--O", "24", "--tileK", "16",
                      "--repeat", "1", "--warmup", "0")
    assert [r["validation"] for r in rows] == ["pass", "pass"]


def test_driver_rejects_bad_flags():
    out = subprocess.run([DRIVER, "--gen", "c1", "--algo", "nope"], capture_output=True, text=True, timeout=60)
    assert out.returncode == 2 and "Unknown algorithm" in out.stderr
