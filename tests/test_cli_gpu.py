"""The drop-in command lines on the GPU.

cwlb-spmm's output lines (per-launch lines, summaries, candidate tables,
results.txt records) must follow the reference's grammar (main.cpp:338-741);
numbers (times, device name, S values that depend on the SM count) differ and
are normalised before comparing with the reference CLI run through oracle/_ref.
"""
import os
import re
import subprocess
import sys

import numpy as np
import pytest

import cwlb_spmm as cs
import graphs
from conftest import ROOT

pytestmark = pytest.mark.gpu

BIN = os.path.join(ROOT, "cwlb-spmm_b200", "bin")
CWLB = os.path.join(BIN, "cwlb-spmm")
COSTWRITE = os.path.join(BIN, "costWrite")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libcwlbref.so")
COSTS = "0.021350\n0.684712\n0.298413\n0.517096\n"

REF_DRIVER = r"""
import ctypes, sys, os
lib = ctypes.CDLL(sys.argv[1])
argv = [a.encode() for a in sys.argv[2:]]
arr = (ctypes.c_char_p * len(argv))(*argv)
rc = lib.cwlbref_main(len(argv), arr)
sys.stdout.flush()
os._exit(rc)
"""


def _env():
    env = dict(os.environ)
    for k in ("CWLB_COSTFILE", "CWLB_DATASET_DIR", "CWLB_RESULTS", "CWLB_COSTS_PER_K",
              "CWLB_COSTFILE_PER_K"):
        env.pop(k, None)
    return env


def run(cmd, cwd, stdin=""):
    p = subprocess.run(cmd, cwd=cwd, input=stdin, capture_output=True, text=True, env=_env(),
                       timeout=900)
    return p.returncode, p.stdout, p.stderr


@pytest.fixture()
def workdir(tmp_path):
    (tmp_path / "resources" / "datasets").mkdir(parents=True)
    (tmp_path / "build").mkdir()
    (tmp_path / "resources" / "spmm_costs.txt").write_text(COSTS)
    rowoff, col, _ = graphs.rmat_np(9, 3000, 0.57, 0.19, 0.19, seed=3, symmetrize=True,
                                    drop_self_loops=True, dedupe=True)
    text = ",".join(map(str, rowoff)) + "\n" + ",".join(map(str, col)) + "\n"
    (tmp_path / "resources" / "datasets" / "g.csr").write_text(text)
    return tmp_path


NUM = re.compile(r"-?\d+(\.\d+)?(e[-+]?\d+)?")


def template(text):
    out = []
    for line in text.splitlines():
        line = re.sub(r"device=\S+( \S+)*? K=", "device=<dev> K=", line)
        out.append(NUM.sub("#", line))
    return out


def _ref_available():
    return os.path.exists(REF_SO)


@pytest.mark.parametrize("argv,stdin", [
    (["g", "16", "--S", "8"], ""),
    (["g", "32", "64"], ""),
    (["g", "16", "4", "12", "4"], ""),
    (["g", "16", "--candidates"], ""),
    (["g", "8", "--candidate-search", "3"], "maybe\nyes\n"),
    (["g", "8", "--candidate-search", "--step", "5"], "no\n"),
])
def test_cli_output_grammar_matches_reference(workdir, argv, stdin):
    rc, out, err = run([CWLB, *argv], workdir / "build", stdin)
    assert rc == 0, err
    assert "SpMM time:" in out or "Search cancelled" in out
    times = [float(m) for m in re.findall(r"SpMM time: ([0-9.]+) us", out)]
    assert all(t > 0 for t in times)
    ours_results = (workdir / "resources" / "results.txt").read_text() \
        if (workdir / "resources" / "results.txt").exists() else ""
    if not _ref_available():
        pytest.skip("oracle/_ref not built: grammar checked on our side only")
    (workdir / "resources" / "results.txt").unlink(missing_ok=True)
    rrc, rout, rerr = run([sys.executable, "-c", REF_DRIVER, REF_SO, "cwlb-spmm", *argv],
                          workdir / "build", stdin)
    assert rrc == 0, rerr
    ours_t, ref_t = template(out), template(rout)
    ref_results = (workdir / "resources" / "results.txt").read_text() \
        if (workdir / "resources" / "results.txt").exists() else ""
    if "--candidate-search" in argv:
        # The search interval follows whichever candidate timed fastest, so
        # the number of search points can differ between runs: compare up to
        # the plan, then check that every planned S value was run once.
        cut = next(i for i, ln in enumerate(ours_t) if ln.startswith("[Search plan]"))
        assert ours_t[:cut] == ref_t[:cut]
        plan = re.search(r"\[Search plan\] S values:((?: \d+)+)", out)
        ran = re.findall(r"\[Search\] running P\d+ S=(\d+)", out)
        if "yes" in stdin:
            assert plan.group(1).split() == ran
            assert out.count("Results appended to") == 1
            assert ours_results.startswith("cwlb-spmm-candidates\t")
        else:
            assert ran == [] and "Search cancelled; results.txt unchanged." in out
    else:
        assert ours_t == ref_t
        assert template(ours_results) == template(ref_results)


def test_cli_missing_cost_file(workdir):
    (workdir / "resources" / "spmm_costs.txt").unlink()
    rc, out, err = run([CWLB, "g", "16", "--S", "8"], workdir / "build")
    assert rc == 1
    assert err.strip() == ("Cannot read microbenchmark cost file: ../resources/spmm_costs.txt. "
                           "Run ./costWrite first.")


def test_cli_large_k_runs(workdir):
    rc, out, err = run([CWLB, "g", "1100", "--S", "16"], workdir / "build")
    assert rc == 0, err
    assert re.search(r"SpMM time: [0-9.]+ us", out)


@pytest.mark.parametrize("argv", [["g", "16", "--S", "8"], ["g", "13", "4"], ["g", "1100", "--S", "16"],
                                  ["g", "8", "--candidates"]])
def test_cli_verify_checks_every_run(workdir, argv):
    rc, out, err = run([CWLB, *argv, "--verify"], workdir / "build")
    assert rc == 0, err
    runs = len(re.findall(r"SpMM time: ", out))
    assert runs >= 1
    assert out.count("Validation passed: all elements satisfy the comparison criteria.") == runs
    assert len(re.findall(r"\[Verify\] S=\d+ ", out)) == runs
    # Without --verify the output carries no verification lines.
    rc, out2, err = run([CWLB, *argv], workdir / "build")
    assert rc == 0 and "[Verify]" not in out2


def test_cli_verify_with_out_of_range_column_fails(workdir):
    # A column beyond the row count is caught by the aggregation's own checks
    # (exit status 1) before any verification.  Mismatch reports themselves
    # are checked against the reference on CPU (test_validate_cpu.py).
    (workdir / "resources" / "datasets" / "bad.csr").write_text("0,1,2\n0,9\n")
    rc, out, err = run([CWLB, "bad", "16", "--S", "4", "--verify"], workdir / "build")
    assert rc == 1 and "[Verify]" not in out


def test_cli_csr_cache(workdir):
    # CWLB_CSR_CACHE=1: the first run writes the binary cache beside the text
    # file, the second reads it; output grammar and the graph are unchanged.
    env = _env()
    env["CWLB_CSR_CACHE"] = "1"
    argv = [CWLB, "g", "16", "--S", "8", "--verify"]
    outs = []
    for _ in range(2):
        p = subprocess.run(argv, cwd=workdir / "build", capture_output=True, text=True, env=env,
                           timeout=900)
        assert p.returncode == 0, p.stderr
        outs.append(p.stdout)
    assert (workdir / "resources" / "datasets" / "g.csr.cwlbbin").exists()
    assert template(outs[0]) == template(outs[1])
    assert "V: 512, E: " in outs[1] and "Validation passed" in outs[1]


def test_cli_deterministic_mode_verifies(workdir):
    env = _env()
    env["CWLB_DETERMINISTIC"] = "1"
    p = subprocess.run([CWLB, "g", "16", "--S", "2", "--verify"], cwd=workdir / "build",
                       capture_output=True, text=True, env=env, timeout=900)
    assert p.returncode == 0, p.stderr
    assert "Validation passed" in p.stdout


def test_costwrite_per_k_table_and_cli_choice(workdir):
    """costWrite --per-k calibrates once per listed K and writes the per-K
    table; cwlb-spmm with CWLB_COSTS_PER_K=1 runs with the entry nearest to K
    and leaves its stdout grammar unchanged."""
    rc, out, err = run([COSTWRITE, "--per-k", "32,128", "5", "8192", "16", "4"], workdir / "build")
    assert rc == 0, err
    assert out.splitlines()[-1] == "Saved per-K cost parameters to: ../resources/spmm_costs_per_k.txt"
    table = cs.read_costs_per_k(str(workdir / "resources" / "spmm_costs_per_k.txt"))
    assert [t.K for t in table] == [32, 128]
    assert all(v > 0 for t in table for v in (t.C_compute_ns, t.C_load_ns, t.C_store_ns,
                                               t.C_atomic_ns))
    env = _env()
    env["CWLB_COSTS_PER_K"] = "1"
    p = subprocess.run([CWLB, "g", "100", "--S", "8"], cwd=workdir / "build", capture_output=True,
                       text=True, env=env, timeout=900)
    assert p.returncode == 0, p.stderr
    assert "costs: per-K table entry K=128" in p.stderr
    assert re.search(r"SpMM time: [0-9.]+ us", p.stdout)
    plain_rc, plain_out, _ = run([CWLB, "g", "100", "--S", "8"], workdir / "build")
    assert plain_rc == 0 and template(plain_out)[:3] == template(p.stdout)[:3]


def test_costwrite_writes_cost_file(workdir):
    rc, out, err = run([COSTWRITE, "32", "5", "8192", "16", "4"], workdir / "build")
    assert rc == 0, err
    lines = out.splitlines()
    assert lines[-6].startswith("device: ")
    for i, k in enumerate(["C_compute_ns", "C_load_ns", "C_store_ns", "C_atomic_ns"]):
        assert lines[-5 + i].startswith(k + ": ")
    assert lines[-1] == "Saved cost parameters to: ../resources/spmm_costs.txt"
    vals = (workdir / "resources" / "spmm_costs.txt").read_text().split("\n")
    assert len(vals) == 5 and vals[-1] == ""
    for v in vals[:4]:
        assert re.fullmatch(r"\d+\.\d{6}", v)
        assert float(v) > 0


def _run_env(cmd, cwd, extra_env, stdin=""):
    env = _env()
    env.update(extra_env)
    p = subprocess.run(cmd, cwd=cwd, input=stdin, capture_output=True, text=True, env=env,
                       timeout=900)
    return p.returncode, p.stdout, p.stderr


@pytest.mark.parametrize("argv", [["g", "16", "--S", "8", "--verify"],
                                  ["g", "24", "--candidates", "--verify"]])
def test_cli_multi_gpu_shards_verify_and_keep_the_grammar(workdir, argv):
    # CWLB_DEVICES=0,0: two shards on one B200 (two contexts, two streams),
    # the multi-GPU runner's whole path; every run verified against the
    # float64 device aggregation of the unsorted graph.
    rc, out, err = _run_env([CWLB, *argv], workdir / "build", {"CWLB_DEVICES": "0,0"})
    assert rc == 0, err
    assert out.count("[Verify]") >= 1 and "PASS" in out.upper()
    assert re.search(r"device=.* x2 K=", out)
    rc1, out1, err1 = run([CWLB, *argv], workdir / "build")
    assert rc1 == 0, err1
    strip = lambda t: [ln for ln in template(t) if not ln.startswith("[Verify]")]  # noqa: E731
    assert strip(out) == strip(out1)


def test_cli_multi_gpu_device_list_errors(workdir):
    rc, out, err = _run_env([CWLB, "g", "16", "--S", "8"], workdir / "build",
                            {"CWLB_DEVICES": "0,99"})
    assert rc == 1 and "CWLB_DEVICES" in err


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except ImportError:
        return 0


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_cli_two_gpus(workdir):
    rc, out, err = _run_env([CWLB, "g", "16", "--S", "8", "--verify"], workdir / "build",
                            {"CWLB_GPUS": "2"})
    assert rc == 0, err
    assert "[Verify]" in out
