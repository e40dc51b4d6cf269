"""Drop-in command lines and loader, checked on CPU against the reference.

* The text-CSR loader (bin/csr-check) accepts and rejects exactly what the
  reference's loader (src/data.cpp:12-130, compiled into oracle/_ref) does,
  with the same messages, and produces the same arrays.
* cwlb-spmm and costWrite reject bad command lines and bad datasets with the
  reference's exit status and messages (main.cpp:432-506, weightCost.cpp:21-41);
  those checks run before any device is used, so they need no GPU.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

BIN = os.path.join(ROOT, "cwlb-spmm_b200", "bin")
CWLB = os.path.join(BIN, "cwlb-spmm")
COSTWRITE = os.path.join(BIN, "costWrite")
CSRCHECK = os.path.join(BIN, "csr-check")

pytestmark = pytest.mark.skipif(not os.path.exists(CWLB), reason="CLI not built")

REF_DRIVER = r"""
import ctypes, sys
lib = ctypes.CDLL(sys.argv[1])
argv = [a.encode() for a in sys.argv[2:]]
arr = (ctypes.c_char_p * len(argv))(*argv)
sys.stdout.flush()
rc = lib.cwlbref_main(len(argv), arr)
sys.stdout.flush()
import os
os._exit(rc)
"""


def _ref_so():
    p = os.path.join(ROOT, "oracle", "_ref", "libcwlbref.so")
    if not os.path.exists(p):
        pytest.skip("oracle/_ref not built")
    return p


def run(cmd, cwd, stdin=""):
    env = dict(os.environ)
    for k in ("CWLB_COSTFILE", "CWLB_DATASET_DIR", "CWLB_RESULTS"):
        env.pop(k, None)
    p = subprocess.run(cmd, cwd=cwd, input=stdin, capture_output=True, text=True, env=env,
                       timeout=300)
    return p.returncode, p.stdout, p.stderr


def run_ref(argv, cwd, stdin=""):
    return run([sys.executable, "-c", REF_DRIVER, _ref_so(), *argv], cwd, stdin)


@pytest.fixture()
def workdir(tmp_path):
    build = tmp_path / "build"
    (tmp_path / "resources" / "datasets").mkdir(parents=True)
    build.mkdir()
    return tmp_path


def write_ds(workdir, name, text):
    (workdir / "resources" / "datasets" / f"{name}.csr").write_text(text)


BAD_DATASETS = {
    "empty": "",
    "oneline": "0,1,2\n",
    "noline2": "0,1,2",
    "emptyoffsets": "\n1,2\n",
    "nnzmismatch": "0,1,3\n0,1\n",
    "firstnonzero": "1,2,3\n0,1\n",
    "nonmonotone": "0,2,1,3\n0,1,2\n",
    "beyondnnz": "0,5,3\n0,1,2\n",
    "negativecol": "0,1,2\n0,-1\n",
    "negativennz": "0,-1\n\n",
    "badcell": "0,1,x\n0,1\n",
    "spacecell": "0,1, ,2\n0,1\n",
    "overflow": "0,1,99999999999\n0\n",
}

GOOD_DATASETS = {
    "plain": "0,2,3,3\n1,2,0\n",
    "crlf": "0,2,3\r\n1,0,2\r\n",
    "trailingcomma": "0,1,2,\n0,1,\n",
    "spaces": " 0, 1 ,2\n 1,0 \n",
    "emptycells": "0,,1,2\n,0,1\n",
    "plus": "+0,+1\n+0\n",
    "emptyline2": "0,0,0\n\n",
    "trailing": "0,1x,2junk\n0abc,1\n",
}


@pytest.mark.parametrize("name", sorted(BAD_DATASETS))
def test_loader_rejects_like_reference(workdir, reference, name):
    write_ds(workdir, name, BAD_DATASETS[name])
    path = str(workdir / "resources" / "datasets" / f"{name}.csr")
    rc, out, err = run([CSRCHECK, path], workdir / "build")
    assert rc == 1
    cwd = os.getcwd()
    os.chdir(workdir / "build")
    try:
        with pytest.raises(Exception) as ei:
            reference.load_csr(name)
    finally:
        os.chdir(cwd)
    want = str(ei.value).replace("../resources/datasets/", "")
    got = err.strip().replace(str(workdir / "resources" / "datasets") + "/", "")
    assert got == want


@pytest.mark.parametrize("name", sorted(GOOD_DATASETS))
def test_loader_accepts_like_reference(workdir, reference, name):
    write_ds(workdir, name, GOOD_DATASETS[name])
    cwd = os.getcwd()
    os.chdir(workdir / "build")
    try:
        ro, col, val, V, E = reference.load_csr(name)
    finally:
        os.chdir(cwd)
    rc, out, err = run([CSRCHECK, str(workdir / "resources" / "datasets" / f"{name}.csr")],
                       workdir)
    assert rc == 0, err
    v2, e2, _ = out.split()
    assert (int(v2), int(e2)) == (V, E)


def test_loader_matches_reference_on_config1_text(workdir, reference):
    from conftest import load_npz
    g = load_npz("cfg1_er4096.npz")
    text = ",".join(map(str, g["rowoff"])) + "\n" + ",".join(map(str, g["col"])) + "\n"
    write_ds(workdir, "er4096", text)
    cwd = os.getcwd()
    os.chdir(workdir / "build")
    try:
        ro, col, val, V, E = reference.load_csr("er4096")
    finally:
        os.chdir(cwd)
    assert np.array_equal(ro, g["rowoff"]) and np.array_equal(col, g["col"])
    rc, out, err = run([CSRCHECK, str(workdir / "resources" / "datasets" / "er4096.csr")], workdir)
    assert rc == 0 and out.split()[:2] == [str(V), str(E)]


CLI_ERRORS = [
    [],
    ["ds"],
    ["ds", "32"],
    ["ds", "abc", "--S", "4"],
    ["ds", "0", "--S", "4"],
    ["ds", "32", "--S", "0"],
    ["ds", "32", "-3"],
    ["ds", "32", "--X", "4"],
    ["ds", "32", "4", "2", "1"],
    ["ds", "32", "4", "8", "0"],
    ["ds", "32", "--candidate-search", "0"],
    ["ds", "32", "--candidate-search", "3x"],
    ["ds", "32", "--candidate-search", "--count", "3"],
    ["ds", "32", "--candidate-search", "--step", "-1"],
    ["", "32", "--S", "4"],
    ["missing", "32", "--S", "4"],
    ["bad", "32", "--candidates"],
    ["a", "b", "c", "d", "e", "f"],
]


@pytest.mark.parametrize("argv", CLI_ERRORS, ids=lambda a: "_".join(a) or "noargs")
def test_cli_errors_match_reference(workdir, argv):
    write_ds(workdir, "bad", "0,2,1\n0,1\n")
    rc, out, err = run([CWLB, *argv], workdir / "build")
    rrc, rout, rerr = run_ref(["cwlb-spmm", *argv], workdir / "build")
    assert (rc, err) == (rrc, rerr)
    assert out == rout == ""


@pytest.mark.parametrize("argv", [["1", "2"], ["0", "1", "1", "1", "1"], ["1", "1", "1", "-1", "1"],
                                  ["x", "1", "1", "1", "1"]])
def test_costwrite_argument_errors(workdir, argv):
    rc, out, err = run([COSTWRITE, *argv], workdir / "build")
    assert rc == 1
    if len(argv) == 2:
        assert err.startswith("Usage:")
    elif argv[0] == "x":
        assert err.strip() == "stoi"
    else:
        assert err.strip() == "All microbenchmark parameters must be positive."


def _big_text(rng, n, nnz):
    deg = rng.multinomial(nnz, np.ones(n) / n)
    ro = np.zeros(n + 1, np.int64)
    np.cumsum(deg, out=ro[1:])
    col = rng.integers(0, n, nnz)
    return ro, col


@pytest.mark.parametrize("damage", [None, "late_letter", "early_overflow", "mid_space"])
def test_loader_parallel_parse_matches_reference(workdir, reference, damage):
    """Lines long enough for the multi-threaded parse (2M column ids, ~16 MB):
    the same arrays as the reference's loader, or the same error."""
    rng = np.random.default_rng(3)
    ro, col = _big_text(rng, 100_000, 2_000_000)
    cells = [str(x) for x in col.tolist()]
    if damage == "late_letter":
        cells[-5] = "x7"
    elif damage == "early_overflow":
        cells[1000] = "99999999999"
        cells[-10] = "y"
    elif damage == "mid_space":
        cells[len(cells) // 2] = " "
    text = ",".join(map(str, ro.tolist())) + "\n" + ",".join(cells) + "\n"
    write_ds(workdir, "big", text)
    path = str(workdir / "resources" / "datasets" / "big.csr")
    rc, out, err = run([CSRCHECK, path], workdir / "build")
    cwd = os.getcwd()
    os.chdir(workdir / "build")
    try:
        if damage is None:
            rro, rcol, _, V, E = reference.load_csr("big")
        else:
            with pytest.raises(Exception) as ei:
                reference.load_csr("big")
    finally:
        os.chdir(cwd)
    if damage is None:
        assert rc == 0, err
        assert out.split()[:2] == [str(V), str(E)]
        h = 1469598103934665603
        for v in np.concatenate([rro, rcol]).astype(np.uint32).tolist():
            for i in range(4):
                h = ((h ^ ((v >> (8 * i)) & 0xFF)) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        assert out.split()[2] == f"{h:016x}"
    else:
        assert rc == 1 and err.strip() == str(ei.value)


def _dump_cli_features(tmp_path, rows, cols):
    path = tmp_path / f"x_{rows}x{cols}.bin"
    p = subprocess.run([CWLB, "--dump-features", str(rows), str(cols), str(path)],
                       capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    return np.fromfile(path, np.float32).reshape(rows, cols)


def test_cli_features_equal_the_reference_bits(tmp_path):
    """The CLI's X (deterministic_features, main.cpp:324-336: mt19937(42),
    U[0,1) floats, row-major) bit for bit: against the reference build's
    digest in the golden fixtures, and, where oracle/_ref exists, against the
    reference's own function on a larger shape."""
    import hashlib
    import json
    from conftest import GOLDEN
    with open(os.path.join(GOLDEN, "helpers.json")) as fh:
        h = json.load(fh)
    x = _dump_cli_features(tmp_path, 33, 17)
    assert hashlib.sha256(x.tobytes()).hexdigest() == h["features_33x17_sha256"]
    assert x.reshape(-1)[:8].tolist() == h["features_33x17_first"]
    so = _ref_so()
    if not os.path.exists(so):
        pytest.skip("oracle/_ref not built: checked against the golden digest only")
    from oracle import Reference
    ref = Reference(so)
    want = ref.features(1000, 96)
    got = _dump_cli_features(tmp_path, 1000, 96)
    assert np.array_equal(got.view(np.uint32), np.asarray(want, np.float32).view(np.uint32))
