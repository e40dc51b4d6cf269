"""The binary CSR cache beside a text dataset (host/src/data.cpp).

Loading through the cache must give exactly what the text loader gives; a
fresh cache is read instead of the text; a stale (text changed or touched),
truncated or corrupted cache is ignored and rewritten; a text file the loader
rejects leaves no cache.  Exercised through bin/csr-check --cache, which
prints the loaded CSR's size and checksum and says on stderr whether the
cache was hit or written; the cache's format is cross-checked by the
binding's own reader.
"""
import os
import subprocess

import numpy as np
import pytest

import cwlb_spmm as cs
from conftest import ROOT, load_npz

CSRCHECK = os.path.join(ROOT, "cwlb-spmm_b200", "bin", "csr-check")

pytestmark = pytest.mark.skipif(not os.path.exists(CSRCHECK), reason="tools not built")


def check(path, cache=True):
    p = subprocess.run([CSRCHECK, *(["--cache"] if cache else []), str(path)], capture_output=True,
                       text=True, timeout=120)
    return p.returncode, p.stdout, p.stderr.strip()


def write_text(path, rowoff, col):
    path.write_text(",".join(map(str, rowoff)) + "\n" + ",".join(map(str, col)) + "\n")


@pytest.fixture()
def dataset(tmp_path):
    g = load_npz("cfg1_er4096.npz")
    path = tmp_path / "er.csr"
    write_text(path, g["rowoff"], g["col"])
    return path, g


def test_cache_written_then_hit_and_identical(dataset):
    path, g = dataset
    rc0, plain, _ = check(path, cache=False)
    rc1, out1, err1 = check(path)
    assert (rc0, rc1) == (0, 0) and err1 == "cache: written"
    assert os.path.exists(str(path) + ".cwlbbin")
    rc2, out2, err2 = check(path)
    assert rc2 == 0 and err2 == "cache: hit"
    assert plain == out1 == out2
    c = cs.read_csr_cache(str(path))
    assert np.array_equal(c.RowOffset, g["rowoff"]) and np.array_equal(c.ColInd, g["col"])
    assert (c.Value == 1.0).all()
    assert os.path.getsize(str(path) + ".cwlbbin") == 64 + 4 * (len(g["rowoff"]) + len(g["col"]))


def test_stale_cache_is_rebuilt(dataset):
    path, g = dataset
    check(path)
    # New content (different size): the cache must follow the text.
    ro = np.array([0, 2, 3, 3], np.int32)
    write_text(path, ro, [1, 2, 0])
    rc, out, err = check(path)
    assert rc == 0 and err == "cache: written" and out.split()[:2] == ["3", "3"]
    # Same content, new modification time: rebuilt as well.
    st = os.stat(path)
    os.utime(path, ns=(st.st_atime_ns, st.st_mtime_ns + 1_000_000_000))
    rc, out2, err = check(path)
    assert rc == 0 and err == "cache: written" and out2 == out
    assert check(path)[2] == "cache: hit"


@pytest.mark.parametrize("damage", ["flip", "truncate", "magic", "extra"])
def test_damaged_cache_is_ignored(dataset, damage):
    path, g = dataset
    rc, want, _ = check(path)
    cpath = str(path) + ".cwlbbin"
    raw = bytearray(open(cpath, "rb").read())
    if damage == "flip":
        raw[-5] ^= 0x10          # inside ColInd: checksum mismatch
    elif damage == "truncate":
        raw = raw[:-4]
    elif damage == "magic":
        raw[0:8] = b"CWLBCSR9"
    else:
        raw += b"\0\0\0\0"
    open(cpath, "wb").write(bytes(raw))
    assert cs.read_csr_cache(str(path)) is None
    rc, out, err = check(path)
    assert rc == 0 and out == want and err == "cache: written"
    assert check(path)[2] == "cache: hit"


def test_rejected_text_leaves_no_cache(tmp_path):
    path = tmp_path / "bad.csr"
    path.write_text("0,2,1\n0,1\n")
    rc_plain, _, err_plain = check(path, cache=False)
    rc, out, err = check(path)
    assert rc == rc_plain == 1 and err == err_plain and out == ""
    assert not os.path.exists(str(path) + ".cwlbbin")


def test_empty_graph_round_trips(tmp_path):
    path = tmp_path / "empty.csr"
    path.write_text("0,0,0\n\n")
    rc1, out1, err1 = check(path)
    rc2, out2, err2 = check(path)
    assert (rc1, rc2) == (0, 0) and (err1, err2) == ("cache: written", "cache: hit")
    assert out1 == out2 and out1.split()[:2] == ["2", "0"]
    c = cs.read_csr_cache(str(path))
    assert list(c.RowOffset) == [0, 0, 0] and c.ColInd.size == 0
