"""Per-K cost table (costWrite --per-k): file format, round trip and the
choice of entry for a row width, through the C ABI (no GPU needed)."""
import os
import subprocess

import pytest

import cwlb_spmm as cs


def _table():
    return [cs.SpmmCostParams(0.01, 0.02, 0.03, 0.5, K=32),
            cs.SpmmCostParams(0.011, 0.018, 0.01, 0.49, K=128),
            cs.SpmmCostParams(0.012, 0.016, 0.009, 0.47, K=512)]


def test_round_trip_and_format(tmp_path):
    p = tmp_path / "sub" / "costs_per_k.txt"
    assert cs.save_costs_per_k(_table(), str(p))
    lines = p.read_text().splitlines()
    assert lines[0].startswith("#")
    assert lines[1] == "32 0.010000 0.020000 0.030000 0.500000"
    back = cs.read_costs_per_k(str(p))
    assert [t.K for t in back] == [32, 128, 512]
    assert back[2].C_atomic_ns == pytest.approx(0.47)


@pytest.mark.parametrize("K,want", [(1, 32), (32, 32), (63, 32), (64, 128), (100, 128),
                                    (128, 128), (256, 512), (255, 128), (4096, 512)])
def test_nearest_width_on_a_log_scale(K, want):
    # 64 is as far from 32 as from 128 (log2): ties go to the larger width.
    assert cs.costs_for_k(_table(), K).K == want


def test_empty_table_and_bad_k():
    with pytest.raises(ValueError):
        cs.costs_for_k([], 128)
    with pytest.raises(ValueError):
        cs.costs_for_k(_table(), 0)


def test_comments_blank_lines_and_malformed_lines(tmp_path):
    p = tmp_path / "t.txt"
    p.write_text("# comment\n\n  64 0.1 0.2 0.3 0.4\n# more\n16 1 2 3 4\n")
    t = cs.read_costs_per_k(str(p))
    assert [e.K for e in t] == [64, 16]
    for bad in ("64 0.1 0.2 0.3\n", "0 1 2 3 4\n", "64 1 2 3 4 5\n", "x 1 2 3 4\n"):
        p.write_text(bad)
        assert cs.read_costs_per_k(str(p)) is None
    assert cs.read_costs_per_k(str(tmp_path / "missing.txt")) is None


def test_save_rejects_entries_without_k(tmp_path):
    assert not cs.save_costs_per_k([cs.SpmmCostParams(1, 2, 3, 4)], str(tmp_path / "x.txt"))


@pytest.mark.parametrize("argv", [["--per-k"], ["--per-k", "32,0"], ["--per-k", "32,x"],
                                  ["--per-k", "32", "1", "2", "3"]])
def test_costwrite_per_k_argument_errors(argv):
    """Argument errors are reported before any device is touched."""
    exe = os.path.join(os.path.dirname(cs.__file__), "bin", "costWrite")
    r = subprocess.run([exe, *argv], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    assert "Usage" in r.stderr or "positive" in r.stderr or "bad K list" in r.stderr
