"""validate_custom_csr_result: the library's version against the reference's.

cwlb_validate_result (the C ABI under the C++ interface's
validate_custom_csr_result) must print what the reference's
validate_custom_csr_result (src/utils.cpp:1117-1265, compiled into oracle/_ref)
prints, on stdout and on stderr, and return the same verdict.  Both write
through the process's std::cout, whose fixed/6-digit mode, once set by a
mismatch report, stays set; so each side runs the whole case sequence in one
fresh process, and the two transcripts are compared as text.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _csr(rows, cols, rng, density=0.3, empty_rows=()):
    ro = [0]
    col, val = [], []
    for r in range(rows):
        if r not in empty_rows:
            for c in range(cols):
                if rng.random() < density:
                    col.append(c)
                    val.append(float(rng.integers(1, 4)) * 0.5)
        ro.append(len(col))
    return np.array(ro, np.int32), np.array(col, np.int32), np.array(val, np.float32)


def cases():
    """(result, reference, rowoff, col, val, dense, tol) tuples, seeded."""
    rng = np.random.default_rng(5)
    out = []
    R, K, V = 12, 6, 9
    ro, col, val = _csr(R, V, rng, empty_rows=(3,))
    dense = rng.uniform(-1, 1, (V, K)).astype(np.float32)
    ref = rng.uniform(-2, 2, (R, K)).astype(np.float32)
    out.append((ref + 1e-6, ref, ro, col, val, dense, 1e-4))  # passes
    r = ref.copy()
    r[1, 2] += 0.5
    r[3, 0] -= 0.25  # a row with no stored entries
    r[11, 5] = 7.0
    out.append((r, ref, ro, col, val, dense, 1e-4))
    out.append((ref + 1.0, ref, ro, col, val, dense, 1e-4))  # more than 10 mismatches
    r = ref.copy()
    f = ref.copy()
    r[0, 0] = np.nan                      # NaN against a number
    r[0, 1] = f[0, 1] = np.nan            # NaN against NaN: equal
    r[0, 2] = f[0, 2] = np.inf            # same infinity: equal
    r[0, 3], f[0, 3] = np.inf, -np.inf    # opposite infinities
    r[0, 4] = -np.inf                     # infinity against a number
    f[2, 2] = np.nan                      # number against NaN
    out.append((r, f, ro, col, val, dense, 1e-4))
    out.append((ref + 0.5, ref, ro, col, val, dense, 0.6))   # large tolerance: passes
    out.append((ref + 0.5, ref, ro, col, val, dense, 0.0))   # zero tolerance
    out.append((ref, ref, ro, col, val, dense, -1.0))        # bad tolerance
    out.append((ref, ref, ro, col, val, dense, float("nan")))
    out.append((ref[:, :5], ref, ro, col, val, dense, 1e-4))   # result shape differs
    out.append((ref[:11], ref[:11], ro, col, val, dense, 1e-4))  # CSR row count differs
    out.append((ref, ref, ro, col, val, dense[:, :4], 1e-4))   # dense columns differ
    out.append((ref, ref, ro, col, val, dense[:0], 1e-4))      # dense has no rows
    # Dense with fewer than 5 rows, large values, a second pass after mismatches.
    ro2, col2, val2 = _csr(4, 3, rng, density=0.9)
    d2 = (rng.uniform(-1, 1, (3, 4)) * 1e5).astype(np.float32)
    f2 = (rng.uniform(-1, 1, (4, 4)) * 1e4).astype(np.float32)
    r2 = f2.copy()
    r2[2, 3] += 3.0
    out.append((r2, f2, ro2, col2, val2, d2, 1e-4))
    out.append((f2, f2, ro2, col2, val2, d2, 1e-4))
    out.append((np.zeros((0, 4), np.float32), np.zeros((0, 4), np.float32),
                np.zeros(1, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32), d2, 1e-4))
    return out


def _run_side(side):
    """Runs every case on one side; prints each verdict after the report."""
    import ctypes
    libc = ctypes.CDLL(None)
    sys.path.insert(0, os.path.join(ROOT, "cwlb-spmm_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    if side == "ours":
        import cwlb_spmm as cs

        def run(r, f, ro, col, val, d, tol):
            return cs.validate_custom_csr_result(r, f, cs.CSR(ro, col, val), d, tol)
    else:
        from oracle import Reference
        ref = Reference()

        def run(r, f, ro, col, val, d, tol):
            return ref.validate_shapes(r, f, ro, col, val, d, tol)
    for i, c in enumerate(cases()):
        ok = run(*c)
        libc.fflush(None)
        os.write(1, f"<case {i}: {int(ok)}>\n".encode())
        os.write(2, f"<case {i}>\n".encode())


def _transcript(side):
    p = subprocess.run([sys.executable, os.path.abspath(__file__), side], capture_output=True,
                       text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    return p.stdout, p.stderr


def test_validation_report_matches_reference(reference):
    ours_out, ours_err = _transcript("ours")
    ref_out, ref_err = _transcript("ref")
    assert ours_out == ref_out
    assert ours_err == ref_err
    verdicts = [ln for ln in ours_out.splitlines() if ln.startswith("<case")]
    assert len(verdicts) == len(cases())
    assert verdicts[0].endswith(": 1>") and verdicts[1].endswith(": 0>")


def test_validation_verdicts_without_reference():
    out, err = _transcript("ours")
    v = [int(ln.rsplit(":", 1)[1].strip(" >")) for ln in out.splitlines() if ln.startswith("<case")]
    assert v == [1, 0, 0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1]
    assert "showing 10 mismatched elements" in out
    assert "Validation error: Validation tolerance must be finite and non-negative." in err
    assert "Validation failed: result matrix shape is (12, 5), but reference matrix shape is (12, 6)." in err


def test_validation_rejects_negative_sizes():
    sys.path.insert(0, os.path.join(ROOT, "cwlb-spmm_b200"))
    import ctypes as C
    import cwlb_spmm as cs
    passed = C.c_int32(7)
    rc = cs._lib.cwlb_validate_result(None, -1, 1, None, 1, 1, None, 2, None, None, None, 1, 1,
                                      1e-4, C.byref(passed))
    assert rc == cs.ERR_INVALID_ARGUMENT and passed.value == 7
    with pytest.raises(ValueError, match="negative size"):
        cs._check(rc)


if __name__ == "__main__":
    _run_side(sys.argv[1])
