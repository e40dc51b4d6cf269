"""CPU-side checks of the product library (no GPU needed, no compute calls).

* libcwlb_spmm.so loads and exports every function include/cwlb_spmm.h
  declares;
* without a CUDA device, creating a context fails loudly (no CPU fallback);
* the host-side helpers (capacity_from_s, the partitioner's S, wave_based_s,
  recommended_candidate_w, the cost-file format) equal the reference's, via
  the golden fixtures produced by the reference itself.
"""
import ctypes
import json
import os

import numpy as np
import pytest

import cwlb_spmm as cs
from conftest import GOLDEN, load_npz


def test_library_exports_every_header_function():
    names = cs.header_functions()
    assert len(names) >= 20
    lib = ctypes.CDLL(cs.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_constants_equal_the_header_defines():
    """The binding's flag and status constants are the header's #defines."""
    import re
    with open(cs.HEADER_PATH) as fh:
        text = fh.read()
    defines = {m.group(1): int(m.group(2), 0)
               for m in re.finditer(r"#define\s+CWLB_(\w+)\s+\(?([0-9xXa-fA-F]+)u?", text)}
    checked = 0
    for name, value in defines.items():
        if hasattr(cs, name):
            assert getattr(cs, name) == value, name
            checked += 1
    for name in ("ROWS_COVERED", "DETERMINISTIC", "TASK_PER_WARP", "TASK_PER_CTA"):
        assert name in defines and getattr(cs, name) == defines[name], name
    assert checked >= 6


def test_header_is_plain_c(tmp_path):
    """include/cwlb_spmm.h is the C ABI: it compiles as pedantic C99 (and C++17)."""
    import shutil
    import subprocess
    inc = os.path.dirname(cs.HEADER_PATH)
    src = tmp_path / "h.c"
    src.write_text('#include "cwlb_spmm.h"\nint main(void) { return CWLB_OK; }\n')
    for cc, std in (("gcc", "-std=c99"), ("g++", "-std=c++17")):
        if shutil.which(cc) is None:
            pytest.skip(f"{cc} not installed")
        lang = ["-x", "c++"] if cc == "g++" else []
        r = subprocess.run([cc, std, "-Wall", "-Wextra", "-pedantic", "-Werror", f"-I{inc}",
                            *lang, "-c", str(src), "-o", str(tmp_path / "h.o")],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_context_without_device_fails_loudly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(cs.NoDeviceError):
        cs.Context(0)


def _golden_helpers():
    with open(os.path.join(GOLDEN, "helpers.json")) as fh:
        return json.load(fh)


def test_capacity_and_segment_size_match_reference():
    h = _golden_helpers()
    sets = load_npz("partition_cases.npz")["cost_sets"]
    for s, ci, cap in h["capacity_from_s"]:
        assert cs.capacity_from_s(s, cs.SpmmCostParams.from_list(sets[ci])) == cap
    assert cs.capacity_from_s(5, cs.SpmmCostParams(0, 0, 1, 2.5)) == h["capacity_from_s_zero_edge"]
    assert cs.capacity_from_s(5, cs.SpmmCostParams(-1, 0.5, 1, -2.5)) == h["capacity_from_s_neg_edge"]


def test_segment_size_reproduces_effective_s(oracle):
    # S recovered from capacity_from_s(S) is sometimes S - 1 in double
    # arithmetic (src/utils.cpp:859-864); the library must reproduce it.
    rng = np.random.default_rng(3)
    seen_shift = False
    for _ in range(2000):
        costs = cs.SpmmCostParams(rng.uniform(0.001, 3), rng.uniform(0.001, 3), rng.uniform(0, 3),
                                  rng.uniform(0, 5))
        S = int(rng.integers(1, 2000))
        cap = cs.capacity_from_s(S, costs)
        got = cs.segment_size(costs, cap)
        wcl = costs.C_compute_ns + costs.C_load_ns
        want = max(1, int(np.floor((cap - costs.C_atomic_ns) / max(1e-30, wcl))))
        assert got == want
        seen_shift |= got == S - 1
    assert seen_shift
    nan_costs = cs.SpmmCostParams(float("nan"), 1, 1, 1)
    assert cs.segment_size(nan_costs, 10.0) == 1
    assert cs.segment_size(cs.SpmmCostParams(1e-300, 0, 0, 0), 1e10) == 1  # overflow -> INT_MIN -> 1


def test_wave_and_candidate_helpers_match_reference():
    h = _golden_helpers()
    for nnz, w in h["recommended_w"]:
        assert cs.recommended_candidate_w(nnz) == w
    for nnz, cu, w, s in h["wave_based_s"]:
        assert cs.wave_based_s(nnz, cu, w) == s
    with pytest.raises(ValueError, match="compute_units and wave must be positive"):
        cs.wave_based_s(100, 0, 4)
    with pytest.raises(ValueError):
        cs.wave_based_s(100, 4, -1)


def test_cost_file_format_matches_reference(tmp_path):
    h = _golden_helpers()
    p = tmp_path / "sub" / "spmm_costs.txt"
    costs = cs.SpmmCostParams(0.0213501, 0.6847129, 2.5, 1234.5678919)
    assert cs.save_costs_one_per_line(costs, str(p))
    assert p.read_text() == h["cost_file_text"]
    back = cs.read_costs_one_per_line(str(p))
    assert back.C_atomic_ns == pytest.approx(1234.567892)
    assert cs.read_costs_one_per_line(str(tmp_path / "missing.txt")) is None
    (tmp_path / "short.txt").write_text("1.0\n2.0\n")
    assert cs.read_costs_one_per_line(str(tmp_path / "short.txt")) is None
    assert cs.save_costs_one_per_line(costs, str(p), append=True)
    assert len(p.read_text().split()) == 8
