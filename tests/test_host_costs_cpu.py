"""C++ drop-in cost-file functions (host/include/utils.h) on the host only:
the reference's four-line file (save/read_costs_one_per_line,
src/utils.cpp:1024-1092) and the per-K table extension, compiled against
libcwlb_host.a and libcwlb_spmm.so the way the cwlb-spmm tool is."""
import os
import shutil
import subprocess

import pytest

from conftest import PKG, ROOT

PROG = r"""
#include <iostream>
#include <stdexcept>
#include <vector>

#include "utils.h"

int main(int argc, char** argv) {
    if (argc != 3) return 1;
    std::vector<SpmmCostParams> t(3);
    const int ks[3] = {32, 128, 512};
    for (int i = 0; i < 3; ++i) {
        t[i].K = ks[i];
        t[i].C_compute_ns = 0.01 * (i + 1);
        t[i].C_load_ns = 0.02 * (i + 1);
        t[i].C_store_ns = 0.03 * (i + 1);
        t[i].C_atomic_ns = 0.5 * (i + 1);
    }
    if (!save_costs_per_k(t, argv[1])) return 2;
    std::vector<SpmmCostParams> back;
    if (!read_costs_per_k(back, argv[1]) || back.size() != 3) return 3;
    std::cout << back[2].K << ' ' << back[2].C_atomic_ns << ' ' << costs_for_k(back, 100).K << ' '
              << costs_for_k(back, 64).K << ' ' << costs_for_k(back, 8).K << '\n';
    try {
        costs_for_k({}, 64);
        return 4;
    } catch (const std::invalid_argument&) {
    }
    SpmmCostParams one = t[1];
    if (!save_costs_one_per_line(one, argv[2])) return 5;
    SpmmCostParams r;
    if (!read_costs_one_per_line(r, argv[2])) return 6;
    std::cout << r.C_compute_ns << ' ' << r.C_load_ns << ' ' << r.C_store_ns << ' '
              << r.C_atomic_ns << '\n';
    return 0;
}
"""


@pytest.fixture(scope="module")
def prog(tmp_path_factory):
    lib = os.path.join(PKG, "lib")
    if not os.path.exists(os.path.join(lib, "libcwlb_host.a")) or not shutil.which("g++"):
        pytest.skip("host library or g++ missing")
    d = tmp_path_factory.mktemp("hostcosts")
    src = d / "prog.cpp"
    src.write_text(PROG)
    exe = d / "prog"
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(PKG, "host", "include"), "-I", "/usr/local/cuda/include",
           str(src), os.path.join(lib, "libcwlb_host.a"), "-L", lib, "-lcwlb_spmm",
           "-L", "/usr/local/cuda/lib64", "-lcudart_static", "-ldl", "-lrt", "-lpthread",
           f"-Wl,-rpath,{lib}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return exe


def test_per_k_table_and_cost_file_through_the_cpp_interface(prog, tmp_path):
    table, one = tmp_path / "a" / "per_k.txt", tmp_path / "costs.txt"
    r = subprocess.run([str(prog), str(table), str(one)], capture_output=True, text=True,
                       timeout=60)
    assert r.returncode == 0, (r.returncode, r.stderr)
    first, second = r.stdout.splitlines()
    # Entry 512 read back; K = 100 -> 128, 64 -> 128 (tie goes to the wider), 8 -> 32.
    assert first.split() == ["512", "1.5", "128", "128", "32"]
    assert [float(v) for v in second.split()] == [0.02, 0.04, 0.06, 1.0]
    assert table.read_text().splitlines()[1] == "32 0.010000 0.020000 0.030000 0.500000"
    assert one.read_text() == "0.020000\n0.040000\n0.060000\n1.000000\n"
