"""ctypes bindings for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Two libraries, both built by oracle/Makefile:
  * libcwlb_oracle.so - the restatement of the reference's hot path
    (cwlb_oracle.cpp); always present once built.
  * _ref/libcwlbref.so - the reference's own unmodified sources compiled
    against the host stand-ins in oracle/shim/ (built only where the
    reference checkout exists; it then travels with the repository).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module.  The product path never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libcwlb_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libcwlbref.so")

_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")


def _c_i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _c_f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class Oracle:
    """The restated reference algorithms (cwlb_oracle.cpp)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        lib = C.CDLL(path)
        lib.oracle_sort_by_degree.argtypes = [C.c_int, C.c_int, _i32p, _i32p, _f32p,
                                              _i32p, _i32p, _i32p, _f32p]
        lib.oracle_sort_by_degree.restype = C.c_int
        lib.oracle_partition.argtypes = [C.c_int, _i32p, _f64p, C.c_double, C.c_void_p,
                                         C.c_int64]
        lib.oracle_partition.restype = C.c_int64
        lib.oracle_spmm_mean.argtypes = [C.c_int, _i32p, _i32p, _f32p, _i32p, _f32p,
                                         C.c_int64, C.c_int64, _i32p, C.c_int64, _f32p,
                                         C.c_int]
        lib.oracle_spmm_mean.restype = C.c_int
        lib.oracle_spmm_mean_f64.argtypes = [C.c_int, _i32p, _i32p, _f32p, _i32p, _f32p,
                                             C.c_int64, _f64p, _f64p, C.c_int]
        lib.oracle_spmm_mean_f64.restype = None
        lib.oracle_capacity_from_s.argtypes = [C.c_int, _f64p]
        lib.oracle_capacity_from_s.restype = C.c_double
        lib.oracle_wave_based_s.argtypes = [C.c_int64, C.c_int, C.c_int]
        lib.oracle_wave_based_s.restype = C.c_int
        lib.oracle_recommended_w.argtypes = [C.c_uint64, _i32p]
        lib.oracle_recommended_w.restype = None
        lib.oracle_features.argtypes = [C.c_int, C.c_int, _f32p]
        lib.oracle_features.restype = None
        self.lib = lib

    def sort_by_degree(self, rowoff, col, val):
        rowoff, col, val = _c_i32(rowoff), _c_i32(col), _c_f32(val)
        n = len(rowoff) - 1
        origin = np.zeros(max(n, 0), np.int32)
        newoff = np.zeros(max(n + 1, 1), np.int32)
        newcol = np.zeros(len(col), np.int32)
        newval = np.zeros(len(val), np.float32)
        rc = self.lib.oracle_sort_by_degree(n, len(col), rowoff, col, val, origin, newoff,
                                            newcol, newval)
        if rc:
            raise RuntimeError("oracle sort: inconsistent NNZ count")
        return origin, newoff, newcol, newval

    def partition(self, rowoff, costs, capacity):
        rowoff = _c_i32(rowoff)
        costs = np.ascontiguousarray(costs, np.float64)
        n = len(rowoff) - 1
        cnt = self.lib.oracle_partition(n, rowoff, costs, float(capacity), None, 0)
        out = np.zeros((max(cnt, 1), 4), np.int32)
        self.lib.oracle_partition(n, rowoff, costs, float(capacity), out.ctypes.data, cnt)
        return out[:cnt]

    def spmm_mean(self, rowoff, col, val, origin, H, tasks, n_threads=0):
        rowoff, col, val, origin = _c_i32(rowoff), _c_i32(col), _c_f32(val), _c_i32(origin)
        H = _c_f32(H)
        tasks = _c_i32(np.asarray(tasks).reshape(-1, 4))
        n = len(rowoff) - 1
        K = H.shape[1]
        out = np.zeros((n, K), np.float32)
        rc = self.lib.oracle_spmm_mean(n, rowoff, col, val, origin, H, H.shape[0], K,
                                       tasks.reshape(-1) if tasks.size else np.zeros(4, np.int32),
                                       len(tasks), out, n_threads)
        if rc:
            raise IndexError("oracle spmm: index out of range")
        return out

    def spmm_mean_f64(self, rowoff, col, val, origin, H, n_threads=0):
        rowoff, col, val, origin = _c_i32(rowoff), _c_i32(col), _c_f32(val), _c_i32(origin)
        H = _c_f32(H)
        n = len(rowoff) - 1
        K = H.shape[1]
        ref = np.zeros((n, K), np.float64)
        cond = np.zeros((n, K), np.float64)
        self.lib.oracle_spmm_mean_f64(n, rowoff, col, val, origin, H, K, ref, cond, n_threads)
        return ref, cond

    def capacity_from_s(self, s, costs):
        return self.lib.oracle_capacity_from_s(int(s), np.ascontiguousarray(costs, np.float64))

    def wave_based_s(self, nnz, compute_units, wave):
        return self.lib.oracle_wave_based_s(int(nnz), int(compute_units), int(wave))

    def recommended_w(self, nnz):
        out = np.zeros(3, np.int32)
        self.lib.oracle_recommended_w(int(nnz), out)
        return [int(x) for x in out]

    def features(self, rows, cols):
        out = np.zeros((rows, cols), np.float32)
        self.lib.oracle_features(rows, cols, out)
        return out


class ReferenceError_(RuntimeError):
    pass


class Reference:
    """The reference's own code (oracle/_ref/libcwlbref.so)."""

    ERRORS = {1: ValueError, 2: RuntimeError, 3: OverflowError, 4: RuntimeError}

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build with `make -C oracle ref`")
        lib = C.CDLL(path)
        lib.cwlbref_last_error.restype = C.c_char_p
        lib.cwlbref_set_device.argtypes = [C.c_long] * 4
        lib.cwlbref_sort_by_degree.argtypes = [C.c_int, C.c_int, _i32p, _i32p, _f32p, _i32p,
                                               _i32p, _i32p, _f32p]
        lib.cwlbref_partition.argtypes = [C.c_int, _i32p, _f64p, C.c_double,
                                          C.POINTER(C.c_int64)]
        lib.cwlbref_partition_fetch.argtypes = [_i32p]
        lib.cwlbref_spmm.argtypes = [C.c_int, C.c_int, C.c_int, _i32p, _i32p, _f32p, _i32p,
                                     _f32p, C.c_long, C.c_long, C.c_int, C.c_int, _i32p,
                                     C.c_long, _f32p, C.POINTER(C.c_double)]
        lib.cwlbref_capacity_from_s.argtypes = [C.c_int, _f64p]
        lib.cwlbref_capacity_from_s.restype = C.c_double
        lib.cwlbref_wave_based_s.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int,
                                             C.POINTER(C.c_int)]
        lib.cwlbref_recommended_w.argtypes = [C.c_uint64, _i32p]
        lib.cwlbref_search_bounds.argtypes = [_i32p, C.c_long, _i32p]
        lib.cwlbref_search_grid.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _i32p,
                                            C.c_int, C.POINTER(C.c_int)]
        lib.cwlbref_positive_search_argument.argtypes = [C.c_char_p, C.POINTER(C.c_int)]
        lib.cwlbref_features.argtypes = [C.c_int, C.c_int, _f32p]
        lib.cwlbref_save_costs.argtypes = [_f64p, C.c_char_p, C.c_int, C.c_int]
        lib.cwlbref_read_costs.argtypes = [_f64p, C.c_char_p]
        lib.cwlbref_load_csr.argtypes = [C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        lib.cwlbref_load_csr_fetch.argtypes = [_i32p, _i32p, _f32p]
        lib.cwlbref_validate.argtypes = [_f32p, _f32p, C.c_long, C.c_long, C.c_int, C.c_int,
                                         _i32p, _i32p, _f32p, _f32p, C.c_long, C.c_float]
        _v, _l = C.c_void_p, C.c_long
        lib.cwlbref_validate_shapes.argtypes = [_v, _l, _l, _v, _l, _l, _v, _l, _v, _l, _v, _v, _l,
                                                _l, C.c_float]
        lib.cwlbref_measure_costs.argtypes = [C.c_int] * 5 + [_f64p]
        lib.cwlbref_main.argtypes = [C.c_int, C.POINTER(C.c_char_p)]
        lib.cwlbref_costwrite_main.argtypes = [C.c_int, C.POINTER(C.c_char_p)]
        self.lib = lib

    def _check(self, rc):
        if rc:
            msg = self.lib.cwlbref_last_error().decode()
            raise self.ERRORS.get(rc, RuntimeError)(msg)

    def set_device(self, max_wg=1024, sub_group=32, local_mem=49152, compute_units=80):
        self.lib.cwlbref_set_device(max_wg, sub_group, local_mem, compute_units)

    def sort_by_degree(self, rowoff, col, val):
        rowoff, col, val = _c_i32(rowoff), _c_i32(col), _c_f32(val)
        n = len(rowoff) - 1
        origin = np.zeros(max(n, 0), np.int32)
        newoff = np.zeros(max(n + 1, 1), np.int32)
        newcol = np.zeros(len(col), np.int32)
        newval = np.zeros(len(val), np.float32)
        self._check(self.lib.cwlbref_sort_by_degree(n, len(col), rowoff, col, val, origin,
                                                    newoff, newcol, newval))
        return origin, newoff, newcol, newval

    def partition(self, rowoff, costs, capacity):
        rowoff = _c_i32(rowoff)
        cnt = C.c_int64()
        self._check(self.lib.cwlbref_partition(len(rowoff) - 1, rowoff,
                                               np.ascontiguousarray(costs, np.float64),
                                               float(capacity), C.byref(cnt)))
        out = np.zeros((max(cnt.value, 1), 4), np.int32)
        self.lib.cwlbref_partition_fetch(out)
        return out[:cnt.value]

    def spmm(self, rowoff, col, val, origin, H, tasks, large_k=False, dim_hint=None,
             local_dimension=None):
        rowoff, col, val, origin = _c_i32(rowoff), _c_i32(col), _c_f32(val), _c_i32(origin)
        H = _c_f32(H)
        tasks = _c_i32(np.asarray(tasks).reshape(-1, 4))
        n = len(origin)
        K = H.shape[1]
        out = np.zeros((n, K), np.float32)
        t = C.c_double()
        dh = K if dim_hint is None else dim_hint
        ld = K if local_dimension is None else local_dimension
        self._check(self.lib.cwlbref_spmm(int(large_k), n, len(col), rowoff, col, val, origin, H,
                                          H.shape[0], K, dh, ld,
                                          tasks.reshape(-1) if tasks.size else np.zeros(4, np.int32),
                                          len(tasks), out if out.size else np.zeros(1, np.float32),
                                          C.byref(t)))
        return out, t.value

    def capacity_from_s(self, s, costs):
        return self.lib.cwlbref_capacity_from_s(int(s), np.ascontiguousarray(costs, np.float64))

    def wave_based_s(self, rowoff, compute_units, wave):
        s = C.c_int()
        if rowoff is None:
            self._check(self.lib.cwlbref_wave_based_s(-1, None, compute_units, wave, C.byref(s)))
        else:
            r = _c_i32(rowoff)
            self._check(self.lib.cwlbref_wave_based_s(len(r) - 1, r.ctypes.data, compute_units,
                                                      wave, C.byref(s)))
        return s.value

    def recommended_w(self, nnz):
        out = np.zeros(3, np.int32)
        self.lib.cwlbref_recommended_w(int(nnz), out)
        return [int(x) for x in out]

    def search_bounds(self, values, best):
        out = np.zeros(2, np.int32)
        self._check(self.lib.cwlbref_search_bounds(_c_i32(values), int(best), out))
        return int(out[0]), int(out[1])

    def search_grid(self, lower, upper, arg, by_step=False):
        out = np.zeros(10001, np.int32)
        n = C.c_int()
        self._check(self.lib.cwlbref_search_grid(int(by_step), lower, upper, arg, out, len(out),
                                                 C.byref(n)))
        return [int(x) for x in out[:n.value]]

    def positive_search_argument(self, text):
        v = C.c_int()
        self._check(self.lib.cwlbref_positive_search_argument(text.encode(), C.byref(v)))
        return v.value

    def features(self, rows, cols):
        out = np.zeros((rows, cols), np.float32)
        self.lib.cwlbref_features(rows, cols, out if out.size else np.zeros(1, np.float32))
        return out

    def save_costs(self, costs, path, append=False, precision=6):
        return self.lib.cwlbref_save_costs(np.ascontiguousarray(costs, np.float64),
                                           path.encode(), int(append), precision) == 0

    def read_costs(self, path):
        out = np.zeros(4, np.float64)
        if self.lib.cwlbref_read_costs(out, path.encode()):
            return None
        return out

    def load_csr(self, name):
        V, E = C.c_int(), C.c_int()
        self._check(self.lib.cwlbref_load_csr(name.encode(), C.byref(V), C.byref(E)))
        rowoff = np.zeros(V.value + 1, np.int32)
        col = np.zeros(max(E.value, 1), np.int32)
        val = np.zeros(max(E.value, 1), np.float32)
        self.lib.cwlbref_load_csr_fetch(rowoff, col, val)
        return rowoff, col[:E.value], val[:E.value], V.value, E.value

    def validate(self, result, reference, rowoff, col, val, dense, abs_tol=1e-4):
        result, reference, dense = _c_f32(result), _c_f32(reference), _c_f32(dense)
        return bool(self.lib.cwlbref_validate(result, reference, result.shape[0],
                                              result.shape[1], len(rowoff) - 1, len(col),
                                              _c_i32(rowoff), _c_i32(col), _c_f32(val), dense,
                                              dense.shape[0], abs_tol))

    def validate_shapes(self, result, reference, rowoff, col, val, dense, abs_tol=1e-4):
        """validate_custom_csr_result with each matrix's own shape (2-D arrays)."""
        r, f, d = (np.ascontiguousarray(a, np.float32) for a in (result, reference, dense))
        ro, c = np.ascontiguousarray(rowoff, np.int32), np.ascontiguousarray(col, np.int32)
        v = np.ascontiguousarray(val, np.float32)
        p = lambda a: a.ctypes.data if a.size else None
        return bool(self.lib.cwlbref_validate_shapes(p(r), r.shape[0], r.shape[1], p(f),
                                                     f.shape[0], f.shape[1], p(ro), len(ro), p(c),
                                                     len(c), p(v), p(d), d.shape[0], d.shape[1],
                                                     float(abs_tol)))

    def main(self, argv):
        arr = (C.c_char_p * len(argv))(*[a.encode() for a in argv])
        return self.lib.cwlbref_main(len(argv), arr)
