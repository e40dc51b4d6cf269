"""Python binding of libcwlb_spmm (the C ABI in include/cwlb_spmm.h).

It mirrors the reference's C++ interface for the hot path, with the same
names, argument meaning and error behaviour:

  CSR, CSR_Order                       include/Matrix.h:15-36
  ParallelDataWeighted, SpmmCostParams include/utils.h:15-33
  sortCSRByDegree                      main.cpp:197-278 (sortCSRByDegreeDPLCPU), on the GPU
  costWeightedTaskPartitioning         src/utils.cpp:832-1021, on the GPU
  spmmKernel                           src/parallelMatrix.cpp:63-254
  spmmKernelLargeKFallback             src/parallelMatrix.cpp:264-683
  capacity_from_s, wave_based_s,
  recommended_candidate_w              main.cpp:87-95, 281-321
  save_costs_one_per_line,
  read_costs_one_per_line              src/utils.cpp:1024-1092

The reference's C++ exceptions map onto Python ones: std::invalid_argument ->
ValueError, std::runtime_error -> RuntimeError, std::overflow_error ->
OverflowError.  `sycl::queue&` becomes a Context (one CUDA device + stream).

There is no CPU fallback: importing this module fails if the shared library
has not been built, and creating a Context fails without a CUDA device.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libcwlb_spmm.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "cwlb_spmm.h")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C cwlb-spmm_b200` "
                      "(or __graft_entry__.build())")

_lib = C.CDLL(LIB_PATH)

OK, ERR_INVALID_ARGUMENT, ERR_RUNTIME, ERR_OVERFLOW, ERR_CUDA, ERR_NO_DEVICE, \
    ERR_BUFFER_TOO_SMALL, ERR_OUT_OF_MEMORY = range(8)
ROWS_COVERED = 1
DETERMINISTIC = 2
TASK_PER_WARP = 4
TASK_PER_CTA = 8
DEVERR_COL_RANGE, DEVERR_ROW_RANGE, DEVERR_OFFSETS, DEVERR_ORIGIN_RANGE = 1, 2, 4, 8


class NoDeviceError(RuntimeError):
    pass


class CudaError(RuntimeError):
    pass


_EXC = {ERR_INVALID_ARGUMENT: ValueError, ERR_RUNTIME: RuntimeError, ERR_OVERFLOW: OverflowError,
        ERR_CUDA: CudaError, ERR_NO_DEVICE: NoDeviceError, ERR_BUFFER_TOO_SMALL: BufferError,
        ERR_OUT_OF_MEMORY: MemoryError}


class cwlb_costs(C.Structure):
    _fields_ = [("C_compute_ns", C.c_double), ("C_load_ns", C.c_double),
                ("C_store_ns", C.c_double), ("C_atomic_ns", C.c_double),
                ("K", C.c_int32), ("WI", C.c_int32), ("repeat", C.c_int32),
                ("atomic_writers_per_addr", C.c_int32)]


_vp = C.c_void_p
_i32, _i64, _u32, _dbl = C.c_int32, C.c_int64, C.c_uint32, C.c_double


def _sig(name, args, res=C.c_int):
    fn = getattr(_lib, name)
    fn.argtypes = args
    fn.restype = res
    return fn


_sig("cwlb_last_error", [], C.c_char_p)
_sig("cwlb_version", [], C.c_char_p)
_sig("cwlb_ctx_create", [C.c_int, C.POINTER(_vp)])
_sig("cwlb_ctx_destroy", [_vp])
_sig("cwlb_ctx_set_stream", [_vp, _vp])
_sig("cwlb_ctx_stream", [_vp], _vp)
_sig("cwlb_ctx_synchronize", [_vp])
_sig("cwlb_ctx_take_device_errors", [_vp, C.POINTER(_u32)])
_sig("cwlb_device_info", [_vp, C.POINTER(_i64), C.POINTER(_i32), C.POINTER(_i64), C.c_char_p,
                          C.c_size_t])
_SPMM_ARGS = [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, _vp, _i64, _vp,
              C.POINTER(_dbl)]
_sig("cwlb_spmm_kernel", _SPMM_ARGS)
_sig("cwlb_spmm_kernel_large_k", _SPMM_ARGS)
_sig("cwlb_spmm_mean_device", [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _i64,
                               _vp, _u32])
_sig("cwlb_tasks_check", [_vp, _i32, _i32, _vp, _vp, _i64, C.POINTER(_i64), C.POINTER(_i64),
                          C.POINTER(_i64)])
_sig("cwlb_sort_by_degree", [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp])
_sig("cwlb_sort_by_degree_device", [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp])
_sig("cwlb_partition", [_vp, _i32, _vp, C.POINTER(cwlb_costs), _dbl, _vp, _i64, C.POINTER(_i64)])
_sig("cwlb_partition_device", [_vp, _i32, _vp, C.POINTER(cwlb_costs), _dbl, C.POINTER(_vp),
                               C.POINTER(_i64)])
_sig("cwlb_capacity_from_s", [_i32, C.POINTER(cwlb_costs)], _dbl)
_sig("cwlb_segment_size", [C.POINTER(cwlb_costs), _dbl], _i32)
_sig("cwlb_wave_based_s", [_i64, _i32, _i32, C.POINTER(_i32)])
_sig("cwlb_recommended_candidate_w", [C.c_uint64, C.POINTER(_i32)], None)
_sig("cwlb_save_costs", [C.POINTER(cwlb_costs), C.c_char_p, _i32, _i32])
_sig("cwlb_measure_spmm_costs", [_vp, _i32, _i32, _i32, _i32, _i32, C.POINTER(cwlb_costs)])
_sig("cwlb_measure_gather_gbs", [_vp, _i32, _i32, _i32, C.POINTER(C.c_double)])
_sig("cwlb_read_costs", [C.POINTER(cwlb_costs), C.c_char_p])
_sig("cwlb_save_costs_per_k", [C.POINTER(cwlb_costs), _i64, C.c_char_p])
_sig("cwlb_read_costs_per_k", [C.POINTER(cwlb_costs), _i64, C.c_char_p, C.POINTER(_i64)])
_sig("cwlb_costs_for_k", [C.POINTER(cwlb_costs), _i64, _i64], _i64)
_sig("cwlb_spmm_mean_reference_device", [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _vp])
_sig("cwlb_shard_bounds", [_i32, _vp, C.POINTER(cwlb_costs), _i32, _vp])
_sig("cwlb_shard_create", [_vp, _i32, _i32, _vp, _vp, _vp, C.POINTER(cwlb_costs), _dbl, _i32,
                           _i32, C.POINTER(_vp)])
_sig("cwlb_shard_create_device", [_vp, _i32, _i32, _vp, _vp, _vp, C.POINTER(cwlb_costs), _dbl,
                                  _i32, _i32, C.POINTER(_vp)])
_sig("cwlb_shard_create_cut", [_vp, _i32, _i32, _vp, _vp, _vp, C.POINTER(cwlb_costs), _dbl, _vp,
                               _i32, _i32, C.POINTER(_vp)])
_sig("cwlb_shard_bounds_rebalance", [_i32, _vp, C.POINTER(cwlb_costs), _i32, _vp, _vp, _vp])
_sig("cwlb_shard_create_device_cut", [_vp, _i32, _i32, _vp, _vp, _vp, C.POINTER(cwlb_costs),
                                      _dbl, _vp, _i32, _i32, C.POINTER(_vp)])
_sig("cwlb_shard_info", [_vp, C.POINTER(_i32), C.POINTER(_i32), C.POINTER(_i32), C.POINTER(_i64),
                         C.POINTER(_i32)])
_sig("cwlb_shard_tasks", [_vp, C.POINTER(_vp)])
_sig("cwlb_shard_aggregate_device", [_vp, _vp, _i64, _i64, _vp, _u32])
_sig("cwlb_shard_destroy", [_vp])
_sig("cwlb_spmm_mean_multi", [C.POINTER(_vp), _i32, _i32, _i32, _vp, _vp, _vp, _vp, _i64, _i64,
                              C.POINTER(cwlb_costs), _dbl, _vp, C.POINTER(_dbl)])
_sig("cwlb_gather_rows_multi", [C.POINTER(_vp), _i32, C.POINTER(_vp), _i64, _i64, _vp])
_sig("cwlb_plan_create", [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _i64, _i32, C.POINTER(_vp)])
_sig("cwlb_plan_info", [_vp, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i32),
                        C.POINTER(_u32)])
_sig("cwlb_plan_aggregate_device", [_vp, _vp, _vp, _i64, _i64, _vp, _u32])
_sig("cwlb_plan_destroy", [_vp])
_sig("cwlb_validate_result", [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _i64,
                              _i64, C.c_float, C.POINTER(_i32)])


def _check(rc):
    if rc != OK:
        msg = _lib.cwlb_last_error().decode()
        raise _EXC.get(rc, RuntimeError)(msg)


def header_functions(path: str = HEADER_PATH):
    """Names of the functions include/cwlb_spmm.h declares."""
    with open(path) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cwlb_[a-z0-9_]+)\s*\(", text)))


def version() -> str:
    return _lib.cwlb_version().decode()


# ---------------------------------------------------------------------------
# data structures (include/Matrix.h, include/utils.h)

@dataclass
class CSR:
    RowOffset: np.ndarray
    ColInd: np.ndarray
    Value: np.ndarray

    def __post_init__(self):
        self.RowOffset = np.ascontiguousarray(self.RowOffset, np.int32)
        self.ColInd = np.ascontiguousarray(self.ColInd, np.int32)
        self.Value = np.ascontiguousarray(self.Value, np.float32)

    @property
    def rows(self) -> int:
        return max(len(self.RowOffset) - 1, 0)

    @property
    def nnz(self) -> int:
        return len(self.ColInd)


@dataclass
class CSR_Order(CSR):
    Origin_local: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))

    def __post_init__(self):
        super().__post_init__()
        self.Origin_local = np.ascontiguousarray(self.Origin_local, np.int32)


TASK_DTYPE = np.dtype([("row_start", np.int32), ("row_end", np.int32),
                       ("first_row_offset", np.int32), ("last_row_nnz", np.int32)])


@dataclass
class SpmmCostParams:
    C_compute_ns: float = 0.0
    C_load_ns: float = 0.0
    C_store_ns: float = 0.0
    C_atomic_ns: float = 0.0
    K: int = 0
    WI: int = 0
    repeat: int = 0
    atomic_writers_per_addr: int = 0

    def c(self) -> cwlb_costs:
        return cwlb_costs(self.C_compute_ns, self.C_load_ns, self.C_store_ns, self.C_atomic_ns,
                          self.K, self.WI, self.repeat, self.atomic_writers_per_addr)

    @classmethod
    def from_list(cls, v):
        return cls(float(v[0]), float(v[1]), float(v[2]), float(v[3]))


def _tasks_i32(tasks) -> np.ndarray:
    t = np.asarray(tasks)
    if t.dtype == TASK_DTYPE:
        t = t.view(np.int32)
    return np.ascontiguousarray(t, np.int32).reshape(-1, 4)


def _p(a: np.ndarray):
    return a.ctypes.data if a.size else None


# ---------------------------------------------------------------------------
# context

class Context:
    """One CUDA device and stream (replaces the reference's sycl::queue)."""

    def __init__(self, device: int = 0):
        h = _vp()
        _check(_lib.cwlb_ctx_create(device, C.byref(h)))
        self._h = h
        self.device = device

    def close(self):
        if getattr(self, "_h", None):
            _lib.cwlb_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self):
        return self._h

    def set_stream(self, cuda_stream: int):
        _check(_lib.cwlb_ctx_set_stream(self._h, _vp(cuda_stream)))

    def synchronize(self):
        _check(_lib.cwlb_ctx_synchronize(self._h))

    def take_device_errors(self) -> int:
        f = _u32()
        _check(_lib.cwlb_ctx_take_device_errors(self._h, C.byref(f)))
        return f.value

    def device_info(self) -> dict:
        mwg, cu, lm = _i64(), _i32(), _i64()
        name = C.create_string_buffer(256)
        _check(_lib.cwlb_device_info(self._h, C.byref(mwg), C.byref(cu), C.byref(lm), name, 256))
        return dict(max_work_group_size=mwg.value, max_compute_units=cu.value,
                    local_mem_size=lm.value, name=name.value.decode())

    # ---- host-buffer entry points (synchronous) --------------------------

    def _spmm(self, fn, adj: CSR_Order, H, dim_hint, local_dimension, tasks, out=None):
        H = np.ascontiguousarray(H, np.float32)
        t = _tasks_i32(tasks)
        n = len(adj.Origin_local)
        K = H.shape[1] if H.ndim == 2 else 0
        if out is None:
            out = np.zeros((n, K), np.float32)
        elif out.shape != (n, K) or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError("out must be a C-contiguous float32 (rows, K) array")
        tm = _dbl()
        _check(fn(self._h, n, adj.nnz, _p(adj.RowOffset), _p(adj.ColInd), _p(adj.Value),
                  _p(adj.Origin_local), _p(H), H.shape[0], K, dim_hint, local_dimension, _p(t),
                  len(t), _p(out), C.byref(tm)))
        return out, tm.value

    def spmmKernel(self, adjOrder: CSR_Order, H, dim_hint, local_dimension, tasks, out=None):
        """spmmKernel (include/parallelMatrix.h:13-20): returns (out, time_us).
        `out` optionally supplies the (rows, K) float32 result buffer (e.g.
        pinned host memory); by default a fresh array is returned, as the
        reference returns a fresh matrix."""
        return self._spmm(_lib.cwlb_spmm_kernel, adjOrder, H, dim_hint, local_dimension, tasks,
                          out)

    def spmmKernelLargeKFallback(self, adjOrder: CSR_Order, H, dim_hint, local_dimension, tasks,
                                 out=None):
        """spmmKernelLargeKFallback (include/parallelMatrix.h:25-32)."""
        return self._spmm(_lib.cwlb_spmm_kernel_large_k, adjOrder, H, dim_hint, local_dimension,
                          tasks, out)

    def sortCSRByDegree(self, csr: CSR) -> CSR_Order:
        """sortCSRByDegreeDPLCPU (main.cpp:197-278) computed on the GPU."""
        n = csr.rows
        if len(csr.ColInd) != len(csr.Value):
            raise RuntimeError("CSR ColInd and Value size mismatch.")
        if n == 0:
            return CSR_Order(np.zeros(0, np.int32), np.zeros(0, np.int32),
                             np.zeros(0, np.float32), np.zeros(0, np.int32))
        origin = np.zeros(n, np.int32)
        ro = np.zeros(n + 1, np.int32)
        col = np.zeros(csr.nnz, np.int32)
        val = np.zeros(csr.nnz, np.float32)
        _check(_lib.cwlb_sort_by_degree(self._h, n, csr.nnz, _p(csr.RowOffset), _p(csr.ColInd),
                                        _p(csr.Value), _p(origin), _p(ro), _p(col), _p(val)))
        return CSR_Order(ro, col, val, origin)

    def costWeightedTaskPartitioning(self, csr: CSR, costs: SpmmCostParams,
                                     capacity_weight: float) -> np.ndarray:
        """costWeightedTaskPartitioning (src/utils.cpp:832-1021) on the GPU.
        Returns an (n_tasks, 4) int32 array of ParallelDataWeighted."""
        n = csr.rows
        c = costs.c()
        cnt = _i64()
        _check(_lib.cwlb_partition(self._h, n, _p(csr.RowOffset), C.byref(c),
                                   float(capacity_weight), None, 0, C.byref(cnt)))
        out = np.zeros((max(cnt.value, 0), 4), np.int32)
        if cnt.value:
            # The first call left the task list on the device; the second call
            # recomputes it and copies it out.
            _check(_lib.cwlb_partition(self._h, n, _p(csr.RowOffset), C.byref(c),
                                       float(capacity_weight), _p(out), cnt.value, C.byref(cnt)))
        return out

    def measure_spmm_costs(self, K=128, repeat=500, WI=131072, data_MB_for_load=512,
                           atomic_target_writers=8) -> "SpmmCostParams":
        """measure_spmm_costs (include/utils.h:47-54): the costWrite calibration."""
        c = cwlb_costs()
        _check(_lib.cwlb_measure_spmm_costs(self._h, K, repeat, WI, data_MB_for_load,
                                            atomic_target_writers, C.byref(c)))
        return SpmmCostParams(c.C_compute_ns, c.C_load_ns, c.C_store_ns, c.C_atomic_ns, c.K,
                              c.WI, c.repeat, c.atomic_writers_per_addr)

    def measure_gather_gbs(self, buffer_MB=48, row_floats=128, repeat=20) -> float:
        """Rate in GB/s of gathering uniformly random rows of row_floats floats
        from a buffer_MB MiB device buffer: the ceiling for rows served from L2
        when the buffer fits in L2, from HBM when it is far larger."""
        g = _dbl()
        _check(_lib.cwlb_measure_gather_gbs(self._h, buffer_MB, row_floats, repeat, C.byref(g)))
        return g.value

    # ---- device-pointer entry points (asynchronous on the context stream) --

    def sort_by_degree_device(self, n_rows, nnz, d_rowoff, d_col, d_val, d_origin, d_new_rowoff,
                              d_new_col, d_new_val):
        _check(_lib.cwlb_sort_by_degree_device(self._h, n_rows, nnz, d_rowoff, d_col, d_val,
                                               d_origin, d_new_rowoff, d_new_col, d_new_val))

    def partition_device(self, n_rows, d_rowoff, costs: SpmmCostParams, capacity):
        """Returns (device pointer to the tasks, n_tasks); the tasks live in
        context memory until the next partition call."""
        ptr, cnt = _vp(), _i64()
        c = costs.c()
        _check(_lib.cwlb_partition_device(self._h, n_rows, d_rowoff, C.byref(c), float(capacity),
                                          C.byref(ptr), C.byref(cnt)))
        return ptr.value, cnt.value

    def spmm_mean_device(self, n_rows, nnz, d_rowoff, d_col, d_val, d_origin, d_H, h_rows, K,
                         d_tasks, n_tasks, d_out, flags=0):
        _check(_lib.cwlb_spmm_mean_device(self._h, n_rows, nnz, d_rowoff, d_col, d_val, d_origin,
                                          d_H, h_rows, K, d_tasks, n_tasks, d_out, flags))

    def spmm_mean_reference_device(self, n_rows, nnz, d_rowoff, d_col, d_val, d_H, h_rows, K,
                                   d_out):
        """Float64 reference aggregation over an unsorted CSR (original row order)."""
        _check(_lib.cwlb_spmm_mean_reference_device(self._h, n_rows, nnz, d_rowoff, d_col, d_val,
                                                    d_H, h_rows, K, d_out))

    def tasks_check(self, n_rows, nnz, d_rowoff, d_tasks, n_tasks):
        bad, unc, nz = _i64(), _i64(), _i64()
        _check(_lib.cwlb_tasks_check(self._h, n_rows, nnz, d_rowoff, d_tasks, n_tasks,
                                     C.byref(bad), C.byref(unc), C.byref(nz)))
        return dict(bad_tasks=bad.value, uncovered_rows=unc.value, nnz_coverage_errors=nz.value)


# ---------------------------------------------------------------------------
# aggregation plans (a task list prepared once for many launches)

PLAN_DISABLED, PLAN_FEW_FRAGMENTS, PLAN_VALUES, PLAN_UNSORTED, PLAN_NO_REUSE = 1, 2, 4, 8, 16


class Plan:
    """cwlb_plan: a reordered CSR's task list prepared once (single-row
    fragment tasks of neighbouring rows grouped, their column unions merged)
    for repeated aggregations.  The device pointers passed in must stay valid
    and unchanged while the plan lives."""

    def __init__(self, ctx: "Context", n_rows, nnz, d_rowoff, d_col, d_val, d_tasks, n_tasks,
                 group_size=0):
        h = _vp()
        _check(_lib.cwlb_plan_create(ctx.handle, n_rows, nnz, d_rowoff, d_col, d_val, d_tasks,
                                     n_tasks, group_size, C.byref(h)))
        self._h = h
        self.ctx = ctx

    def info(self) -> dict:
        gt, gn, ue, gs, why = _i64(), _i64(), _i64(), _i32(), _u32()
        _check(_lib.cwlb_plan_info(self._h, C.byref(gt), C.byref(gn), C.byref(ue), C.byref(gs),
                                   C.byref(why)))
        return dict(grouped_tasks=gt.value, grouped_nnz=gn.value, union_entries=ue.value,
                    group_size=gs.value, off_reason=why.value)

    def aggregate_device(self, d_origin, d_H, h_rows, K, d_out, flags=0):
        """One aggregation (cwlb_spmm_mean_device's flags), asynchronous on
        the context's stream."""
        _check(_lib.cwlb_plan_aggregate_device(self._h, d_origin, d_H, h_rows, K, d_out, flags))

    def close(self):
        if getattr(self, "_h", None):
            _lib.cwlb_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# several GPUs of one node (no counterpart in the reference, which runs on one
# sycl::queue, main.cpp:514-516)

def shard_bounds(row_offset, costs: SpmmCostParams, n_shards: int) -> np.ndarray:
    """Cut points of the cost-balanced contiguous row shards (n_shards + 1
    ints): shard s = original rows [b[s], b[s+1]), equal summed whole-row
    weight (Cc + Cl) * deg + Cs (src/utils.cpp:850-852).  Host code."""
    ro = np.ascontiguousarray(row_offset, np.int32)
    n = max(len(ro) - 1, 0)
    b = np.zeros(n_shards + 1, np.int32)
    c = costs.c()
    _check(_lib.cwlb_shard_bounds(n, _p(ro), C.byref(c), n_shards, _p(b)))
    return b


def shard_bounds_rebalance(row_offset, costs: SpmmCostParams, bounds, shard_time) -> np.ndarray:
    """The cut of shard_bounds re-weighted by measured shard times: every row
    of shard g under `bounds` weighs its whole-row weight times
    shard_time[g] / (the shard's summed weight).  Host code."""
    ro = np.ascontiguousarray(row_offset, np.int32)
    n = max(len(ro) - 1, 0)
    b = np.ascontiguousarray(bounds, np.int32)
    t = np.ascontiguousarray(shard_time, np.float64)
    G = len(b) - 1
    if G < 1 or len(t) != G:
        raise ValueError("need n_shards + 1 bounds and n_shards times")
    nb = np.zeros(G + 1, np.int32)
    c = costs.c()
    _check(_lib.cwlb_shard_bounds_rebalance(n, _p(ro), C.byref(c), G, _p(b), _p(t), _p(nb)))
    return nb


class Shard:
    """One GPU's resident share of a multi-GPU aggregation: original rows
    [row_begin, row_end) sorted by degree and partitioned on that GPU."""

    def __init__(self, ctx: "Context", handle):
        self.ctx = ctx
        self._h = handle
        rb, re_, nz, nt, seg = _i32(), _i32(), _i32(), _i64(), _i32()
        _check(_lib.cwlb_shard_info(self._h, C.byref(rb), C.byref(re_), C.byref(nz), C.byref(nt),
                                    C.byref(seg)))
        self.row_begin, self.row_end, self.nnz = rb.value, re_.value, nz.value
        self.n_tasks, self.segment_size = nt.value, seg.value

    @classmethod
    def from_host(cls, ctx: "Context", csr: CSR, costs: SpmmCostParams, capacity: float,
                  shard: int, n_shards: int, cut=None) -> "Shard":
        """cut: n_shards + 1 cut points (e.g. from shard_bounds_rebalance);
        None cuts as shard_bounds."""
        h = _vp()
        c = costs.c()
        cb = None
        if cut is not None:
            cb = np.ascontiguousarray(cut, np.int32)
            if len(cb) != n_shards + 1:
                raise ValueError("cut needs n_shards + 1 entries")
        _check(_lib.cwlb_shard_create_cut(ctx.handle, csr.rows, csr.nnz, _p(csr.RowOffset),
                                          _p(csr.ColInd), _p(csr.Value), C.byref(c),
                                          float(capacity), None if cb is None else _p(cb),
                                          shard, n_shards, C.byref(h)))
        return cls(ctx, h)

    @classmethod
    def from_device(cls, ctx: "Context", n_rows, nnz, d_rowoff, d_col, d_val,
                    costs: SpmmCostParams, capacity: float, shard: int, n_shards: int,
                    cut=None) -> "Shard":
        """cut: n_shards + 1 cut points (e.g. from shard_bounds_rebalance);
        None cuts as shard_bounds."""
        h = _vp()
        c = costs.c()
        if cut is None:
            _check(_lib.cwlb_shard_create_device(ctx.handle, n_rows, nnz, d_rowoff, d_col, d_val,
                                                 C.byref(c), float(capacity), shard, n_shards,
                                                 C.byref(h)))
        else:
            cb = np.ascontiguousarray(cut, np.int32)
            if len(cb) != n_shards + 1:
                raise ValueError("cut needs n_shards + 1 entries")
            _check(_lib.cwlb_shard_create_device_cut(ctx.handle, n_rows, nnz, d_rowoff, d_col,
                                                     d_val, C.byref(c), float(capacity), _p(cb),
                                                     shard, n_shards, C.byref(h)))
        return cls(ctx, h)

    @property
    def rows(self) -> int:
        return self.row_end - self.row_begin

    def tasks_ptr(self) -> int:
        p = _vp()
        _check(_lib.cwlb_shard_tasks(self._h, C.byref(p)))
        return p.value or 0

    def aggregate_device(self, d_H, h_rows, K, d_out, flags=0):
        """Rows [row_begin, row_end) of the mean aggregation into d_out
        ((rows, K), device memory); asynchronous on the context's stream."""
        _check(_lib.cwlb_shard_aggregate_device(self._h, d_H, h_rows, K, d_out, flags))

    def close(self):
        if getattr(self, "_h", None):
            _lib.cwlb_shard_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def spmm_mean_multi(ctxs, csr: CSR, H, costs: SpmmCostParams, capacity: float, out=None):
    """The whole pipeline (sort -> partition -> aggregation) over the GPUs of
    `ctxs`, one host thread each, from an UNSORTED host CSR and host H to the
    (rows, K) output in ORIGINAL row order.  Returns (out, time_us), time_us
    the largest per-GPU device time of the aggregation."""
    H = np.ascontiguousarray(H, np.float32)
    K = H.shape[1] if H.ndim == 2 else 0
    n = csr.rows
    if out is None:
        out = np.zeros((n, K), np.float32)
    elif out.shape != (n, K) or out.dtype != np.float32 or not out.flags.c_contiguous:
        raise ValueError("out must be a C-contiguous float32 (rows, K) array")
    arr = (_vp * len(ctxs))(*[c.handle for c in ctxs])
    tm = _dbl()
    c = costs.c()
    _check(_lib.cwlb_spmm_mean_multi(arr, len(ctxs), n, csr.nnz, _p(csr.RowOffset),
                                     _p(csr.ColInd), _p(csr.Value), _p(H), H.shape[0], K,
                                     C.byref(c), float(capacity), _p(out), C.byref(tm)))
    return out, tm.value


def gather_rows_multi(ctxs, d_ptrs, rows: int, K: int, bounds):
    """All-gather of a row-sharded (rows, K) float32 matrix over the contexts'
    GPUs by peer copies; d_ptrs[g] holds rows [bounds[g], bounds[g+1])."""
    b = np.ascontiguousarray(bounds, np.int32)
    arr = (_vp * len(ctxs))(*[c.handle for c in ctxs])
    ptrs = (_vp * len(d_ptrs))(*d_ptrs)
    _check(_lib.cwlb_gather_rows_multi(arr, len(ctxs), ptrs, rows, K, _p(b)))


# ---------------------------------------------------------------------------
# host helpers (main.cpp, src/utils.cpp)

def capacity_from_s(s: int, costs: SpmmCostParams) -> float:
    c = costs.c()
    return _lib.cwlb_capacity_from_s(int(s), C.byref(c))


def segment_size(costs: SpmmCostParams, capacity: float) -> int:
    c = costs.c()
    return _lib.cwlb_segment_size(C.byref(c), float(capacity))


def wave_based_s(nnz: int, compute_units: int, wave: int) -> int:
    s = _i32()
    _check(_lib.cwlb_wave_based_s(int(nnz), int(compute_units), int(wave), C.byref(s)))
    return s.value


def recommended_candidate_w(nnz: int):
    out = (_i32 * 3)()
    _lib.cwlb_recommended_candidate_w(int(nnz), out)
    return [int(x) for x in out]


def validate_custom_csr_result(result, reference, csr: CSR, dense_matrix,
                               abs_tolerance: float = 1e-4) -> bool:
    """validate_custom_csr_result (src/utils.cpp:1117-1265): element-wise check
    of `result` against `reference`, printing the reference's report on the
    process's stdout/stderr.  Host only."""
    r = np.ascontiguousarray(result, np.float32)
    f = np.ascontiguousarray(reference, np.float32)
    d = np.ascontiguousarray(dense_matrix, np.float32)
    r2, f2, d2 = (a if a.ndim == 2 else a.reshape(-1, 1) for a in (r, f, d))
    passed = _i32()
    _check(_lib.cwlb_validate_result(_p(r2), r2.shape[0], r2.shape[1], _p(f2), f2.shape[0],
                                     f2.shape[1], _p(csr.RowOffset), len(csr.RowOffset),
                                     _p(csr.ColInd), _p(csr.Value), _p(d2), d2.shape[0],
                                     d2.shape[1], float(abs_tolerance), C.byref(passed)))
    return passed.value != 0


CSR_CACHE_MAGIC = b"CWLBCSR1"


def read_csr_cache(text_path: str):
    """Reads the binary cache the C++ loader writes beside a text CSR
    ("<file>.csr.cwlbbin": 64-byte header, int32 RowOffset[V+1], int32
    ColInd[E]; values 1.0f).  Returns a CSR, or None when the cache is
    missing, stale (the text file's size or modification time changed) or
    corrupt."""
    import os
    path = text_path + ".cwlbbin"
    try:
        st = os.stat(text_path)
        with open(path, "rb") as f:
            raw = f.read()
    except OSError:
        return None
    if len(raw) < 64 or raw[:8] != CSR_CACHE_MAGIC:
        return None
    ver, hdr = np.frombuffer(raw, "<u4", 2, 8)
    size, mtime, rows, nnz, checksum = (np.frombuffer(raw, "<u8", 1, 16)[0],
                                        *np.frombuffer(raw, "<i8", 3, 24),
                                        np.frombuffer(raw, "<u8", 1, 48)[0])
    if (ver != 1 or hdr != 64 or size != st.st_size or mtime != st.st_mtime_ns or rows < 0 or
            nnz < 0 or len(raw) != 64 + 4 * (rows + 1) + 4 * nnz):
        return None
    words = np.frombuffer(raw, "<u4", (len(raw) - 64) // 4, 64)
    h = 1469598103934665603
    for w in words.tolist():
        h = ((h ^ w) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    if h != int(checksum):
        return None
    ro = words[:rows + 1].view("<i4")
    col = words[rows + 1:].view("<i4")
    return CSR(ro, col, np.ones(nnz, np.float32))


def save_costs_one_per_line(costs: SpmmCostParams, filepath: str, append: bool = False,
                            precision: int = 6) -> bool:
    c = costs.c()
    return _lib.cwlb_save_costs(C.byref(c), filepath.encode(), int(append), precision) == OK


def read_costs_one_per_line(filepath: str):
    c = cwlb_costs()
    if _lib.cwlb_read_costs(C.byref(c), filepath.encode()) != OK:
        return None
    return SpmmCostParams(c.C_compute_ns, c.C_load_ns, c.C_store_ns, c.C_atomic_ns)


def save_costs_per_k(table, filepath: str) -> bool:
    """Per-K cost table (costWrite --per-k): one line per entry, K then the
    four costs; every entry needs a positive K."""
    arr = (cwlb_costs * max(len(table), 1))(*[t.c() for t in table])
    return _lib.cwlb_save_costs_per_k(arr, len(table), filepath.encode()) == OK


def read_costs_per_k(filepath: str):
    """The per-K table as a list of SpmmCostParams (K set), or None."""
    n = _i64()
    if _lib.cwlb_read_costs_per_k(None, 0, filepath.encode(), C.byref(n)) != OK:
        return None
    arr = (cwlb_costs * max(n.value, 1))()
    if n.value and _lib.cwlb_read_costs_per_k(arr, n.value, filepath.encode(), C.byref(n)) != OK:
        return None
    return [SpmmCostParams(a.C_compute_ns, a.C_load_ns, a.C_store_ns, a.C_atomic_ns, a.K)
            for a in arr[:n.value]]


def costs_for_k(table, K: int) -> SpmmCostParams:
    """The entry calibrated at the row width nearest to K on a log scale
    (ties go to the larger width)."""
    arr = (cwlb_costs * max(len(table), 1))(*[t.c() for t in table])
    i = _lib.cwlb_costs_for_k(arr, len(table), int(K))
    if i < 0:
        raise ValueError("no per-K cost entry for this K")
    return table[i]
