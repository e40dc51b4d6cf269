#pragma once
// Mean-aggregation SpMM entry points (reference: include/parallelMatrix.h:13-32).
#include <vector>

#include "Matrix.h"
#include "config.h"
#include "cwlb_queue.h"
#include "utils.h"

// One task per work unit; returns the mean aggregation in ORIGINAL row order.
// `time` receives the device time of the aggregation kernels in microseconds
// (transfers excluded).  Throws std::invalid_argument for K > the device's
// max work-group size (use spmmKernelLargeKFallback).
Defined::RowMajorMatrixXf spmmKernel(cwlb::Queue& q, const CSR_Order& adjOrder,
                                     const Defined::RowMajorMatrixXf& H, int dim_hint,
                                     int local_dimension, std::vector<ParallelDataWeighted> tasks,
                                     double& time);

// Same contract for K above the device's max work-group size.
Defined::RowMajorMatrixXf spmmKernelLargeKFallback(cwlb::Queue& q, const CSR_Order& adjOrder,
                                                   const Defined::RowMajorMatrixXf& H,
                                                   int dim_hint, int local_dimension,
                                                   std::vector<ParallelDataWeighted> tasks,
                                                   double& time);

// Several GPUs of one node (no counterpart in the reference, which runs on one
// sycl::queue, main.cpp:514-516): the whole per-graph pipeline of the
// reference -- sortCSRByDegree, costWeightedTaskPartitioning at `capacity`,
// spmmKernel -- on every queue's GPU for a contiguous, cost-balanced block of
// ORIGINAL rows (cwlb_spmm_mean_multi; one host thread per queue, H
// replicated).  Takes the UNSORTED CSR; returns the mean aggregation in
// original row order.  `time` receives the largest per-GPU device time of the
// aggregation kernels in microseconds.  Each queue must be a different
// object, used by no other thread during the call.
Defined::RowMajorMatrixXf spmmKernelMultiGPU(const std::vector<cwlb::Queue*>& queues,
                                             const CSR& adj, const Defined::RowMajorMatrixXf& H,
                                             const SpmmCostParams& costs, double capacity,
                                             double& time);
