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
