// spmmKernel / spmmKernelLargeKFallback over libcwlb_spmm.
#include "parallelMatrix.h"

namespace {

Defined::RowMajorMatrixXf run(cwlb::Queue& q, bool large_k, const CSR_Order& a,
                              const Defined::RowMajorMatrixXf& H, int dim_hint,
                              int local_dimension, const std::vector<ParallelDataWeighted>& tasks,
                              double& time) {
    const long rows = static_cast<long>(a.Origin_local.size());
    Defined::RowMajorMatrixXf out(rows, H.cols());
    auto fn = large_k ? cwlb_spmm_kernel_large_k : cwlb_spmm_kernel;
    cwlb::check(fn(q.ctx(), static_cast<int32_t>(rows), static_cast<int32_t>(a.ColInd.size()),
                   a.RowOffset.data(), a.ColInd.data(), a.Value.data(), a.Origin_local.data(),
                   H.data(), H.rows(), H.cols(), dim_hint, local_dimension,
                   reinterpret_cast<const cwlb_task*>(tasks.data()),
                   static_cast<int64_t>(tasks.size()), out.data(), &time));
    return out;
}

}  // namespace

Defined::RowMajorMatrixXf spmmKernel(cwlb::Queue& q, const CSR_Order& adjOrder,
                                     const Defined::RowMajorMatrixXf& H, int dim_hint,
                                     int local_dimension, std::vector<ParallelDataWeighted> tasks,
                                     double& time) {
    return run(q, false, adjOrder, H, dim_hint, local_dimension, tasks, time);
}

Defined::RowMajorMatrixXf spmmKernelLargeKFallback(cwlb::Queue& q, const CSR_Order& adjOrder,
                                                   const Defined::RowMajorMatrixXf& H,
                                                   int dim_hint, int local_dimension,
                                                   std::vector<ParallelDataWeighted> tasks,
                                                   double& time) {
    return run(q, true, adjOrder, H, dim_hint, local_dimension, tasks, time);
}
