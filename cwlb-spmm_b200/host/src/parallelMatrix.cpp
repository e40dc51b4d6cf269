// spmmKernel / spmmKernelLargeKFallback over libcwlb_spmm.
#include "parallelMatrix.h"

#include <stdexcept>

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

Defined::RowMajorMatrixXf spmmKernelMultiGPU(const std::vector<cwlb::Queue*>& queues,
                                             const CSR& adj, const Defined::RowMajorMatrixXf& H,
                                             const SpmmCostParams& costs, double capacity,
                                             double& time) {
    std::vector<cwlb_ctx*> ctxs;
    for (cwlb::Queue* q : queues) {
        if (!q) throw std::invalid_argument("spmmKernelMultiGPU: null queue");
        ctxs.push_back(q->ctx());
    }
    const long rows = adj.RowOffset.empty() ? 0 : static_cast<long>(adj.RowOffset.size()) - 1;
    Defined::RowMajorMatrixXf out(rows, H.cols());
    const cwlb_costs c{costs.C_compute_ns, costs.C_load_ns, costs.C_store_ns, costs.C_atomic_ns,
                       costs.K, costs.WI, costs.repeat, costs.atomic_writers_per_addr};
    const int32_t zero = 0;
    cwlb::check(cwlb_spmm_mean_multi(ctxs.data(), static_cast<int32_t>(ctxs.size()),
                                     static_cast<int32_t>(rows),
                                     static_cast<int32_t>(adj.ColInd.size()),
                                     adj.RowOffset.empty() ? &zero : adj.RowOffset.data(),
                                     adj.ColInd.data(), adj.Value.data(), H.data(), H.rows(),
                                     H.cols(), &c, capacity, out.data(), &time));
    return out;
}
