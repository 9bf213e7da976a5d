// Launch builders for the non-structured ops of a plan.  Each returns a
// closure that resolves device pointers from the runtime's buffers and
// enqueues one kernel.  Defined in runtime.cpp.
#pragma once

#include <functional>
#include <vector>

#include "../kernels/kernels.h"
#include "plan.h"

namespace gawee {

// B-operand packing source: element (b, k, n) of the logical [batch, K, N]
// operand (see kern::PackBParams).
struct PackSpec {
  View src;
  int64_t batch = 1, K = 0, N = 0;
  int64_t sn = 0;
  int64_t row_off = 0;  // first plane row written (several operands packed into one pair of planes)
  std::vector<int64_t> k_shape, k_st, k_valid;
  std::vector<int64_t> batch_shape, batch_st;
};

namespace launch {
using Fn = std::function<void(Runtime&, void*)>;
Fn remap(kern::RemapParams rp, const View& in, const View& out);
Fn nchw_to_nhwc4(const View& in, const View& out, int64_t N, int C, int C4, int64_t HW, int64_t in_sn, int64_t in_sc);
Fn reduce(const View& in, const View& out, const std::vector<bool>& red, bool mean, float count);
Fn generic_reduce(const View& in, const View& out, const std::vector<bool>& red, const EProgram& body);
Fn pool(kern::PoolParams pp, const View& in, const View& out);
Fn softmax(const View& in, const View& out, int axis);
Fn gather(const View& data, const View& idx, const View& out, int64_t pre, int64_t axis_len, int64_t nidx,
          int64_t post);
Fn gather_elements(const View& data, const View& idx, const View& out, int axis);
Fn range(kern::RangeParams rp, const View& out);
Fn topk(const View& in, const View& vals, const View& idxs, const View& used, int64_t k);
Fn pack(const PackSpec& ps, int64_t ldk, int hi, int lo);
// x, cs, sn: views over out's shape (broadcast strides 0); out dense
Fn rope(const View& x, const View& cs, const View& sn, const View& out);
// x: [rows][cols] with row stride x_rs (cols contiguous); w, b: per-column views (b.buf < 0: none)
Fn rownorm(const View& x, int64_t rows, int64_t cols, int64_t x_rs, const View& w, int64_t w_st, const View& b,
           int64_t b_st, const View& out, float eps, bool centered);
}  // namespace launch

}  // namespace gawee
