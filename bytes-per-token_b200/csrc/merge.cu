// merged[b, h, :] = sum_s softmax_s(lse[b, h, :]) * outs[b, h, s, :], the exact recombination of split
// partial attentions (kernels/reference.py:205-211). One warp per (sequence, query head); a row whose splits
// all have lse -inf (no tokens) merges to 0, as the reference's nan_to_num does.
#include <math_constants.h>

#include "common.cuh"

namespace bpt {
namespace {

template <int ODT>
__global__ void merge_kernel(const float* __restrict__ outs, const float* __restrict__ lses, int64_t rows, int S, int D,
                             void* __restrict__ merged) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  pdl_wait();
  const float* l = lses + row * S;
  float mx = -CUDART_INF_F;
  for (int s = lane; s < S; s += 32) mx = fmaxf(mx, l[s]);
  mx = warp_max(mx);
  float wsum = 0.f;
  for (int s = lane; s < S; s += 32) wsum += (mx == -CUDART_INF_F) ? 0.f : expf(l[s] - mx);
  wsum = warp_sum(wsum);
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
    if (mx != -CUDART_INF_F)
      for (int s = 0; s < S; ++s) acc += expf(l[s] - mx) * outs[(row * S + s) * D + d];
    store_from_float<ODT>(merged, row * D + d, acc * inv);
  }
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" int bpt_merge_partials(const float* outs, const float* lses, int64_t B, int64_t Hq, int64_t S, int64_t D,
                                  void* merged, int out_dtype, void* stream) {
  BPT_REQUIRE(outs && lses && merged, BPT_ERR_INVALID, "merge: null pointer");
  BPT_REQUIRE(B >= 0 && Hq >= 1 && S >= 1 && D >= 1 && S < (1 << 30) && D < (1 << 30), BPT_ERR_INVALID,
              "merge: bad shape");
  const int64_t rows = B * Hq;
  if (rows == 0) return BPT_OK;
  const int threads = 256;
  const int64_t blocks = (rows * 32 + threads - 1) / threads;
  BPT_REQUIRE(blocks < (1ll << 31), BPT_ERR_INVALID, "merge: too many rows");
  auto s = static_cast<cudaStream_t>(stream);
  switch (out_dtype) {
    case BPT_DTYPE_F32:
      merge_kernel<BPT_DTYPE_F32><<<unsigned(blocks), threads, 0, s>>>(outs, lses, rows, int(S), int(D), merged);
      break;
    case BPT_DTYPE_F16:
      merge_kernel<BPT_DTYPE_F16><<<unsigned(blocks), threads, 0, s>>>(outs, lses, rows, int(S), int(D), merged);
      break;
    case BPT_DTYPE_BF16:
      merge_kernel<BPT_DTYPE_BF16><<<unsigned(blocks), threads, 0, s>>>(outs, lses, rows, int(S), int(D), merged);
      break;
    default:
      return set_error(BPT_ERR_INVALID, "merge: out dtype %d", out_dtype);
  }
  return check_launch("merge partials");
}
