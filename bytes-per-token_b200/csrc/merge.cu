// merged[b, h, :] = sum_s softmax_s(lse[b, h, :]) * outs[b, h, s, :], the exact recombination of split
// partial attentions (kernels/reference.py:205-211); a row whose splits all have lse -inf (no tokens) merges to
// 0, as the reference's nan_to_num does, and a split of weight 0 is skipped (its partial is never read).
//
// merge_rows_kernel: one CTA per (sequence, query head). The splits' weights exp(lse - max) are formed once per
// split, 1,024 at a time, in shared memory; the threads then split the row's D values (four floats at a time)
// and its splits between them, each summing its own splits in order with the loads of several splits in flight,
// and the CTA adds the per-thread sums in a fixed order. A long context (hundreds of splits for a few rows) is
// then spread over a whole CTA per row rather than walked by one warp. merge_kernel (one warp per row) remains
// for rows wider than the CTA covers.
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

constexpr int kMergeThreads = 256;
constexpr int kMergeChunk = 1024;  // splits whose weights sit in shared memory at once

template <int ODT, int U>
__global__ void __launch_bounds__(kMergeThreads) merge_rows_kernel(const float* __restrict__ outs,
                                                                   const float* __restrict__ lses, int S, int D,
                                                                   void* __restrict__ merged) {
  __shared__ float w_s[kMergeChunk];
  __shared__ float red[kMergeThreads / 32];
  __shared__ float part[kMergeThreads * U];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  const float* l = lses + row * S;
  const float* o = outs + row * int64_t(S) * D;
  auto block_reduce = [&](float v, bool is_max) {
    v = is_max ? warp_max(v) : warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < kMergeThreads / 32; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
    __syncthreads();
    return r;
  };
  float mx = -CUDART_INF_F;
  for (int s = tid; s < S; s += kMergeThreads) mx = fmaxf(mx, l[s]);
  mx = block_reduce(mx, true);

  const int nd = D / U;                 // units (U floats) of a split's row; nd <= kMergeThreads
  const int lanes = kMergeThreads / nd;  // threads per unit, each taking every lanes-th split
  const int unit = tid % nd, sl = tid / nd;
  float acc[U];
#pragma unroll
  for (int u = 0; u < U; ++u) acc[u] = 0.f;
  float wpart = 0.f;
  for (int c0 = 0; c0 < S; c0 += kMergeChunk) {
    const int cn = min(kMergeChunk, S - c0);
    __syncthreads();  // the previous chunk's weights are consumed
    for (int i = tid; i < cn; i += kMergeThreads) {
      const float w = mx == -CUDART_INF_F ? 0.f : expf(l[c0 + i] - mx);
      w_s[i] = w;
      wpart += w;
    }
    __syncthreads();
    if (sl < lanes) {
#pragma unroll 4
      for (int i = sl; i < cn; i += lanes) {
        const float w = w_s[i];
        if (w != 0.f) {
          const float* src = o + int64_t(c0 + i) * D + unit * U;
          if constexpr (U == 4) {
            const float4 x = __ldcs(reinterpret_cast<const float4*>(src));
            acc[0] += w * x.x;
            acc[1] += w * x.y;
            acc[2] += w * x.z;
            acc[3] += w * x.w;
          } else {
            acc[0] += w * __ldcs(src);
          }
        }
      }
    }
  }
  const float wsum = block_reduce(wpart, false);
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
  for (int u = 0; u < U; ++u) part[tid * U + u] = acc[u];
  __syncthreads();
  for (int e = tid; e < D; e += kMergeThreads) {  // value e: unit e / U, element e % U, summed over the lanes in order
    const int un = e / U, el = e % U;
    float v = 0.f;
    for (int k = 0; k < lanes; ++k) v += part[(k * nd + un) * U + el];
    store_from_float<ODT>(merged, row * D + e, v * inv);
  }
}

template <int ODT>
void launch_merge(const float* outs, const float* lses, int64_t rows, int S, int D, void* merged, cudaStream_t s) {
  const bool vec4 = D % 4 == 0 && (reinterpret_cast<uintptr_t>(outs) & 15u) == 0;
  if (vec4 && D / 4 <= kMergeThreads) {
    merge_rows_kernel<ODT, 4><<<unsigned(rows), kMergeThreads, 0, s>>>(outs, lses, S, D, merged);
  } else if (!vec4 && D <= kMergeThreads) {
    merge_rows_kernel<ODT, 1><<<unsigned(rows), kMergeThreads, 0, s>>>(outs, lses, S, D, merged);
  } else {
    const int threads = 256;
    const int64_t blocks = (rows * 32 + threads - 1) / threads;
    merge_kernel<ODT><<<unsigned(blocks), threads, 0, s>>>(outs, lses, rows, S, D, merged);
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
  BPT_REQUIRE(rows < (1ll << 31) / 32, BPT_ERR_INVALID, "merge: too many rows");
  BPT_REQUIRE(S * D < (1ll << 40), BPT_ERR_INVALID, "merge: rows too long");
  auto s = static_cast<cudaStream_t>(stream);
  switch (out_dtype) {
    case BPT_DTYPE_F32: launch_merge<BPT_DTYPE_F32>(outs, lses, rows, int(S), int(D), merged, s); break;
    case BPT_DTYPE_F16: launch_merge<BPT_DTYPE_F16>(outs, lses, rows, int(S), int(D), merged, s); break;
    case BPT_DTYPE_BF16: launch_merge<BPT_DTYPE_BF16>(outs, lses, rows, int(S), int(D), merged, s); break;
    default:
      return set_error(BPT_ERR_INVALID, "merge: out dtype %d", out_dtype);
  }
  return check_launch("merge partials");
}
