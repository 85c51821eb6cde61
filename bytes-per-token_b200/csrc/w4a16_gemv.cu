// W4A16 linear for small M (decode): y[M, N] = x[M, K] . (scale * (q - zero))^T on CUDA cores.
//
// Memory path. Each CTA owns a contiguous slab of weight rows; its whole slab ((rows x K/2) bytes, contiguous
// in the [N, K/8] int32 layout) is requested at once with cp.async.bulk (the TMA engine), split over up to
// eight mbarriers so compute starts on the first rows while the rest stream in. The weight copies do not
// depend on the previous kernel, so they are issued before griddepcontrol.wait: under programmatic dependent
// launch they overlap the previous kernel's tail, and only the activations wait for it.
//
// Compute. A warp owns a 1024-input slice of K (one 16-byte chunk = 32 codes per lane) and walks the slab's
// rows; the lane keeps its 32 activations in registers as fp32 pairs. Eight codes of one int32 word become
// four bf16 pairs with one shift and one LOP3 each, (w >> 4i) & 0x000F000F | 0x43004300 = bf16 (128 + q_i,
// 128 + q_{i+4}) exactly, widened to fp32 by a shift or a mask. The chunk's dot product is accumulated with
// packed fp32x2 FMAs against those offset codes, and the grid is applied once per chunk (a chunk never spans
// two groups):  sum_k x_k * s * (q_k - z) = s * (sum_k x_k * (128 + q_k) - (128 + z) * sum_k x_k).
// Lanes reduce with shuffles; slices (and, fused, the gate/up row pair) combine in shared memory in a fixed
// order, so results are deterministic.
#include <cstdlib>

#include "common.cuh"

namespace bpt {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxChunks = 8;
constexpr int kSlabBudget = 96 * 1024;  // two CTAs per SM

struct GemvArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  const uint8_t* qweight;  // [N, K/2] bytes
  const __half* scales;    // [N, G]
  const uint32_t* qzeros;  // [N, ZW] or null
  __nv_bfloat16* y;
  int64_t ldy;
  int M, N, K, group, G, ZW;
  int rows_per_cta;  // even when fused
  int S;             // 1024-input slices
  int RW;            // row slots: warps / S
  int slab_bytes;    // rows_per_cta * K/2, rounded up to 128
};

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

template <int MT, bool FUSED>
__global__ void __launch_bounds__(kThreads) w4a16_gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * a.rows_per_cta;
  const int rows = min(a.rows_per_cta, a.N - row0);
  const int m0 = blockIdx.y * MT;
  const int mt = min(MT, a.M - m0);
  const int row_bytes = a.K >> 1;

  uint8_t* slab = smem;
  float* red = reinterpret_cast<float*>(smem + a.slab_bytes);  // [rows_per_cta][S][MT]
  // mbarriers need 8-byte alignment: round the offset after the reduction buffer up to 16 bytes
  const int bar_off = (a.slab_bytes + a.rows_per_cta * a.S * MT * int(sizeof(float)) + 15) & ~15;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + bar_off);
  const int rows_per_chunk = (rows + kMaxChunks - 1) / kMaxChunks;
  const int n_chunks = (rows + rows_per_chunk - 1) / rows_per_chunk;  // every chunk holds at least one row

  if (tid == 0) {
    for (int c = 0; c < n_chunks; ++c) mbar_init(&bars[c], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint64_t policy = l2_policy_evict_first();
    for (int c = 0; c < n_chunks; ++c) {
      const int rb = c * rows_per_chunk;
      const int re = min(rows, rb + rows_per_chunk);
      const uint32_t bytes = uint32_t(re - rb) * uint32_t(row_bytes);
      mbar_arrive_expect_tx(&bars[c], bytes);
      bulk_g2s_evict_first(slab + size_t(rb) * row_bytes, a.qweight + (size_t(row0) + rb) * row_bytes, bytes,
                           &bars[c], policy);
    }
  }
  pdl_launch_dependents();
  pdl_wait();  // the activations (and the output buffer) belong to the previous kernel until here

  const int slice = warp % a.S;
  const int rslot = warp / a.S;
  const int nwarp_used = a.S * a.RW;
  const int chunk = slice * 32 + lane;
  const bool active = (warp < nwarp_used) && (chunk < (a.K >> 5));

  float2 xp[MT][16];
  float xs[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    xs[m] = 0.f;
#pragma unroll
    for (int p = 0; p < 16; ++p) xp[m][p] = make_float2(0.f, 0.f);
    if (active && m < mt) {
      const uint4* src = reinterpret_cast<const uint4*>(a.x + (int64_t)(m0 + m) * a.ldx + chunk * 32);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = src[j];  // 8 bf16: inputs 8j .. 8j+7 of the chunk
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        float f[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          f[2 * e] = bf16_bits_to_float(w[e] & 0xFFFFu);
          f[2 * e + 1] = bf16_bits_to_float(w[e] >> 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) xp[m][4 * j + i] = make_float2(f[i], f[i + 4]);
#pragma unroll
        for (int e = 0; e < 8; ++e) xs[m] += f[e];
      }
    }
  }

  if (warp < nwarp_used) {
    for (int r = rslot; r < rows; r += a.RW) {
      const int c_id = r / rows_per_chunk;
      if (!mbar_wait_warp(&bars[c_id], 0)) break;  // recorded; the drain below bounds the exit
      float part[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) part[m] = 0.f;
      if (active) {
        const uint4 wq = *reinterpret_cast<const uint4*>(slab + size_t(r) * row_bytes + chunk * 16);
        const int grow = row0 + r;
        const int g = (chunk * 32) / a.group;
        const float s = __half2float(a.scales[(int64_t)grow * a.G + g]);
        const float z = a.qzeros ? float((a.qzeros[(int64_t)grow * a.ZW + (g >> 3)] >> (4 * (g & 7))) & 15u) : 8.f;
        float2 acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = make_float2(0.f, 0.f);
        const uint32_t words[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t t = ((words[j] >> (4 * i)) & 0x000F000Fu) | 0x43004300u;
            const float2 wv = make_float2(__uint_as_float(t << 16), __uint_as_float(t & 0xFFFF0000u));
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[m] = ffma2(xp[m][4 * j + i], wv, acc[m]);
          }
        }
        const float zz = 128.f + z;
#pragma unroll
        for (int m = 0; m < MT; ++m) part[m] = s * ((acc[m].x + acc[m].y) - zz * xs[m]);
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) part[m] = warp_sum(part[m]);
      if (lane == 0) {
        if (a.S == 1 && !FUSED) {
#pragma unroll
          for (int m = 0; m < MT; ++m)
            if (m < mt) a.y[(int64_t)(m0 + m) * a.ldy + row0 + r] = __float2bfloat16_rn(part[m]);
        } else {
#pragma unroll
          for (int m = 0; m < MT; ++m) red[(r * a.S + slice) * MT + m] = part[m];
        }
      }
    }
  }
  // Every copy has landed before the CTA exits, even on the error path (bounded).
  __syncthreads();
  if (tid == 0)
    for (int c = 0; c < n_chunks; ++c) (void)mbar_wait(&bars[c], 0, 50000000ull);
  if (a.S == 1 && !FUSED) return;
  if constexpr (FUSED) {
    const int pairs = rows >> 1;
    for (int idx = tid; idx < pairs * mt; idx += kThreads) {
      const int p = idx / mt, m = idx % mt;
      float gsum = 0.f, usum = 0.f;
      for (int sl = 0; sl < a.S; ++sl) {
        gsum += red[((2 * p) * a.S + sl) * MT + m];
        usum += red[((2 * p + 1) * a.S + sl) * MT + m];
      }
      a.y[(int64_t)(m0 + m) * a.ldy + (row0 >> 1) + p] = __float2bfloat16_rn(silu(gsum) * usum);
    }
  } else {
    for (int idx = tid; idx < rows * mt; idx += kThreads) {
      const int r = idx / mt, m = idx % mt;
      float sum = 0.f;
      for (int sl = 0; sl < a.S; ++sl) sum += red[(r * a.S + sl) * MT + m];
      a.y[(int64_t)(m0 + m) * a.ldy + row0 + r] = __float2bfloat16_rn(sum);
    }
  }
}

template <int MT, bool FUSED>
int launch(GemvArgs a, int grid_x, int grid_y, int smem, int flags, cudaStream_t stream) {
  auto kernel = w4a16_gemv_kernel<MT, FUSED>;
  int st = set_max_smem(reinterpret_cast<const void*>(kernel), smem);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid_x, grid_y, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BPT_FLAG_PDL) ? 1 : 0;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "w4a16 gemv launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

}  // namespace

// Validates the arguments shared by the W4A16 entry points.
int w4a16_check(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* y,
                int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused) {
  BPT_REQUIRE(x && qweight && scales && y, BPT_ERR_INVALID, "w4a16: null pointer argument");
  BPT_REQUIRE(M >= 1 && N >= 1 && K >= 1, BPT_ERR_INVALID, "w4a16: empty shape M=%lld N=%lld K=%lld",
              (long long)M, (long long)N, (long long)K);
  BPT_REQUIRE(group >= 32 && group % 32 == 0 && K % group == 0, BPT_ERR_INVALID,
              "w4a16: group %lld must be a multiple of 32 that divides K=%lld", (long long)group, (long long)K);
  BPT_REQUIRE(K <= 32768, BPT_ERR_UNSUPPORTED, "w4a16: K=%lld above 32768", (long long)K);
  BPT_REQUIRE(N < (1ll << 31) && M < (1ll << 31), BPT_ERR_INVALID, "w4a16: N or M too large");
  BPT_REQUIRE(ldx >= K && ldx % 8 == 0, BPT_ERR_ALIGNMENT, "w4a16: ldx=%lld must be >= K and a multiple of 8",
              (long long)ldx);
  BPT_REQUIRE(aligned16(x) && aligned16(qweight), BPT_ERR_ALIGNMENT, "w4a16: x and qweight must be 16-byte aligned");
  BPT_REQUIRE(!fused || N % 2 == 0, BPT_ERR_INVALID, "w4a16 gate_up: N=%lld must be even (gate/up pairs)", (long long)N);
  BPT_REQUIRE(ldy >= (fused ? N / 2 : N), BPT_ERR_INVALID, "w4a16: ldy=%lld too small", (long long)ldy);
  return BPT_OK;
}

bool w4a16_mma_applies(int64_t M, int64_t N, int64_t K, int64_t group);
int w4a16_mma(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros, void* y,
              int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags, cudaStream_t stream);

bool w4a16_stream_applies(int64_t M, int64_t N, int64_t K, int64_t group, bool zeros);
int w4a16_stream(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros,
                 void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags,
                 cudaStream_t stream);

bool w4a16_tc_applies(int64_t M, int64_t N, int64_t K, int64_t group);
int w4a16_tc(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros, void* y,
             int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags, cudaStream_t stream);

bool w4a16_gemm_applies(int64_t M, int64_t N, int64_t K, int64_t group);
int w4a16_gemm(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros, void* y,
               int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags, cudaStream_t stream);

// The kernel for a shape: M >= 16 the tcgen05 GEMM (w4a16_tc.cu), else the mma.sync tiled GEMM (w4a16_gemm.cu);
// M <= 8 the persistent streaming GEMV (w4a16_stream.cu); otherwise the tensor-core GEMV (w4a16_mma.cu) where
// its staging fits, the CUDA-core kernel below last. The bulk-copy kernels need 16-byte aligned scales and zero
// points.
int w4a16_pick(int64_t M, int64_t N, int64_t K, int64_t group, bool zeros, bool aligned) {
  if (w4a16_tc_applies(M, N, K, group)) return BPT_W4A16_KERNEL_TCGEN05;
  if (w4a16_gemm_applies(M, N, K, group)) return BPT_W4A16_KERNEL_MMA_GEMM;
  if (aligned && w4a16_stream_applies(M, N, K, group, zeros)) return BPT_W4A16_KERNEL_STREAM;
  if (aligned && w4a16_mma_applies(M, N, K, group)) return BPT_W4A16_KERNEL_MMA_GEMV;
  return BPT_W4A16_KERNEL_CUDA_CORES;
}

int w4a16_gemv(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros,
               void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags,
               cudaStream_t stream) {
  switch (w4a16_pick(M, N, K, group, qzeros != nullptr, aligned16(scales) && (!qzeros || aligned16(qzeros)))) {
    case BPT_W4A16_KERNEL_TCGEN05:
      return w4a16_tc(x, ldx, qweight, scales, qzeros, y, ldy, M, N, K, group, fused, flags, stream);
    case BPT_W4A16_KERNEL_MMA_GEMM:
      return w4a16_gemm(x, ldx, qweight, scales, qzeros, y, ldy, M, N, K, group, fused, flags, stream);
    case BPT_W4A16_KERNEL_STREAM:
      return w4a16_stream(x, ldx, qweight, scales, qzeros, y, ldy, M, N, K, group, fused, flags, stream);
    case BPT_W4A16_KERNEL_MMA_GEMV:
      return w4a16_mma(x, ldx, qweight, scales, qzeros, y, ldy, M, N, K, group, fused, flags, stream);
    default:
      break;
  }
  GemvArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.qweight = reinterpret_cast<const uint8_t*>(qweight);
  a.scales = static_cast<const __half*>(scales);
  a.qzeros = reinterpret_cast<const uint32_t*>(qzeros);
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.M = int(M);
  a.N = int(N);
  a.K = int(K);
  a.group = int(group);
  a.G = int(K / group);
  a.ZW = (a.G + 7) / 8;
  a.S = int((K + 1023) / 1024);
  const int warps = kThreads / 32;
  if (a.S > warps) return set_error(BPT_ERR_UNSUPPORTED, "w4a16 gemv: K=%lld needs more than %d warps", (long long)K, warps);
  a.RW = warps / a.S;
  const int MT = M >= 4 ? 4 : (M >= 2 ? 2 : 1);
  const int row_bytes = int(K / 2);
  // Rows per CTA: about two CTAs per SM, bounded by the slab budget; even when fused (gate/up pairs).
  const int sms = num_sms();
  int rows = int((N + 2 * sms - 1) / (2 * sms));
  rows = max(rows, 1);
  rows = min(rows, max(1, kSlabBudget / row_bytes));
  if (fused) rows = max(2, rows & ~1);
  a.rows_per_cta = rows;
  a.slab_bytes = (rows * row_bytes + 127) & ~127;
  const int smem = ((a.slab_bytes + rows * a.S * MT * int(sizeof(float)) + 15) & ~15) + kMaxChunks * 8;
  const int grid_x = int((N + rows - 1) / rows);
  const int grid_y = int((M + MT - 1) / MT);
  if (MT == 4) return fused ? launch<4, true>(a, grid_x, grid_y, smem, flags, stream)
                            : launch<4, false>(a, grid_x, grid_y, smem, flags, stream);
  if (MT == 2) return fused ? launch<2, true>(a, grid_x, grid_y, smem, flags, stream)
                            : launch<2, false>(a, grid_x, grid_y, smem, flags, stream);
  return fused ? launch<1, true>(a, grid_x, grid_y, smem, flags, stream)
               : launch<1, false>(a, grid_x, grid_y, smem, flags, stream);
}

}  // namespace bpt
