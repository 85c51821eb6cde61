// W4A16 entry points: argument checks, dispatch, and the RTN quantize + pack kernel.
#include "common.cuh"

namespace bpt {

int w4a16_check(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* y,
                int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused);
int w4a16_pick(int64_t M, int64_t N, int64_t K, int64_t group, bool zeros, bool aligned);
int w4a16_gemv(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros,
               void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags,
               cudaStream_t stream);

namespace {

// One warp per (row, zero-point word): up to 8 groups of the row. For each group the warp finds the range,
// derives the fp16 scale and the zero-point exactly as the CPU reference does (IEEE division, rounding half
// to even), then writes the group's code words. Lane l handles the 8-code words l, l+32, ... of the group.
template <typename T>
__global__ void w4a16_quantize_kernel(const T* __restrict__ w, int N, int K, int group, uint32_t* __restrict__ qweight,
                                      __half* __restrict__ scales, uint32_t* __restrict__ qzeros) {
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int G = K / group, ZW = (G + 7) / 8;
  if (warp_global >= N * ZW) return;
  const int n = warp_global / ZW, zw = warp_global % ZW;
  const int words_per_group = group / 8;
  uint32_t zword = 0;
  for (int gi = 0; gi < 8; ++gi) {
    const int g = zw * 8 + gi;
    if (g >= G) break;
    const T* src = w + (int64_t)n * K + (int64_t)g * group;
    float lo = 0.f, hi = 0.f;  // the range always includes 0
    for (int wd = lane; wd < words_per_group; wd += 32) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float v = float(src[wd * 8 + e]);
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    __half s16 = __float2half_rn(__fdiv_rn(hi - lo, 15.0f));
    if (!(__half2float(s16) > 0.f)) s16 = __float2half_rn(1.0f);
    const float s = __half2float(s16);
    const float z = fminf(fmaxf(rintf(__fdiv_rn(-lo, s)), 0.f), 15.f);
    for (int wd = lane; wd < words_per_group; wd += 32) {
      uint32_t word = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float c = fminf(fmaxf(rintf(__fdiv_rn(float(src[wd * 8 + e]), s)) + z, 0.f), 15.f);
        word |= uint32_t(c) << (4 * e);
      }
      qweight[(int64_t)n * (K / 8) + (int64_t)g * words_per_group + wd] = word;
    }
    if (lane == 0) scales[(int64_t)n * G + g] = s16;
    zword |= uint32_t(z) << (4 * gi);
  }
  if (lane == 0) qzeros[(int64_t)n * ZW + zw] = zword;
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" int bpt_w4a16_linear(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                                const int32_t* qzeros, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                                int64_t group, int flags, void* stream) {
  int st = w4a16_check(x, ldx, qweight, scales, y, ldy, M, N, K, group, false);
  if (st) return st;
  return w4a16_gemv(x, ldx, qweight, scales, qzeros, y, ldy, M, N, K, group, false, flags,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int bpt_w4a16_gate_up_silu(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                                      const int32_t* qzeros, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                                      int64_t group, int flags, void* stream) {
  int st = w4a16_check(x, ldx, qweight, scales, y, ldy, M, N, K, group, true);
  if (st) return st;
  return w4a16_gemv(x, ldx, qweight, scales, qzeros, y, ldy, M, N, K, group, true, flags,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int bpt_w4a16_kernel(int64_t M, int64_t N, int64_t K, int64_t group, int has_zeros) {
  return w4a16_pick(M, N, K, group, has_zeros != 0, true);
}

extern "C" int bpt_w4a16_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int64_t group, int32_t* qweight,
                                  void* scales, int32_t* qzeros, void* stream) {
  BPT_REQUIRE(w && qweight && scales && qzeros, BPT_ERR_INVALID, "w4a16_quantize: null pointer argument");
  BPT_REQUIRE(N >= 1 && K >= 1 && N < (1ll << 31) && K < (1ll << 31), BPT_ERR_INVALID, "w4a16_quantize: bad shape");
  BPT_REQUIRE(group >= 8 && group % 8 == 0 && K % group == 0, BPT_ERR_INVALID,
              "w4a16_quantize: group %lld must be a multiple of 8 that divides K=%lld", (long long)group, (long long)K);
  BPT_REQUIRE(w_dtype == BPT_DTYPE_F32 || w_dtype == BPT_DTYPE_BF16, BPT_ERR_UNSUPPORTED,
              "w4a16_quantize: weights must be fp32 or bf16");
  const int64_t warps = N * ((K / group + 7) / 8);
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  BPT_REQUIRE(blocks < (1ll << 31), BPT_ERR_INVALID, "w4a16_quantize: too large");
  auto s = static_cast<cudaStream_t>(stream);
  if (w_dtype == BPT_DTYPE_F32)
    w4a16_quantize_kernel<float><<<unsigned(blocks), threads, 0, s>>>(
        static_cast<const float*>(w), int(N), int(K), int(group), reinterpret_cast<uint32_t*>(qweight),
        static_cast<__half*>(scales), reinterpret_cast<uint32_t*>(qzeros));
  else
    w4a16_quantize_kernel<__nv_bfloat16><<<unsigned(blocks), threads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(w), int(N), int(K), int(group), reinterpret_cast<uint32_t*>(qweight),
        static_cast<__half*>(scales), reinterpret_cast<uint32_t*>(qzeros));
  return check_launch("w4a16_quantize");
}
