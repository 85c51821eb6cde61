// RMSNorm fused with per-token symmetric INT8 quantization: the activation quantizer in front of a W8A8 linear.
//
// For every row x of a [rows, d] tensor (kernels/norm_quant.py:42-67 computes the same, kernels/reference.py:44-55
// is its definition):
//   y      = x * (1 / sqrt(sum(x^2) / d + eps)) * weight      fp32 throughout
//   scale  = max(max|y| / 127, 1e-12)                          one fp32 per row
//   codes  = clamp(rint(y / scale), -128, 127)                 int8, round half to even
// With a residual (vLLM's fused add + RMSNorm): x is first replaced by x + delta, rounded to x's dtype as the
// model's residual tensor is, and that sum is also written out.
//
// The row is read once: its elements stay in registers (16-byte loads when the row, the weight and the strides
// allow it, else one element at a time) and the three passes (sum of squares, max of |y|, the codes) run on that
// copy. Two launch shapes:
// - 512 rows or more, each of up to 1,024 chunks (8,192 16-bit or 4,096 fp32 elements; 1,024 on the one-element
//   path; past 512 chunks one CTA per SM): one WARP per row, eight rows per CTA, warps persistent over rows,
//   reductions by shuffles only. A row
//   is a few KB, so an SM needs many rows in flight to cover HBM latency: the row is kept as packed 16-byte
//   words, there is no block barrier, and the arithmetic runs two elements per instruction on the packed fp32
//   pipe (the kernel is otherwise instruction-bound: ~20 operations per element).
// - fewer or longer rows: one CTA per row (up to 256 threads); a row longer than the CTA's registers hold (more
//   than 16,384 16-bit or 8,192 fp32 elements) reads its remainder again, from L2.
// Divisions and the square root are IEEE-rounded, as the reference's fp32 tensor ops are, so results differ from
// it only through the order of the row's sums.
#include "common.cuh"

namespace bpt {
namespace {

constexpr int kMaxThreads = 256;
constexpr int kMaxCached = 8;  // chunks of a row a thread keeps in registers

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  if constexpr (std::is_same_v<T, float>) return v;
  else if constexpr (std::is_same_v<T, __half>) return __half2float(v);
  else return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T from_f(float v) {
  if constexpr (std::is_same_v<T, float>) return v;
  else if constexpr (std::is_same_v<T, __half>) return __float2half_rn(v);
  else return __float2bfloat16_rn(v);
}

// CH consecutive elements of type T at p (CH * sizeof(T) bytes, aligned to that size when CH > 1) as floats.
template <typename T, int CH>
__device__ __forceinline__ void load_chunk(const T* p, float (&v)[CH]) {
  if constexpr (CH == 1) {
    v[0] = to_f(p[0]);
  } else {
    constexpr int kBytes = CH * int(sizeof(T));
    static_assert(kBytes % 8 == 0, "vector chunks are 8, 16 or 32 bytes");
    alignas(16) T tmp[CH];
    if constexpr (kBytes == 8) {
      *reinterpret_cast<uint2*>(tmp) = *reinterpret_cast<const uint2*>(p);
    } else {
#pragma unroll
      for (int i = 0; i < kBytes / 16; ++i) reinterpret_cast<uint4*>(tmp)[i] = reinterpret_cast<const uint4*>(p)[i];
    }
#pragma unroll
    for (int i = 0; i < CH; ++i) v[i] = to_f(tmp[i]);
  }
}

template <typename T, int CH>
__device__ __forceinline__ void store_chunk(T* p, const float (&v)[CH]) {
  alignas(16) T tmp[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) tmp[i] = from_f<T>(v[i]);
  if constexpr (CH == 1) {
    p[0] = tmp[0];
  } else {
    constexpr int kBytes = CH * int(sizeof(T));
    if constexpr (kBytes == 8) {
      *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(tmp);
    } else {
#pragma unroll
      for (int i = 0; i < kBytes / 16; ++i) reinterpret_cast<uint4*>(p)[i] = reinterpret_cast<const uint4*>(tmp)[i];
    }
  }
}

// div_by (common.cuh): y / b correctly rounded from the divisor's reciprocal; its only exception, an underflowing
// remainder, touches quotients far below 0.5 here (code 0 either way).

// clamp(rint(v), -128, 127) as int8: round to nearest even and saturate in one conversion
__device__ __forceinline__ int8_t to_code(float v) {
  int r;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(v));
  return int8_t(r);
}

// Pairs of fp32 lanes on the packed two-wide fp32 pipe of sm_100 (add/mul/fma .f32x2): each half rounds exactly
// as the scalar instruction would.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// four codes clamp(rint(v), -128, 127), v0 in the lowest byte: round to nearest even into s32, then two
// saturating packs (each puts its two values in the low bytes above the third operand's bits)
__device__ __forceinline__ uint32_t to_codes4(float v0, float v1, float v2, float v3) {
  int i0, i1, i2, i3;
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(i0) : "f"(v0));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(i1) : "f"(v1));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(i2) : "f"(v2));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(i3) : "f"(v3));
  uint32_t hi, w;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(i3), "r"(i2), "r"(0));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(i1), "r"(i0), "r"(hi));
  return w;
}

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  v = is_max ? warp_max(v) : warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < nw; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];  // the same order in every thread
  __syncthreads();
  return r;
}

struct NormQuantArgs {
  const void* x;
  int64_t ldx;  // elements between rows of x
  const void* weight;
  const void* delta;  // [rows, d] contiguous, x's dtype, or null
  void* x_out;        // [rows, d] contiguous, x's dtype: x + delta (with delta)
  int8_t* codes;      // [rows, d] contiguous
  float* scale;       // [rows]
  int d;
  float eps;
};

// CH elements per chunk: 16 / sizeof(T) on the vector path, 1 otherwise.
template <typename T, typename W, int CH>
__global__ void __launch_bounds__(kMaxThreads) rms_norm_int8_kernel(const NormQuantArgs a) {
  __shared__ float red[kMaxThreads / 32];
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  const int d = a.d, nchunks = d / CH, nt = blockDim.x;
  const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
  const T* dr = a.delta ? static_cast<const T*>(a.delta) + row * int64_t(d) : nullptr;
  T* xo = a.x_out ? static_cast<T*>(a.x_out) + row * int64_t(d) : nullptr;
  const W* w = static_cast<const W*>(a.weight);
  pdl_wait();  // x (and delta) may come from the previous kernel

  // the row's chunk at index ci: x, or x + delta rounded to T (written out once, in pass 1)
  auto fetch = [&](int ci, float (&v)[CH], bool write_sum) {
    load_chunk<T, CH>(xr + int64_t(ci) * CH, v);
    if (dr) {
      float e[CH];
      load_chunk<T, CH>(dr + int64_t(ci) * CH, e);
#pragma unroll
      for (int i = 0; i < CH; ++i) v[i] = to_f(from_f<T>(v[i] + e[i]));
      if (write_sum && xo) store_chunk<T, CH>(xo + int64_t(ci) * CH, v);
    }
  };

  // pass 1: sum of squares; the first kMaxCached chunks of this thread stay in registers
  float cache[kMaxCached][CH];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxCached; ++i) {
    const int ci = threadIdx.x + i * nt;
    if (ci < nchunks) {
      fetch(ci, cache[i], true);
#pragma unroll
      for (int e = 0; e < CH; ++e) ss = fmaf(cache[i][e], cache[i][e], ss);
    }
  }
  for (int ci = threadIdx.x + kMaxCached * nt; ci < nchunks; ci += nt) {
    float v[CH];
    fetch(ci, v, true);
#pragma unroll
    for (int e = 0; e < CH; ++e) ss = fmaf(v[e], v[e], ss);
  }
  const float ms = __fdiv_rn(block_reduce(ss, red, false), float(d));
  const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(ms, a.eps)));

  // pass 2: y = x * inv * weight, its largest magnitude
  auto norm = [&](int ci, const float (&v)[CH], float (&y)[CH]) {
    float wv[CH];
    load_chunk<W, CH>(w + int64_t(ci) * CH, wv);
#pragma unroll
    for (int e = 0; e < CH; ++e) y[e] = __fmul_rn(__fmul_rn(v[e], inv), wv[e]);
  };
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxCached; ++i) {
    const int ci = threadIdx.x + i * nt;
    if (ci < nchunks) {
      float y[CH];
      norm(ci, cache[i], y);
#pragma unroll
      for (int e = 0; e < CH; ++e) amax = fmaxf(amax, fabsf(y[e]));
    }
  }
  for (int ci = threadIdx.x + kMaxCached * nt; ci < nchunks; ci += nt) {
    float v[CH], y[CH];
    fetch(ci, v, false);
    norm(ci, v, y);
#pragma unroll
    for (int e = 0; e < CH; ++e) amax = fmaxf(amax, fabsf(y[e]));
  }
  const float scale = fmaxf(__fdiv_rn(block_reduce(amax, red, true), 127.f), 1e-12f);
  const float rscale = __frcp_rn(scale);
  if (threadIdx.x == 0) a.scale[row] = scale;

  // pass 3: the codes
  int8_t* cr = a.codes + row * int64_t(d);
  auto quant = [&](int ci, const float (&y)[CH]) {
    alignas(8) int8_t q[CH];
#pragma unroll
    for (int e = 0; e < CH; ++e) q[e] = to_code(div_by(y[e], scale, rscale));
    if constexpr (CH == 8) {
      *reinterpret_cast<uint2*>(cr + int64_t(ci) * CH) = *reinterpret_cast<const uint2*>(q);
    } else if constexpr (CH == 4) {
      *reinterpret_cast<uint32_t*>(cr + int64_t(ci) * CH) = *reinterpret_cast<const uint32_t*>(q);
    } else {
#pragma unroll
      for (int e = 0; e < CH; ++e) cr[int64_t(ci) * CH + e] = q[e];
    }
  };
#pragma unroll
  for (int i = 0; i < kMaxCached; ++i) {
    const int ci = threadIdx.x + i * nt;
    if (ci < nchunks) {
      float y[CH];
      norm(ci, cache[i], y);
      quant(ci, y);
    }
  }
  for (int ci = threadIdx.x + kMaxCached * nt; ci < nchunks; ci += nt) {
    float v[CH], y[CH];
    fetch(ci, v, false);
    norm(ci, v, y);
    quant(ci, y);
  }
}

// ---- one warp per row ---------------------------------------------------------------------------------------
constexpr int kRowsPerCta = 8;

template <typename T>
__device__ __forceinline__ void unpack16(const uint4 u, float (&v)[16 / sizeof(T)]) {
  alignas(16) T tmp[16 / sizeof(T)];
  *reinterpret_cast<uint4*>(tmp) = u;
#pragma unroll
  for (int i = 0; i < int(16 / sizeof(T)); ++i) v[i] = to_f(tmp[i]);
}
template <typename T>
__device__ __forceinline__ uint4 pack16(const float (&v)[16 / sizeof(T)]) {
  alignas(16) T tmp[16 / sizeof(T)];
#pragma unroll
  for (int i = 0; i < int(16 / sizeof(T)); ++i) tmp[i] = from_f<T>(v[i]);
  return *reinterpret_cast<const uint4*>(tmp);
}

// CH weights at element offset off, whatever the weight's dtype (a uniform branch; the weight sits in L1)
template <int CH>
__device__ __forceinline__ void load_weight(const void* w, int w_dtype, int64_t off, float (&v)[CH]) {
  if (w_dtype == BPT_DTYPE_F32) load_chunk<float, CH>(static_cast<const float*>(w) + off, v);
  else if (w_dtype == BPT_DTYPE_F16) load_chunk<__half, CH>(static_cast<const __half*>(w) + off, v);
  else load_chunk<__nv_bfloat16, CH>(static_cast<const __nv_bfloat16*>(w) + off, v);
}

// the 128-byte lines of bytes [0, n) at p, one per lane in turn, requested into L2
__device__ __forceinline__ void prefetch_l2(const void* p, int64_t n, int lane) {
  const char* c = static_cast<const char*>(p);
  for (int64_t o = int64_t(lane) * 128; o < n; o += 32 * 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(c + o));
}

// CH = 16 / sizeof(T) (16-byte chunks) or 1; lane l holds chunks l, l + 32, ..., NPER of them at most. Warps are
// persistent over rows (row, row + all warps, ...); each asks L2 for its next row before working on this one.
template <typename T, int CH, int NPER>
__global__ void __launch_bounds__(32 * kRowsPerCta, NPER <= 16 ? 2 : 1) rms_norm_int8_rows_kernel(const NormQuantArgs a, int64_t rows,
                                                                             int w_dtype) {
  pdl_launch_dependents();
  pdl_wait();  // x (and delta) may come from the previous kernel
  const int lane = threadIdx.x & 31;
  const int64_t stride = int64_t(gridDim.x) * kRowsPerCta;
  const int64_t row_bytes = int64_t(a.d) * int64_t(sizeof(T));
  for (int64_t row = int64_t(blockIdx.x) * kRowsPerCta + (threadIdx.x >> 5); row < rows; row += stride) {
  if (row + stride < rows) {
    prefetch_l2(static_cast<const T*>(a.x) + (row + stride) * a.ldx, row_bytes, lane);
    if (a.delta) prefetch_l2(static_cast<const T*>(a.delta) + (row + stride) * int64_t(a.d), row_bytes, lane);
  }
  const int d = a.d, nchunks = d / CH;
  const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
  const T* dr = a.delta ? static_cast<const T*>(a.delta) + row * int64_t(d) : nullptr;
  T* xo = a.x_out ? static_cast<T*>(a.x_out) + row * int64_t(d) : nullptr;
  constexpr bool kVec = CH > 1;
  using Raw = std::conditional_t<kVec, uint4, float>;
  Raw raw[NPER];  // the row (or row + delta), as loaded: packed 16-byte words on the vector path

  // every load first, then the sums
#pragma unroll
  for (int i = 0; i < NPER; ++i) {
    const int ci = lane + 32 * i;
    if (ci < nchunks) {
      if constexpr (kVec) raw[i] = *reinterpret_cast<const uint4*>(xr + int64_t(ci) * CH);
      else raw[i] = to_f(xr[ci]);
    }
  }
  float ss = 0.f;
  uint64_t ss2 = pk2(0.f, 0.f);  // the vector path sums even and odd elements apart, then adds the two
#pragma unroll
  for (int i = 0; i < NPER; ++i) {
    const int ci = lane + 32 * i;
    if (ci < nchunks) {
      float v[CH];
      if constexpr (kVec) unpack16<T>(raw[i], v);
      else v[0] = raw[i];
      if (dr) {  // x + delta, rounded to T like the model's residual tensor
        float e[CH];
        load_chunk<T, CH>(dr + int64_t(ci) * CH, e);
#pragma unroll
        for (int k = 0; k < CH; ++k) v[k] = to_f(from_f<T>(v[k] + e[k]));
        if constexpr (kVec) raw[i] = pack16<T>(v);
        else raw[i] = v[0];
        if (xo) store_chunk<T, CH>(xo + int64_t(ci) * CH, v);
      }
      if constexpr (kVec) {
#pragma unroll
        for (int k = 0; k < CH; k += 2) {
          const uint64_t v2 = pk2(v[k], v[k + 1]);
          ss2 = fma2(v2, v2, ss2);
        }
      } else {
        ss = fmaf(v[0], v[0], ss);
      }
    }
  }
  if constexpr (kVec) {
    float s0, s1;
    upk2(ss2, s0, s1);
    ss = s0 + s1;
  }
  const float ms = __fdiv_rn(warp_sum(ss), float(d));
  const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
  const uint64_t inv2 = pk2(inv, inv);

  auto norm = [&](int i, int ci, float (&y)[CH]) {
    float v[CH], wv[CH];
    if constexpr (kVec) unpack16<T>(raw[i], v);
    else v[0] = raw[i];
    load_weight<CH>(a.weight, w_dtype, int64_t(ci) * CH, wv);
    if constexpr (kVec) {
#pragma unroll
      for (int k = 0; k < CH; k += 2)
        upk2(mul2(mul2(pk2(v[k], v[k + 1]), inv2), pk2(wv[k], wv[k + 1])), y[k], y[k + 1]);
    } else {
      y[0] = __fmul_rn(__fmul_rn(v[0], inv), wv[0]);
    }
  };
  // up to 64 values in 8 chunks a lane, y stays in registers for the codes (the packed row dies as it forms);
  // longer rows form it again
  constexpr bool kKeepY = NPER * CH <= 64 && NPER <= 8;
  float amax = 0.f;
  float yv[kKeepY ? NPER : 1][CH];
#pragma unroll
  for (int i = 0; i < NPER; ++i) {
    const int ci = lane + 32 * i;
    if (ci < nchunks) {
      float (&y)[CH] = yv[kKeepY ? i : 0];
      norm(i, ci, y);
#pragma unroll
      for (int k = 0; k < CH; ++k) amax = fmaxf(amax, fabsf(y[k]));
    }
  }
  const float scale = fmaxf(__fdiv_rn(warp_max(amax), 127.f), 1e-12f);
  const float rscale = __frcp_rn(scale);
  const uint64_t r2 = pk2(rscale, rscale), nb2 = pk2(-scale, -scale);
  if (lane == 0) a.scale[row] = scale;
  int8_t* cr = a.codes + row * int64_t(d);
#pragma unroll
  for (int i = 0; i < NPER; ++i) {
    const int ci = lane + 32 * i;
    if (ci < nchunks) {
      float (&y)[CH] = yv[kKeepY ? i : 0];
      if constexpr (!kKeepY) norm(i, ci, y);
      if constexpr (kVec) {  // div_by two at a time: q = y r, e = y - q b, q + e r
        float t[CH];
#pragma unroll
        for (int k = 0; k < CH; k += 2) {
          const uint64_t y2 = pk2(y[k], y[k + 1]);
          const uint64_t q2 = mul2(y2, r2);
          upk2(fma2(fma2(q2, nb2, y2), r2, q2), t[k], t[k + 1]);
        }
        uint32_t w[CH / 4];
#pragma unroll
        for (int k = 0; k < CH / 4; ++k) w[k] = to_codes4(t[4 * k], t[4 * k + 1], t[4 * k + 2], t[4 * k + 3]);
        if constexpr (CH == 8) *reinterpret_cast<uint2*>(cr + int64_t(ci) * CH) = make_uint2(w[0], w[1]);
        else *reinterpret_cast<uint32_t*>(cr + int64_t(ci) * CH) = w[0];
      } else {
        cr[ci] = to_code(div_by(y[0], scale, rscale));
      }
    }
  }
  }  // rows
}

template <typename T, int CH, int NPER>
int launch_rows_t(const NormQuantArgs& a, int64_t rows, int w_dtype, int flags, cudaStream_t stream) {
  static int resident = 0;  // CTAs of this instantiation one SM holds at once
  if (resident == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, rms_norm_int8_rows_kernel<T, CH, NPER>, 32 * kRowsPerCta,
                                                      0) != cudaSuccess || n < 1)
      n = 1;
    resident = n;
  }
  const int64_t grid = std::min<int64_t>((rows + kRowsPerCta - 1) / kRowsPerCta, int64_t(resident) * num_sms());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(32 * kRowsPerCta);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BPT_FLAG_PDL) ? 1 : 0;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, rms_norm_int8_rows_kernel<T, CH, NPER>, a, rows, w_dtype);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "rms_norm_int8 launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

constexpr int kWarpMaxChunks = 32 * 32;  // the warp-per-row kernel's longest row, in chunks
constexpr int64_t kWarpMinRows = 512;    // below this a CTA per row finishes sooner (more SMs share a call)

template <typename T, int CH>
int launch_rows(const NormQuantArgs& a, int64_t rows, int w_dtype, int flags, cudaStream_t stream) {
  const int per = (a.d / CH + 31) / 32;  // chunks per lane
  if (per <= 2) return launch_rows_t<T, CH, 2>(a, rows, w_dtype, flags, stream);
  if (per <= 4) return launch_rows_t<T, CH, 4>(a, rows, w_dtype, flags, stream);
  if (per <= 8) return launch_rows_t<T, CH, 8>(a, rows, w_dtype, flags, stream);
  if (per <= 16) return launch_rows_t<T, CH, 16>(a, rows, w_dtype, flags, stream);
  // longer rows: one CTA of eight warps per SM, whose registers hold 24 or 32 chunks a lane
  if (per <= 24) return launch_rows_t<T, CH, 24>(a, rows, w_dtype, flags, stream);
  return launch_rows_t<T, CH, 32>(a, rows, w_dtype, flags, stream);
}

// ---- one CTA per row ----------------------------------------------------------------------------------------
template <typename T, typename W, int CH>
int launch_t(const NormQuantArgs& a, int64_t rows, int flags, cudaStream_t stream) {
  const int64_t nchunks = a.d / CH;
  const int threads = int(std::min<int64_t>(kMaxThreads, std::max<int64_t>(32, (nchunks + 31) / 32 * 32)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(rows));
  cfg.blockDim = dim3(unsigned(threads));
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BPT_FLAG_PDL) ? 1 : 0;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, rms_norm_int8_kernel<T, W, CH>, a);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "rms_norm_int8 launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

template <typename T, typename W>
int launch_w(const NormQuantArgs& a, int64_t rows, bool vec, int flags, cudaStream_t stream) {
  if (vec) return launch_t<T, W, 16 / int(sizeof(T))>(a, rows, flags, stream);
  return launch_t<T, W, 1>(a, rows, flags, stream);
}

template <typename T>
int launch_x(const NormQuantArgs& a, int w_dtype, int64_t rows, bool vec, int flags, cudaStream_t stream) {
  // a warp per row once there are enough rows to fill the GPU with warps; fewer rows: a CTA each
  constexpr int kCh = 16 / int(sizeof(T));
  const bool many = rows >= kWarpMinRows;
  if (many && vec && a.d / kCh <= kWarpMaxChunks) return launch_rows<T, kCh>(a, rows, w_dtype, flags, stream);
  if (many && !vec && a.d <= kWarpMaxChunks) return launch_rows<T, 1>(a, rows, w_dtype, flags, stream);
  switch (w_dtype) {
    case BPT_DTYPE_F32: return launch_w<T, float>(a, rows, vec, flags, stream);
    case BPT_DTYPE_F16: return launch_w<T, __half>(a, rows, vec, flags, stream);
    default: return launch_w<T, __nv_bfloat16>(a, rows, vec, flags, stream);
  }
}

int dtype_size(int dt) { return dt == BPT_DTYPE_F32 ? 4 : 2; }
bool dtype_ok(int dt) { return dt == BPT_DTYPE_F32 || dt == BPT_DTYPE_F16 || dt == BPT_DTYPE_BF16; }

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" int bpt_rms_norm_int8(const void* x, int x_dtype, int64_t x_row_stride, const void* weight, int w_dtype,
                                 const void* delta, void* x_out, void* codes, void* scale, int64_t rows, int64_t d,
                                 float eps, int flags, void* stream) {
  BPT_REQUIRE(dtype_ok(x_dtype) && dtype_ok(w_dtype), BPT_ERR_INVALID, "rms_norm_int8: dtype codes %d, %d",
              x_dtype, w_dtype);
  BPT_REQUIRE(rows >= 0 && rows < (1ll << 31), BPT_ERR_INVALID, "rms_norm_int8: rows=%lld", (long long)rows);
  if (rows == 0) return BPT_OK;  // nothing to read or write (empty tensors may have null data pointers)
  BPT_REQUIRE(x && weight && codes && scale, BPT_ERR_INVALID, "rms_norm_int8: null pointer argument");
  BPT_REQUIRE(d >= 1 && d < (1ll << 28), BPT_ERR_INVALID, "rms_norm_int8: d=%lld", (long long)d);
  BPT_REQUIRE(x_row_stride >= d || rows <= 1, BPT_ERR_INVALID, "rms_norm_int8: row stride %lld < d=%lld",
              (long long)x_row_stride, (long long)d);
  BPT_REQUIRE(!x_out || delta, BPT_ERR_INVALID, "rms_norm_int8: x_out is the residual sum and needs delta");
  BPT_REQUIRE(eps >= 0.f, BPT_ERR_INVALID, "rms_norm_int8: eps=%g", double(eps));
  // the vector path: 16-byte chunks of x (and delta, x_out), the weight's chunk aligned to its size, 4- or 8-code
  // stores aligned
  const int xs = dtype_size(x_dtype), ws = dtype_size(w_dtype), ch = 16 / xs;
  auto al = [](const void* p, int b) { return (reinterpret_cast<uintptr_t>(p) % uintptr_t(b)) == 0; };
  const bool vec = d % ch == 0 && (x_row_stride * xs) % 16 == 0 && al(x, 16) && al(weight, ch * ws) &&
                   (!delta || al(delta, 16)) && (!x_out || al(x_out, 16)) && al(codes, ch);
  NormQuantArgs a{x, x_row_stride, weight, delta, x_out, static_cast<int8_t*>(codes), static_cast<float*>(scale),
                  int(d), eps};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (x_dtype) {
    case BPT_DTYPE_F32: return launch_x<float>(a, w_dtype, rows, vec, flags, st);
    case BPT_DTYPE_F16: return launch_x<__half>(a, w_dtype, rows, vec, flags, st);
    default: return launch_x<__nv_bfloat16>(a, w_dtype, rows, vec, flags, st);
  }
}
