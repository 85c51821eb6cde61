// The quantized KV-cache write path.
//
// bpt_paged_kv_write: rows that start on 16 bytes, with at least 4 new tokens, take paged_kv_write_vec_kernel (8 values
// per lane, up to 8 tokens per warp); otherwise one warp per (K or V, sequence, KV head, new token). The warp reads the head vector (one
// vector load per lane where strides allow), quantizes it (FP8: x / scale rounded to E4M3 with saturation; INT8:
// an fp16 scale from the vector's absmax, then codes), and stores D bytes to slot (block, offset) of the pool (one
// word per lane), plus the scale for INT8. Quotients are correctly rounded (div_by: the divisor's reciprocal and
// one remainder correction) and rounding is half-to-even, so the codes equal the CPU reference's bit for bit.
//
// bpt_kivi_quantize: the KIVI grids of kernels/reference.py for whole key groups. At D = 128 with groups of 32 and
// 16-bit inputs: keys one warp per (sequence, head, group), 4 channels per lane over all 32 rows at once; values one
// warp per 8 tokens, 8 channels per lane. Otherwise keys one thread per (sequence, head, group, channel [pair]) over
// the group's tokens and values one warp per token over its head vector. 4-bit codes are packed channel d low /
// d + D/2 high.
#include "common.cuh"

namespace bpt {
namespace {

template <int DT>
__device__ __forceinline__ float ld(const void* p, int64_t i) {
  return load_as_float<DT>(p, i);
}

// VPL values of type DT (VPL * sizeof(DT) bytes, aligned to that size up to 16) as floats
template <int DT, int VPL>
__device__ __forceinline__ void load_vec(const void* src, int64_t i, float (&x)[VPL]) {
  constexpr int kBytes = VPL * (DT == BPT_DTYPE_F32 ? 4 : 2);
  struct alignas(kBytes < 16 ? kBytes : 16) Chunk {
    uint8_t b[kBytes];
  };
  const Chunk c = *reinterpret_cast<const Chunk*>(static_cast<const uint8_t*>(src) + i * (kBytes / VPL));
#pragma unroll
  for (int j = 0; j < VPL; ++j) x[j] = load_as_float<DT>(c.b, j);
}

// VEC: a lane's VPL values load as one aligned vector and its codes store as one VPL-byte word (the host checks
// strides and pointers); otherwise element by element.
template <int DT, int VPL, int KIND, bool VEC>
__global__ void paged_kv_write_kernel(const void* __restrict__ k, const void* __restrict__ v, int64_t sb, int64_t sh,
                                      int64_t sq, int B, int Hkv, int Q, const int32_t* __restrict__ wblocks,
                                      const int32_t* __restrict__ woffsets, uint8_t* __restrict__ k_pool,
                                      uint8_t* __restrict__ v_pool, float k_scale, float v_scale,
                                      __half* __restrict__ k_scales, __half* __restrict__ v_scales, int block_size,
                                      int64_t num_blocks) {
  constexpr int D = VPL * 32;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t per_tensor = (int64_t)B * Hkv * Q;
  if (wid >= 2 * per_tensor) return;
  pdl_wait();
  const bool is_v = wid >= per_tensor;
  const int64_t idx = is_v ? wid - per_tensor : wid;
  int q, h, b;
  if (per_tensor < (int64_t(1) << 31)) {  // 32-bit index arithmetic (64-bit division is a long sequence)
    const uint32_t i32 = uint32_t(idx), qh = uint32_t(Q) * uint32_t(Hkv);
    b = int(i32 / qh);
    const uint32_t rest = i32 - uint32_t(b) * qh;
    h = int(rest / uint32_t(Q));
    q = int(rest - uint32_t(h) * uint32_t(Q));
  } else {
    q = int(idx % Q);
    h = int((idx / Q) % Hkv);
    b = int(idx / ((int64_t)Q * Hkv));
  }
  const void* src = is_v ? v : k;
  const int64_t base = (int64_t)b * sb + (int64_t)h * sh + (int64_t)q * sq + lane * VPL;
  // lane owns dims [lane*VPL, lane*VPL + VPL): contiguous bytes in the pool row; the values are requested with
  // the slot, before either is used
  float x[VPL];
  if constexpr (VEC) {
    load_vec<DT, VPL>(src, base, x);
  } else {
#pragma unroll
    for (int j = 0; j < VPL; ++j) x[j] = ld<DT>(src, base + j);
  }
  const int32_t blk = wblocks[(int64_t)b * Q + q];
  const int32_t off = woffsets[(int64_t)b * Q + q];
  if (blk < 0 || blk >= num_blocks || off < 0 || off >= block_size) {
    if (lane == 0) record_error(blk < 0 || blk >= num_blocks ? kDevErrBlockIndex : kDevErrSlotIndex);
    return;
  }
  const int64_t slot = ((int64_t)blk * block_size + off) * Hkv + h;
  uint8_t* dst = (is_v ? v_pool : k_pool) + slot * D + lane * VPL;
  alignas(8) uint8_t bytes[VPL];
  if constexpr (KIND == BPT_KV_FP8) {
    const float s = is_v ? v_scale : k_scale;
    const float rs = __frcp_rn(s);
#pragma unroll
    for (int j = 0; j < VPL; j += 2) {
      // the quotient carries x's sign, a zero's included (div_by alone turns -0 into +0; E4M3 keeps the sign)
      const uint16_t two = float2_to_e4m3x2(copysignf(div_by(x[j], s, rs), x[j]), copysignf(div_by(x[j + 1], s, rs), x[j + 1]));
      bytes[j] = uint8_t(two & 0xFF);
      bytes[j + 1] = uint8_t(two >> 8);
    }
  } else {
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) amax = fmaxf(amax, fabsf(x[j]));
    amax = warp_max(amax);
    __half s16 = __float2half_rn(__fdiv_rn(amax, 127.0f));
    if (!(__half2float(s16) > 0.f)) s16 = __float2half_rn(1.0f);
    const float s = __half2float(s16);
    const float rs = __frcp_rn(s);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const float c = fminf(fmaxf(rintf(div_by(x[j], s, rs)), -128.f), 127.f);
      bytes[j] = uint8_t(int8_t(int(c)));
    }
    if (lane == 0) (is_v ? v_scales : k_scales)[slot] = s16;
  }
  if constexpr (VEC && VPL == 8) {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(bytes);
  } else if constexpr (VEC && VPL == 4) {
    *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(bytes);
  } else if constexpr (VEC && VPL == 2) {
    *reinterpret_cast<uint16_t*>(dst) = *reinterpret_cast<const uint16_t*>(bytes);
  } else {
#pragma unroll
    for (int j = 0; j < VPL; ++j) dst[j] = bytes[j];
  }
}

// The same write for rows whose starts are 16-byte aligned (strides multiples of 8 elements, D of 64, 128 or 256):
// a lane takes 8 consecutive values of one head vector with one 16-byte load (two for fp32), so D / 8 lanes cover
// a token's head and a warp 32 / (D / 8) tokens per pass. A warp owns up to kWriteTokens consecutive new tokens of
// one (K or V, sequence, KV head): all their loads and write slots are requested before any is quantized, the
// quotients come in pairs from packed FMAs (the same correctly rounded division as div_by), INT8 codes are rounded
// half to even by the 1.5 * 2^23 magic number after the clamp, and each lane stores its 8 codes as one word.
constexpr int kWriteTokens = 8;

template <int DT>
__device__ __forceinline__ void eight_as_float(const uint8_t* p, float2 (&x)[4]) {
  if constexpr (DT == BPT_DTYPE_F32) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 16);
    x[0] = make_float2(a.x, a.y); x[1] = make_float2(a.z, a.w); x[2] = make_float2(b.x, b.y); x[3] = make_float2(b.z, b.w);
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (DT == BPT_DTYPE_BF16) {
        x[i] = make_float2(__uint_as_float(wv[i] << 16), __uint_as_float(wv[i] & 0xFFFF0000u));
      } else {
        x[i] = __half22float2(*reinterpret_cast<const __half2*>(&wv[i]));
      }
    }
  }
}

// y / b for a pair, correctly rounded (div_by on two lanes): q = RN(y r) (adding -0 keeps the sign of a zero
// product), e = y - q b exactly, RN(q + e r).
__device__ __forceinline__ float2 div_by2(float2 y, float b, float r) {
  const float2 q = ffma2(y, make_float2(r, r), make_float2(-0.f, -0.f));
  const float2 e = ffma2(q, make_float2(-b, -b), y);
  return ffma2(e, make_float2(r, r), q);
}

template <int DT, int D, int KIND>
__global__ void __launch_bounds__(256) paged_kv_write_vec_kernel(
    const void* __restrict__ k, const void* __restrict__ v, int64_t sb, int64_t sh, int64_t sq, int B, int Hkv, int Q,
    const int32_t* __restrict__ wblocks, const int32_t* __restrict__ woffsets, uint8_t* __restrict__ k_pool,
    uint8_t* __restrict__ v_pool, float k_scale, float v_scale, __half* __restrict__ k_scales,
    __half* __restrict__ v_scales, int block_size, int64_t num_blocks) {
  constexpr int LPT = D / 8;                 // lanes per token's head vector
  constexpr int TPP = 32 / LPT;              // tokens per pass
  constexpr int NP = kWriteTokens / TPP;     // passes
  constexpr int ESZ = DT == BPT_DTYPE_F32 ? 4 : 2;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int QG = (Q + kWriteTokens - 1) / kWriteTokens;  // token groups per (sequence, head)
  const int64_t per_tensor = (int64_t)B * Hkv * QG;
  if (wid >= 2 * per_tensor) return;
  pdl_wait();
  const bool is_v = wid >= per_tensor;
  const int64_t idx = is_v ? wid - per_tensor : wid;
  int qg, h, b;
  if (per_tensor < (int64_t(1) << 31)) {  // 32-bit index arithmetic (64-bit division is a long sequence)
    const uint32_t i32 = uint32_t(idx), qh = uint32_t(QG) * uint32_t(Hkv);
    b = int(i32 / qh);
    const uint32_t rest = i32 - uint32_t(b) * qh;
    h = int(rest / uint32_t(QG));
    qg = int(rest - uint32_t(h) * uint32_t(QG));
  } else {
    qg = int(idx % QG);
    h = int((idx / QG) % Hkv);
    b = int(idx / ((int64_t)QG * Hkv));
  }
  const int q0 = qg * kWriteTokens;
  const int nq = min(kWriteTokens, Q - q0);
  const int sub = lane / LPT, li = lane % LPT;
  int32_t my_blk = 0, my_off = 0;  // lane t < nq: token q0 + t's write slot
  if (lane < nq) {
    my_blk = wblocks[(int64_t)b * Q + q0 + lane];
    my_off = woffsets[(int64_t)b * Q + q0 + lane];
  }
  const uint8_t* src = static_cast<const uint8_t*>(is_v ? v : k) +
                       ((int64_t)b * sb + (int64_t)h * sh + (int64_t)q0 * sq + li * 8) * ESZ;
  float2 x[NP][4];
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int t = p * TPP + sub;
    if (t < nq) {
      eight_as_float<DT>(src + (int64_t)t * sq * ESZ, x[p]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) x[p][i] = make_float2(0.f, 0.f);
    }
  }
  uint8_t* pool = is_v ? v_pool : k_pool;
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int t = p * TPP + sub;
    const int32_t blk = __shfl_sync(0xffffffffu, my_blk, t < nq ? t : 0);
    const int32_t off = __shfl_sync(0xffffffffu, my_off, t < nq ? t : 0);
    const bool bad = blk < 0 || blk >= num_blocks || off < 0 || off >= block_size;
    const int64_t slot = ((int64_t)blk * block_size + off) * Hkv + h;
    uint2 word;
    if constexpr (KIND == BPT_KV_FP8) {
      const float s = is_v ? v_scale : k_scale;
      const float rs = __frcp_rn(s);
      uint16_t c[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 y = div_by2(x[p][i], s, rs);  // with x's sign restored on a zero quotient (E4M3 keeps -0)
        c[i] = float2_to_e4m3x2(copysignf(y.x, x[p][i].x), copysignf(y.y, x[p][i].y));
      }
      word = make_uint2(uint32_t(c[0]) | (uint32_t(c[1]) << 16), uint32_t(c[2]) | (uint32_t(c[3]) << 16));
    } else {
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fmaxf(fabsf(x[p][i].x), fabsf(x[p][i].y)));
#pragma unroll
      for (int o = LPT / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      __half s16 = __float2half_rn(__fdiv_rn(amax, 127.0f));
      if (!(__half2float(s16) > 0.f)) s16 = __float2half_rn(1.0f);
      const float s = __half2float(s16);
      const float rs = __frcp_rn(s);
      uint32_t t4[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 y = div_by2(x[p][i], s, rs);
        y.x = fminf(fmaxf(y.x, -128.f), 127.f);
        y.y = fminf(fmaxf(y.y, -128.f), 127.f);
        // y + 1.5 * 2^23 rounds y to an integer half to even; its low byte is the code (two's complement)
        const float2 m = ffma2(y, make_float2(1.f, 1.f), make_float2(12582912.f, 12582912.f));
        t4[2 * i] = __float_as_uint(m.x);
        t4[2 * i + 1] = __float_as_uint(m.y);
      }
      word = make_uint2(__byte_perm(__byte_perm(t4[0], t4[1], 0x0040), __byte_perm(t4[2], t4[3], 0x0040), 0x5410),
                        __byte_perm(__byte_perm(t4[4], t4[5], 0x0040), __byte_perm(t4[6], t4[7], 0x0040), 0x5410));
      if (li == 0 && t < nq && !bad) (is_v ? v_scales : k_scales)[slot] = s16;
    }
    if (t < nq) {
      if (bad) {
        if (li == 0) record_error(blk < 0 || blk >= num_blocks ? kDevErrBlockIndex : kDevErrSlotIndex);
      } else {
        *reinterpret_cast<uint2*>(pool + slot * D + li * 8) = word;
      }
    }
  }
}

template <int DT>
int paged_write_dt(const void* k, const void* v, int64_t sb, int64_t sh, int64_t sq, int64_t B, int64_t Hkv,
                   int64_t Q, int64_t D, const int32_t* wb, const int32_t* wo, void* kp, void* vp, int kind, float ks,
                   float vs, void* kss, void* vss, int64_t bs, int64_t nb, cudaStream_t stream) {
  const int64_t warps = 2 * B * Hkv * Q;
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  BPT_REQUIRE(blocks < (1ll << 31), BPT_ERR_INVALID, "paged kv write: too many tokens");
  // vector accesses: every row start (and each lane's VPL values) aligned to the vector, pools to the code word
  const int64_t vpl = D / 32, esz = DT == BPT_DTYPE_F32 ? 4 : 2;
  const int64_t vbytes = std::min<int64_t>(vpl * esz, 16);
  auto al = [](const void* p, int64_t n) { return (reinterpret_cast<uintptr_t>(p) % uintptr_t(n)) == 0; };
  const bool vec = sb % vpl == 0 && sh % vpl == 0 && sq % vpl == 0 && al(k, vbytes) && al(v, vbytes) &&
                   al(kp, vpl) && al(vp, vpl);
  // rows that start on 16 bytes and at least 4 new tokens per sequence: eight values per lane, up to kWriteTokens
  // tokens per warp (one or two tokens, as in a decode step, keep one warp per token: measured faster there)
  if (Q >= 4 && (D == 64 || D == 128 || D == 256) && sb % 8 == 0 && sh % 8 == 0 && sq % 8 == 0 && al(k, 16) && al(v, 16) &&
      al(kp, 8) && al(vp, 8)) {
    const int64_t vwarps = 2 * B * Hkv * ((Q + kWriteTokens - 1) / kWriteTokens);
    const int64_t vblocks = (vwarps * 32 + threads - 1) / threads;
#define BPT_KVW8(DD, KIND)                                                                                         \
  paged_kv_write_vec_kernel<DT, DD, KIND><<<unsigned(vblocks), threads, 0, stream>>>(                              \
      k, v, sb, sh, sq, int(B), int(Hkv), int(Q), wb, wo, static_cast<uint8_t*>(kp), static_cast<uint8_t*>(vp), ks,  \
      vs, static_cast<__half*>(kss), static_cast<__half*>(vss), int(bs), nb)
    if (kind == BPT_KV_FP8) {
      if (D == 64) BPT_KVW8(64, BPT_KV_FP8);
      else if (D == 128) BPT_KVW8(128, BPT_KV_FP8);
      else BPT_KVW8(256, BPT_KV_FP8);
    } else {
      if (D == 64) BPT_KVW8(64, BPT_KV_INT8);
      else if (D == 128) BPT_KVW8(128, BPT_KV_INT8);
      else BPT_KVW8(256, BPT_KV_INT8);
    }
#undef BPT_KVW8
    return check_launch("paged kv write");
  }
#define BPT_KVW(VPL, KIND)                                                                                        \
  if (vec)                                                                                                        \
    paged_kv_write_kernel<DT, VPL, KIND, true><<<unsigned(blocks), threads, 0, stream>>>(                         \
        k, v, sb, sh, sq, int(B), int(Hkv), int(Q), wb, wo, static_cast<uint8_t*>(kp), static_cast<uint8_t*>(vp),   \
        ks, vs, static_cast<__half*>(kss), static_cast<__half*>(vss), int(bs), nb);                               \
  else                                                                                                            \
    paged_kv_write_kernel<DT, VPL, KIND, false><<<unsigned(blocks), threads, 0, stream>>>(                        \
        k, v, sb, sh, sq, int(B), int(Hkv), int(Q), wb, wo, static_cast<uint8_t*>(kp), static_cast<uint8_t*>(vp),   \
        ks, vs, static_cast<__half*>(kss), static_cast<__half*>(vss), int(bs), nb)
  if (kind == BPT_KV_FP8) {
    if (D == 64) BPT_KVW(2, BPT_KV_FP8);
    else if (D == 128) BPT_KVW(4, BPT_KV_FP8);
    else BPT_KVW(8, BPT_KV_FP8);
  } else {
    if (D == 64) BPT_KVW(2, BPT_KV_INT8);
    else if (D == 128) BPT_KVW(4, BPT_KV_INT8);
    else BPT_KVW(8, BPT_KV_INT8);
  }
#undef BPT_KVW
  return check_launch("paged kv write");
}

// ---- KIVI -----------------------------------------------------------------------------------------------------

// Keys: per (b, h, group, channel c) over `group` tokens. With bits 4 the thread owns channels c and c + D/2.
template <int DT>
__global__ void kivi_keys_kernel(const void* __restrict__ k, int B, int Hkv, int T, int D, int bits, int group,
                                 uint8_t* __restrict__ codes, __half* __restrict__ kscale, __half* __restrict__ kzero,
                                 int64_t t_max, int64_t n_groups, int64_t t0) {
  const int per_group = bits == 4 ? D / 2 : D;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)B * Hkv * (T / group) * per_group;
  if (tid >= total) return;
  int c, gi, h, b;
  if (total < (int64_t(1) << 31)) {  // 32-bit index arithmetic (64-bit division is a long sequence)
    const uint32_t i = uint32_t(tid), pg = uint32_t(per_group), ng = uint32_t(T / group);
    const uint32_t r1 = i / pg, r2 = r1 / ng;
    c = int(i - r1 * pg);
    gi = int(r1 - r2 * ng);
    b = int(r2 / uint32_t(Hkv));
    h = int(r2 - uint32_t(b) * uint32_t(Hkv));
  } else {
    c = int(tid % per_group);
    gi = int((tid / per_group) % (T / group));
    h = int((tid / ((int64_t)per_group * (T / group))) % Hkv);
    b = int(tid / ((int64_t)per_group * (T / group) * Hkv));
  }
  const float qmax = float((1 << bits) - 1);
  const int nch = bits == 4 ? 2 : 1;
  uint8_t out_codes[2][64];  // at most group 64 tokens per thread
  for (int ch = 0; ch < nch; ++ch) {
    const int d = c + ch * (D / 2);
    const int64_t src0 = (((int64_t)b * Hkv + h) * T + (int64_t)gi * group) * D + d;
    float lo = 0.f, hi = 0.f;
    for (int t = 0; t < group; ++t) {
      const float x = load_as_float<DT>(k, src0 + (int64_t)t * D);
      lo = fminf(lo, x);
      hi = fmaxf(hi, x);
    }
    __half s16 = __float2half_rn(__fdiv_rn(hi - lo, qmax));
    if (!(__half2float(s16) > 0.f)) s16 = __float2half_rn(1.0f);
    const float s = __half2float(s16);
    const float rs = __frcp_rn(s);
    const float z = fminf(fmaxf(rintf(div_by(-lo, s, rs)), 0.f), qmax);
    const int64_t g_out = ((int64_t)b * Hkv + h) * n_groups + (t0 / group) + gi;
    kscale[g_out * D + d] = s16;
    kzero[g_out * D + d] = __float2half_rn(z);
    for (int t = 0; t < group; ++t) {
      const float x = load_as_float<DT>(k, src0 + (int64_t)t * D);
      out_codes[ch][t] = uint8_t(fminf(fmaxf(rintf(div_by(x, s, rs)) + z, 0.f), qmax));
    }
  }
  const int row_bytes = bits == 4 ? D / 2 : D;
  for (int t = 0; t < group; ++t) {
    const int64_t tok = t0 + (int64_t)gi * group + t;
    const uint8_t byte = bits == 4 ? uint8_t(out_codes[0][t] | (out_codes[1][t] << 4)) : out_codes[0][t];
    codes[(((int64_t)b * Hkv + h) * t_max + tok) * row_bytes + c] = byte;
  }
}

// Values: one warp per (b, h, token) over the head vector.
template <int DT>
__global__ void kivi_values_kernel(const void* __restrict__ v, int B, int Hkv, int T, int D, int bits,
                                   uint8_t* __restrict__ codes, __half* __restrict__ vscale, __half* __restrict__ vzero,
                                   int64_t t_max, int64_t t0) {
  __shared__ uint8_t stage[8][256];
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int64_t total = (int64_t)B * Hkv * T;
  if (wid >= total) return;  // whole warps exit together (blockDim a multiple of 32)
  int t;
  int64_t bh;
  if (total < (int64_t(1) << 31)) {  // 32-bit index arithmetic
    const uint32_t w = uint32_t(wid), q = w / uint32_t(T);
    bh = q;
    t = int(w - q * uint32_t(T));
  } else {
    t = int(wid % T);
    bh = wid / T;
  }
  const int64_t src0 = (bh * T + t) * D;
  float lo = 0.f, hi = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float x = load_as_float<DT>(v, src0 + d);
    lo = fminf(lo, x);
    hi = fmaxf(hi, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  const float qmax = float((1 << bits) - 1);
  __half s16 = __float2half_rn(__fdiv_rn(hi - lo, qmax));
  if (!(__half2float(s16) > 0.f)) s16 = __float2half_rn(1.0f);
  const float s = __half2float(s16);
  const float rs = __frcp_rn(s);
  const float z = fminf(fmaxf(rintf(div_by(-lo, s, rs)), 0.f), qmax);
  for (int d = lane; d < D; d += 32) {
    const float x = load_as_float<DT>(v, src0 + d);
    stage[wl][d] = uint8_t(fminf(fmaxf(rintf(div_by(x, s, rs)) + z, 0.f), qmax));
  }
  __syncwarp();
  const int64_t tok = t0 + t;
  const int row_bytes = bits == 4 ? D / 2 : D;
  uint8_t* dst = codes + (bh * t_max + tok) * row_bytes;
  for (int j = lane; j < row_bytes; j += 32)
    dst[j] = bits == 4 ? uint8_t(stage[wl][j] | (stage[wl][j + D / 2] << 4)) : stage[wl][j];
  if (lane == 0) {
    vscale[bh * t_max + tok] = s16;
    vzero[bh * t_max + tok] = __float2half_rn(z);
  }
}

// Fast paths for the configs' shape (D = 128, groups of 32 tokens, 16-bit inputs, aligned buffers), with the same
// grid and code arithmetic as the kernels above (so the same bits).
// Two 16-bit values of a packed word as floats (low half first).
template <int DT>
__device__ __forceinline__ float2 pair_as_float(uint32_t w) {
  if constexpr (DT == BPT_DTYPE_BF16) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// Packed 16-bit minimum / maximum of two words: exact, and a NaN loses to a number, as with fminf / fmaxf.
template <int DT>
__device__ __forceinline__ uint32_t min16x2(uint32_t a, uint32_t b) {
  if constexpr (DT == BPT_DTYPE_BF16) {
    const __nv_bfloat162 r = __hmin2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  } else {
    const __half2 r = __hmin2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
}
template <int DT>
__device__ __forceinline__ uint32_t max16x2(uint32_t a, uint32_t b) {
  if constexpr (DT == BPT_DTYPE_BF16) {
    const __nv_bfloat162 r = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  } else {
    const __half2 r = __hmax2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
}

// y / b for a pair with a divisor per lane, correctly rounded (div_by on two lanes).
__device__ __forceinline__ float2 div_by2v(float2 y, float2 b, float2 r) {
  const float2 q = ffma2(y, r, make_float2(-0.f, -0.f));
  const float2 e = ffma2(q, make_float2(-b.x, -b.y), y);
  return ffma2(e, r, q);
}

// The codes of a pair, clamp(rint(x / s) + z, 0, qmax) with the correctly rounded quotient, as
// rint(clamp(x / s, -z, qmax - z)) + z (the same integer: z and the bounds are integers, and a NaN quotient gives 0 in
// both); the rounding is the 1.5 * 2^23 magic number, whose bits less those of 1.5 * 2^23 are rint(y).
__device__ __forceinline__ void kivi_code2(float2 x, float2 s, float2 rs, float2 z, float qmax, uint32_t& c0,
                                           uint32_t& c1) {
  float2 y = div_by2v(x, s, rs);
  y.x = fminf(fmaxf(y.x, -z.x), qmax - z.x);
  y.y = fminf(fmaxf(y.y, -z.y), qmax - z.y);
  const float2 m = ffma2(y, make_float2(1.f, 1.f), make_float2(12582912.f, 12582912.f));
  c0 = __float_as_uint(m.x) - (0x4B400000u - uint32_t(int(z.x)));
  c1 = __float_as_uint(m.y) - (0x4B400000u - uint32_t(int(z.y)));
}

// Four codes (each below 256) as the bytes of one word, the first lowest.
__device__ __forceinline__ uint32_t pack4(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3) {
  return __byte_perm(__byte_perm(c0, c1, 0x0040), __byte_perm(c2, c3, 0x0040), 0x5410);
}

// Keys: one warp per (sequence, head, group of 32 tokens); lane l owns channels 4l .. 4l + 3, reads its 8 bytes of
// all 32 rows at once (one pass over the input), and writes each token's codes as one word. 4-bit codes pack
// channel d (low nibble) with d + 64 (high), whose codes lane l + 16 holds.
template <int DT, int BITS>
__global__ void __launch_bounds__(128, 4) kivi_keys128_kernel(const void* __restrict__ k, int B, int Hkv, int T,
                                                           uint8_t* __restrict__ codes, __half* __restrict__ kscale,
                                                           __half* __restrict__ kzero, int64_t t_max, int64_t n_groups,
                                                           int64_t t0) {
  constexpr int D = 128, G = 32;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int ng = T / G;
  if (wid >= (int64_t)B * Hkv * ng) return;  // whole warps
  const int64_t bh = wid / ng;
  const int gi = int(wid - bh * ng);
  const uint8_t* src = static_cast<const uint8_t*>(k) + ((bh * T + (int64_t)gi * G) * D + 4 * lane) * 2;
  uint2 raw[G];
#pragma unroll
  for (int t = 0; t < G; ++t) raw[t] = *reinterpret_cast<const uint2*>(src + (int64_t)t * D * 2);
  uint32_t mn[2] = {0u, 0u}, mx[2] = {0u, 0u};  // packed per channel pair; the range always includes 0
#pragma unroll
  for (int t = 0; t < G; ++t) {
    mn[0] = min16x2<DT>(mn[0], raw[t].x);
    mn[1] = min16x2<DT>(mn[1], raw[t].y);
    mx[0] = max16x2<DT>(mx[0], raw[t].x);
    mx[1] = max16x2<DT>(mx[1], raw[t].y);
  }
  float lo[4], hi[4];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const float2 l = pair_as_float<DT>(mn[p]), u = pair_as_float<DT>(mx[p]);
    lo[2 * p] = l.x; lo[2 * p + 1] = l.y;
    hi[2 * p] = u.x; hi[2 * p + 1] = u.y;
  }
  constexpr float qmax = float((1 << BITS) - 1);
  float s[4], rs[4], z[4];
  __half s16[4], z16[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    s16[j] = __float2half_rn(__fdiv_rn(hi[j] - lo[j], qmax));
    if (!(__half2float(s16[j]) > 0.f)) s16[j] = __float2half_rn(1.0f);
    s[j] = __half2float(s16[j]);
    rs[j] = __frcp_rn(s[j]);
    z[j] = fminf(fmaxf(rintf(div_by(-lo[j], s[j], rs[j])), 0.f), qmax);
    z16[j] = __float2half_rn(z[j]);
  }
  const int64_t g_out = (bh * n_groups + t0 / G + gi) * D + 4 * lane;
  *reinterpret_cast<uint2*>(kscale + g_out) =
      make_uint2(uint32_t(__half_as_ushort(s16[0])) | (uint32_t(__half_as_ushort(s16[1])) << 16),
                 uint32_t(__half_as_ushort(s16[2])) | (uint32_t(__half_as_ushort(s16[3])) << 16));
  *reinterpret_cast<uint2*>(kzero + g_out) =
      make_uint2(uint32_t(__half_as_ushort(z16[0])) | (uint32_t(__half_as_ushort(z16[1])) << 16),
                 uint32_t(__half_as_ushort(z16[2])) | (uint32_t(__half_as_ushort(z16[3])) << 16));
  constexpr int row_bytes = BITS == 4 ? D / 2 : D;
  uint8_t* dst = codes + (bh * t_max + t0 + (int64_t)gi * G) * row_bytes + 4 * lane;
#pragma unroll
  for (int t = 0; t < G; ++t) {
    uint32_t c[4];
    kivi_code2(pair_as_float<DT>(raw[t].x), make_float2(s[0], s[1]), make_float2(rs[0], rs[1]), make_float2(z[0], z[1]),
               qmax, c[0], c[1]);
    kivi_code2(pair_as_float<DT>(raw[t].y), make_float2(s[2], s[3]), make_float2(rs[2], rs[3]), make_float2(z[2], z[3]),
               qmax, c[2], c[3]);
    const uint32_t word = pack4(c[0], c[1], c[2], c[3]);
    if constexpr (BITS == 4) {
      const uint32_t up = __shfl_down_sync(0xffffffffu, word, 16);  // channels 4l + 64 .. 4l + 67
      if (lane < 16) *reinterpret_cast<uint32_t*>(dst + (int64_t)t * row_bytes) = word | (up << 4);
    } else {
      *reinterpret_cast<uint32_t*>(dst + (int64_t)t * row_bytes) = word;
    }
  }
}

// Values: one warp per 8 consecutive tokens of a (sequence, head), 16 lanes per token with 8 channels each (one
// 16-byte load), two tokens per pass; min and max over the token's lanes by shuffles. 4-bit codes pack channel d
// (low nibble) with d + 64, held by lane li + 8 of the token's 16.
template <int DT, int BITS>
__global__ void __launch_bounds__(256) kivi_values128_kernel(const void* __restrict__ v, int B, int Hkv, int T,
                                                             uint8_t* __restrict__ codes, __half* __restrict__ vscale,
                                                             __half* __restrict__ vzero, int64_t t_max, int64_t t0) {
  constexpr int D = 128, TW = 8, NP = TW / 2;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int tg = (T + TW - 1) / TW;
  if (wid >= (int64_t)B * Hkv * tg) return;  // whole warps
  const int64_t bh = wid / tg;
  const int tb = int(wid - bh * tg) * TW;
  const int nt = min(TW, T - tb);
  const int sub = lane >> 4, li = lane & 15;
  const uint8_t* src = static_cast<const uint8_t*>(v) + ((bh * T + tb) * D + 8 * li) * 2;
  uint4 raw[NP];
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int t = 2 * p + sub;
    raw[p] = t < nt ? *reinterpret_cast<const uint4*>(src + (int64_t)t * D * 2) : make_uint4(0u, 0u, 0u, 0u);
  }
  constexpr float qmax = float((1 << BITS) - 1);
  constexpr int row_bytes = BITS == 4 ? D / 2 : D;
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int t = 2 * p + sub;
    const uint32_t wv[4] = {raw[p].x, raw[p].y, raw[p].z, raw[p].w};
    // the range: packed 16-bit minima and maxima (the range always includes 0), then (-lo, hi) as one packed word
    // whose maximum the token's 16 lanes share
    uint32_t mn = 0u, mx = 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      mn = min16x2<DT>(mn, wv[q]);
      mx = max16x2<DT>(mx, wv[q]);
    }
    mn = min16x2<DT>(mn, __byte_perm(mn, 0u, 0x1032));  // both halves: the lane's minimum
    mx = max16x2<DT>(mx, __byte_perm(mx, 0u, 0x1032));
    uint32_t nh = __byte_perm(mn ^ 0x80008000u, mx, 0x7610);  // (-lo, hi), exact
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) nh = max16x2<DT>(nh, __shfl_xor_sync(0xffffffffu, nh, o));
    const float2 nhf = pair_as_float<DT>(nh);
    const float lo = -nhf.x, hi = nhf.y;
    __half s16 = __float2half_rn(__fdiv_rn(hi - lo, qmax));
    if (!(__half2float(s16) > 0.f)) s16 = __float2half_rn(1.0f);
    const float s = __half2float(s16);
    const float rs = __frcp_rn(s);
    const float z = fminf(fmaxf(rintf(div_by(-lo, s, rs)), 0.f), qmax);
    uint32_t c[8];  // channels 8 li .. 8 li + 7
#pragma unroll
    for (int q = 0; q < 4; ++q)
      kivi_code2(pair_as_float<DT>(wv[q]), make_float2(s, s), make_float2(rs, rs), make_float2(z, z), qmax, c[2 * q],
                 c[2 * q + 1]);
    const uint32_t w0 = pack4(c[0], c[1], c[2], c[3]), w1 = pack4(c[4], c[5], c[6], c[7]);
    const int64_t row = bh * t_max + t0 + tb + t;
    if constexpr (BITS == 4) {
      const uint32_t u0 = __shfl_down_sync(0xffffffffu, w0, 8), u1 = __shfl_down_sync(0xffffffffu, w1, 8);
      if (t < nt && li < 8) *reinterpret_cast<uint2*>(codes + row * row_bytes + 8 * li) = make_uint2(w0 | (u0 << 4), w1 | (u1 << 4));
    } else {
      if (t < nt) *reinterpret_cast<uint2*>(codes + row * row_bytes + 8 * li) = make_uint2(w0, w1);
    }
    if (t < nt && li == 0) {
      vscale[row] = s16;
      vzero[row] = __float2half_rn(z);
    }
  }
}

template <int DT>
int kivi_quantize_dt(const void* k, const void* v, int64_t B, int64_t Hkv, int64_t T, int64_t D, int bits,
                     int64_t group, void* kc, void* vc, void* ks, void* kz, void* vs, void* vz, int64_t t_max,
                     int64_t n_groups, int64_t t0, cudaStream_t stream) {
  auto al = [](const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
  if (DT != BPT_DTYPE_F32 && D == 128 && group == 32 && al(k, 16) && al(v, 16) && al(kc, 4) && al(vc, 8) &&
      al(ks, 8) && al(kz, 8)) {
    const int64_t kwarps = B * Hkv * (T / 32), vwarps = B * Hkv * ((T + 7) / 8);
    if constexpr (DT != BPT_DTYPE_F32) {
      if (kwarps > 0) {
        if (bits == 4)
          kivi_keys128_kernel<DT, 4><<<unsigned((kwarps * 32 + 127) / 128), 128, 0, stream>>>(
              k, int(B), int(Hkv), int(T), static_cast<uint8_t*>(kc), static_cast<__half*>(ks), static_cast<__half*>(kz),
              t_max, n_groups, t0);
        else
          kivi_keys128_kernel<DT, 8><<<unsigned((kwarps * 32 + 127) / 128), 128, 0, stream>>>(
              k, int(B), int(Hkv), int(T), static_cast<uint8_t*>(kc), static_cast<__half*>(ks), static_cast<__half*>(kz),
              t_max, n_groups, t0);
      }
      if (vwarps > 0) {
        if (bits == 4)
          kivi_values128_kernel<DT, 4><<<unsigned((vwarps * 32 + 255) / 256), 256, 0, stream>>>(
              v, int(B), int(Hkv), int(T), static_cast<uint8_t*>(vc), static_cast<__half*>(vs), static_cast<__half*>(vz),
              t_max, t0);
        else
          kivi_values128_kernel<DT, 8><<<unsigned((vwarps * 32 + 255) / 256), 256, 0, stream>>>(
              v, int(B), int(Hkv), int(T), static_cast<uint8_t*>(vc), static_cast<__half*>(vs), static_cast<__half*>(vz),
              t_max, t0);
      }
    }
    return check_launch("kivi quantize");
  }
  const int per_group = bits == 4 ? int(D / 2) : int(D);
  const int64_t kthreads = B * Hkv * (T / group) * per_group;
  if (kthreads > 0)
    kivi_keys_kernel<DT><<<unsigned((kthreads + 127) / 128), 128, 0, stream>>>(
        k, int(B), int(Hkv), int(T), int(D), bits, int(group), static_cast<uint8_t*>(kc), static_cast<__half*>(ks),
        static_cast<__half*>(kz), t_max, n_groups, t0);
  const int64_t vwarps = B * Hkv * T;
  if (vwarps > 0)
    kivi_values_kernel<DT><<<unsigned((vwarps * 32 + 255) / 256), 256, 0, stream>>>(
        v, int(B), int(Hkv), int(T), int(D), bits, static_cast<uint8_t*>(vc), static_cast<__half*>(vs),
        static_cast<__half*>(vz), t_max, t0);
  return check_launch("kivi quantize");
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" int bpt_paged_kv_write(const void* k, const void* v, int in_dtype, int64_t stride_b, int64_t stride_h,
                                  int64_t stride_q, int64_t B, int64_t Hkv, int64_t Q, int64_t D,
                                  const int32_t* write_blocks, const int32_t* write_offsets, void* k_pool, void* v_pool,
                                  int kind, float k_scale_f32, float v_scale_f32, void* k_scales, void* v_scales,
                                  int64_t block_size, int64_t num_blocks, void* stream) {
  BPT_REQUIRE(k && v && write_blocks && write_offsets && k_pool && v_pool, BPT_ERR_INVALID,
              "paged kv write: null pointer");
  BPT_REQUIRE(kind == BPT_KV_FP8 || (kind == BPT_KV_INT8 && k_scales && v_scales), BPT_ERR_INVALID,
              "paged kv write: kind %d (INT8 needs scale pools)", kind);
  BPT_REQUIRE(D == 64 || D == 128 || D == 256, BPT_ERR_UNSUPPORTED, "paged kv write: D=%lld", (long long)D);
  BPT_REQUIRE(B >= 0 && Hkv >= 1 && Q >= 0 && block_size >= 1 && num_blocks >= 1, BPT_ERR_INVALID,
              "paged kv write: bad shape");
  BPT_REQUIRE(kind != BPT_KV_FP8 || (k_scale_f32 > 0.f && v_scale_f32 > 0.f), BPT_ERR_INVALID,
              "paged kv write: FP8 scales must be positive");
  if (B == 0 || Q == 0) return BPT_OK;
  auto s = static_cast<cudaStream_t>(stream);
  switch (in_dtype) {
    case BPT_DTYPE_F32:
      return paged_write_dt<BPT_DTYPE_F32>(k, v, stride_b, stride_h, stride_q, B, Hkv, Q, D, write_blocks, write_offsets,
                                           k_pool, v_pool, kind, k_scale_f32, v_scale_f32, k_scales, v_scales,
                                           block_size, num_blocks, s);
    case BPT_DTYPE_F16:
      return paged_write_dt<BPT_DTYPE_F16>(k, v, stride_b, stride_h, stride_q, B, Hkv, Q, D, write_blocks, write_offsets,
                                           k_pool, v_pool, kind, k_scale_f32, v_scale_f32, k_scales, v_scales,
                                           block_size, num_blocks, s);
    case BPT_DTYPE_BF16:
      return paged_write_dt<BPT_DTYPE_BF16>(k, v, stride_b, stride_h, stride_q, B, Hkv, Q, D, write_blocks,
                                            write_offsets, k_pool, v_pool, kind, k_scale_f32, v_scale_f32, k_scales,
                                            v_scales, block_size, num_blocks, s);
  }
  return set_error(BPT_ERR_INVALID, "paged kv write: dtype %d", in_dtype);
}

extern "C" int bpt_kivi_quantize(const void* k, const void* v, int in_dtype, int64_t B, int64_t Hkv, int64_t T,
                                 int64_t D, int bits, int64_t group, void* k_codes, void* v_codes, void* k_scale,
                                 void* k_zero, void* v_scale, void* v_zero, int64_t t_max, int64_t n_groups, int64_t t0,
                                 void* stream) {
  BPT_REQUIRE(k && v && k_codes && v_codes && k_scale && k_zero && v_scale && v_zero, BPT_ERR_INVALID,
              "kivi quantize: null pointer");
  BPT_REQUIRE(bits == 4 || bits == 8, BPT_ERR_INVALID, "kivi quantize: bits %d (4 or 8)", bits);
  BPT_REQUIRE(group >= 1 && group <= 64 && T % group == 0 && t0 % group == 0, BPT_ERR_INVALID,
              "kivi quantize: T=%lld and t0=%lld must be whole groups of %lld (group <= 64)", (long long)T,
              (long long)t0, (long long)group);
  BPT_REQUIRE(D >= 2 && D <= 256 && D % 2 == 0, BPT_ERR_UNSUPPORTED, "kivi quantize: D=%lld", (long long)D);
  BPT_REQUIRE(t0 + T <= t_max && (t0 + T) / group <= n_groups, BPT_ERR_INVALID, "kivi quantize: writes past the cache");
  auto s = static_cast<cudaStream_t>(stream);
  switch (in_dtype) {
    case BPT_DTYPE_F32:
      return kivi_quantize_dt<BPT_DTYPE_F32>(k, v, B, Hkv, T, D, bits, group, k_codes, v_codes, k_scale, k_zero, v_scale,
                                             v_zero, t_max, n_groups, t0, s);
    case BPT_DTYPE_F16:
      return kivi_quantize_dt<BPT_DTYPE_F16>(k, v, B, Hkv, T, D, bits, group, k_codes, v_codes, k_scale, k_zero, v_scale,
                                             v_zero, t_max, n_groups, t0, s);
    case BPT_DTYPE_BF16:
      return kivi_quantize_dt<BPT_DTYPE_BF16>(k, v, B, Hkv, T, D, bits, group, k_codes, v_codes, k_scale, k_zero,
                                              v_scale, v_zero, t_max, n_groups, t0, s);
  }
  return set_error(BPT_ERR_INVALID, "kivi quantize: dtype %d", in_dtype);
}
