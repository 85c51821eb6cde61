// The decode step's small ops around the hot path, fused (the caller side of the path: config 5's Qwen3 step).
//
// rms_norm_residual: h' = h + delta (bf16, optional), x = weight * bf16(h' * rsqrt(mean(h'^2) + eps)) with the
//   statistics in fp32 — engine/model.py:24-36 (RMSNorm) and the residual adds of DecoderLayer.forward
//   (:109-111), each rounding where the reference's tensors round. One CTA per row.
// qk_norm_rope_kv_write: for one new token per sequence, from the fused q/k/v projection output:
//   q head: RMSNorm over head_dim (q_norm), rotate-half RoPE (engine/rope.py:31-43) -> q_out (bf16);
//   k head: RMSNorm (k_norm), RoPE, then the FP8 E4M3 store x / k_scale at slot (block, offset) of the pool;
//   v head: the FP8 store only.
//   One warp per (sequence, head); head_dim 128 (4 elements per lane; the rotate-half partner of lane l's
//   elements sits in lane l ^ 16). Every bf16 rounding of the reference's tensors is kept: normalised values,
//   times the norm weight, x * cos, rot * sin, their sum.
#include "common.cuh"

namespace bpt {
namespace {

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 rn(float v) { return __float2bfloat16_rn(v); }

template <int kThreads>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) s += red[w];  // every thread adds in the same order
  __syncthreads();
  return s;
}

// h, delta, h_out, x_out: [rows, hidden] bf16 (row stride = hidden); weight [hidden] bf16; hidden % 8 == 0.
constexpr int kNormThreads = 256;
__global__ void __launch_bounds__(kNormThreads) rms_norm_residual_kernel(
    const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ delta,
    const __nv_bfloat16* __restrict__ weight, __nv_bfloat16* __restrict__ h_out, __nv_bfloat16* __restrict__ x_out,
    int hidden, float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* hr = h + row * hidden;
  constexpr int kMaxPer = 8;  // up to 8 x 8 x 256 = 16384 features per row in registers
  uint4 hv[kMaxPer];
  float ss = 0.f;
  const int n8 = hidden / 8;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < n8) {
      uint4 u = reinterpret_cast<const uint4*>(hr)[c];
      if (delta) {  // h + delta, rounded to bf16 like the reference's residual tensor
        const uint4 d = reinterpret_cast<const uint4*>(delta + row * hidden)[c];
        const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&u);
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&d);
        uint4 o;
        __nv_bfloat162* r = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) r[e] = __hadd2(a[e], b[e]);
        u = o;
      }
      hv[i] = u;
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p[e]);
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
  }
  const float inv = rsqrtf(block_sum<kNormThreads>(ss, red) / float(hidden) + eps);
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < n8) {
      if (h_out) reinterpret_cast<uint4*>(h_out + row * hidden)[c] = hv[i];
      const uint4 wv = reinterpret_cast<const uint4*>(weight)[c];
      const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(&hv[i]);
      const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(&wv);
      uint4 o;
      __nv_bfloat16* r = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = rn(bf(w[e]) * bf(rn(bf(p[e]) * inv)));
      reinterpret_cast<uint4*>(x_out + row * hidden)[c] = o;
    }
  }
}

struct QkArgs {
  const __nv_bfloat16* qkv;  // [B, ld]: q heads, then k heads, then v heads, D each
  int64_t ld;
  const __nv_bfloat16* q_norm;  // [D]
  const __nv_bfloat16* k_norm;  // [D]
  const __nv_bfloat16* cos;     // [B, D]
  const __nv_bfloat16* sin;     // [B, D]
  __nv_bfloat16* q_out;         // [B, Hq, D]
  const int32_t* blocks;        // [B]
  const int32_t* offsets;       // [B]
  uint8_t* k_pool;              // [num_blocks, block_size, Hkv, D]
  uint8_t* v_pool;
  float k_scale, v_scale, eps;
  int B, Hq, Hkv, block_size, num_blocks;
};

constexpr int kHeadDim = 128;

__global__ void __launch_bounds__(256) qk_norm_rope_kv_write_kernel(const QkArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int item = int(blockIdx.x) * 8 + int(threadIdx.x >> 5);
  const int heads = a.Hq + 2 * a.Hkv;
  if (item >= a.B * heads) return;  // whole warps leave together
  const int b = item / heads, slot = item - b * heads;
  const int e0 = 4 * lane;  // this lane's elements e0 .. e0 + 3
  const uint2 raw = *reinterpret_cast<const uint2*>(a.qkv + int64_t(b) * a.ld + int64_t(slot) * kHeadDim + e0);
  const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&raw);
  float x[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) x[e] = bf(xv[e]);
  const bool is_v = slot >= a.Hq + a.Hkv;
  if (!is_v) {
    // RMSNorm over the head (fp32 statistics), rounded, times the norm weight, rounded
    const float inv = rsqrtf(warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]) / float(kHeadDim) + a.eps);
    const __nv_bfloat16* w = (slot < a.Hq ? a.q_norm : a.k_norm) + e0;
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = bf(rn(bf(w[e]) * bf(rn(x[e] * inv))));
    // rotate-half RoPE: rot = (-x[i + 64] for i < 64, x[i - 64] above), out = x cos + rot sin, each rounded
    float partner[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const __nv_bfloat16* cs = a.cos + int64_t(b) * kHeadDim + e0;
    const __nv_bfloat16* sn = a.sin + int64_t(b) * kHeadDim + e0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float rot = lane < 16 ? -partner[e] : partner[e];
      x[e] = bf(rn(bf(rn(x[e] * bf(cs[e]))) + bf(rn(rot * bf(sn[e])))));
    }
  }
  if (slot < a.Hq) {
    uint2 o;
    __nv_bfloat16* r = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) r[e] = rn(x[e]);
    *reinterpret_cast<uint2*>(a.q_out + (int64_t(b) * a.Hq + slot) * kHeadDim + e0) = o;
    return;
  }
  // the FP8 store: x / scale rounded to E4M3 with saturation (as the paged KV write)
  const int blk = a.blocks[b], off = a.offsets[b];
  if (blk < 0 || blk >= a.num_blocks) {
    if (lane == 0) record_error(kDevErrBlockIndex);
    return;
  }
  if (off < 0 || off >= a.block_size) {
    if (lane == 0) record_error(kDevErrSlotIndex);
    return;
  }
  const int h = is_v ? slot - a.Hq - a.Hkv : slot - a.Hq;
  const float s = is_v ? a.v_scale : a.k_scale;
  const uint16_t lo = float2_to_e4m3x2(__fdiv_rn(x[0], s), __fdiv_rn(x[1], s));
  const uint16_t hi = float2_to_e4m3x2(__fdiv_rn(x[2], s), __fdiv_rn(x[3], s));
  uint8_t* pool = is_v ? a.v_pool : a.k_pool;
  *reinterpret_cast<uint32_t*>(pool + ((int64_t(blk) * a.block_size + off) * a.Hkv + h) * kHeadDim + e0) =
      uint32_t(lo) | (uint32_t(hi) << 16);
}

int launch_pdl(const void* kernel, dim3 grid, dim3 block, void** args, int flags, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BPT_FLAG_PDL) ? 1 : 0;
  const cudaError_t err = cudaLaunchKernelExC(&cfg, kernel, args);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "decode fused launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" int bpt_rms_norm_residual(const void* h, const void* delta, const void* weight, void* h_out, void* x_out,
                                     int64_t rows, int64_t hidden, float eps, int flags, void* stream) {
  BPT_REQUIRE(h && weight && x_out, BPT_ERR_INVALID, "rms_norm_residual: null pointer argument");
  BPT_REQUIRE(rows >= 1 && rows < (1ll << 31), BPT_ERR_INVALID, "rms_norm_residual: rows=%lld", (long long)rows);
  BPT_REQUIRE(hidden >= 8 && hidden % 8 == 0 && hidden <= 8 * 8 * kNormThreads, BPT_ERR_UNSUPPORTED,
              "rms_norm_residual: hidden=%lld must be a multiple of 8 up to 16384", (long long)hidden);
  BPT_REQUIRE(aligned16(h) && aligned16(weight) && aligned16(x_out) && (!delta || aligned16(delta)) &&
                  (!h_out || aligned16(h_out)),
              BPT_ERR_ALIGNMENT, "rms_norm_residual: tensors must be 16-byte aligned");
  const __nv_bfloat16* hp = static_cast<const __nv_bfloat16*>(h);
  const __nv_bfloat16* dp = static_cast<const __nv_bfloat16*>(delta);
  const __nv_bfloat16* wp = static_cast<const __nv_bfloat16*>(weight);
  __nv_bfloat16* hop = static_cast<__nv_bfloat16*>(h_out);
  __nv_bfloat16* xop = static_cast<__nv_bfloat16*>(x_out);
  int hid = int(hidden);
  void* args[] = {&hp, &dp, &wp, &hop, &xop, &hid, &eps};
  return launch_pdl(reinterpret_cast<const void*>(rms_norm_residual_kernel), dim3(unsigned(rows)),
                    dim3(kNormThreads), args, flags, static_cast<cudaStream_t>(stream));
}

extern "C" int bpt_qk_norm_rope_kv_write(const void* qkv, int64_t ld, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                         const void* q_norm, const void* k_norm, const void* cos, const void* sin,
                                         float eps, void* q_out, const int32_t* write_blocks,
                                         const int32_t* write_offsets, void* k_pool, void* v_pool, float k_scale,
                                         float v_scale, int64_t block_size, int64_t num_blocks, int flags,
                                         void* stream) {
  BPT_REQUIRE(qkv && q_norm && k_norm && cos && sin && q_out && write_blocks && write_offsets && k_pool && v_pool,
              BPT_ERR_INVALID, "qk_norm_rope_kv_write: null pointer argument");
  BPT_REQUIRE(D == kHeadDim, BPT_ERR_UNSUPPORTED, "qk_norm_rope_kv_write: head_dim %lld (128 only)", (long long)D);
  BPT_REQUIRE(B >= 1 && Hq >= 1 && Hkv >= 1 && B * (Hq + 2 * Hkv) < (1ll << 31), BPT_ERR_INVALID,
              "qk_norm_rope_kv_write: bad shape");
  BPT_REQUIRE(ld >= (Hq + 2 * Hkv) * D && ld % 4 == 0, BPT_ERR_INVALID, "qk_norm_rope_kv_write: ld=%lld",
              (long long)ld);
  BPT_REQUIRE(k_scale > 0.f && v_scale > 0.f, BPT_ERR_INVALID, "qk_norm_rope_kv_write: FP8 scales must be positive");
  BPT_REQUIRE(block_size >= 1 && num_blocks >= 1 && num_blocks < (1ll << 31), BPT_ERR_INVALID,
              "qk_norm_rope_kv_write: bad pool shape");
  BPT_REQUIRE((reinterpret_cast<uintptr_t>(qkv) & 7) == 0 && (reinterpret_cast<uintptr_t>(q_out) & 7) == 0 &&
                  (reinterpret_cast<uintptr_t>(k_pool) & 3) == 0 && (reinterpret_cast<uintptr_t>(v_pool) & 3) == 0,
              BPT_ERR_ALIGNMENT, "qk_norm_rope_kv_write: misaligned tensors");
  QkArgs a;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ld = ld;
  a.q_norm = static_cast<const __nv_bfloat16*>(q_norm);
  a.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.blocks = write_blocks;
  a.offsets = write_offsets;
  a.k_pool = static_cast<uint8_t*>(k_pool);
  a.v_pool = static_cast<uint8_t*>(v_pool);
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.eps = eps;
  a.B = int(B);
  a.Hq = int(Hq);
  a.Hkv = int(Hkv);
  a.block_size = int(block_size);
  a.num_blocks = int(num_blocks);
  const int64_t items = B * (Hq + 2 * Hkv);
  void* args[] = {&a};
  return launch_pdl(reinterpret_cast<const void*>(qk_norm_rope_kv_write_kernel), dim3(unsigned((items + 7) / 8)),
                    dim3(256), args, flags, static_cast<cudaStream_t>(stream));
}
