// Paged decode attention over an FP8 (E4M3, per-tensor scale) or INT8 (fp16 scale per token and KV head)
// KV cache, with GQA head sharing and split-K.
//
// Grid (n_splits, B): one CTA per (sequence, split of `split` tokens), one warp per KV head, so every cached
// byte is read once and serves the REP query heads of its KV head. The pool layout is the reference's
// [num_blocks, block_size, Hkv, D]: a page of all KV heads is one contiguous block, so each page of K and of
// V (and, for INT8, its scales) arrives with one cp.async.bulk (TMA engine) into a ring of shared-memory
// stages. The block table is read on the device; the last warp to finish a stage refills it with the page
// NST ahead, so nothing waits on a dedicated producer.
//
// Per page and warp: QK with D/16 lanes per token (16 bytes = 16 codes per lane, dequantized in registers,
// packed fp32x2 FMAs, a shuffle reduction), an online softmax in base 2 (log2(e), the softmax scale and the
// FP8 key scale folded into q; the INT8 key scale applied per token), the weights published to shared memory,
// then PV with D/32 dims per lane (the INT8 value scale folded into the weight, the FP8 one into the epilogue).
//
// Outputs: either the per-split partials (out f32 [B, Hq, S, D], lse f32 [B, Hq, S]: the contract of the
// reference's kernel 2), or the merged attention: every CTA of a sequence with more than one split stores
// its partial in the workspace, takes a ticket from an atomic counter, and the last one merges (exactly
// reference.merge_partials) and resets the counter. No CTA ever waits on another.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math_constants.h>

#include <cstring>

#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"

namespace bpt {
namespace {

constexpr int kBS = 16;  // tokens per page
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct PagedArgs {
  const void* q;
  int q_dtype;
  int64_t q_sb, q_sh;
  const uint8_t* k_pool;
  const uint8_t* v_pool;
  float k_scale, v_scale;
  const __half* k_scales;
  const __half* v_scales;
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* lengths;
  int B, Hq, Hkv;
  int64_t num_blocks;
  int split, n_splits;
  float sm_scale;
  // partial mode
  float* out_partial;
  float* lse_partial;
  // merge mode
  int merge;
  void* out;
  int out_dtype;
  float* ws_out;           // [B][n_splits][Hq][D]
  float* ws_lse;           // [B][n_splits][Hq]
  unsigned int* ws_count;  // tickets: [B] (split kernels) or [B][Hkv] (persistent kernel)
  // layout
  int page_bytes;   // kBS * Hkv * D
  int scale_bytes;  // kBS * Hkv * 2 (INT8) or 0
  int nst;          // pipeline stages
  // persistent kernel
  int early;          // BPT_FLAG_KV_READY under PDL: map the pages and copy them before waiting on the predecessor
  int persist_ctas;   // CTAs (one per SM)
  int max_cta_pages;  // capacity of a CTA's page list
  int stall;          // BPT_FLAG_TEST_STALL: CTA 0's producer stops before one page (bounded-wait tests)
  uint64_t wait_ns;   // limit of every wait on a page's arrival
};

__device__ __forceinline__ float q_load(const void* q, int dt, int64_t i) {
  if (dt == BPT_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(q)[i]);
  if (dt == BPT_DTYPE_F16) return __half2float(static_cast<const __half*>(q)[i]);
  return static_cast<const float*>(q)[i];
}

__device__ __forceinline__ void out_store(void* o, int dt, int64_t i, float v) {
  if (dt == BPT_DTYPE_BF16)
    static_cast<__nv_bfloat16*>(o)[i] = __float2bfloat16_rn(v);
  else if (dt == BPT_DTYPE_F16)
    static_cast<__half*>(o)[i] = __float2half_rn(v);
  else
    static_cast<float*>(o)[i] = v;
}

// Four stored bytes -> four fp32 values (before any scale).
template <int KIND>
__device__ __forceinline__ void dequant4(uint32_t w, float* f) {
  if constexpr (KIND == BPT_KV_FP8) {
    const float2 a = e4m3x2_to_float2(uint16_t(w & 0xFFFFu));
    const float2 b = e4m3x2_to_float2(uint16_t(w >> 16));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
  } else {
    // int8 -> fp32 exactly: the byte, sign bit flipped, becomes the low mantissa byte of 2^23 + 128 + v.
    const uint32_t u = w ^ 0x80808080u;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      f[j] = __uint_as_float(__byte_perm(u, 0x4B000000u, j | 0x7440u)) - 8388736.0f;
  }
}

template <int D, int REP, int KIND>
__global__ void __launch_bounds__(512) paged_attn_kernel(const PagedArgs a) {
  constexpr int LPT = D / 16;    // lanes per token in QK
  constexpr int TPS = 32 / LPT;  // tokens per QK step
  constexpr int STEPS = kBS / TPS;
  constexpr int DPL = D / 32;  // dims per lane in PV
  static_assert(kBS % TPS == 0, "page must be a whole number of QK steps");

  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.y, s = blockIdx.x;
  const int h = warp;  // KV head

  pdl_launch_dependents();
  pdl_wait();  // the KV write of this step, the block table and the lengths come from earlier work

  const int L = a.lengths[b];
  const int t0 = s * a.split;
  const int t1 = min(L, t0 + a.split);
  const int nsplit_b = min(a.n_splits, (L + a.split - 1) / a.split);

  if (t0 >= t1) {  // nothing in this split
    if (!a.merge) {
      for (int i = tid; i < a.Hq * D; i += blockDim.x) {
        const int hq = i / D, d = i % D;
        a.out_partial[(((int64_t)b * a.Hq + hq) * a.n_splits + s) * D + d] = 0.f;
        if (d == 0) a.lse_partial[((int64_t)b * a.Hq + hq) * a.n_splits + s] = -CUDART_INF_F;
      }
    } else if (s == 0) {  // an empty sequence: its attention output is 0
      for (int i = tid; i < a.Hq * D; i += blockDim.x) out_store(a.out, a.out_dtype, (int64_t)b * a.Hq * D + i, 0.f);
    }
    return;
  }

  const int stage_bytes = 2 * (a.page_bytes + a.scale_bytes);
  uint8_t* stages = smem;
  float* pbuf = reinterpret_cast<float*>(smem + a.nst * stage_bytes);  // [Hkv][kBS][REP]
  uint64_t* bars = reinterpret_cast<uint64_t*>(pbuf + a.Hkv * kBS * REP);
  int* consumed = reinterpret_cast<int*>(bars + a.nst);
  int* valid = consumed + a.nst;
  int* issued = valid + a.nst;  // pages issued into each stage so far
  int* ticket = issued + a.nst;

  const int p_first = t0 / kBS;
  const int npages = (t1 - 1) / kBS - p_first + 1;
  const int32_t* table = a.block_table + (int64_t)b * a.bt_stride;

  // Issue page i into its stage (called by one thread).
  auto issue = [&](int i) {
    const int st = i % a.nst;
    uint8_t* base = stages + st * stage_bytes;
    issued[st] += 1;
    // A page past the table's row, or an entry outside the pool, is recorded and skipped, never addressed.
    const int32_t blk = (p_first + i < a.bt_stride) ? table[p_first + i] : -1;
    if (blk < 0 || blk >= a.num_blocks) {
      record_error(kDevErrBlockIndex);
      valid[st] = 0;
      mbar_arrive_expect_tx(&bars[st], 0);
      return;
    }
    valid[st] = 1;
    const uint32_t bytes = 2u * uint32_t(a.page_bytes + a.scale_bytes);
    mbar_arrive_expect_tx(&bars[st], bytes);
    const uint64_t policy = l2_policy_evict_first();
    bulk_g2s_evict_first(base, a.k_pool + (int64_t)blk * a.page_bytes, a.page_bytes, &bars[st], policy);
    bulk_g2s_evict_first(base + a.page_bytes, a.v_pool + (int64_t)blk * a.page_bytes, a.page_bytes, &bars[st],
                         policy);
    if constexpr (KIND == BPT_KV_INT8) {
      const uint8_t* ks = reinterpret_cast<const uint8_t*>(a.k_scales) + (int64_t)blk * a.scale_bytes;
      const uint8_t* vs = reinterpret_cast<const uint8_t*>(a.v_scales) + (int64_t)blk * a.scale_bytes;
      bulk_g2s(base + 2 * a.page_bytes, ks, a.scale_bytes, &bars[st]);
      bulk_g2s(base + 2 * a.page_bytes + a.scale_bytes, vs, a.scale_bytes, &bars[st]);
    }
  };

  if (tid == 0) {
    for (int i = 0; i < a.nst; ++i) {
      mbar_init(&bars[i], 1);
      consumed[i] = 0;
      issued[i] = 0;
    }
    fence_mbar_init();
    for (int i = 0; i < min(a.nst, npages); ++i) issue(i);
  }
  __syncthreads();

  // q for this lane's QK chunk (dims [16c, 16c+16)), pre-scaled into the base-2 softmax domain.
  const int qc = lane % LPT;
  float qscale = a.sm_scale * kLog2e;
  if constexpr (KIND == BPT_KV_FP8) qscale *= a.k_scale;
  float2 q2[REP][8];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    const int64_t qb = (int64_t)b * a.q_sb + (int64_t)(h * REP + r) * a.q_sh + qc * 16;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      q2[r][j] = make_float2(q_load(a.q, a.q_dtype, qb + 2 * j) * qscale, q_load(a.q, a.q_dtype, qb + 2 * j + 1) * qscale);
  }

  float m[REP], l[REP];
  float2 acc[REP][DPL / 2];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -CUDART_INF_F;
    l[r] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL / 2; ++j) acc[r][j] = make_float2(0.f, 0.f);
  }
  float* my_p = pbuf + h * kBS * REP;

  for (int i = 0; i < npages; ++i) {
    const int st = i % a.nst;
    const uint32_t parity = (i / a.nst) & 1;
    if (!mbar_wait_warp(&bars[st], parity)) break;  // recorded; the drain below bounds the exit
    const uint8_t* kpage = stages + st * stage_bytes;
    const uint8_t* vpage = kpage + a.page_bytes;
    const __half* kscl = reinterpret_cast<const __half*>(kpage + 2 * a.page_bytes);
    const __half* vscl = reinterpret_cast<const __half*>(kpage + 2 * a.page_bytes + a.scale_bytes);
    const int tb = (p_first + i) * kBS;
    const int lo = max(t0 - tb, 0), hi = min(t1 - tb, kBS);
    const bool usable = valid[st] != 0;

    // ---- QK: scores for tokens step*TPS + lane/LPT ----
    float sc[STEPS][REP];
#pragma unroll
    for (int step = 0; step < STEPS; ++step) {
      const int t = step * TPS + lane / LPT;
      const uint4 kb = *reinterpret_cast<const uint4*>(kpage + (t * a.Hkv + h) * D + qc * 16);
      const uint32_t kw[4] = {kb.x, kb.y, kb.z, kb.w};
      float2 dot[REP];
#pragma unroll
      for (int r = 0; r < REP; ++r) dot[r] = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float f[4];
        dequant4<KIND>(kw[j], f);
#pragma unroll
        for (int r = 0; r < REP; ++r) {
          dot[r] = ffma2(q2[r][2 * j], make_float2(f[0], f[1]), dot[r]);
          dot[r] = ffma2(q2[r][2 * j + 1], make_float2(f[2], f[3]), dot[r]);
        }
      }
      float ks = 1.f;
      if constexpr (KIND == BPT_KV_INT8) ks = __half2float(kscl[t * a.Hkv + h]);
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        float v = dot[r].x + dot[r].y;
#pragma unroll
        for (int o = LPT / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        sc[step][r] = (usable && t >= lo && t < hi) ? v * ks : -CUDART_INF_F;
      }
    }

    // ---- online softmax over the page (base 2) ----
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float pm = sc[0][r];
#pragma unroll
      for (int step = 1; step < STEPS; ++step) pm = fmaxf(pm, sc[step][r]);
#pragma unroll
      for (int o = LPT; o < 32; o <<= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, o));
      const float m_new = fmaxf(m[r], pm);
      const float m_use = (m_new == -CUDART_INF_F) ? 0.f : m_new;  // a page with no usable token
      const float alpha = exp2f(m[r] - m_use);
      float ps = 0.f;
#pragma unroll
      for (int step = 0; step < STEPS; ++step) {
        const float p = exp2f(sc[step][r] - m_use);
        sc[step][r] = p;
        ps += p;
      }
#pragma unroll
      for (int o = LPT; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[r] = l[r] * alpha + ps;
      m[r] = m_new;
#pragma unroll
      for (int j = 0; j < DPL / 2; ++j) {
        acc[r][j].x *= alpha;
        acc[r][j].y *= alpha;
      }
    }
    if (qc == 0) {
#pragma unroll
      for (int step = 0; step < STEPS; ++step) {
        const int t = step * TPS + lane / LPT;
        float vs = 1.f;
        if constexpr (KIND == BPT_KV_INT8) vs = __half2float(vscl[t * a.Hkv + h]);
#pragma unroll
        for (int r = 0; r < REP; ++r) my_p[t * REP + r] = sc[step][r] * vs;
      }
    }
    __syncwarp();

    // ---- PV: dims [lane*DPL, lane*DPL + DPL) ----
    if (usable) {
      for (int t = lo; t < hi; ++t) {
        const uint8_t* vrow = vpage + (t * a.Hkv + h) * D + lane * DPL;
        float f[DPL];
        if constexpr (DPL == 2) {
          const float2 v2 = (KIND == BPT_KV_FP8) ? e4m3x2_to_float2(*reinterpret_cast<const uint16_t*>(vrow))
                                                 : make_float2(float(int8_t(vrow[0])), float(int8_t(vrow[1])));
          f[0] = v2.x;
          f[1] = v2.y;
        } else if constexpr (DPL == 4) {
          dequant4<KIND>(*reinterpret_cast<const uint32_t*>(vrow), f);
        } else {
          const uint2 w2 = *reinterpret_cast<const uint2*>(vrow);
          dequant4<KIND>(w2.x, f);
          dequant4<KIND>(w2.y, f + 4);
        }
        float pr[REP];
#pragma unroll
        for (int r = 0; r < REP; ++r) pr[r] = my_p[t * REP + r];
#pragma unroll
        for (int r = 0; r < REP; ++r)
#pragma unroll
          for (int j = 0; j < DPL / 2; ++j)
            acc[r][j] = ffma2(make_float2(pr[r], pr[r]), make_float2(f[2 * j], f[2 * j + 1]), acc[r][j]);
      }
    }
    __syncwarp();

    // ---- release the stage; the last warp refills it with the page nst ahead ----
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&consumed[st], 1) == a.Hkv - 1) {
        consumed[st] = 0;
        if (i + a.nst < npages) issue(i + a.nst);
      }
    }
  }

  // ---- drain: every copy issued into a stage has landed before the CTA can exit (bounded) ----
  __syncthreads();
  if (tid == 0)
    for (int st = 0; st < a.nst; ++st)
      if (issued[st] > 0) (void)mbar_wait(&bars[st], (issued[st] - 1) & 1, 50000000ull);

  // ---- epilogue ----
  float vscale = 1.f;
  if constexpr (KIND == BPT_KV_FP8) vscale = a.v_scale;
  const bool single = a.merge && nsplit_b == 1;
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    const int hq = h * REP + r;
    const float inv = l[r] > 0.f ? vscale / l[r] : 0.f;
    const float lse = l[r] > 0.f ? (m[r] + log2f(l[r])) * kLn2 : -CUDART_INF_F;
    float o[DPL];
#pragma unroll
    for (int j = 0; j < DPL / 2; ++j) {
      o[2 * j] = acc[r][j].x * inv;
      o[2 * j + 1] = acc[r][j].y * inv;
    }
    if (!a.merge) {
      float* dst = a.out_partial + (((int64_t)b * a.Hq + hq) * a.n_splits + s) * D + lane * DPL;
#pragma unroll
      for (int j = 0; j < DPL; ++j) dst[j] = o[j];
      if (lane == 0) a.lse_partial[((int64_t)b * a.Hq + hq) * a.n_splits + s] = lse;
    } else if (single) {
#pragma unroll
      for (int j = 0; j < DPL; ++j) out_store(a.out, a.out_dtype, ((int64_t)b * a.Hq + hq) * D + lane * DPL + j, o[j]);
    } else {
      float* dst = a.ws_out + (((int64_t)b * a.n_splits + s) * a.Hq + hq) * D + lane * DPL;
#pragma unroll
      for (int j = 0; j < DPL; ++j) dst[j] = o[j];
      if (lane == 0) a.ws_lse[((int64_t)b * a.n_splits + s) * a.Hq + hq] = lse;
    }
  }
  if (!a.merge || single) return;

  // ---- fused merge: the last CTA of this sequence combines the splits ----
  __threadfence();
  __syncthreads();
  if (tid == 0) *ticket = int(atomicAdd(&a.ws_count[b], 1u));
  __syncthreads();
  if (*ticket != nsplit_b - 1) return;
  __threadfence();
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    const int hq = h * REP + r;
    float mx = -CUDART_INF_F;
    for (int sp = lane; sp < nsplit_b; sp += 32) mx = fmaxf(mx, __ldcg(&a.ws_lse[((int64_t)b * a.n_splits + sp) * a.Hq + hq]));
    mx = warp_max(mx);
    float o[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[j] = 0.f;
    float wsum = 0.f;
    for (int sp = 0; sp < nsplit_b; ++sp) {
      const float w = __expf(__ldcg(&a.ws_lse[((int64_t)b * a.n_splits + sp) * a.Hq + hq]) - mx);
      wsum += w;
      const float* src = a.ws_out + (((int64_t)b * a.n_splits + sp) * a.Hq + hq) * D + lane * DPL;
#pragma unroll
      for (int j = 0; j < DPL; ++j) o[j] += w * __ldcg(src + j);
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) out_store(a.out, a.out_dtype, ((int64_t)b * a.Hq + hq) * D + lane * DPL + j, o[j] * inv);
  }
  if (tid == 0) a.ws_count[b] = 0u;
}

template <int D, int REP, int KIND>
int launch_t(const PagedArgs& a, int flags, cudaStream_t stream) {
  auto kernel = paged_attn_kernel<D, REP, KIND>;
  const int stage_bytes = 2 * (a.page_bytes + a.scale_bytes);
  const int smem = a.nst * stage_bytes + a.Hkv * kBS * REP * 4 + a.nst * 8 + a.nst * 12 + 16;
  int st = set_max_smem(reinterpret_cast<const void*>(kernel), smem);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_splits, a.B, 1);
  cfg.blockDim = dim3(32 * a.Hkv, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BPT_FLAG_PDL) ? 1 : 0;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "paged attention launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

template <int D, int KIND>
int launch_rep(const PagedArgs& a, int rep, int flags, cudaStream_t stream) {
  switch (rep) {
    case 1: return launch_t<D, 1, KIND>(a, flags, stream);
    case 2: return launch_t<D, 2, KIND>(a, flags, stream);
    case 4: return launch_t<D, 4, KIND>(a, flags, stream);
    case 8: return launch_t<D, 8, KIND>(a, flags, stream);
  }
  return set_error(BPT_ERR_UNSUPPORTED, "paged attention: REP=%d not in {1, 2, 4, 8}", rep);
}

template <int KIND>
int launch_d(const PagedArgs& a, int D, int rep, int flags, cudaStream_t stream) {
  switch (D) {
    case 64: return launch_rep<64, KIND>(a, rep, flags, stream);
    case 128: return launch_rep<128, KIND>(a, rep, flags, stream);
    case 256: return launch_rep<256, KIND>(a, rep, flags, stream);
  }
  return set_error(BPT_ERR_UNSUPPORTED, "paged attention: D=%d not in {64, 128, 256}", D);
}

#include "paged_attention_mma.cuh"
#include "paged_attention_persistent.cuh"

int paged_common(PagedArgs& a, const void* q, int q_dtype, int64_t q_sb, int64_t q_sh, const void* k_pool,
                 const void* v_pool, int kind, float k_scale, float v_scale, const void* k_scales,
                 const void* v_scales, const int32_t* block_table, int64_t bt_stride, const int32_t* lengths,
                 int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t block_size, int64_t num_blocks,
                 int64_t split, int64_t n_splits, float sm_scale) {
  BPT_REQUIRE(q && k_pool && v_pool && block_table && lengths, BPT_ERR_INVALID, "paged attention: null pointer");
  BPT_REQUIRE(kind == BPT_KV_FP8 || kind == BPT_KV_INT8, BPT_ERR_INVALID, "paged attention: kind %d", kind);
  BPT_REQUIRE(kind == BPT_KV_FP8 || (k_scales && v_scales), BPT_ERR_INVALID, "paged attention: INT8 needs scales");
  BPT_REQUIRE(q_dtype == BPT_DTYPE_F32 || q_dtype == BPT_DTYPE_F16 || q_dtype == BPT_DTYPE_BF16, BPT_ERR_INVALID,
              "paged attention: q dtype %d", q_dtype);
  BPT_REQUIRE(B >= 1 && Hkv >= 1 && Hq >= Hkv && Hq % Hkv == 0, BPT_ERR_INVALID,
              "paged attention: B=%lld Hq=%lld Hkv=%lld", (long long)B, (long long)Hq, (long long)Hkv);
  BPT_REQUIRE(Hkv <= 16, BPT_ERR_UNSUPPORTED, "paged attention: Hkv=%lld above 16", (long long)Hkv);
  BPT_REQUIRE(block_size == kBS, BPT_ERR_UNSUPPORTED, "paged attention: block_size %lld (this build: 16)",
              (long long)block_size);
  BPT_REQUIRE(split >= kBS && split % kBS == 0, BPT_ERR_INVALID, "paged attention: split %lld not a multiple of %d",
              (long long)split, kBS);
  BPT_REQUIRE(n_splits >= 1 && n_splits < 65536 && B < 65536, BPT_ERR_INVALID, "paged attention: grid too large");
  BPT_REQUIRE(num_blocks >= 1 && bt_stride >= 1, BPT_ERR_INVALID, "paged attention: empty pool or table");
  BPT_REQUIRE(aligned16(k_pool) && aligned16(v_pool) && (kind == BPT_KV_FP8 || (aligned16(k_scales) && aligned16(v_scales))),
              BPT_ERR_ALIGNMENT, "paged attention: pools and scales must be 16-byte aligned");
  a.q = q;
  a.q_dtype = q_dtype;
  a.q_sb = q_sb;
  a.q_sh = q_sh;
  a.k_pool = static_cast<const uint8_t*>(k_pool);
  a.v_pool = static_cast<const uint8_t*>(v_pool);
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.k_scales = static_cast<const __half*>(k_scales);
  a.v_scales = static_cast<const __half*>(v_scales);
  a.block_table = block_table;
  a.bt_stride = bt_stride;
  a.lengths = lengths;
  a.B = int(B);
  a.Hq = int(Hq);
  a.Hkv = int(Hkv);
  a.num_blocks = num_blocks;
  a.split = int(split);
  a.n_splits = int(n_splits);
  a.sm_scale = sm_scale;
  a.page_bytes = int(kBS * Hkv * D);
  a.scale_bytes = kind == BPT_KV_INT8 ? int(kBS * Hkv * 2) : 0;
  const int stage_bytes = 2 * (a.page_bytes + a.scale_bytes);
  a.nst = max(2, min(8, (96 * 1024) / stage_bytes));
  BPT_REQUIRE(a.nst * stage_bytes <= 200 * 1024, BPT_ERR_UNSUPPORTED, "paged attention: pages of %d bytes too large",
              a.page_bytes);
  a.out_partial = nullptr;
  a.lse_partial = nullptr;
  a.merge = 0;
  a.out = nullptr;
  a.out_dtype = BPT_DTYPE_F32;
  a.ws_out = nullptr;
  a.ws_lse = nullptr;
  a.ws_count = nullptr;
  a.persist_ctas = 0;
  a.max_cta_pages = 0;
  a.stall = 0;
  a.wait_ns = kWaitNs;
  return BPT_OK;
}

// The tensor-core kernel serves head dims 64 and 128 with up to 8 KV heads; the scalar kernel the rest.
int paged_dispatch(const PagedArgs& a, int kind, int64_t D, int flags, cudaStream_t stream) {
  const int rep = a.Hq / a.Hkv;
  if ((D == 64 || D == 128) && a.Hkv <= kMmaMaxHkv) {
    if (kind == BPT_KV_FP8)
      return D == 64 ? launch_mma_rep<64, BPT_KV_FP8>(a, rep, flags, stream)
                     : launch_mma_rep<128, BPT_KV_FP8>(a, rep, flags, stream);
    return D == 64 ? launch_mma_rep<64, BPT_KV_INT8>(a, rep, flags, stream)
                   : launch_mma_rep<128, BPT_KV_INT8>(a, rep, flags, stream);
  }
  if (kind == BPT_KV_FP8) return launch_d<BPT_KV_FP8>(a, int(D), rep, flags, stream);
  return launch_d<BPT_KV_INT8>(a, int(D), rep, flags, stream);
}

// Workspace layouts. Both start with the ticket counters (kMaxSeqs x u32) at a fixed offset, so the zeros every
// call leaves behind are found by the next call whatever its shape or kernel.
//   split kernels:      [counters][lse: B x S x Hq f32][outs: B x S x Hq x D f32]
//   persistent kernel:  [counters][lse: (B + CTAs) x Hq f32][outs: (B + CTAs) x Hq x D f32]
// The split kernels count per sequence, the persistent kernel per (sequence, KV head).
constexpr int64_t kMaxSeqs = 65536;
constexpr int64_t kCounterBytes = kMaxSeqs * 4;
static_assert(kCounterBytes == kCounterBytesP, "one counter region for every merge kernel");
static_assert(int64_t(kPersistMaxSeqs) * kMmaMaxHkv <= kMaxSeqs, "persistent tickets fit the counter region");

int64_t split_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int64_t n_splits) {
  const int64_t outs = B * n_splits * Hq * D * 4;
  const int64_t lses = B * n_splits * Hq * 4;
  return kCounterBytes + ((lses + 255) / 256) * 256 + ((outs + 255) / 256) * 256;
}

bool persistent_applies(const PagedArgs& a, int64_t D, int64_t& cap) {
  const int G = num_sms();
  // a CTA owns at most W pages, W = ceil((pages + kStartCost B) / CTAs) (the cost-weighted split)
  cap = (int64_t(a.B) * a.bt_stride + int64_t(kStartCost) * a.B + G - 1) / G;
  return (D == 64 || D == 128) && a.Hkv <= kMmaMaxHkv &&
         a.B <= kPersistMaxSeqs && cap <= kPersistMaxCtaPages && a.q_sh == D && a.q_sb == a.Hq * D &&
         aligned16(a.q);
}

// The fused-merge launch: the persistent kernel where it applies, the split kernels otherwise; `ws` is the
// workspace (caller's or the no-allocation array) of `ws_bytes` bytes.
int merge_launch(PagedArgs& a, int kind, int64_t D, int flags, cudaStream_t stream, uint8_t* ws, int64_t ws_bytes,
                 const char* who) {
  const int64_t B = a.B, Hq = a.Hq;
  int64_t cap = 0;
  a.merge = 1;
  if (persistent_applies(a, D, cap)) {
    const int G = num_sms();
    const int64_t need = persist_workspace_bytes(B, Hq, D, G);
    BPT_REQUIRE(ws_bytes >= need, BPT_ERR_WORKSPACE, "%s: workspace of %lld bytes, need %lld", who, (long long)ws_bytes,
                (long long)need);
    const int64_t lses = (((B + G) * Hq * 4 + 255) / 256) * 256;
    a.persist_ctas = G;
    a.max_cta_pages = int(cap);
    a.ws_count = reinterpret_cast<unsigned int*>(ws);
    a.ws_lse = reinterpret_cast<float*>(ws + kCounterBytes);
    a.ws_out = reinterpret_cast<float*>(ws + kCounterBytes + lses);
    const int rep = a.Hq / a.Hkv;
    if (kind == BPT_KV_FP8)
      return D == 64 ? launch_persist<64, BPT_KV_FP8>(a, rep, flags, stream) : launch_persist<128, BPT_KV_FP8>(a, rep, flags, stream);
    return D == 64 ? launch_persist<64, BPT_KV_INT8>(a, rep, flags, stream) : launch_persist<128, BPT_KV_INT8>(a, rep, flags, stream);
  }
  const int64_t need = split_workspace_bytes(B, Hq, D, a.n_splits);
  BPT_REQUIRE(ws_bytes >= need, BPT_ERR_WORKSPACE, "%s: workspace of %lld bytes, need %lld", who, (long long)ws_bytes,
              (long long)need);
  const int64_t lses = ((B * a.n_splits * Hq * 4 + 255) / 256) * 256;
  a.ws_count = reinterpret_cast<unsigned int*>(ws);
  a.ws_lse = reinterpret_cast<float*>(ws + kCounterBytes);
  a.ws_out = reinterpret_cast<float*>(ws + kCounterBytes + lses);
  return paged_dispatch(a, kind, D, flags, stream);
}

}  // namespace

int64_t paged_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int64_t n_splits) {
  return std::max(split_workspace_bytes(B, Hq, D, n_splits), persist_workspace_bytes(B, Hq, D, num_sms()));
}

}  // namespace bpt

using namespace bpt;

extern "C" int bpt_paged_decode_partials(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                         const void* k_pool, const void* v_pool, int kind, float k_scale_f32,
                                         float v_scale_f32, const void* k_scales, const void* v_scales,
                                         const int32_t* block_table, int64_t bt_stride, const int32_t* lengths,
                                         int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t block_size,
                                         int64_t num_blocks, int64_t split, int64_t n_splits, float sm_scale,
                                         float* out_partial, float* lse_partial, int flags, void* stream) {
  PagedArgs a;
  int st = paged_common(a, q, q_dtype, q_stride_b, q_stride_h, k_pool, v_pool, kind, k_scale_f32, v_scale_f32,
                        k_scales, v_scales, block_table, bt_stride, lengths, B, Hq, Hkv, D, block_size, num_blocks,
                        split, n_splits, sm_scale);
  if (st) return st;
  BPT_REQUIRE(out_partial && lse_partial, BPT_ERR_INVALID, "paged partials: null output");
  a.out_partial = out_partial;
  a.lse_partial = lse_partial;
  return paged_dispatch(a, kind, D, flags, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t bpt_paged_attend_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int64_t n_splits) {
  return paged_workspace_bytes(B, Hq, D, n_splits);
}

extern "C" int bpt_paged_attend(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h, const void* k_pool,
                                const void* v_pool, int kind, float k_scale_f32, float v_scale_f32,
                                const void* k_scales, const void* v_scales, const int32_t* block_table,
                                int64_t bt_stride, const int32_t* lengths, int64_t B, int64_t Hq, int64_t Hkv,
                                int64_t D, int64_t block_size, int64_t num_blocks, int64_t split, int64_t n_splits,
                                float sm_scale, void* out, int out_dtype, void* workspace, int64_t workspace_bytes,
                                int flags, void* stream) {
  PagedArgs a;
  int st = paged_common(a, q, q_dtype, q_stride_b, q_stride_h, k_pool, v_pool, kind, k_scale_f32, v_scale_f32,
                        k_scales, v_scales, block_table, bt_stride, lengths, B, Hq, Hkv, D, block_size, num_blocks,
                        split, n_splits, sm_scale);
  if (st) return st;
  BPT_REQUIRE(out, BPT_ERR_INVALID, "paged attend: null output");
  BPT_REQUIRE(out_dtype == BPT_DTYPE_F32 || out_dtype == BPT_DTYPE_F16 || out_dtype == BPT_DTYPE_BF16,
              BPT_ERR_INVALID, "paged attend: out dtype %d", out_dtype);
  BPT_REQUIRE(workspace, BPT_ERR_WORKSPACE, "paged attend: no workspace");
  BPT_REQUIRE(aligned16(workspace), BPT_ERR_ALIGNMENT, "paged attend: workspace must be 16-byte aligned");
  a.out = out;
  a.out_dtype = out_dtype;
  return merge_launch(a, kind, D, flags, static_cast<cudaStream_t>(stream), static_cast<uint8_t*>(workspace),
                      workspace_bytes, "paged attend");
}

// ---- the no-allocation variant of bpt_paged_attend ------------------------------------------------------------
// For callers that cannot allocate device memory: the workspace is a fixed file-scope device array instead of a
// caller buffer. The array's name is a host-side stand-in in host code, so its device address is looked up
// once per device (cudaGetSymbolAddress, with that device current) and passed to the kernel like any workspace.

#include <cudaTypedefs.h>

#include <mutex>

namespace bpt {
namespace {

constexpr int64_t kNoAllocBytes = BPT_NOALLOC_SCRATCH_BYTES;
static_assert(kNoAllocBytes > kCounterBytes, "the scratch must hold the ticket counters");

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

// The array's device address per device, with the context it was looked up in: a new context (after a
// cudaDeviceReset, or a primary context that was released and retained again) loads the module anew and may
// place the array elsewhere, so the address is looked up again whenever the current context changes.
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kMaxDevices] = {};
void* g_noalloc_ctx[kMaxDevices] = {};

PFN_cuCtxGetCurrent_v4000 ctx_get_current() {
  static PFN_cuCtxGetCurrent_v4000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  }();
  return fn;
}

int noalloc_scratch(const void* q, void** addr) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "paged attend (no alloc): no current device: %s", cudaGetErrorString(err));
  BPT_REQUIRE(dev >= 0 && dev < kMaxDevices, BPT_ERR_UNSUPPORTED, "paged attend (no alloc): device %d", dev);
  // The library picks the scratch of the current device: the caller's tensors must live there too.
  cudaPointerAttributes attr;
  err = cudaPointerGetAttributes(&attr, q);
  BPT_REQUIRE(err == cudaSuccess && attr.type == cudaMemoryTypeDevice && attr.device == dev, BPT_ERR_INVALID,
              "paged attend (no alloc): q is not device memory of the current device %d", dev);
  PFN_cuCtxGetCurrent_v4000 get_ctx = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get_ctx == nullptr || get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return set_error(BPT_ERR_CUDA, "paged attend (no alloc): no current context on device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr || g_noalloc_ctx[dev] != static_cast<void*>(ctx)) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr)
      return set_error(BPT_ERR_CUDA, "paged attend (no alloc): cannot find the scratch array on device %d: %s", dev,
                       cudaGetErrorString(err));
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = static_cast<void*>(ctx);
  }
  *addr = g_noalloc_addr[dev];
  return BPT_OK;
}

}  // namespace
}  // namespace bpt

extern "C" int bpt_paged_attend_noalloc(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                        const void* k_pool, const void* v_pool, int kind, float k_scale_f32,
                                        float v_scale_f32, const void* k_scales, const void* v_scales,
                                        const int32_t* block_table, int64_t bt_stride, const int32_t* lengths,
                                        int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t block_size,
                                        int64_t num_blocks, int64_t split, int64_t n_splits, float sm_scale, void* out,
                                        int out_dtype, int flags, void* stream) {
  PagedArgs a;
  int st = paged_common(a, q, q_dtype, q_stride_b, q_stride_h, k_pool, v_pool, kind, k_scale_f32, v_scale_f32,
                        k_scales, v_scales, block_table, bt_stride, lengths, B, Hq, Hkv, D, block_size, num_blocks,
                        split, n_splits, sm_scale);
  if (st) return st;
  BPT_REQUIRE(out, BPT_ERR_INVALID, "paged attend (no alloc): null output");
  BPT_REQUIRE(out_dtype == BPT_DTYPE_F32 || out_dtype == BPT_DTYPE_F16 || out_dtype == BPT_DTYPE_BF16,
              BPT_ERR_INVALID, "paged attend (no alloc): out dtype %d", out_dtype);
  int64_t cap = 0;
  const int64_t need = persistent_applies(a, D, cap) ? persist_workspace_bytes(B, Hq, D, num_sms())
                                                     : split_workspace_bytes(B, Hq, D, n_splits);
  BPT_REQUIRE(need <= kNoAllocBytes, BPT_ERR_WORKSPACE,
              "paged attend (no alloc): B=%lld x n_splits=%lld x Hq=%lld x D=%lld needs %lld bytes of scratch, above the "
              "fixed %lld (use larger splits, or bpt_paged_attend with a caller workspace)",
              (long long)B, (long long)n_splits, (long long)Hq, (long long)D, (long long)need, (long long)kNoAllocBytes);
  void* scratch = nullptr;
  st = noalloc_scratch(q, &scratch);
  if (st) return st;
  auto s = static_cast<cudaStream_t>(stream);
  // The array keeps whatever the last call left: the tickets this call uses (one per sequence, or per sequence
  // and KV head for the persistent kernel) must start at zero.
  const size_t tickets = size_t(B) * (persistent_applies(a, D, cap) ? size_t(Hkv) : 1u);
  cudaError_t err = cudaMemsetAsync(scratch, 0, tickets * sizeof(unsigned int), s);
  if (err != cudaSuccess)
    return set_error(BPT_ERR_CUDA, "paged attend (no alloc): clearing the tickets: %s", cudaGetErrorString(err));
  a.out = out;
  a.out_dtype = out_dtype;
  return merge_launch(a, kind, D, flags, s, static_cast<uint8_t*>(scratch), kNoAllocBytes, "paged attend (no alloc)");
}
