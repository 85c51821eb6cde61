// Tensor-core variant of the paged decode attention (included by paged_attention.cu, inside its namespace).
//
// Same grid, pages, pipeline and outputs as paged_attn_kernel; the per-page math runs on mma.sync.m16n8k16
// (f16 x f16 -> f32) instead of dequantize-and-FMA loops:
//
//   QK  S[16 x 8 tokens] = Q[16 x 16 dims] . K^T      rows g < REP: q of head g rounded to f16 ("hi"),
//                                                     rows 8 + g: the rest, q - hi, rounded to f16 ("lo")
//   PV  O[16 x 8 dims]  += P[16 x 16 tokens] . V     rows g: f16(p), rows 8 + g: f16(p - f16(p))
//
// With the hi/lo split every product is exact in the fp32 accumulator and the operands carry 22 bits, so the
// result matches fp32 arithmetic to the reference kernel's tolerance; lane (c, g) reads head g's score as
// c0 + c2 and its output as c0 + c2, c1 + c3, with no shuffle. The QK accumulator fragment of a lane holds the
// very tokens its PV A-fragment needs (tokens 2c, 2c+1, 8+2c, 9+2c), so P never leaves registers.
//
// Operand layouts. MMA k-slots are mapped to head dims so that each lane's key bytes are contiguous: in QK
// k-step ks, lane c's slots {2c, 2c+1, 2c+8, 2c+9} hold dims c*D/4 + 4ks + {0, 1, 2, 3}, i.e. one 32-bit word
// of the row, whose two byte pairs convert straight into the two B registers (cvt.rn.f16x2.e4m3x2, or, for
// INT8, a byte permute into f16 1024 + u and one subtraction). In PV, column n of n-tile nt is head dim
// n * D/8 + nt, so lane g needs bytes [g*D/8, (g+1)*D/8) of four token rows; a byte permute pairs the two
// tokens of each B register. The output dims of a lane are then [c*D/4, (c+1)*D/4), written contiguously.
//
// Shared memory: token rows are copied one per bulk copy to a pitch of Hkv*D + 16 bytes, which makes both
// fragment loads (different tokens, same column) bank-conflict free. A warp issues a page's 32 row copies
// cooperatively.

constexpr int kMmaMaxHkv = 8;

// (not volatile: a pure register operation the compiler may schedule freely around loads and other math)
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint32_t two_bytes) {
  uint32_t r;
  const uint16_t v = uint16_t(two_bytes);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// Two int8 bytes (sign bits already flipped) -> f16x2, exactly: 0x64uu is f16 1024 + u, minus 1152.
__device__ __forceinline__ uint32_t s8x2_f16x2(uint32_t flipped, uint32_t sel) {
  const uint32_t biased = __byte_perm(flipped, 0x64646464u, sel);
  __half2 h = *reinterpret_cast<const __half2*>(&biased);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));  // 1152
  return *reinterpret_cast<uint32_t*>(&h);
}

// A 32-bit word of 4 stored bytes -> the two f16x2 B registers (bytes 0,1) and (bytes 2,3).
template <int KIND>
__device__ __forceinline__ void word_to_b(uint32_t w, uint32_t& b0, uint32_t& b1) {
  if constexpr (KIND == BPT_KV_FP8) {
    asm("{\n\t.reg .b16 lo, hi;\n\t"
        "mov.b32 {lo, hi}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
        "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
        : "=r"(b0), "=r"(b1)
        : "r"(w));
  } else {
    const uint32_t f = w ^ 0x80808080u;
    b0 = s8x2_f16x2(f, 0x5140u);
    b1 = s8x2_f16x2(f, 0x7362u);
  }
}

// Four e4m3 codes -> two f16x2 words on the integer pipe: lo = codes (0, 2), hi = codes (1, 3), each 2^-8 times
// the code's value, exactly. The f16 bits (c & 0x7F) << 7 | (c & 0x80) << 8 put the e4m3 exponent and mantissa
// into the f16 fields with the exponent bias 8 short (15 - 7); e4m3 subnormals land on f16 subnormals with the
// same factor. (The conversion instruction does the same work on the quarter-rate conversion unit.)
__device__ __forceinline__ void e4m3x4_to_f16_scaled(uint32_t w, uint32_t& lo, uint32_t& hi) {
  constexpr uint32_t m = 0x3F803F80u;  // exponent and mantissa fields of both halves
  const uint32_t s = w & 0x80808080u;  // sign bits
  lo = ((w << 7) & m) | ((s << 8) & ~m);
  hi = ((w >> 1) & m) | (s & ~m);
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// f16 "hi" parts of two values and their f16 "lo" remainders.
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  hi = pack_half2(__half2float(h0), __half2float(h1));
  lo = pack_half2(x0 - __half2float(h0), x1 - __half2float(h1));
}

template <int D, int REP, int KIND, int COPY>
__global__ void __launch_bounds__(32 * kMmaMaxHkv, 1) paged_attn_mma_kernel(const PagedArgs a) {
  constexpr int KS = D / 16;  // QK k-steps
  constexpr int DQ = D / 4;   // key bytes per lane per token; output dims per lane
  constexpr int VB = D / 8;   // value bytes per lane per token; PV n-tiles
  static_assert(REP <= 8, "hi/lo rows: at most 8 query heads per KV head");
  static_assert(DQ % 16 == 0 && VB % 8 == 0, "D must be 64 or 128");

  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int b = blockIdx.y, s = blockIdx.x;
  const int h = warp;

  pdl_launch_dependents();
  pdl_wait();

  const int L = a.lengths[b];
  const int t0 = s * a.split;
  const int t1 = min(L, t0 + a.split);
  const int nsplit_b = min(a.n_splits, (L + a.split - 1) / a.split);

  if (t0 >= t1) {
    if (!a.merge) {
      for (int i = tid; i < a.Hq * D; i += blockDim.x) {
        const int hq = i / D, d = i % D;
        a.out_partial[(((int64_t)b * a.Hq + hq) * a.n_splits + s) * D + d] = 0.f;
        if (d == 0) a.lse_partial[((int64_t)b * a.Hq + hq) * a.n_splits + s] = -CUDART_INF_F;
      }
    } else if (s == 0) {
      for (int i = tid; i < a.Hq * D; i += blockDim.x) out_store(a.out, a.out_dtype, (int64_t)b * a.Hq * D + i, 0.f);
    }
    return;
  }

  const int rowb = a.Hkv * D;                         // bytes of one token row (all KV heads) in the pool
  const int kpitch = (COPY & 1) ? rowb + 16 : rowb;   // token rows in shared memory: padded when copied one by one
  const int vpitch = (COPY & 2) ? rowb + 16 : rowb;
  const int kpage = kBS * kpitch, vpage_bytes = kBS * vpitch;
  const int stage_bytes = kpage + vpage_bytes + 2 * a.scale_bytes;
  uint8_t* stages = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.nst * stage_bytes);
  int* consumed = reinterpret_cast<int*>(bars + a.nst);
  int* valid = consumed + a.nst;
  int* issued = valid + a.nst;
  int* ticket = issued + a.nst;
  int* blocks = ticket + 1;  // this split's block-table entries, read once up front

  const int p_first = t0 / kBS;
  const int npages = (t1 - 1) / kBS - p_first + 1;
  const int32_t* table = a.block_table + (int64_t)b * a.bt_stride;

  // Warp-cooperative issue of page i. A tensor copied row by row uses one lane per token row (keys: lanes 0-15,
  // values: lanes 16-31); a tensor copied whole uses one lane.
  auto issue_warp = [&](int i) {
    const int st = i % a.nst;
    uint8_t* base = stages + st * stage_bytes;
    const int32_t blk = blocks[i];
    const bool ok = blk >= 0 && blk < a.num_blocks;
    if (lane == 0) {
      issued[st] += 1;
      valid[st] = ok ? 1 : 0;
      if (!ok) record_error(kDevErrBlockIndex);
      mbar_arrive_expect_tx(&bars[st], ok ? uint32_t(2 * kBS * rowb + 2 * a.scale_bytes) : 0u);
    }
    __syncwarp();
    if (ok) {
      const uint64_t policy = l2_policy_evict_first();
      const int t = lane & 15;
      const uint8_t* ksrc = a.k_pool + (int64_t)blk * a.page_bytes;
      const uint8_t* vsrc = a.v_pool + (int64_t)blk * a.page_bytes;
      if constexpr (COPY & 1) {
        if (lane < 16) bulk_g2s_evict_first(base + t * kpitch, ksrc + t * rowb, rowb, &bars[st], policy);
      } else {
        if (lane == 0) bulk_g2s_evict_first(base, ksrc, a.page_bytes, &bars[st], policy);
      }
      if constexpr (COPY & 2) {
        if (lane >= 16) bulk_g2s_evict_first(base + kpage + t * vpitch, vsrc + t * rowb, rowb, &bars[st], policy);
      } else {
        if (lane == 16) bulk_g2s_evict_first(base + kpage, vsrc, a.page_bytes, &bars[st], policy);
      }
      if constexpr (KIND == BPT_KV_INT8) {
        if (lane == 1)
          bulk_g2s(base + kpage + vpage_bytes, reinterpret_cast<const uint8_t*>(a.k_scales) + (int64_t)blk * a.scale_bytes,
                   a.scale_bytes, &bars[st]);
        if (lane == 2)
          bulk_g2s(base + kpage + vpage_bytes + a.scale_bytes,
                   reinterpret_cast<const uint8_t*>(a.v_scales) + (int64_t)blk * a.scale_bytes, a.scale_bytes, &bars[st]);
      }
    }
  };

  if (tid == 0) {
    for (int i = 0; i < a.nst; ++i) {
      mbar_init(&bars[i], 1);
      consumed[i] = 0;
      issued[i] = 0;
    }
    fence_mbar_init();
  }
  // A page past the table's row reads as -1 (recorded and skipped, never addressed).
  for (int i = tid; i < npages; i += blockDim.x) blocks[i] = (p_first + i < a.bt_stride) ? table[p_first + i] : -1;
  __syncthreads();
  if (warp == 0)
    for (int i = 0; i < min(a.nst, npages); ++i) issue_warp(i);

  // q as MMA A-fragments: rows g (hi) and 8 + g (lo) of head g, dims c*DQ + 4ks + {0..3}.
  uint32_t qa[KS][4];
  {
    const bool real = g < REP;
    const int64_t qb = (int64_t)b * a.q_sb + (int64_t)(h * REP + (real ? g : 0)) * a.q_sh + c * DQ;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      float x[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = real ? q_load(a.q, a.q_dtype, qb + 4 * ks + j) : 0.f;
      split2(x[0], x[1], qa[ks][0], qa[ks][1]);
      split2(x[2], x[3], qa[ks][2], qa[ks][3]);
    }
  }
  float qscale = a.sm_scale * kLog2e;
  if constexpr (KIND == BPT_KV_FP8) qscale *= a.k_scale;

  float m = -CUDART_INF_F, l = 0.f;  // this lane's head g
  float o[VB][4];
#pragma unroll
  for (int nt = 0; nt < VB; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  __syncthreads();  // the barriers are armed before anyone waits

  for (int i = 0; i < npages; ++i) {
    const int st = i % a.nst;
    if (!mbar_wait_warp(&bars[st], (i / a.nst) & 1)) break;
    const uint8_t* kp = stages + st * stage_bytes;
    const uint8_t* vp = kp + kpage;
    const __half* kscl = reinterpret_cast<const __half*>(kp + kpage + vpage_bytes);
    const __half* vscl = reinterpret_cast<const __half*>(kp + kpage + vpage_bytes + a.scale_bytes);
    const int tb = (p_first + i) * kBS;
    const int lo = max(t0 - tb, 0), hi = min(t1 - tb, kBS);
    const bool usable = valid[st] != 0;

    // ---- QK: two n-tiles of 8 tokens; this lane owns tokens 2c, 2c+1 of each ----
    float sc[4];  // tokens 2c, 2c+1, 8+2c, 9+2c
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint8_t* row = kp + (nt * 8 + g) * kpitch + h * D + c * DQ;
      uint32_t kw[DQ / 4];
#pragma unroll
      for (int v = 0; v < DQ / 16; ++v) {
        const uint4 u = *reinterpret_cast<const uint4*>(row + 16 * v);
        kw[4 * v] = u.x;
        kw[4 * v + 1] = u.y;
        kw[4 * v + 2] = u.z;
        kw[4 * v + 3] = u.w;
      }
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t b0, b1;
        word_to_b<KIND>(kw[ks], b0, b1);
        mma_f16(acc, qa[ks], b0, b1);
      }
      sc[2 * nt] = (acc[0] + acc[2]) * qscale;
      sc[2 * nt + 1] = (acc[1] + acc[3]) * qscale;
    }
    int tok[4] = {2 * c, 2 * c + 1, 8 + 2 * c, 9 + 2 * c};
    bool live[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      live[j] = usable && tok[j] >= lo && tok[j] < hi;
      float v = sc[j];
      if constexpr (KIND == BPT_KV_INT8) v *= live[j] ? __half2float(kscl[tok[j] * a.Hkv + h]) : 0.f;
      sc[j] = live[j] ? v : -CUDART_INF_F;
    }

    // ---- online softmax for head g over the page (the four lanes of this g) ----
    float pm = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 1));
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 2));
    const float m_new = fmaxf(m, pm);
    const float m_use = (m_new == -CUDART_INF_F) ? 0.f : m_new;
    const float alpha = exp2f(m - m_use);
    float p[4], ps = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      p[j] = exp2f(sc[j] - m_use);
      ps += p[j];
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l = l * alpha + ps;
    m = m_new;
    if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
      for (int nt = 0; nt < VB; ++nt) {
        o[nt][0] *= alpha;
        o[nt][1] *= alpha;
        o[nt][2] *= alpha;
        o[nt][3] *= alpha;
      }
    }
    if (usable) {  // an unusable page contributes nothing, but its stage is still released below
    // ---- P as the PV A-fragment (INT8: the value scale folds into the weight) ----
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (KIND == BPT_KV_INT8) p[j] = live[j] ? p[j] * __half2float(vscl[tok[j] * a.Hkv + h]) : 0.f;
    }
    uint32_t pa[4];
    split2(p[0], p[1], pa[0], pa[1]);
    split2(p[2], p[3], pa[2], pa[3]);

    // ---- PV: value rows of tokens 2c, 2c+1, 8+2c, 9+2c, bytes [g*VB, (g+1)*VB) ----
    uint32_t vr[4][VB / 4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint8_t* row = vp + tok[j] * vpitch + h * D + g * VB;
#pragma unroll
      for (int v = 0; v < VB / 16; ++v) {
        const uint4 u = *reinterpret_cast<const uint4*>(row + 16 * v);
        vr[j][4 * v] = u.x;
        vr[j][4 * v + 1] = u.y;
        vr[j][4 * v + 2] = u.z;
        vr[j][4 * v + 3] = u.w;
      }
      if constexpr (VB % 16 == 8) {
        const uint2 u = *reinterpret_cast<const uint2*>(row + 16 * (VB / 16));
        vr[j][VB / 4 - 2] = u.x;
        vr[j][VB / 4 - 1] = u.y;
      }
      if (!live[j]) {  // rows past the sequence may hold any bytes: a zero weight must not meet a NaN code
#pragma unroll
        for (int w = 0; w < VB / 4; ++w) vr[j][w] = 0u;
      }
    }
#pragma unroll
    for (int w = 0; w < VB / 4; ++w) {
      // pair token 2c with 2c+1 (B row 2c, 2c+1) and 8+2c with 9+2c (rows 2c+8, 2c+9), per value dim
      const uint32_t lo01 = __byte_perm(vr[0][w], vr[1][w], 0x5140u), lo23 = __byte_perm(vr[0][w], vr[1][w], 0x7362u);
      const uint32_t hi01 = __byte_perm(vr[2][w], vr[3][w], 0x5140u), hi23 = __byte_perm(vr[2][w], vr[3][w], 0x7362u);
      uint32_t b0[4], b1[4];
      if constexpr (KIND == BPT_KV_FP8) {
        b0[0] = cvt_e4m3x2_f16x2(lo01 & 0xFFFFu);
        b0[1] = cvt_e4m3x2_f16x2(lo01 >> 16);
        b0[2] = cvt_e4m3x2_f16x2(lo23 & 0xFFFFu);
        b0[3] = cvt_e4m3x2_f16x2(lo23 >> 16);
        b1[0] = cvt_e4m3x2_f16x2(hi01 & 0xFFFFu);
        b1[1] = cvt_e4m3x2_f16x2(hi01 >> 16);
        b1[2] = cvt_e4m3x2_f16x2(hi23 & 0xFFFFu);
        b1[3] = cvt_e4m3x2_f16x2(hi23 >> 16);
      } else {
        const uint32_t f01 = lo01 ^ 0x80808080u, f23 = lo23 ^ 0x80808080u;
        const uint32_t g01 = hi01 ^ 0x80808080u, g23 = hi23 ^ 0x80808080u;
        b0[0] = s8x2_f16x2(f01, 0x5140u);
        b0[1] = s8x2_f16x2(f01, 0x7362u);
        b0[2] = s8x2_f16x2(f23, 0x5140u);
        b0[3] = s8x2_f16x2(f23, 0x7362u);
        b1[0] = s8x2_f16x2(g01, 0x5140u);
        b1[1] = s8x2_f16x2(g01, 0x7362u);
        b1[2] = s8x2_f16x2(g23, 0x5140u);
        b1[3] = s8x2_f16x2(g23, 0x7362u);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) mma_f16(o[4 * w + e], pa, b0[e], b1[e]);
    }
    }  // usable

    // ---- release the stage; the last warp refills it ----
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&consumed[st], 1) == a.Hkv - 1;
      if (last) consumed[st] = 0;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last && i + a.nst < npages) issue_warp(i + a.nst);
  }
  __syncthreads();
  if (tid == 0)
    for (int st = 0; st < a.nst; ++st)
      if (issued[st] > 0) (void)mbar_wait(&bars[st], (issued[st] - 1) & 1, 50000000ull);

  // ---- epilogue: lane (c, g < REP) holds head g's dims [c*DQ, (c+1)*DQ) ----
  float vscale = 1.f;
  if constexpr (KIND == BPT_KV_FP8) vscale = a.v_scale;
  const bool single = a.merge && nsplit_b == 1;
  if (g < REP) {
    const int hq = h * REP + g;
    const float inv = l > 0.f ? vscale / l : 0.f;
    const float lse = l > 0.f ? (m + log2f(l)) * kLn2 : -CUDART_INF_F;
    float res[DQ];
#pragma unroll
    for (int nt = 0; nt < VB; ++nt) {
      res[nt] = (o[nt][0] + o[nt][2]) * inv;
      res[VB + nt] = (o[nt][1] + o[nt][3]) * inv;
    }
    if (!a.merge) {
      float* dst = a.out_partial + (((int64_t)b * a.Hq + hq) * a.n_splits + s) * D + c * DQ;
#pragma unroll
      for (int j = 0; j < DQ; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(res[j], res[j + 1], res[j + 2], res[j + 3]);
      if (c == 0) a.lse_partial[((int64_t)b * a.Hq + hq) * a.n_splits + s] = lse;
    } else if (single) {
#pragma unroll
      for (int j = 0; j < DQ; ++j) out_store(a.out, a.out_dtype, ((int64_t)b * a.Hq + hq) * D + c * DQ + j, res[j]);
    } else {
      float* dst = a.ws_out + (((int64_t)b * a.n_splits + s) * a.Hq + hq) * D + c * DQ;
#pragma unroll
      for (int j = 0; j < DQ; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(res[j], res[j + 1], res[j + 2], res[j + 3]);
      if (c == 0) a.ws_lse[((int64_t)b * a.n_splits + s) * a.Hq + hq] = lse;
    }
  }
  if (!a.merge || single) return;

  // ---- fused merge by the last CTA of the sequence (as in paged_attn_kernel) ----
  __threadfence();
  __syncthreads();
  if (tid == 0) *ticket = int(atomicAdd(&a.ws_count[b], 1u));
  __syncthreads();
  if (*ticket != nsplit_b - 1) return;
  __threadfence();
  for (int r = 0; r < REP; ++r) {
    const int hq = h * REP + r;
    float mx = -CUDART_INF_F;
    for (int sp = lane; sp < nsplit_b; sp += 32) mx = fmaxf(mx, __ldcg(&a.ws_lse[((int64_t)b * a.n_splits + sp) * a.Hq + hq]));
    mx = warp_max(mx);
    constexpr int DPL = D / 32;
    float acc[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
    float wsum = 0.f;
    for (int sp = 0; sp < nsplit_b; ++sp) {
      const float w = __expf(__ldcg(&a.ws_lse[((int64_t)b * a.n_splits + sp) * a.Hq + hq]) - mx);
      wsum += w;
      const float* src = a.ws_out + (((int64_t)b * a.n_splits + sp) * a.Hq + hq) * D + lane * DPL;
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[j] += w * __ldcg(src + j);
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) out_store(a.out, a.out_dtype, ((int64_t)b * a.Hq + hq) * D + lane * DPL + j, acc[j] * inv);
  }
  if (tid == 0) a.ws_count[b] = 0u;
}

// Pages are copied token row by token row to a padded pitch (COPY bit 0: keys, bit 1: values), four stages deep
// where they fit.
constexpr int kMmaCopy = 3;
constexpr int kMmaStages = 4;

template <int D, int REP, int KIND, int COPY>
int launch_mma_t(const PagedArgs& a0, int flags, cudaStream_t stream) {
  PagedArgs a = a0;
  const int rowb = a.Hkv * D;
  const int stage_bytes = kBS * (rowb + ((COPY & 1) ? 16 : 0)) + kBS * (rowb + ((COPY & 2) ? 16 : 0)) + 2 * a.scale_bytes;
  a.nst = max(2, min(kMmaStages, (200 * 1024) / stage_bytes));
  auto kernel = paged_attn_mma_kernel<D, REP, KIND, COPY>;
  const int max_pages = a.split / kBS + 1;
  const int smem = a.nst * stage_bytes + a.nst * 8 + a.nst * 12 + 16 + 4 * max_pages;
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
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "paged attention (mma) launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

template <int D, int KIND>
int launch_mma_rep(const PagedArgs& a, int rep, int flags, cudaStream_t stream) {
  switch (rep) {
    case 1: return launch_mma_t<D, 1, KIND, kMmaCopy>(a, flags, stream);
    case 2: return launch_mma_t<D, 2, KIND, kMmaCopy>(a, flags, stream);
    case 4: return launch_mma_t<D, 4, KIND, kMmaCopy>(a, flags, stream);
    case 8: return launch_mma_t<D, 8, KIND, kMmaCopy>(a, flags, stream);
  }
  return set_error(BPT_ERR_UNSUPPORTED, "paged attention: REP=%d not in {1, 2, 4, 8}", rep);
}
