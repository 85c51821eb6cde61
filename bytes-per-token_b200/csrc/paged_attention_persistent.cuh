// Persistent, warp-specialized paged decode attention with the split merge fused in (included by
// paged_attention.cu, inside its namespace; uses the MMA helpers of paged_attention_mma.cuh).
//
// Work split. The pages of all sequences, laid end to end, are cut into one contiguous range per CTA (one CTA per
// SM) of equal cost, a page costing 1 and a sequence's first page kStartCost more, so ragged lengths never
// unbalance the GPU and a range that opens a sequence takes fewer pages. The piece of a sequence that falls inside one
// CTA's range is a "part": it has its own online-softmax state and leaves one partial (out, lse). A
// sequence's parts are the CTAs first_b .. last_b whose ranges meet it; part (c, b) writes workspace slot
// c + b, so a launch needs at most #CTAs + B slots. The CTA that finishes a sequence's last part merges its
// partials (an atomic ticket per sequence; nothing waits), exactly as reference.merge_partials.
//
// Roles. Warp Hkv is the producer: it walks the CTA's pages and, per page, waits until the consumers have
// released the stage (an "empty" mbarrier), arms the "full" mbarrier and issues the page's bulk copies: K and V
// (whole pages, or token rows to a padded pitch), INT8 scales, and, with the first page of a part, the
// sequence's q rows. Warps 0 .. Hkv-1 are the consumers, one per KV head, with the tensor-core math of
// paged_attn_mma_kernel; they arrive on "empty" when done with a page and never issue copies themselves.
//
// Prologue. All threads read the lengths into shared memory; warp 0 scans them into page offsets; every thread
// then resolves a share of the CTA's pages to (sequence, page, block) with one block-table read each. Those
// are the only global round trips before the producer starts.

constexpr int kPersistMaxSeqs = 4096;
constexpr int kMaxSmemPerCta = 227 * 1024;  // sm_100 opt-in dynamic shared memory per block
constexpr int kPersistMaxCtaPages = 4096;
constexpr int kPersistStages = 6;
// Each sequence's first page carries this many pages' worth of extra cost in the work split (the part it opens
// costs a q copy, a partial, a ticket and shorter steps at its edges): CTA ranges cut the cost evenly, not the
// page count, so a CTA whose range holds a sequence start gets correspondingly fewer pages. (Config 2 with the
// swizzled tiles: 34.10, 33.68 and 33.89 us per call at 2, 3 and 4; with the split merge's loads of both items in
// flight together, attention alone / GEMV + attention step: 33.09 / 40.11 at 2, 32.91-33.05 / 39.77-39.97 at 3,
// 32.84-32.94 / 39.46-39.56 at 4, 33.08 / 39.82 at 5, 33.15 / 39.58 at 6.)
constexpr int kStartCost = 4;

constexpr int64_t kCounterBytesP = 65536 * 4;  // the ticket counters, at the workspace's start (as paged_attend)

// A stage is a page of K then one of V (stage_bytes); its INT8 scales (K then V) and, when the page opens a part, the
// sequence's q rows sit in the stage's aux slot (aux_bytes; q at q_off), the aux slots after all the stages, so the
// stages keep the tiles' alignment without padding.
struct PersistLayout {
  int stage_bytes, aux_bytes, kpitch, vpitch, kpage, vpage, q_off, q_bytes;
};

// COPY: how a page lands in its stage. 0: K and V pages as stored ([token][head][D], one bulk copy each); 4 (D = 128):
// K and V as 4-D tensor copies into head-major tiles [head][token][128 bytes] with the 128-byte swizzle (16-byte chunk
// j of token row t at chunk j ^ (t mod 8)), so the consumers' row reads meet no bank conflict with one copy per page
// (stages then start on 1 KB boundaries). (Row-by-row copies to a padded pitch, the split kernels' form, measured
// much slower here: 32 small copies per page swamp the TMA engine.)
template <int D, int COPY>
__host__ __device__ inline PersistLayout persist_layout(int Hkv, int Hq, int q_esize, int scale_bytes) {
  static_assert(COPY == 0 || COPY == 4, "pages as stored, or swizzled head-major tiles");
  PersistLayout p;
  const int rowb = Hkv * D;
  p.kpitch = (COPY & 4) ? D : rowb;
  p.vpitch = (COPY & 4) ? D : rowb;
  p.kpage = kBS * rowb;
  p.vpage = kBS * rowb;
  p.q_bytes = Hq * D * q_esize;
  p.q_off = 2 * scale_bytes;
  p.stage_bytes = (COPY & 4) ? (p.kpage + p.vpage + 1023) & ~1023 : (p.kpage + p.vpage + 127) & ~127;
  p.aux_bytes = (p.q_off + p.q_bytes + 127) & ~127;
  return p;
}

// Stage st's aux slot (its INT8 scales, then q at q_off) in a ring of nst stages starting at `stages`.
__host__ __device__ inline uint8_t* stage_aux(uint8_t* stages, const PersistLayout& lay, int nst, int st) {
  return stages + nst * lay.stage_bytes + st * lay.aux_bytes;
}

// Byte offset in a stage's K (or V) page of token t's 16-byte chunk j (bytes 16 j .. 16 j + 15 of the head's D)
// for KV head h.
template <int D, int COPY>
__device__ __forceinline__ int page_chunk(const PersistLayout& lay, int pitch, int h, int t, int j) {
  if constexpr (COPY & 4) {
    static_assert(D == 128, "swizzled tiles hold 128-byte rows");
    return (h * kBS + t) * D + ((j ^ (t & 7)) << 4);
  } else {
    return t * pitch + h * D + 16 * j;
  }
}

// Atomic add at GPU scope with release (prior writes, and those ordered before by a barrier, are visible first)
// and acquire (later reads see what the other arrivals released) semantics; returns the old value.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(unsigned int* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}


__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}


// The part's partials are all in: out[b, hq] = sum_p w_p out_p / sum_p w_p, w_p = exp(lse_p - max lse), for
// the query heads hq0 .. hq0 + nheads - 1. Each of the group's nthr threads takes two (query head, 4 dims) items at
// a time (items i and i + nthr) and reads the parts in batches of four with the loads of both items issued before
// any is used, folding each batch in with a running maximum: a warp merging two heads of D = 128 pays one round
// trip to L2 per batch of parts, not one per item (as many values in flight as batches of eight for one item, so
// no more registers).
template <int D>
__device__ __forceinline__ void merge_parts(const PagedArgs& a, int b, int64_t s0, int nparts, int hq0, int nheads,
                                            int tid, int nthr) {
  constexpr int kBatch = 4;
  const int items = nheads * (D / 4);
  const int64_t ostride = int64_t(a.Hq) * D;
  for (int i0 = tid; i0 < items; i0 += 2 * nthr) {
    int hq[2], d[2];
    bool use[2];
    const float* lse[2];
    const float* po[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = i0 + u * nthr;
      use[u] = i < items;
      hq[u] = hq0 + (use[u] ? i : i0) / (D / 4);
      d[u] = 4 * ((use[u] ? i : i0) % (D / 4));
      lse[u] = a.ws_lse + s0 * a.Hq + hq[u];
      po[u] = a.ws_out + (s0 * a.Hq + hq[u]) * D + d[u];
    }
    float mx[2] = {-CUDART_INF_F, -CUDART_INF_F}, wsum[2] = {0.f, 0.f};
    float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    for (int p0 = 0; p0 < nparts; p0 += kBatch) {
      float lv[2][kBatch];
      float4 ov[2][kBatch];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const bool v = use[u] && p0 + j < nparts;
          lv[u][j] = v ? __ldcg(lse[u] + int64_t(p0 + j) * a.Hq) : -CUDART_INF_F;
          ov[u][j] = v ? __ldcg(reinterpret_cast<const float4*>(po[u] + (p0 + j) * ostride))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float bm = lv[u][0];
#pragma unroll
        for (int j = 1; j < kBatch; ++j) bm = fmaxf(bm, lv[u][j]);
        const float nm = fmaxf(mx[u], bm);
        if (nm == -CUDART_INF_F) continue;  // no tokens in any part so far
        const float f = expf(mx[u] - nm);
        wsum[u] *= f;
        acc[u].x *= f; acc[u].y *= f; acc[u].z *= f; acc[u].w *= f;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const float w = expf(lv[u][j] - nm);
          wsum[u] += w;
          acc[u].x += w * ov[u][j].x; acc[u].y += w * ov[u][j].y; acc[u].z += w * ov[u][j].z;
          acc[u].w += w * ov[u][j].w;
        }
        mx[u] = nm;
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!use[u]) continue;
      const int64_t o = ((int64_t)b * a.Hq + hq[u]) * D + d[u];
      out_store(a.out, a.out_dtype, o, wsum[u] > 0.f ? acc[u].x / wsum[u] : 0.f);
      out_store(a.out, a.out_dtype, o + 1, wsum[u] > 0.f ? acc[u].y / wsum[u] : 0.f);
      out_store(a.out, a.out_dtype, o + 2, wsum[u] > 0.f ? acc[u].z / wsum[u] : 0.f);
      out_store(a.out, a.out_dtype, o + 3, wsum[u] > 0.f ? acc[u].w / wsum[u] : 0.f);
    }
  }
}

// Consumers with tokens on the MMA's M dimension (REP <= 4). Per page:
//   QK   S^T[16 tokens x 8] = K[16 tokens x 16 dims] . Q^T
//   PV   O^T[16 dims x 8]  += V^T[16 dims x 16 tokens] . P^T
// B column n = 2 * head + part: part 0 is the f16 rounding of q (or p), part 1 the f16 rounding of what is left,
// so the f16 products add up to fp32-grade results. A page costs D/16 MMAs for each product, q is a constant B
// fragment (D/8 registers) and the output accumulator D/4 registers. Lane (g, c) gets columns 2c and 2c+1 of
// every C tile: both parts of head c, summed in the lane, so each lane owns one head. P goes from the QK layout
// (tokens on g) to the PV layout (tokens on c) through a small per-warp tile in shared memory. A step takes one
// or two pages of the same part as straight-line code, so their load, convert and MMA chains interleave.
// CONV (FP8 only): bit 0 converts keys, bit 1 values on the integer pipe (2^-8-scaled, codes paired (0, 2) and
// (1, 3)) instead of the conversion unit.
template <int D, int REP, int KIND, int COPY, int CONV>
__device__ __forceinline__ void consume_transposed(const PagedArgs& a, const PersistLayout& lay, uint8_t* stages,
                                                   uint64_t* full, uint64_t* empty, const int* off, const int* slen,
                                                   const int* pblk, const int* pseq, const int* plp, volatile int* misc,
                                                   float* ptile_all, int n, int per) {
  static_assert(REP <= 4, "four query heads per KV head at most in this layout");
  constexpr int KS = D / 16;  // QK k-steps
  constexpr int DQ = D / 4;   // key bytes per lane per token
  constexpr int VD = D / 8;   // value bytes (dims) per lane per token
  constexpr int MT = D / 16;  // PV m-tiles
  constexpr bool kKAlu = KIND == BPT_KV_FP8 && (CONV & 1);
  constexpr bool kVAlu = KIND == BPT_KV_FP8 && (CONV & 2);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int h = warp, Hkv = a.Hkv, cta = blockIdx.x, nst = a.nst;
  const int q_esize = a.q_dtype == BPT_DTYPE_F32 ? 4 : 2;
  const int bhead = g >> 1, bpart = g & 1;  // the B column this lane feeds
  float* ptile = ptile_all + warp * 32 * 4;
  float qscale = a.sm_scale * kLog2e;
  if constexpr (KIND == BPT_KV_FP8) qscale *= a.k_scale * (kKAlu ? 256.f : 1.f);
  float vscale = 1.f;
  if constexpr (KIND == BPT_KV_FP8) vscale = a.v_scale * (kVAlu ? 256.f : 1.f);

  uint32_t qb[KS][2];
  float m = -CUDART_INF_F, l = 0.f;
  float o[MT][4];
  int waited = 0;

  auto wait_page = [&](int k, int st, uint32_t ph) {
    if (!misc[2]) {
      if (mbar_wait_warp(&full[st], ph, a.wait_ns))
        waited = k + 1;
      else if (lane == 0)
        misc[2] = 1;
    }
  };

  // One step over pages k .. k + NP - 1 (stages st[0 .. NP - 1]) of a sequence of L tokens.
  auto step = [&](auto npc, int k, const int* st, int L) {
    constexpr int NP = decltype(npc)::value;
    const uint8_t* sp[NP];
    int hi_tok[NP];  // live tokens of the page (0 for a block index outside the pool)
#pragma unroll
    for (int pg = 0; pg < NP; ++pg) {
      sp[pg] = stages + st[pg] * lay.stage_bytes;
      const int blk = pblk[k + pg];
      hi_tok[pg] = (blk >= 0 && blk < a.num_blocks) ? min(kBS, L - plp[k + pg] * kBS) : 0;
    }

    // ---- key rows g and g + 8 of each page; this lane's DQ bytes of the warp's head ----
    uint32_t w[NP][2][DQ / 4];
#pragma unroll
    for (int pg = 0; pg < NP; ++pg) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int v = 0; v < DQ / 16; ++v) {
          const uint4 u = *reinterpret_cast<const uint4*>(
              sp[pg] + page_chunk<D, COPY>(lay, lay.kpitch, h, g + 8 * r, c * (DQ / 16) + v));
          w[pg][r][4 * v] = u.x; w[pg][r][4 * v + 1] = u.y; w[pg][r][4 * v + 2] = u.z; w[pg][r][4 * v + 3] = u.w;
        }
      }
    }

    // ---- S^T = K . Q^T, two accumulators per page (even and odd k-steps) ----
    float acc[NP][2][4];
#pragma unroll
    for (int pg = 0; pg < NP; ++pg)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[pg][0][e] = acc[pg][1][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int pg = 0; pg < NP; ++pg) {
        uint32_t af[4];
        if constexpr (kKAlu) {  // k slots (2c, 2c+1) = dims (0, 2) of the word, (2c+8, 2c+9) = dims (1, 3)
          e4m3x4_to_f16_scaled(w[pg][0][ks], af[0], af[2]);
          e4m3x4_to_f16_scaled(w[pg][1][ks], af[1], af[3]);
        } else {  // k slots (2c, 2c+1) = dims (0, 1) of the word, (2c+8, 2c+9) = dims (2, 3)
          word_to_b<KIND>(w[pg][0][ks], af[0], af[2]);  // token g
          word_to_b<KIND>(w[pg][1][ks], af[1], af[3]);  // token g + 8
        }
        mma_f16(acc[pg][ks & 1], af, qb[ks][0], qb[ks][1]);
      }
    }
    float s[NP][2];  // head c at tokens g and g + 8, log2 units
#pragma unroll
    for (int pg = 0; pg < NP; ++pg) {
      const float v0 = (acc[pg][0][0] + acc[pg][0][1]) + (acc[pg][1][0] + acc[pg][1][1]);
      const float v1 = (acc[pg][0][2] + acc[pg][0][3]) + (acc[pg][1][2] + acc[pg][1][3]);
      const bool live0 = g < hi_tok[pg], live1 = g + 8 < hi_tok[pg];
      float k0 = qscale, k1 = qscale;
      if constexpr (KIND == BPT_KV_INT8) {
        const __half* kscl = reinterpret_cast<const __half*>(stage_aux(stages, lay, nst, st[pg]));
        k0 *= live0 ? __half2float(kscl[g * Hkv + h]) : 0.f;
        k1 *= live1 ? __half2float(kscl[(g + 8) * Hkv + h]) : 0.f;
      }
      s[pg][0] = live0 ? v0 * k0 : -CUDART_INF_F;
      s[pg][1] = live1 ? v1 * k1 : -CUDART_INF_F;
    }

    // ---- online softmax of head c over the step's tokens (the lanes with this c) ----
    float pm = fmaxf(s[0][0], s[0][1]);
#pragma unroll
    for (int pg = 1; pg < NP; ++pg) pm = fmaxf(pm, fmaxf(s[pg][0], s[pg][1]));
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 4));
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 8));
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 16));
    const float m_new = fmaxf(m, pm);
    const float m_use = (m_new == -CUDART_INF_F) ? 0.f : m_new;
    const float alpha = exp2f(m - m_use);
    float ps = 0.f;
#pragma unroll
    for (int pg = 0; pg < NP; ++pg) {
      s[pg][0] = exp2f(s[pg][0] - m_use);
      s[pg][1] = exp2f(s[pg][1] - m_use);
      ps += s[pg][0] + s[pg][1];
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
    l = l * alpha + ps;
    m = m_new;
    if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        o[mt][0] *= alpha; o[mt][1] *= alpha; o[mt][2] *= alpha; o[mt][3] *= alpha;
      }
    }

    // ---- P through the warp's tile [token][head] (INT8: times the value scale) ----
#pragma unroll
    for (int pg = 0; pg < NP; ++pg) {
      float vs0 = 1.f, vs1 = 1.f;
      if constexpr (KIND == BPT_KV_INT8) {
        const __half* vscl = reinterpret_cast<const __half*>(stage_aux(stages, lay, nst, st[pg]) + a.scale_bytes);
        vs0 = g < hi_tok[pg] ? __half2float(vscl[g * Hkv + h]) : 0.f;
        vs1 = g + 8 < hi_tok[pg] ? __half2float(vscl[(g + 8) * Hkv + h]) : 0.f;
      }
      ptile[(pg * 16 + g) * 4 + c] = s[pg][0] * vs0;
      ptile[(pg * 16 + g + 8) * 4 + c] = s[pg][1] * vs1;
    }
    __syncwarp();

    // ---- O^T += V^T . P^T: value rows of tokens 2c, 2c+1, 2c+8, 2c+9; dims [g*VD, (g+1)*VD) ----
#pragma unroll
    for (int pg = 0; pg < NP; ++pg) {
      const uint8_t* vp = sp[pg] + lay.kpage;
      float pw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) pw[j] = ptile[(pg * 16 + 2 * c + (j & 1) + 8 * (j >> 1)) * 4 + bhead];
      uint32_t b0, b1;
      {
        uint32_t h01, l01, h23, l23;
        split2(pw[0], pw[1], h01, l01);
        split2(pw[2], pw[3], h23, l23);
        b0 = bpart ? l01 : h01;
        b1 = bpart ? l23 : h23;
      }
      uint32_t vr[4][VD / 4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tok = 2 * c + (j & 1) + 8 * (j >> 1);
        const uint8_t* row = (COPY & 4) ? vp + page_chunk<D, COPY>(lay, lay.vpitch, h, tok, g)
                                        : vp + tok * lay.vpitch + h * D + g * VD;
        if constexpr (VD == 16) {
          const uint4 u = *reinterpret_cast<const uint4*>(row);
          vr[j][0] = u.x; vr[j][1] = u.y; vr[j][2] = u.z; vr[j][3] = u.w;
        } else {
          const uint2 u = *reinterpret_cast<const uint2*>(row);
          vr[j][0] = u.x; vr[j][1] = u.y;
        }
      }
      if constexpr (KIND == BPT_KV_FP8) {
        if (hi_tok[pg] < kBS) {  // rows past the sequence may hold NaN codes; int8 codes are all finite
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const bool live = 2 * c + (j & 1) + 8 * (j >> 1) < hi_tok[pg];
#pragma unroll
            for (int q = 0; q < VD / 4; ++q) vr[j][q] = live ? vr[j][q] : 0u;
          }
        }
      }
      uint32_t p01[VD], p89[VD];  // f16x2 (token pair) per lane dim
#pragma unroll
      for (int q = 0; q < VD / 4; ++q) {
        const uint32_t* r = &vr[0][0];
        constexpr int R = VD / 4;  // words per row
        if constexpr (kVAlu) {  // [t0 d0, t0 d1, t1 d0, t1 d1] -> (t0, t1) of d0 and of d1
          e4m3x4_to_f16_scaled(__byte_perm(r[q], r[R + q], 0x5410u), p01[4 * q], p01[4 * q + 1]);
          e4m3x4_to_f16_scaled(__byte_perm(r[q], r[R + q], 0x7632u), p01[4 * q + 2], p01[4 * q + 3]);
          e4m3x4_to_f16_scaled(__byte_perm(r[2 * R + q], r[3 * R + q], 0x5410u), p89[4 * q], p89[4 * q + 1]);
          e4m3x4_to_f16_scaled(__byte_perm(r[2 * R + q], r[3 * R + q], 0x7632u), p89[4 * q + 2], p89[4 * q + 3]);
        } else {  // [t0 d0, t1 d0, t0 d1, t1 d1] -> (t0, t1) of d0 and of d1
          word_to_b<KIND>(__byte_perm(r[q], r[R + q], 0x5140u), p01[4 * q], p01[4 * q + 1]);
          word_to_b<KIND>(__byte_perm(r[q], r[R + q], 0x7362u), p01[4 * q + 2], p01[4 * q + 3]);
          word_to_b<KIND>(__byte_perm(r[2 * R + q], r[3 * R + q], 0x5140u), p89[4 * q], p89[4 * q + 1]);
          word_to_b<KIND>(__byte_perm(r[2 * R + q], r[3 * R + q], 0x7362u), p89[4 * q + 2], p89[4 * q + 3]);
        }
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint32_t af[4] = {p01[mt], p01[VD / 2 + mt], p89[mt], p89[VD / 2 + mt]};
        mma_f16(o[mt], af, b0, b1);
      }
    }
    __syncwarp();  // all reads of the stages and of the P tile are done
    if (lane == 0) {
#pragma unroll
      for (int pg = 0; pg < NP; ++pg) mbar_arrive(&empty[st[pg]]);
    }
  };

  // A part's ticket (per sequence and KV head) is taken at the part's end and read at the next part's end, or
  // after the last page, so the warp does not wait for the atomic's round trip between its pages. The last of
  // a sequence's parts to arrive merges them.
  int pend_b = -1, pend_nparts = 0;
  int64_t pend_s0 = 0;
  uint32_t pend_ticket = 0;
  auto settle = [&]() {
    if (pend_b < 0) return;
    const int t = __shfl_sync(0xffffffffu, int(pend_ticket), 0);
    __syncwarp();  // lane 0's acquire, then every lane's reads
    if (t == pend_nparts - 1) {
      merge_parts<D>(a, pend_b, pend_s0, pend_nparts, h * REP, REP, lane, 32);
      if (lane == 0) a.ws_count[int64_t(pend_b) * Hkv + h] = 0u;
    }
    pend_b = -1;
  };

  int st0 = 0;       // stage of page k
  uint32_t ph = 0;   // its full-barrier parity
  for (int k = 0; k < n;) {
    const int b = pseq[k];
    const bool first = (k == 0) || (pseq[k - 1] != b);
    const int np = (k + 1 < n && pseq[k + 1] == b) ? 2 : 1;
    const bool last = (k + np >= n) || (pseq[k + np] != b);
    const int L = slen[b];
    int st[2];
    uint32_t phs[2];
    st[0] = st0; phs[0] = ph;
    st[1] = st0 + 1 == nst ? 0 : st0 + 1;
    phs[1] = st0 + 1 == nst ? ph ^ 1u : ph;
    wait_page(k, st[0], phs[0]);
    if (np == 2) wait_page(k + 1, st[1], phs[1]);

    if (first) {  // q of this sequence as the QK B fragment: column g = head g / 2, part g % 2
      const uint8_t* qrow = stage_aux(stages, lay, nst, st0) + lay.q_off +
                            (int64_t)(h * REP + (bhead < REP ? bhead : 0)) * D * q_esize;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        float x[4];
        const int d0 = c * DQ + 4 * ks;
        if (a.q_dtype == BPT_DTYPE_F32) {
          const float4 v = *reinterpret_cast<const float4*>(qrow + d0 * 4);
          x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else {
          const uint2 v = *reinterpret_cast<const uint2*>(qrow + d0 * 2);
          if (a.q_dtype == BPT_DTYPE_BF16) {
            x[0] = bf16_bits_to_float(v.x & 0xFFFFu); x[1] = bf16_bits_to_float(v.x >> 16);
            x[2] = bf16_bits_to_float(v.y & 0xFFFFu); x[3] = bf16_bits_to_float(v.y >> 16);
          } else {
            x[0] = __half2float(__ushort_as_half(uint16_t(v.x & 0xFFFFu))); x[1] = __half2float(__ushort_as_half(uint16_t(v.x >> 16)));
            x[2] = __half2float(__ushort_as_half(uint16_t(v.y & 0xFFFFu))); x[3] = __half2float(__ushort_as_half(uint16_t(v.y >> 16)));
          }
        }
        if (bhead >= REP) x[0] = x[1] = x[2] = x[3] = 0.f;
        uint32_t hi01, lo01, hi23, lo23;
        if constexpr (kKAlu) {  // the keys' pairing: dims (0, 2) and (1, 3)
          split2(x[0], x[2], hi01, lo01);
          split2(x[1], x[3], hi23, lo23);
        } else {
          split2(x[0], x[1], hi01, lo01);
          split2(x[2], x[3], hi23, lo23);
        }
        qb[ks][0] = bpart ? lo01 : hi01;
        qb[ks][1] = bpart ? lo23 : hi23;
      }
      m = -CUDART_INF_F;
      l = 0.f;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    }

    if (np == 2)
      step(std::integral_constant<int, 2>(), k, st, L);
    else
      step(std::integral_constant<int, 1>(), k, st, L);
    k += np;
    st0 = np == 2 ? st[1] : st[0];
    ph = np == 2 ? phs[1] : phs[0];
    if (++st0 == nst) { st0 = 0; ph ^= 1u; }
    if (!last) continue;

    // ---- end of a part: lane (g, c) holds head c at dims g*VD + [0, VD) ----
    const int first_cta = (off[b] + kStartCost * (b + 1)) / per;  // the CTAs owning b's first and last pages
    const int last_cta = (off[b + 1] - 1 + kStartCost * (b + 1)) / per;
    const int nparts = last_cta - first_cta + 1;
    if (c < REP) {
      const int hq = h * REP + c;
      const float inv = l > 0.f ? vscale / l : 0.f;
      const float lse = l > 0.f ? (m + log2f(l)) * kLn2 : -CUDART_INF_F;
      float res[VD];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        res[mt] = (o[mt][0] + o[mt][1]) * inv;
        res[VD / 2 + mt] = (o[mt][2] + o[mt][3]) * inv;
      }
      if (nparts == 1) {
#pragma unroll
        for (int j = 0; j < VD; ++j) out_store(a.out, a.out_dtype, ((int64_t)b * a.Hq + hq) * D + g * VD + j, res[j]);
      } else {
        const int64_t slot = cta + b;
        float* dst = a.ws_out + (slot * a.Hq + hq) * D + g * VD;
#pragma unroll
        for (int j = 0; j < VD; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(res[j], res[j + 1], res[j + 2], res[j + 3]);
        if (g == 0) a.ws_lse[slot * a.Hq + hq] = lse;
      }
    }
    if (nparts == 1) continue;
    settle();
    __syncwarp();  // the lanes' partial writes before lane 0's release
    if (lane == 0) pend_ticket = atom_add_acq_rel_gpu(&a.ws_count[int64_t(b) * Hkv + h], 1u);
    pend_b = b;
    pend_nparts = nparts;
    pend_s0 = first_cta + b;
  }
  settle();
  if (misc[2] && warp == 0 && lane == 0) {
    const int issued = misc[1];
    for (int k = waited; k < issued; ++k) (void)mbar_wait(&full[k % nst], (k / nst) & 1, (a.wait_ns < 20000000ull ? a.wait_ns : 20000000ull));
  }
}

// tm_k, tm_v: the pools' tensor maps for COPY 4 (unused otherwise).
template <int D, int REP, int KIND, int COPY, bool TR, int CONV>
__global__ void __launch_bounds__(32 * (kMmaMaxHkv + 1), 1)
    paged_attn_persistent_kernel(const PagedArgs a, const __grid_constant__ CUtensorMap tm_k,
                                 const __grid_constant__ CUtensorMap tm_v) {
  constexpr int KS = D / 16, DQ = D / 4, VB = D / 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // COPY 4: swizzled tiles need 1 KB aligned stages (the launch reserves the slack)
  uint8_t* smem = (COPY & 4) ? smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) : smem_raw;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int Hkv = a.Hkv, B = a.B, G = gridDim.x, cta = blockIdx.x;
  const int q_esize = a.q_dtype == BPT_DTYPE_F32 ? 4 : 2;
  const PersistLayout lay = persist_layout<D, COPY>(Hkv, a.Hq, q_esize, a.scale_bytes);
  const int rowb = Hkv * D;

  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.nst * (lay.stage_bytes + lay.aux_bytes));
  uint64_t* empty = full + a.nst;
  int* off = reinterpret_cast<int*>(empty + a.nst);  // [B + 1] page offsets of the sequences
  int* slen = off + B + 1;                            // [B] lengths in tokens
  int* pblk = slen + B;                               // [cap] block of each of this CTA's pages
  int* pseq = pblk + a.max_cta_pages;                 // [cap] its sequence
  int* plp = pseq + a.max_cta_pages;                  // [cap] its page index in the sequence
  volatile int* misc = plp + a.max_cta_pages;         // [0] ticket, [1] pages issued, [2] abort
  // [Hkv][32 tokens][4 heads] P tiles of the transposed consumers, 16-byte aligned after misc[0..2]
  float* ptile = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(misc + 3) + 15) & ~uintptr_t(15));

  pdl_launch_dependents();
  // Under BPT_FLAG_KV_READY the lengths, block table and pools are final already: the prologue and the first
  // stages' page copies run while the previous kernel finishes; q, the output and the workspace wait for it.
  if (!a.early) pdl_wait();

  // ---- prologue: offsets, this CTA's range, its pages' blocks ----
  for (int b = tid; b < B; b += blockDim.x) {
    const int L = a.lengths[b];
    const int np = L > 0 ? (L + kBS - 1) / kBS : 0;
    slen[b] = L;
    off[b + 1] = min(np, int(a.bt_stride));  // pages past the table's row are never read
  }
  if (tid == 0) {
    off[0] = 0;
    misc[0] = 0;
    misc[1] = 0;
    misc[2] = 0;
    for (int i = 0; i < a.nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], Hkv);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {  // inclusive scan of off[1 .. B] in chunks of 32
    int carry = 0;
    for (int base = 1; base <= B; base += 32) {
      int v = (base + lane <= B) ? off[base + lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      if (base + lane <= B) off[base + lane] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  const int P = off[B];
  // CTA c owns the pages whose cost position lies in [c W, (c + 1) W), W the total cost over the CTAs
  const int per = (P + kStartCost * B + G - 1) / G;
  // The first page whose cost position is >= t (P if none): sequence b's pages sit at positions p + kStartCost (b + 1),
  // so with b the last sequence whose first position is <= t, it is t - kStartCost (b + 1) clamped to b's pages
  // (past b's last page: the next page in order, whose position is above t). One binary search over sequences.
  auto first_page_at = [&](int64_t t) -> int {
    if (t < kStartCost) return 0;
    int lo = 0, hi = B;  // invariant: start position of lo <= t (sequence 0's is kStartCost)
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (off[mid] + int64_t(kStartCost) * (mid + 1) <= t) lo = mid; else hi = mid;
    }
    const int64_t p = t - int64_t(kStartCost) * (lo + 1);
    return int(min(int64_t(off[lo + 1]), max(int64_t(off[lo]), p)));
  };
  const int g0 = first_page_at(int64_t(cta) * per), g1 = first_page_at(int64_t(cta + 1) * per);
  const int n = g1 - g0;
  for (int k = tid; k < n; k += blockDim.x) {
    const int gp = g0 + k;
    int lo = 0, hi = B;  // the sequence b with off[b] <= gp < off[b + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (off[mid] <= gp) lo = mid; else hi = mid;
    }
    const int lp = gp - off[lo];
    pseq[k] = lo;
    plp[k] = lp;
    pblk[k] = a.block_table[(int64_t)lo * a.bt_stride + lp];
  }
  __syncthreads();
  const bool producer = warp == Hkv;
  // A sequence with no tokens is in nobody's range and gets a zero output: sequence b from CTA b mod G, one warp
  // each (the consumer warps; every warp of a CTA without pages), after the wait on the previous kernel.
  if (!producer || n <= 0) {
    if (a.early) pdl_wait();
    const int nw = n <= 0 ? int(blockDim.x >> 5) : Hkv;
    for (int b = cta + G * warp; b < B; b += G * nw)
      if (off[b + 1] == off[b])
        for (int i = lane; i < a.Hq * D; i += 32) out_store(a.out, a.out_dtype, (int64_t)b * a.Hq * D + i, 0.f);
  }
  if (n <= 0) return;

  if (producer) {
    // ---------------- producer warp ----------------
    const uint64_t policy = l2_policy_evict_first();
    // Early start: pages 0 .. pre - 1 are requested before the wait on the previous kernel, their q copies after it.
    const int pre = a.early ? min(n, a.nst) : 0;
    auto q_copies_of_first_pages = [&]() {
      pdl_wait();
      for (int k = 0; k < pre; ++k)
        if ((k == 0 || pseq[k - 1] != pseq[k]) && lane == 3)
          bulk_g2s(stage_aux(stages, lay, a.nst, k) + lay.q_off,
                   static_cast<const uint8_t*>(a.q) + (int64_t)pseq[k] * lay.q_bytes, lay.q_bytes, &full[k]);
    };
    int st = 0;        // stage of page k
    uint32_t eph = 1;  // parity of the empty phase that frees it: (k / nst - 1) & 1
    for (int k = 0; k < n; ++k, st = (st + 1 == a.nst) ? 0 : st + 1, eph ^= (st == 0) ? 1u : 0u) {
      if (k == pre && pre > 0) q_copies_of_first_pages();
      if (misc[2]) break;
      // BPT_FLAG_TEST_STALL: the CTA holding the first page issues nothing from its second page on (its first, if it
      // has one page). Every page it did issue is awaited by the consumers before they reach the missing one, so
      // no copy is in flight.
      if (a.stall && g0 == 0 && k == min(1, n - 1)) break;
      if (k >= a.nst && !mbar_wait_warp(&empty[st], eph, a.wait_ns)) {
        misc[2] = 1;
        break;
      }
      if (misc[2]) break;  // a consumer gave up while this warp waited for the stage
      uint8_t* base = stages + st * lay.stage_bytes;
      const int b = pseq[k];
      const int blk = pblk[k];
      const bool ok = blk >= 0 && blk < a.num_blocks;
      const bool first = (k == 0) || (pseq[k - 1] != b);
      uint32_t bytes = ok ? uint32_t(2 * kBS * rowb + 2 * a.scale_bytes) : 0u;
      if (first) bytes += uint32_t(lay.q_bytes);
      if (lane == 0) {
        if (!ok) record_error(kDevErrBlockIndex);
        mbar_arrive_expect_tx(&full[st], bytes);
      }
      __syncwarp();
      if (ok) {
        const uint8_t* ksrc = a.k_pool + (int64_t)blk * a.page_bytes;
        const uint8_t* vsrc = a.v_pool + (int64_t)blk * a.page_bytes;
        if constexpr (COPY & 4) {
          if (lane == 0) tma_load_4d_hint(base, &tm_k, 0, 0, 0, blk, &full[st], policy);
          if (lane == 16) tma_load_4d_hint(base + lay.kpage, &tm_v, 0, 0, 0, blk, &full[st], policy);
        } else {
          if (lane == 0) bulk_g2s_evict_first(base, ksrc, a.page_bytes, &full[st], policy);
          if (lane == 16) bulk_g2s_evict_first(base + lay.kpage, vsrc, a.page_bytes, &full[st], policy);
        }
        if constexpr (KIND == BPT_KV_INT8) {
          if (lane == 1)
            bulk_g2s(stage_aux(stages, lay, a.nst, st), reinterpret_cast<const uint8_t*>(a.k_scales) + (int64_t)blk * a.scale_bytes,
                     a.scale_bytes, &full[st]);
          if (lane == 2)
            bulk_g2s(stage_aux(stages, lay, a.nst, st) + a.scale_bytes,
                     reinterpret_cast<const uint8_t*>(a.v_scales) + (int64_t)blk * a.scale_bytes, a.scale_bytes, &full[st]);
        }
      }
      if (first && lane == 3 && k >= pre)
        bulk_g2s(stage_aux(stages, lay, a.nst, st) + lay.q_off, static_cast<const uint8_t*>(a.q) + (int64_t)b * lay.q_bytes,
                 lay.q_bytes, &full[st]);
      __syncwarp();
      if (lane == 0) misc[1] = k + 1;
    }
    if (pre == n && pre > 0) q_copies_of_first_pages();  // every page fitted in the first stages
    return;
  }

  // ---------------- consumer warps: one per KV head ----------------
  if constexpr (TR) {
    consume_transposed<D, REP, KIND, COPY, CONV>(a, lay, stages, full, empty, off, slen, pblk, pseq, plp, misc, ptile, n, per);
    return;
  } else {
  // A step covers one page, or two consecutive pages of the same part (32 tokens): the two pages' QK chains and
  // PV accumulations interleave, and the softmax, barrier wait and release costs are paid once per two pages.
  const int h = warp;
  float qscale = a.sm_scale * kLog2e;
  if constexpr (KIND == BPT_KV_FP8) qscale *= a.k_scale;
  float vscale = 1.f;
  if constexpr (KIND == BPT_KV_FP8) vscale = a.v_scale;

  uint32_t qa[KS][4];
  float m = -CUDART_INF_F, l = 0.f;
  float o[VB][4];
  int waited = 0;  // pages whose data this warp saw arrive

  // After a wait gives up, every later wait is skipped (the abort flag) but the loop still runs to the end, so
  // all consumer warps meet the same named barriers; the data they read then is stale but in bounds.
  auto wait_page = [&](int k) {
    if (!misc[2]) {
      if (mbar_wait_warp(&full[k % a.nst], (k / a.nst) & 1, a.wait_ns))
        waited = k + 1;
      else if (lane == 0)
        misc[2] = 1;
    }
  };

  for (int k = 0; k < n;) {
    const int b = pseq[k];
    const bool first = (k == 0) || (pseq[k - 1] != b);
    const int np = (k + 1 < n && pseq[k + 1] == b) ? 2 : 1;
    const bool last = (k + np >= n) || (pseq[k + np] != b);
    const int L = slen[b];
    wait_page(k);
    if (np == 2) wait_page(k + 1);

    if (first) {  // a new part: this sequence's q (copied with the part's first page), fresh softmax state
      const uint8_t* kp0 = stage_aux(stages, lay, a.nst, k % a.nst);
      const bool real = g < REP;
      const int hq = h * REP + (real ? g : 0);
      const uint8_t* qrow = kp0 + lay.q_off + (int64_t)hq * D * q_esize;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        float x[4];
        const int d0 = c * DQ + 4 * ks;
        if (a.q_dtype == BPT_DTYPE_F32) {
          const float4 v = *reinterpret_cast<const float4*>(qrow + d0 * 4);
          x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else {
          const uint2 v = *reinterpret_cast<const uint2*>(qrow + d0 * 2);
          if (a.q_dtype == BPT_DTYPE_BF16) {
            x[0] = bf16_bits_to_float(v.x & 0xFFFFu); x[1] = bf16_bits_to_float(v.x >> 16);
            x[2] = bf16_bits_to_float(v.y & 0xFFFFu); x[3] = bf16_bits_to_float(v.y >> 16);
          } else {
            x[0] = __half2float(__ushort_as_half(uint16_t(v.x & 0xFFFFu))); x[1] = __half2float(__ushort_as_half(uint16_t(v.x >> 16)));
            x[2] = __half2float(__ushort_as_half(uint16_t(v.y & 0xFFFFu))); x[3] = __half2float(__ushort_as_half(uint16_t(v.y >> 16)));
          }
        }
        if (!real) x[0] = x[1] = x[2] = x[3] = 0.f;
        split2(x[0], x[1], qa[ks][0], qa[ks][1]);
        split2(x[2], x[3], qa[ks][2], qa[ks][3]);
      }
      m = -CUDART_INF_F;
      l = 0.f;
#pragma unroll
      for (int nt = 0; nt < VB; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    }

    // ---- QK for up to two pages: scores of tokens 2c, 2c+1, 8+2c, 9+2c of each ----
    float sc[2][4];
    bool live[2][4];
    bool usable[2];
#pragma unroll
    for (int pg = 0; pg < 2; ++pg) {
      usable[pg] = false;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[pg][j] = -CUDART_INF_F;
        live[pg][j] = false;
      }
      if (pg < np) {
        const int kk = k + pg;
        const uint8_t* kp = stages + (kk % a.nst) * lay.stage_bytes;
        const __half* kscl = reinterpret_cast<const __half*>(stage_aux(stages, lay, a.nst, kk % a.nst));
        usable[pg] = pblk[kk] >= 0 && pblk[kk] < a.num_blocks;
        const int hi = min(kBS, L - plp[kk] * kBS);
        float acc[2][2][4];  // [n-tile][even/odd k-steps][c-fragment]
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint8_t* row = kp + (nt * 8 + g) * lay.kpitch + h * D + c * DQ;
          uint32_t kw[DQ / 4];
#pragma unroll
          for (int v = 0; v < DQ / 16; ++v) {
            const uint4 u = *reinterpret_cast<const uint4*>(row + 16 * v);
            kw[4 * v] = u.x; kw[4 * v + 1] = u.y; kw[4 * v + 2] = u.z; kw[4 * v + 3] = u.w;
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) acc[nt][e][0] = acc[nt][e][1] = acc[nt][e][2] = acc[nt][e][3] = 0.f;
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            uint32_t b0, b1;
            word_to_b<KIND>(kw[ks], b0, b1);
            mma_f16(acc[nt][ks & 1], qa[ks], b0, b1);
          }
        }
        const bool full_page = usable[pg] && hi == kBS;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = 2 * nt + e;
            const int t = nt * 8 + 2 * c + e;
            float v = (acc[nt][0][e] + acc[nt][0][e + 2] + acc[nt][1][e] + acc[nt][1][e + 2]) * qscale;
            live[pg][j] = full_page || (usable[pg] && t < hi);
            if constexpr (KIND == BPT_KV_INT8) v *= live[pg][j] ? __half2float(kscl[t * Hkv + h]) : 0.f;
            sc[pg][j] = live[pg][j] ? v : -CUDART_INF_F;
          }
        }
      }
    }

    // ---- online softmax over the step's tokens (the four lanes of head g) ----
    float pm = fmaxf(fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[0][2], sc[0][3])),
                     fmaxf(fmaxf(sc[1][0], sc[1][1]), fmaxf(sc[1][2], sc[1][3])));
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 1));
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 2));
    const float m_new = fmaxf(m, pm);
    const float m_use = (m_new == -CUDART_INF_F) ? 0.f : m_new;
    const float alpha = exp2f(m - m_use);
    float p[2][4], ps = 0.f;
#pragma unroll
    for (int pg = 0; pg < 2; ++pg)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        p[pg][j] = exp2f(sc[pg][j] - m_use);
        ps += p[pg][j];
      }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l = l * alpha + ps;
    m = m_new;
    if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
      for (int nt = 0; nt < VB; ++nt) {
        o[nt][0] *= alpha; o[nt][1] *= alpha; o[nt][2] *= alpha; o[nt][3] *= alpha;
      }
    }

    // ---- PV: one 16-token k-step per page ----
#pragma unroll
    for (int pg = 0; pg < 2; ++pg) {
      if (pg < np && usable[pg]) {
        const int kk = k + pg;
        const uint8_t* vp = stages + (kk % a.nst) * lay.stage_bytes + lay.kpage;
        const __half* vscl = reinterpret_cast<const __half*>(stage_aux(stages, lay, a.nst, kk % a.nst) + a.scale_bytes);
        const int tok[4] = {2 * c, 2 * c + 1, 8 + 2 * c, 9 + 2 * c};
        float pw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          pw[j] = p[pg][j];
          if constexpr (KIND == BPT_KV_INT8) pw[j] = live[pg][j] ? pw[j] * __half2float(vscl[tok[j] * Hkv + h]) : 0.f;
        }
        uint32_t pa[4];
        split2(pw[0], pw[1], pa[0], pa[1]);
        split2(pw[2], pw[3], pa[2], pa[3]);
        uint32_t vr[4][VB / 4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint8_t* row = vp + tok[j] * lay.vpitch + h * D + g * VB;
#pragma unroll
          for (int v = 0; v < VB / 16; ++v) {
            const uint4 u = *reinterpret_cast<const uint4*>(row + 16 * v);
            vr[j][4 * v] = u.x; vr[j][4 * v + 1] = u.y; vr[j][4 * v + 2] = u.z; vr[j][4 * v + 3] = u.w;
          }
          if constexpr (VB % 16 == 8) {
            const uint2 u = *reinterpret_cast<const uint2*>(row + 16 * (VB / 16));
            vr[j][VB / 4 - 2] = u.x;
            vr[j][VB / 4 - 1] = u.y;
          }
          if (!live[pg][j]) {  // rows past the sequence may hold any bytes: a zero weight must not meet a NaN code
#pragma unroll
            for (int w = 0; w < VB / 4; ++w) vr[j][w] = 0u;
          }
        }
#pragma unroll
        for (int w = 0; w < VB / 4; ++w) {
          const uint32_t lo01 = __byte_perm(vr[0][w], vr[1][w], 0x5140u), lo23 = __byte_perm(vr[0][w], vr[1][w], 0x7362u);
          const uint32_t hi01 = __byte_perm(vr[2][w], vr[3][w], 0x5140u), hi23 = __byte_perm(vr[2][w], vr[3][w], 0x7362u);
          uint32_t b0[4], b1[4];
          word_to_b<KIND>(lo01, b0[0], b0[1]);
          word_to_b<KIND>(lo23, b0[2], b0[3]);
          word_to_b<KIND>(hi01, b1[0], b1[1]);
          word_to_b<KIND>(hi23, b1[2], b1[3]);
#pragma unroll
          for (int e = 0; e < 4; ++e) mma_f16(o[4 * w + e], pa, b0[e], b1[e]);
        }
      }
    }

    // ---- release the step's stages to the producer ----
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty[k % a.nst]);
      if (np == 2) mbar_arrive(&empty[(k + 1) % a.nst]);
    }
    k += np;

    if (!last) continue;

    // ---- end of a part: its partial, then the ticket; the last part of a sequence merges ----
    const int first_cta = (off[b] + kStartCost * (b + 1)) / per;  // the CTAs owning b's first and last pages
    const int last_cta = (off[b + 1] - 1 + kStartCost * (b + 1)) / per;
    const int nparts = last_cta - first_cta + 1;
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
      if (nparts == 1) {
#pragma unroll
        for (int j = 0; j < DQ; ++j) out_store(a.out, a.out_dtype, ((int64_t)b * a.Hq + hq) * D + c * DQ + j, res[j]);
      } else {
        const int64_t slot = cta + b;
        float* dst = a.ws_out + (slot * a.Hq + hq) * D + c * DQ;
#pragma unroll
        for (int j = 0; j < DQ; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(res[j], res[j + 1], res[j + 2], res[j + 3]);
        if (c == 0) a.ws_lse[slot * a.Hq + hq] = lse;
      }
    }
    if (nparts == 1) continue;
    // Each warp (KV head) takes its own ticket for (sequence, KV head). The warp barrier orders the lanes'
    // partial writes before lane 0's fence; the fence after the ticket orders the other parts' partials before
    // the lanes' reads, again through the warp barrier.
    __syncwarp();
    int ticket = 0;
    if (lane == 0) {
      __threadfence();
      ticket = int(atomicAdd(&a.ws_count[int64_t(b) * Hkv + h], 1u));
      __threadfence();
    }
    __syncwarp();
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket == nparts - 1) {
      merge_parts<D>(a, b, first_cta + b, nparts, h * REP, REP, lane, 32);
      if (lane == 0) a.ws_count[int64_t(b) * Hkv + h] = 0u;
    }
  }
  // After an abort, wait (bounded) for every page the producer issued beyond the last one seen, so no copy
  // lands in shared memory after the CTA is gone.
  if (misc[2] && warp == 0 && lane == 0) {
    const int issued = misc[1];
    for (int k = waited; k < issued; ++k)
      (void)mbar_wait(&full[k % a.nst], (k / a.nst) & 1, (a.wait_ns < 20000000ull ? a.wait_ns : 20000000ull));
  }
  }  // !TR
}

int64_t persist_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int sms) {
  const int64_t slots = B + sms;
  return kCounterBytesP + ((slots * Hq * 4 + 255) / 256) * 256 + ((slots * Hq * D * 4 + 255) / 256) * 256;
}

using PersistKernel = void (*)(PagedArgs, CUtensorMap, CUtensorMap);

// The kernel for (D, REP, KIND): up to four query heads per KV head take the transposed consumers, eight the
// head-major ones. FP8 keys and values convert on the conversion unit (CONV 0) at D 128 with two query heads per
// KV head (the configs' shape, where that measured fastest), on the integer pipe (CONV 3) elsewhere.
template <int D, int REP>
constexpr int persist_copy() { return (REP <= 4 && D == 128) ? 4 : 0; }

template <int D, int REP, int KIND>
PersistKernel persist_kernel() {
  if constexpr (REP <= 4) {
    constexpr int kCopy = persist_copy<D, REP>();
    if constexpr (KIND == BPT_KV_FP8 && !(D == 128 && REP == 2)) return paged_attn_persistent_kernel<D, REP, KIND, kCopy, true, 3>;
    return paged_attn_persistent_kernel<D, REP, KIND, kCopy, true, 0>;
  } else {
    return paged_attn_persistent_kernel<D, REP, KIND, 0, false, 0>;
  }
}

template <int D, int REP, int KIND>
int launch_persist_t(const PagedArgs& a0, int flags, cudaStream_t stream) {
  PagedArgs a = a0;
  a.stall = (flags & BPT_FLAG_TEST_STALL) ? 1 : 0;
  a.wait_ns = a.stall ? kTestWaitNs : kWaitNs;
  // (the stall test needs every issued copy awaited in order: no early copies before the dependency wait)
  a.early = (flags & BPT_FLAG_PDL) && (flags & BPT_FLAG_KV_READY) && !a.stall ? 1 : 0;
  const int q_esize = a.q_dtype == BPT_DTYPE_F32 ? 4 : 2;
  constexpr int kCopy = persist_copy<D, REP>();
  const PersistLayout lay = persist_layout<D, kCopy>(a.Hkv, a.Hq, q_esize, a.scale_bytes);
  const int G = a.persist_ctas;
  // Everything but the stages and their two barriers: offsets, lengths, page lists, misc, the P tiles.
  const int fixed = 4 * (2 * a.B + 1) + 12 * a.max_cta_pages + 16 + 16 + a.Hkv * 32 * 4 * 4;
  // six stages of one page (32 KB for 8 KV heads at D 128) where they fit: config 2 measured 40.5, 37.3 and 37.0 us
  // per call at 4, 5 and 6
  const int slack = (kCopy & 4) ? 1024 : 0;  // the swizzled tiles' 1 KB alignment
  a.nst = max(2, min(kPersistStages, (kMaxSmemPerCta - fixed - slack) / (lay.stage_bytes + lay.aux_bytes + 16)));
  const int smem = a.nst * (lay.stage_bytes + lay.aux_bytes + 16) + fixed + slack;
  CUtensorMap tm_k, tm_v;
  std::memset(&tm_k, 0, sizeof(tm_k));
  std::memset(&tm_v, 0, sizeof(tm_v));
  if constexpr ((kCopy & 4) != 0) {
    // a pool [blocks][16 tokens][Hkv][D] of bytes as a 4-D tensor (D, tokens, heads, blocks): one box of a whole page
    // lands head-major, [head][token][D] with the 128-byte swizzle
    auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
    if (!encode) return set_error(BPT_ERR_UNSUPPORTED, "paged attention: the driver has no tensor-map encoder");
    const cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(kBS), cuuint64_t(a.Hkv), cuuint64_t(a.num_blocks)};
    const cuuint64_t strides[3] = {cuuint64_t(a.Hkv * D), cuuint64_t(D), cuuint64_t(a.page_bytes)};
    const cuuint32_t box[4] = {cuuint32_t(D), cuuint32_t(kBS), cuuint32_t(a.Hkv), 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int which = 0; which < 2; ++which) {
      CUresult r = encode(which ? &tm_v : &tm_k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4,
                          const_cast<uint8_t*>(which ? a.v_pool : a.k_pool), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) return set_error(BPT_ERR_CUDA, "paged attention: pool tensor map (%d)", int(r));
    }
  }
  const PersistKernel kernel = persist_kernel<D, REP, KIND>();
  int st = set_max_smem(reinterpret_cast<const void*>(kernel), smem);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G, 1, 1);
  cfg.blockDim = dim3(32 * (a.Hkv + 1), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BPT_FLAG_PDL) ? 1 : 0;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a, tm_k, tm_v);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "paged attention (persistent) launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

template <int D, int KIND>
int launch_persist(const PagedArgs& a, int rep, int flags, cudaStream_t stream) {
  switch (rep) {
    case 1: return launch_persist_t<D, 1, KIND>(a, flags, stream);
    case 2: return launch_persist_t<D, 2, KIND>(a, flags, stream);
    case 4: return launch_persist_t<D, 4, KIND>(a, flags, stream);
    case 8: return launch_persist_t<D, 8, KIND>(a, flags, stream);
  }
  return set_error(BPT_ERR_UNSUPPORTED, "paged attention: REP=%d not in {1, 2, 4, 8}", rep);
}
