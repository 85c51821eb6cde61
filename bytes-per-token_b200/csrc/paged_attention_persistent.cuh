// Persistent, warp-specialized paged decode attention with the split merge fused in (included by
// paged_attention.cu, inside its namespace; uses the MMA helpers of paged_attention_mma.cuh).
//
// Work split. The pages of all sequences, laid end to end, are cut into one equal contiguous range per CTA
// (one CTA per SM), so ragged lengths never unbalance the GPU. The piece of a sequence that falls inside one
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
constexpr int kPersistMaxCtaPages = 4096;
constexpr int64_t kCounterBytesP = 65536 * 4;  // the ticket counters, at the workspace's start (as paged_attend)

struct PersistLayout {
  int stage_bytes, kpitch, vpitch, kpage, vpage, q_off, q_bytes;
};

template <int D, int COPY>
__host__ __device__ inline PersistLayout persist_layout(int Hkv, int Hq, int q_esize, int scale_bytes) {
  PersistLayout p;
  const int rowb = Hkv * D;
  p.kpitch = (COPY & 1) ? rowb + 16 : rowb;
  p.vpitch = (COPY & 2) ? rowb + 16 : rowb;
  p.kpage = kBS * p.kpitch;
  p.vpage = kBS * p.vpitch;
  p.q_bytes = Hq * D * q_esize;
  p.q_off = p.kpage + p.vpage + 2 * scale_bytes;
  p.stage_bytes = (p.q_off + p.q_bytes + 127) & ~127;
  return p;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}


// The part's partials are all in: out[b] = sum_p w_p out_p / sum_p w_p, w_p = exp(lse_p - max lse), with the
// consumer threads spread over (query head, dim).
template <int D>
__device__ __forceinline__ void merge_parts(const PagedArgs& a, int b, int64_t s0, int nparts, int tid, int ncons) {
  for (int i = tid; i < a.Hq * D; i += ncons) {
    const int hq = i / D, d = i % D;
    float mx = -CUDART_INF_F;
    for (int p2 = 0; p2 < nparts; ++p2) mx = fmaxf(mx, __ldcg(&a.ws_lse[(s0 + p2) * a.Hq + hq]));
    float acc = 0.f, wsum = 0.f;
    if (mx != -CUDART_INF_F) {
#pragma unroll 4
      for (int p2 = 0; p2 < nparts; ++p2) {
        const float w = expf(__ldcg(&a.ws_lse[(s0 + p2) * a.Hq + hq]) - mx);
        wsum += w;
        acc += w * __ldcg(&a.ws_out[((s0 + p2) * a.Hq + hq) * D + d]);
      }
    }
    out_store(a.out, a.out_dtype, ((int64_t)b * a.Hq + hq) * D + d, wsum > 0.f ? acc / wsum : 0.f);
  }
}

// Consumers with tokens on the MMA's M dimension (REP <= 4). Per page:
//   QK   S^T[16 tokens x 8] = K[16 tokens x 16 dims] . Q^T      B columns: hi parts of heads 0..3, then lo parts
//   PV   O^T[16 dims x 8]  += V^T[16 dims x 16 tokens] . P^T   B columns: f16(p) of heads 0..3, then p - f16(p)
// so a page costs D/16 MMAs for each product, q is a constant B fragment (D/8 registers) and the output
// accumulator is D/4 registers. Lane (c, g) owns the columns 2c, 2c+1: heads hA = 2(c & 1), hA + 1, part c >> 1;
// hi and lo parts of a head meet with one shuffle (lane ^ 2). P goes from the QK layout (tokens on g) to the PV
// layout (tokens on c) through a small per-warp tile in shared memory.
template <int D, int REP, int KIND, int COPY>
__device__ __forceinline__ void consume_transposed(const PagedArgs& a, const PersistLayout& lay, uint8_t* stages,
                                                   uint64_t* full, uint64_t* empty, const int* off, const int* slen,
                                                   const int* pblk, const int* pseq, const int* plp, volatile int* misc,
                                                   float* ptile_all, int n, int per) {
  static_assert(REP <= 4, "four query heads per KV head at most in this layout");
  constexpr int KS = D / 16;  // QK k-steps
  constexpr int DQ = D / 4;   // key bytes per lane per token
  constexpr int VD = D / 8;   // value bytes (dims) per lane per token
  constexpr int MT = D / 16;  // PV m-tiles
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int h = warp, Hkv = a.Hkv, ncons = 32 * Hkv, cta = blockIdx.x;
  const int q_esize = a.q_dtype == BPT_DTYPE_F32 ? 4 : 2;
  const int hA = 2 * (c & 1);          // this lane's heads: hA, hA + 1
  const int ccol = g & 3, cpart = g >> 2;  // the B column this lane feeds: head ccol, part cpart
  float* ptile = ptile_all + warp * 32 * 4;
  float qscale = a.sm_scale * kLog2e;
  if constexpr (KIND == BPT_KV_FP8) qscale *= a.k_scale;
  float vscale = 1.f;
  if constexpr (KIND == BPT_KV_FP8) vscale = a.v_scale;

  uint32_t qb[KS][2];
  float m[2] = {-CUDART_INF_F, -CUDART_INF_F}, l[2] = {0.f, 0.f};
  float o[MT][4];
  int waited = 0;

  auto wait_page = [&](int k) {
    if (!misc[2]) {
      if (mbar_wait_warp(&full[k % a.nst], (k / a.nst) & 1))
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

    if (first) {  // q of this sequence as the QK B fragment: column g = head ccol, hi or lo part
      const uint8_t* qrow = stages + (k % a.nst) * lay.stage_bytes + lay.q_off +
                            (int64_t)(h * REP + (ccol < REP ? ccol : 0)) * D * q_esize;
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
        if (ccol >= REP) x[0] = x[1] = x[2] = x[3] = 0.f;
        uint32_t hi01, lo01, hi23, lo23;
        split2(x[0], x[1], hi01, lo01);
        split2(x[2], x[3], hi23, lo23);
        qb[ks][0] = cpart ? lo01 : hi01;
        qb[ks][1] = cpart ? lo23 : hi23;
      }
      m[0] = m[1] = -CUDART_INF_F;
      l[0] = l[1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    }

    // ---- QK^T: scores of heads hA, hA+1 at tokens g and g+8 of each page ----
    float s[2][4];  // [page][token g: hA, hA+1, token g+8: hA, hA+1]
    bool usable[2] = {false, false};
    int hi_tok[2] = {0, 0};
#pragma unroll
    for (int pg = 0; pg < 2; ++pg) {
      s[pg][0] = s[pg][1] = s[pg][2] = s[pg][3] = -CUDART_INF_F;
      if (pg < np) {
        const int kk = k + pg;
        const uint8_t* kp = stages + (kk % a.nst) * lay.stage_bytes;
        const __half* kscl = reinterpret_cast<const __half*>(kp + lay.kpage + lay.vpage);
        usable[pg] = pblk[kk] >= 0 && pblk[kk] < a.num_blocks;
        hi_tok[pg] = min(kBS, L - plp[kk] * kBS);
        const uint8_t* r0 = kp + g * lay.kpitch + h * D + c * DQ;
        const uint8_t* r1 = kp + (g + 8) * lay.kpitch + h * D + c * DQ;
        uint32_t w0[DQ / 4], w1[DQ / 4];
#pragma unroll
        for (int v = 0; v < DQ / 16; ++v) {
          const uint4 u0 = *reinterpret_cast<const uint4*>(r0 + 16 * v);
          const uint4 u1 = *reinterpret_cast<const uint4*>(r1 + 16 * v);
          w0[4 * v] = u0.x; w0[4 * v + 1] = u0.y; w0[4 * v + 2] = u0.z; w0[4 * v + 3] = u0.w;
          w1[4 * v] = u1.x; w1[4 * v + 1] = u1.y; w1[4 * v + 2] = u1.z; w1[4 * v + 3] = u1.w;
        }
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t af[4];
          word_to_b<KIND>(w0[ks], af[0], af[2]);  // token g: slots (2c, 2c+1) and (2c+8, 2c+9)
          word_to_b<KIND>(w1[ks], af[1], af[3]);  // token g+8
          mma_f16(acc[ks & 1], af, qb[ks][0], qb[ks][1]);
        }
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[e] = acc[0][e] + acc[1][e];
          v[e] += __shfl_xor_sync(0xffffffffu, v[e], 2);  // hi + lo parts of the head
        }
        const bool live0 = usable[pg] && g < hi_tok[pg];
        const bool live1 = usable[pg] && g + 8 < hi_tok[pg];
        float k0 = qscale, k1 = qscale;
        if constexpr (KIND == BPT_KV_INT8) {
          k0 *= live0 ? __half2float(kscl[g * Hkv + h]) : 0.f;
          k1 *= live1 ? __half2float(kscl[(g + 8) * Hkv + h]) : 0.f;
        }
        s[pg][0] = live0 ? v[0] * k0 : -CUDART_INF_F;
        s[pg][1] = live0 ? v[1] * k0 : -CUDART_INF_F;
        s[pg][2] = live1 ? v[2] * k1 : -CUDART_INF_F;
        s[pg][3] = live1 ? v[3] * k1 : -CUDART_INF_F;
      }
    }

    // ---- online softmax for heads hA, hA+1 over the step's tokens (lanes with the same c) ----
    float alpha[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float pm = fmaxf(fmaxf(s[0][hh], s[0][2 + hh]), fmaxf(s[1][hh], s[1][2 + hh]));
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 4));
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 8));
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 16));
      const float m_new = fmaxf(m[hh], pm);
      const float m_use = (m_new == -CUDART_INF_F) ? 0.f : m_new;
      alpha[hh] = exp2f(m[hh] - m_use);
      float ps = 0.f;
#pragma unroll
      for (int pg = 0; pg < 2; ++pg) {
        s[pg][hh] = exp2f(s[pg][hh] - m_use);
        s[pg][2 + hh] = exp2f(s[pg][2 + hh] - m_use);
        ps += s[pg][hh] + s[pg][2 + hh];
      }
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      l[hh] = l[hh] * alpha[hh] + ps;
      m[hh] = m_new;
    }
    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        o[mt][0] *= alpha[0]; o[mt][2] *= alpha[0];
        o[mt][1] *= alpha[1]; o[mt][3] *= alpha[1];
      }
    }

    // ---- P through the warp's tile: [token][head], written by the hi-part lanes (INT8: times the value scale) ----
    if (c < 2) {
#pragma unroll
      for (int pg = 0; pg < 2; ++pg) {
        if (pg < np) {
          float vs0 = 1.f, vs1 = 1.f;
          if constexpr (KIND == BPT_KV_INT8) {
            const uint8_t* kp = stages + ((k + pg) % a.nst) * lay.stage_bytes;
            const __half* vscl = reinterpret_cast<const __half*>(kp + lay.kpage + lay.vpage + a.scale_bytes);
            vs0 = (usable[pg] && g < hi_tok[pg]) ? __half2float(vscl[g * Hkv + h]) : 0.f;
            vs1 = (usable[pg] && g + 8 < hi_tok[pg]) ? __half2float(vscl[(g + 8) * Hkv + h]) : 0.f;
          }
          *reinterpret_cast<float2*>(ptile + (pg * 16 + g) * 4 + hA) = make_float2(s[pg][0] * vs0, s[pg][1] * vs0);
          *reinterpret_cast<float2*>(ptile + (pg * 16 + g + 8) * 4 + hA) = make_float2(s[pg][2] * vs1, s[pg][3] * vs1);
        }
      }
    }
    __syncwarp();

    // ---- PV^T: value rows of tokens 2c, 2c+1, 2c+8, 2c+9; dims [g*VD, (g+1)*VD) ----
#pragma unroll
    for (int pg = 0; pg < 2; ++pg) {
      if (pg < np && usable[pg]) {
        const uint8_t* vp = stages + ((k + pg) % a.nst) * lay.stage_bytes + lay.kpage;
        const int tok[4] = {2 * c, 2 * c + 1, 8 + 2 * c, 9 + 2 * c};
        float pw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) pw[j] = ptile[(pg * 16 + tok[j]) * 4 + ccol];
        uint32_t b0, b1;
        {
          uint32_t h01, l01, h23, l23;
          split2(pw[0], pw[1], h01, l01);
          split2(pw[2], pw[3], h23, l23);
          b0 = cpart ? l01 : h01;
          b1 = cpart ? l23 : h23;
        }
        uint32_t vr[4][VD / 4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint8_t* row = vp + tok[j] * lay.vpitch + h * D + g * VD;
          if constexpr (VD == 16) {
            const uint4 u = *reinterpret_cast<const uint4*>(row);
            vr[j][0] = u.x; vr[j][1] = u.y; vr[j][2] = u.z; vr[j][3] = u.w;
          } else {
            const uint2 u = *reinterpret_cast<const uint2*>(row);
            vr[j][0] = u.x; vr[j][1] = u.y;
          }
          if (!(tok[j] < hi_tok[pg])) {  // rows past the sequence may hold any bytes
#pragma unroll
            for (int w = 0; w < VD / 4; ++w) vr[j][w] = 0u;
          }
        }
        uint32_t p01[VD], p89[VD];  // f16x2 (token pair) per lane dim
#pragma unroll
        for (int w = 0; w < VD / 4; ++w) {
          word_to_b<KIND>(__byte_perm(vr[0][w], vr[1][w], 0x5140u), p01[4 * w], p01[4 * w + 1]);
          word_to_b<KIND>(__byte_perm(vr[0][w], vr[1][w], 0x7362u), p01[4 * w + 2], p01[4 * w + 3]);
          word_to_b<KIND>(__byte_perm(vr[2][w], vr[3][w], 0x5140u), p89[4 * w], p89[4 * w + 1]);
          word_to_b<KIND>(__byte_perm(vr[2][w], vr[3][w], 0x7362u), p89[4 * w + 2], p89[4 * w + 3]);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint32_t af[4] = {p01[mt], p01[VD / 2 + mt], p89[mt], p89[VD / 2 + mt]};
          mma_f16(o[mt], af, b0, b1);
        }
      }
    }
    __syncwarp();

    // ---- release the step's stages ----
    if (lane == 0) {
      mbar_arrive(&empty[k % a.nst]);
      if (np == 2) mbar_arrive(&empty[(k + 1) % a.nst]);
    }
    k += np;
    if (!last) continue;

    // ---- end of a part ----
    const int first_cta = off[b] / per;
    const int last_cta = (off[b + 1] - 1) / per;
    const int nparts = last_cta - first_cta + 1;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][e] += __shfl_xor_sync(0xffffffffu, o[mt][e], 2);
    if (c < 2) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int head = hA + hh;
        if (head >= REP) continue;
        const int hq = h * REP + head;
        const float inv = l[hh] > 0.f ? vscale / l[hh] : 0.f;
        const float lse = l[hh] > 0.f ? (m[hh] + log2f(l[hh])) * kLn2 : -CUDART_INF_F;
        float res[VD];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          res[mt] = o[mt][hh] * inv;
          res[VD / 2 + mt] = o[mt][2 + hh] * inv;
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
    }
    if (nparts == 1) continue;
    __threadfence();
    consumer_sync(ncons);
    if (tid == 0) misc[0] = int(atomicAdd(&a.ws_count[b], 1u));
    consumer_sync(ncons);
    if (misc[0] == nparts - 1) {
      __threadfence();
      merge_parts<D>(a, b, first_cta + b, nparts, tid, ncons);
      if (tid == 0) a.ws_count[b] = 0u;
    }
    consumer_sync(ncons);
  }
  if (misc[2] && warp == 0 && lane == 0) {
    const int issued = misc[1];
    for (int k = waited; k < issued; ++k) (void)mbar_wait(&full[k % a.nst], (k / a.nst) & 1, 20000000ull);
  }
}

template <int D, int REP, int KIND, int COPY, bool TR>
__global__ void __launch_bounds__(32 * (kMmaMaxHkv + 1), 1) paged_attn_persistent_kernel(const PagedArgs a) {
  constexpr int KS = D / 16, DQ = D / 4, VB = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int Hkv = a.Hkv, B = a.B, G = gridDim.x, cta = blockIdx.x;
  const int q_esize = a.q_dtype == BPT_DTYPE_F32 ? 4 : 2;
  const PersistLayout lay = persist_layout<D, COPY>(Hkv, a.Hq, q_esize, a.scale_bytes);
  const int rowb = Hkv * D;

  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.nst * lay.stage_bytes);
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
  pdl_wait();

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
  const int per = (P + G - 1) / G;
  const int g0 = min(P, cta * per), g1 = min(P, g0 + per);
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
  if (cta == 0)  // a sequence with no tokens gets a zero output and is in nobody's range
    for (int i = tid; i < B * a.Hq * D; i += blockDim.x)
      if (off[i / (a.Hq * D) + 1] == off[i / (a.Hq * D)]) out_store(a.out, a.out_dtype, i, 0.f);
  __syncthreads();
  if (n <= 0) return;

  const bool producer = warp == Hkv;
  if (producer) {
    // ---------------- producer warp ----------------
    const uint64_t policy = l2_policy_evict_first();
    for (int k = 0; k < n; ++k) {
      const int st = k % a.nst;
      if (misc[2]) break;
      if (k >= a.nst && !mbar_wait_warp(&empty[st], ((k / a.nst) - 1) & 1)) {
        misc[2] = 1;
        break;
      }
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
        const int t = lane & 15;
        if constexpr (COPY & 1) {
          if (lane < 16) bulk_g2s_evict_first(base + t * lay.kpitch, ksrc + t * rowb, rowb, &full[st], policy);
        } else {
          if (lane == 0) bulk_g2s_evict_first(base, ksrc, a.page_bytes, &full[st], policy);
        }
        if constexpr (COPY & 2) {
          if (lane >= 16) bulk_g2s_evict_first(base + lay.kpage + t * lay.vpitch, vsrc + t * rowb, rowb, &full[st], policy);
        } else {
          if (lane == 16) bulk_g2s_evict_first(base + lay.kpage, vsrc, a.page_bytes, &full[st], policy);
        }
        if constexpr (KIND == BPT_KV_INT8) {
          if (lane == 1)
            bulk_g2s(base + lay.kpage + lay.vpage, reinterpret_cast<const uint8_t*>(a.k_scales) + (int64_t)blk * a.scale_bytes,
                     a.scale_bytes, &full[st]);
          if (lane == 2)
            bulk_g2s(base + lay.kpage + lay.vpage + a.scale_bytes,
                     reinterpret_cast<const uint8_t*>(a.v_scales) + (int64_t)blk * a.scale_bytes, a.scale_bytes, &full[st]);
        }
      }
      if (first && lane == 3)
        bulk_g2s(base + lay.q_off, static_cast<const uint8_t*>(a.q) + (int64_t)b * lay.q_bytes, lay.q_bytes, &full[st]);
      __syncwarp();
      if (lane == 0) misc[1] = k + 1;
    }
    return;
  }

  // ---------------- consumer warps: one per KV head ----------------
  if constexpr (TR) {
    consume_transposed<D, REP, KIND, COPY>(a, lay, stages, full, empty, off, slen, pblk, pseq, plp, misc, ptile, n, per);
    return;
  } else {
  // A step covers one page, or two consecutive pages of the same part (32 tokens): the two pages' QK chains and
  // PV accumulations interleave, and the softmax, barrier wait and release costs are paid once per two pages.
  const int h = warp;
  const int ncons = 32 * Hkv;
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
      if (mbar_wait_warp(&full[k % a.nst], (k / a.nst) & 1))
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
      const uint8_t* kp0 = stages + (k % a.nst) * lay.stage_bytes;
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
        const __half* kscl = reinterpret_cast<const __half*>(kp + lay.kpage + lay.vpage);
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
        const __half* vscl = reinterpret_cast<const __half*>(vp + lay.vpage + a.scale_bytes);
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
    const int first_cta = off[b] / per;
    const int last_cta = (off[b + 1] - 1) / per;
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
    __threadfence();
    consumer_sync(ncons);
    if (tid == 0) misc[0] = int(atomicAdd(&a.ws_count[b], 1u));
    consumer_sync(ncons);
    if (misc[0] == nparts - 1) {
      __threadfence();
      // out[b, hq, d] = sum_parts w_p * out_p / sum_parts w_p, w_p = exp(lse_p - max lse); consumer threads over (hq, d)
      const int64_t s0 = first_cta + b;
      for (int i = tid; i < a.Hq * D; i += ncons) {
        const int hq = i / D, d = i % D;
        float mx = -CUDART_INF_F;
        for (int p2 = 0; p2 < nparts; ++p2) mx = fmaxf(mx, __ldcg(&a.ws_lse[(s0 + p2) * a.Hq + hq]));
        float acc = 0.f, wsum = 0.f;
        if (mx != -CUDART_INF_F) {
#pragma unroll 4
          for (int p2 = 0; p2 < nparts; ++p2) {
            const float w = expf(__ldcg(&a.ws_lse[(s0 + p2) * a.Hq + hq]) - mx);
            wsum += w;
            acc += w * __ldcg(&a.ws_out[((s0 + p2) * a.Hq + hq) * D + d]);
          }
        }
        out_store(a.out, a.out_dtype, ((int64_t)b * a.Hq + hq) * D + d, wsum > 0.f ? acc / wsum : 0.f);
      }
      if (tid == 0) a.ws_count[b] = 0u;
    }
    consumer_sync(ncons);
  }
  // After an abort, wait (bounded) for every page the producer issued beyond the last one seen, so no copy
  // lands in shared memory after the CTA is gone.
  if (misc[2] && warp == 0 && lane == 0) {
    const int issued = misc[1];
    for (int k = waited; k < issued; ++k) (void)mbar_wait(&full[k % a.nst], (k / a.nst) & 1, 20000000ull);
  }
  }  // !TR
}

int64_t persist_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int sms) {
  const int64_t slots = B + sms;
  return kCounterBytesP + ((slots * Hq * 4 + 255) / 256) * 256 + ((slots * Hq * D * 4 + 255) / 256) * 256;
}

template <int D, int REP, int KIND, int COPY>
int launch_persist_t(const PagedArgs& a0, int flags, cudaStream_t stream) {
  static const int transposed = env_int("BPT_PAGED_TRANSPOSED", 1);
  constexpr bool kTR = REP <= 4;
  PagedArgs a = a0;
  const int q_esize = a.q_dtype == BPT_DTYPE_F32 ? 4 : 2;
  const PersistLayout lay = persist_layout<D, COPY>(a.Hkv, a.Hq, q_esize, a.scale_bytes);
  const int G = a.persist_ctas;
  const int fixed = 2 * 8 * 8 + 4 * (2 * a.B + 1) + 12 * a.max_cta_pages + 16 + 16 + a.Hkv * 32 * 4 * 4;
  a.nst = max(2, min(env_int("BPT_PAGED_STAGES", 5), (210 * 1024 - fixed) / lay.stage_bytes));
  const int smem = a.nst * lay.stage_bytes + 2 * 8 * a.nst + 4 * (2 * a.B + 1) + 12 * a.max_cta_pages + 16 + 16 +
                   a.Hkv * 32 * 4 * 4;
  auto kernel = (kTR && transposed) ? paged_attn_persistent_kernel<D, REP, KIND, COPY, kTR>
                                    : paged_attn_persistent_kernel<D, REP, KIND, COPY, false>;
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
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "paged attention (persistent) launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

template <int D, int KIND, int COPY>
int launch_persist_rep(const PagedArgs& a, int rep, int flags, cudaStream_t stream) {
  switch (rep) {
    case 1: return launch_persist_t<D, 1, KIND, COPY>(a, flags, stream);
    case 2: return launch_persist_t<D, 2, KIND, COPY>(a, flags, stream);
    case 4: return launch_persist_t<D, 4, KIND, COPY>(a, flags, stream);
    case 8: return launch_persist_t<D, 8, KIND, COPY>(a, flags, stream);
  }
  return set_error(BPT_ERR_UNSUPPORTED, "paged attention: REP=%d not in {1, 2, 4, 8}", rep);
}

template <int D, int KIND>
int launch_persist(const PagedArgs& a, int rep, int flags, cudaStream_t stream) {
  static const int copy = env_int("BPT_PAGED_PCOPY", 0);
  if (copy == 3) return launch_persist_rep<D, KIND, 3>(a, rep, flags, stream);
  return launch_persist_rep<D, KIND, 0>(a, rep, flags, stream);
}
