// Decode attention over the reference's contiguous KIVI cache (kernels/reference.py QuantKV), bits 4, 8 or 16:
// the drop-in for kernel 2 behind decode_attention (kernels/kv_attention.py:190-245), same per-split outputs.
//
// Grid (n_splits, B * Hkv), four warps per CTA. The split's tokens are walked in key groups of 32; warp w takes
// groups w, w + 4, ... with its own online softmax, and the four states are combined at the end. Inside a group
// lane t owns token t: it streams its key row with 16-byte loads and dots it against the group's scaled query
// (the key grid folded into q once per group, as the reference kernel does: score = sum_d (q_d s_d) code_d -
// sum_d q_d s_d z_d), so the softmax of the group is a plain warp reduction. Values are read row by row with
// lanes across the head dim; the value grid folds into the weight (p_t s_t) and one shift per group.
#include <math_constants.h>

#include "common.cuh"

namespace bpt {
namespace {

constexpr int kWarps = 4;
constexpr int kGroup = 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct KiviArgs {
  const void* q;
  int q_dtype;
  int64_t q_sb, q_sh;
  const uint8_t* k_codes;
  const uint8_t* v_codes;
  const __half* k_scale;
  const __half* k_zero;
  const __half* v_scale;
  const __half* v_zero;
  const int32_t* lengths;
  int B, Hq, Hkv;
  int64_t t_max, n_groups;
  int split, n_splits;
  float sm_scale;
  float* out_partial;
  float* lse_partial;
};

__device__ __forceinline__ float qload(const void* q, int dt, int64_t i) {
  if (dt == BPT_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(q)[i]);
  if (dt == BPT_DTYPE_F16) return __half2float(static_cast<const __half*>(q)[i]);
  return static_cast<const float*>(q)[i];
}

// Byte k of a word, an unsigned code 0..255, as a float, exactly: the byte becomes the low mantissa byte of 2^23 + code
// (one PRMT and one FADD at full rate, where a conversion instruction runs at the conversion unit's lower rate).
__device__ __forceinline__ float code_f(uint32_t w, int k) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | uint32_t(k))) - 8388608.0f;
}

// Stored element e of a row as a float (its code for bits 4/8 low nibble handled by the caller).
template <int BITS, int CDT>
__device__ __forceinline__ float elem(const uint8_t* row, int e) {
  if constexpr (BITS == 8) return float(row[e]);
  if constexpr (BITS == 16 && CDT == BPT_DTYPE_F32) return reinterpret_cast<const float*>(row)[e];
  if constexpr (BITS == 16 && CDT == BPT_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(row)[e]);
  if constexpr (BITS == 16 && CDT == BPT_DTYPE_BF16)
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[e]);
  return 0.f;
}

template <int D, int REP, int BITS, int CDT>
__global__ void __launch_bounds__(kWarps * 32) kivi_attn_kernel(const KiviArgs a) {
  constexpr int ESZ = BITS == 16 ? (CDT == BPT_DTYPE_F32 ? 4 : 2) : 1;        // bytes per stored element
  constexpr int ROWB = BITS == 4 ? D / 2 : D * ESZ;                          // bytes per token row
  constexpr int CB = ROWB < 16 ? ROWB : 16;                                   // bytes per load
  constexpr int NCH = ROWB / CB;                                              // loads per row
  constexpr int PV_E = BITS == 4 ? D / 2 : D;                                 // stored elements per row
  constexpr int EPL = PV_E >= 32 ? PV_E / 32 : 1;                             // elements per lane in PV
  constexpr int NACC = BITS == 4 ? 2 * EPL : EPL;

  __shared__ float q_s[REP][D];
  __shared__ __align__(16) float qs_buf[kWarps * REP * D];  // the group's scaled queries; reused to combine the warps
  __shared__ float bias_s[kWarps][REP];
  __shared__ float p_s[kWarps][kGroup][REP];
  __shared__ float m_s[kWarps][REP], l_s[kWarps][REP];
  float (*qs_s)[REP][D] = reinterpret_cast<float (*)[REP][D]>(qs_buf);
  float (*acc_s)[REP][D] = reinterpret_cast<float (*)[REP][D]>(qs_buf);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.Hkv, h = bh % a.Hkv;
  pdl_wait();
  const int L = min(a.lengths[b], int(a.t_max));  // the cache holds t_max tokens
  const int t0 = s * a.split;
  const int t1 = min(L, t0 + a.split);

  // The split's code rows and grids are requested into L2 up front (one 128-byte line per thread in turn): the
  // group loop's chain of dependent loads (grids, key rows, value grids, value rows) then waits on L2, not DRAM.
  if (t1 > t0) {
    const int64_t r0 = (int64_t)bh * a.t_max + t0, nt = t1 - t0;
    auto prefetch = [&](const void* p, int64_t bytes) {
      const char* c = static_cast<const char*>(p);
      for (int64_t o = int64_t(tid) * 128; o < bytes; o += int64_t(kWarps * 32) * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(c + o));
    };
    prefetch(a.k_codes + r0 * ROWB, nt * ROWB);
    prefetch(a.v_codes + r0 * ROWB, nt * ROWB);
    if constexpr (BITS != 16) {
      prefetch(a.v_scale + r0, nt * 2);
      prefetch(a.v_zero + r0, nt * 2);
      const int64_t g0 = (int64_t)bh * a.n_groups + t0 / kGroup, ng = (nt + kGroup - 1) / kGroup;
      prefetch(a.k_scale + g0 * D, ng * D * 2);
      prefetch(a.k_zero + g0 * D, ng * D * 2);
    }
  }

  for (int i = tid; i < REP * D; i += kWarps * 32) {
    const int r = i / D, d = i % D;
    q_s[r][d] = qload(a.q, a.q_dtype, (int64_t)b * a.q_sb + (int64_t)(h * REP + r) * a.q_sh + d) * a.sm_scale * kLog2e;
  }
  __syncthreads();

  float m[REP], l[REP], acc[REP][NACC];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -CUDART_INF_F;
    l[r] = 0.f;
#pragma unroll
    for (int j = 0; j < NACC; ++j) acc[r][j] = 0.f;
  }

  const int64_t row0 = (int64_t)bh * a.t_max;
  for (int g0 = t0; g0 < t1; g0 += kGroup * kWarps) {
    const int gs = g0 + warp * kGroup;  // this warp's group start
    if (gs >= t1) continue;
    const int valid = min(kGroup, t1 - gs);

    // ---- fold this group's key grid into q ----
    if constexpr (BITS != 16) {
      const int64_t grid = ((int64_t)bh * a.n_groups + gs / kGroup) * D;
      float bias[REP];
#pragma unroll
      for (int r = 0; r < REP; ++r) bias[r] = 0.f;
#pragma unroll
      for (int d = lane; d < D; d += 32) {
        const float ks = __half2float(a.k_scale[grid + d]);
        const float kz = __half2float(a.k_zero[grid + d]);
#pragma unroll
        for (int r = 0; r < REP; ++r) {
          const float qs = q_s[r][d] * ks;
          qs_s[warp][r][d] = qs;
          bias[r] -= qs * kz;
        }
      }
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        bias[r] = warp_sum(bias[r]);
        if (lane == 0) bias_s[warp][r] = bias[r];
      }
    } else {
      for (int d = lane; d < D; d += 32)
#pragma unroll
        for (int r = 0; r < REP; ++r) qs_s[warp][r][d] = q_s[r][d];
      if (lane < REP) bias_s[warp][lane] = 0.f;
    }
    __syncwarp();

    // ---- QK: lane t owns token gs + t (its value grid requested first, so that load overlaps the dot) ----
    const int t = lane;
    float vsc = 1.f, vz = 0.f;
    if constexpr (BITS != 16) {
      if (t < valid) {
        vsc = __half2float(a.v_scale[row0 + gs + t]);
        vz = __half2float(a.v_zero[row0 + gs + t]);
      }
    }
    float sc[REP];
#pragma unroll
    for (int r = 0; r < REP; ++r) sc[r] = 0.f;
    if (t < valid) {
      const uint8_t* krow = a.k_codes + (row0 + gs + t) * ROWB;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        uint8_t buf[CB];
        if constexpr (CB == 16) {
          *reinterpret_cast<uint4*>(buf) = __ldg(reinterpret_cast<const uint4*>(krow + c * CB));
        } else if constexpr (CB == 8) {
          *reinterpret_cast<uint2*>(buf) = __ldg(reinterpret_cast<const uint2*>(krow + c * CB));
        } else {
#pragma unroll
          for (int j = 0; j < CB; ++j) buf[j] = krow[c * CB + j];
        }
        if constexpr (BITS == 4 && CB == 16) {  // byte e: dims e (low nibble) and e + D/2 (high nibble)
          const uint32_t* wv = reinterpret_cast<const uint32_t*>(buf);
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const int e0 = c * CB + 4 * k4;
            const uint32_t lo = wv[k4] & 0x0F0F0F0Fu, hi = (wv[k4] >> 4) & 0x0F0F0F0Fu;
            float xl[4], xh[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              xl[k] = code_f(lo, k);
              xh[k] = code_f(hi, k);
            }
#pragma unroll
            for (int r = 0; r < REP; ++r) {
              const float4 ql = *reinterpret_cast<const float4*>(&qs_s[warp][r][e0]);
              const float4 qh = *reinterpret_cast<const float4*>(&qs_s[warp][r][e0 + D / 2]);
              sc[r] = fmaf(ql.x, xl[0], fmaf(ql.y, xl[1], fmaf(ql.z, xl[2], fmaf(ql.w, xl[3], sc[r]))));
              sc[r] = fmaf(qh.x, xh[0], fmaf(qh.y, xh[1], fmaf(qh.z, xh[2], fmaf(qh.w, xh[3], sc[r]))));
            }
          }
        } else if constexpr (BITS == 4) {
#pragma unroll
          for (int j = 0; j < CB; ++j) {
            const int e = c * CB + j;
            const float lo = float(buf[j] & 0xF), hi = float(buf[j] >> 4);
#pragma unroll
            for (int r = 0; r < REP; ++r) sc[r] += qs_s[warp][r][e] * lo + qs_s[warp][r][e + D / 2] * hi;
          }
        } else if constexpr (BITS == 8 && CB == 16) {
          const uint32_t* wv = reinterpret_cast<const uint32_t*>(buf);
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const int e0 = c * CB + 4 * k4;
            float x[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) x[k] = code_f(wv[k4], k);
#pragma unroll
            for (int r = 0; r < REP; ++r) {
              const float4 qv = *reinterpret_cast<const float4*>(&qs_s[warp][r][e0]);
              sc[r] = fmaf(qv.x, x[0], fmaf(qv.y, x[1], fmaf(qv.z, x[2], fmaf(qv.w, x[3], sc[r]))));
            }
          }
        } else if constexpr (BITS == 16 && CB == 16 && CDT != BPT_DTYPE_F32) {  // eight 16-bit elements per load
          const int e0 = c * 8;
          float x[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) x[j] = elem<BITS, CDT>(buf, j);
#pragma unroll
          for (int r = 0; r < REP; ++r) {
            const float4 q0 = *reinterpret_cast<const float4*>(&qs_s[warp][r][e0]);
            const float4 q1 = *reinterpret_cast<const float4*>(&qs_s[warp][r][e0 + 4]);
            sc[r] = fmaf(q0.x, x[0], fmaf(q0.y, x[1], fmaf(q0.z, x[2], fmaf(q0.w, x[3], sc[r]))));
            sc[r] = fmaf(q1.x, x[4], fmaf(q1.y, x[5], fmaf(q1.z, x[6], fmaf(q1.w, x[7], sc[r]))));
          }
        } else if constexpr (BITS == 16 && CB == 16) {  // four fp32 elements per load
          const int e0 = c * 4;
          const float* xf = reinterpret_cast<const float*>(buf);
#pragma unroll
          for (int r = 0; r < REP; ++r) {
            const float4 q0 = *reinterpret_cast<const float4*>(&qs_s[warp][r][e0]);
            sc[r] = fmaf(q0.x, xf[0], fmaf(q0.y, xf[1], fmaf(q0.z, xf[2], fmaf(q0.w, xf[3], sc[r]))));
          }
        } else {
          constexpr int EPC = CB / ESZ;
#pragma unroll
          for (int j = 0; j < EPC; ++j) {
            const int e = c * EPC + j;
            const float x = elem<BITS, CDT>(buf, j);
#pragma unroll
            for (int r = 0; r < REP; ++r) sc[r] += qs_s[warp][r][e] * x;
          }
        }
      }
    }
    // ---- online softmax over the group (base 2): lanes are tokens ----
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float score = t < valid ? sc[r] + bias_s[warp][r] : -CUDART_INF_F;
      const float m_new = fmaxf(m[r], warp_max(score));
      const float alpha = exp2f(m[r] - m_new);
      const float p = exp2f(score - m_new);
      l[r] = l[r] * alpha + warp_sum(p);
      m[r] = m_new;
#pragma unroll
      for (int j = 0; j < NACC; ++j) acc[r][j] *= alpha;
      const float pw = p * vsc;  // the value grid folds into the weight
      p_s[warp][t][r] = pw;
      if constexpr (BITS != 16) {
        const float shift = warp_sum(pw * vz);
#pragma unroll
        for (int j = 0; j < NACC; ++j) acc[r][j] -= shift;
      }
    }
    __syncwarp();

    // ---- PV: lane owns stored elements [lane*EPL, lane*EPL + EPL) of each row; unrolled by 8 so eight rows'
    // loads are in flight together (4 and 16 measured slower overall) ----
    if (lane * EPL < PV_E) {
#pragma unroll 8
      for (int tt = 0; tt < valid; ++tt) {
        const uint8_t* vrow = a.v_codes + (row0 + gs + tt) * ROWB;
        float pr[REP];
#pragma unroll
        for (int r = 0; r < REP; ++r) pr[r] = p_s[warp][tt][r];
        if constexpr ((BITS == 4 || BITS == 8) && (EPL == 2 || EPL == 4)) {
          // the lane's EPL bytes in one load: codes as floats without the conversion unit
          const uint32_t w = EPL == 4 ? *reinterpret_cast<const uint32_t*>(vrow + lane * EPL)
                                      : uint32_t(*reinterpret_cast<const uint16_t*>(vrow + lane * EPL));
          const uint32_t lo = BITS == 4 ? (w & 0x0F0F0F0Fu) : w, hi = (w >> 4) & 0x0F0F0F0Fu;
#pragma unroll
          for (int j = 0; j < EPL; ++j) {
            const float xl = code_f(lo, j);
#pragma unroll
            for (int r = 0; r < REP; ++r) acc[r][j] = fmaf(pr[r], xl, acc[r][j]);
            if constexpr (BITS == 4) {
              const float xh = code_f(hi, j);
#pragma unroll
              for (int r = 0; r < REP; ++r) acc[r][EPL + j] = fmaf(pr[r], xh, acc[r][EPL + j]);
            }
          }
        } else if constexpr (BITS == 16 && CDT != BPT_DTYPE_F32 && EPL == 4) {  // four 16-bit elements in one load
          const uint2 w = *reinterpret_cast<const uint2*>(vrow + lane * EPL * ESZ);
          const uint32_t ww[2] = {w.x, w.y};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t bits16 = (j & 1) ? (ww[j >> 1] >> 16) : (ww[j >> 1] & 0xFFFFu);
            const float x = CDT == BPT_DTYPE_BF16 ? __uint_as_float(bits16 << 16)
                                                  : __half2float(__ushort_as_half(uint16_t(bits16)));
#pragma unroll
            for (int r = 0; r < REP; ++r) acc[r][j] = fmaf(pr[r], x, acc[r][j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < EPL; ++j) {
            const int e = lane * EPL + j;
            if constexpr (BITS == 4) {
              const uint8_t byte = vrow[e];
              const float lo = float(byte & 0xF), hi = float(byte >> 4);
#pragma unroll
              for (int r = 0; r < REP; ++r) {
                acc[r][j] += pr[r] * lo;
                acc[r][EPL + j] += pr[r] * hi;
              }
            } else {
              const float x = elem<BITS, CDT>(vrow, e);
#pragma unroll
              for (int r = 0; r < REP; ++r) acc[r][j] += pr[r] * x;
            }
          }
        }
      }
    }
    __syncwarp();
  }

  // ---- combine the four warps (acc_s aliases qs_s: every warp is done with its queries first) ----
  __syncthreads();
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    if (lane == 0) {
      m_s[warp][r] = m[r];
      l_s[warp][r] = l[r];
    }
    if (lane * EPL < PV_E) {
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const int e = lane * EPL + j;
        acc_s[warp][r][e] = acc[r][j];
        if constexpr (BITS == 4) acc_s[warp][r][e + D / 2] = acc[r][EPL + j];
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < REP * D; i += kWarps * 32) {
    const int r = i / D, d = i % D;
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, m_s[w][r]);
    float lsum = 0.f, o = 0.f;
    if (mx != -CUDART_INF_F) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float f = exp2f(m_s[w][r] - mx);
        lsum += l_s[w][r] * f;
        o += acc_s[w][r][d] * f;
      }
    }
    const int hq = h * REP + r;
    const int64_t orow = ((int64_t)b * a.Hq + hq) * a.n_splits + s;
    a.out_partial[orow * D + d] = lsum > 0.f ? o / lsum : 0.f;
    if (d == 0) a.lse_partial[orow] = lsum > 0.f ? (mx + log2f(lsum)) * kLn2 : -CUDART_INF_F;
  }
}

template <int D, int REP, int BITS, int CDT>
int launch_k(const KiviArgs& a, cudaStream_t stream) {
  kivi_attn_kernel<D, REP, BITS, CDT><<<dim3(a.n_splits, a.B * a.Hkv), kWarps * 32, 0, stream>>>(a);
  return check_launch("kivi attention");
}

template <int D, int REP>
int launch_bits(const KiviArgs& a, int bits, int cdt, cudaStream_t stream) {
  if (bits == 4) return launch_k<D, REP, 4, BPT_DTYPE_F32>(a, stream);
  if (bits == 8) return launch_k<D, REP, 8, BPT_DTYPE_F32>(a, stream);
  if (cdt == BPT_DTYPE_F32) return launch_k<D, REP, 16, BPT_DTYPE_F32>(a, stream);
  if (cdt == BPT_DTYPE_F16) return launch_k<D, REP, 16, BPT_DTYPE_F16>(a, stream);
  return launch_k<D, REP, 16, BPT_DTYPE_BF16>(a, stream);
}

template <int D>
int launch_rep(const KiviArgs& a, int rep, int bits, int cdt, cudaStream_t stream) {
  switch (rep) {
    case 1: return launch_bits<D, 1>(a, bits, cdt, stream);
    case 2: return launch_bits<D, 2>(a, bits, cdt, stream);
    case 4: return launch_bits<D, 4>(a, bits, cdt, stream);
    case 8: return launch_bits<D, 8>(a, bits, cdt, stream);
  }
  return set_error(BPT_ERR_UNSUPPORTED, "kivi attention: REP=%d not in {1, 2, 4, 8}", rep);
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" int bpt_kivi_decode_partials(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h, int bits,
                                        int code_dtype, const void* k_codes, const void* v_codes, const void* k_scale,
                                        const void* k_zero, const void* v_scale, const void* v_zero,
                                        const int32_t* lengths, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                        int64_t t_max, int64_t n_groups, int64_t group, int64_t split, int64_t n_splits,
                                        float sm_scale, float* out_partial, float* lse_partial, void* stream) {
  BPT_REQUIRE(q && k_codes && v_codes && lengths && out_partial && lse_partial, BPT_ERR_INVALID,
              "kivi attention: null pointer");
  BPT_REQUIRE(bits == 4 || bits == 8 || bits == 16, BPT_ERR_INVALID, "kivi attention: bits %d", bits);
  BPT_REQUIRE(bits == 16 || (k_scale && k_zero && v_scale && v_zero), BPT_ERR_INVALID, "kivi attention: grids missing");
  BPT_REQUIRE(bits != 16 || code_dtype == BPT_DTYPE_F32 || code_dtype == BPT_DTYPE_F16 || code_dtype == BPT_DTYPE_BF16,
              BPT_ERR_INVALID, "kivi attention: 16-bit cache dtype %d", code_dtype);
  BPT_REQUIRE(q_dtype == BPT_DTYPE_F32 || q_dtype == BPT_DTYPE_F16 || q_dtype == BPT_DTYPE_BF16, BPT_ERR_INVALID,
              "kivi attention: q dtype %d", q_dtype);
  BPT_REQUIRE(group == kGroup, BPT_ERR_UNSUPPORTED, "kivi attention: key group %lld (this build: 32)", (long long)group);
  BPT_REQUIRE(split >= kGroup && split % kGroup == 0, BPT_ERR_INVALID,
              "kivi attention: split %lld must be a multiple of the key group %lld", (long long)split, (long long)group);
  BPT_REQUIRE(B >= 1 && Hkv >= 1 && Hq % Hkv == 0 && n_splits >= 1 && n_splits < 65536 && B * Hkv < 65536,
              BPT_ERR_INVALID, "kivi attention: bad shape");
  BPT_REQUIRE(t_max >= 1 && n_groups * group >= t_max, BPT_ERR_INVALID, "kivi attention: grids do not cover t_max");
  const int esz = bits == 16 ? (code_dtype == BPT_DTYPE_F32 ? 4 : 2) : 1;
  const int64_t rowb = bits == 4 ? D / 2 : D * esz;
  BPT_REQUIRE(rowb % 16 == 0 || rowb == 8, BPT_ERR_UNSUPPORTED, "kivi attention: row of %lld bytes", (long long)rowb);
  BPT_REQUIRE(aligned16(k_codes) && aligned16(v_codes), BPT_ERR_ALIGNMENT, "kivi attention: codes must be 16-byte aligned");
  KiviArgs a;
  a.q = q;
  a.q_dtype = q_dtype;
  a.q_sb = q_stride_b;
  a.q_sh = q_stride_h;
  a.k_codes = static_cast<const uint8_t*>(k_codes);
  a.v_codes = static_cast<const uint8_t*>(v_codes);
  a.k_scale = static_cast<const __half*>(k_scale);
  a.k_zero = static_cast<const __half*>(k_zero);
  a.v_scale = static_cast<const __half*>(v_scale);
  a.v_zero = static_cast<const __half*>(v_zero);
  a.lengths = lengths;
  a.B = int(B);
  a.Hq = int(Hq);
  a.Hkv = int(Hkv);
  a.t_max = t_max;
  a.n_groups = n_groups;
  a.split = int(split);
  a.n_splits = int(n_splits);
  a.sm_scale = sm_scale;
  a.out_partial = out_partial;
  a.lse_partial = lse_partial;
  const int rep = int(Hq / Hkv);
  auto s = static_cast<cudaStream_t>(stream);
  switch (D) {
    case 16: return launch_rep<16>(a, rep, bits, code_dtype, s);
    case 32: return launch_rep<32>(a, rep, bits, code_dtype, s);
    case 64: return launch_rep<64>(a, rep, bits, code_dtype, s);
    case 128: return launch_rep<128>(a, rep, bits, code_dtype, s);
    case 256: return launch_rep<256>(a, rep, bits, code_dtype, s);
  }
  return set_error(BPT_ERR_UNSUPPORTED, "kivi attention: D=%lld not in {16, 32, 64, 128, 256}", (long long)D);
}
