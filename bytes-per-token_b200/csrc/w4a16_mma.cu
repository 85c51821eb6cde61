// W4A16 linear for small M on the tensor cores: y[M, N] = x[M, K] . (scale * (q - zero))^T, M <= 16.
//
// One CTA owns 8 weight rows (one MMA N tile; M <= 8) or 16 (two tiles sharing every x fragment; M up to 16) and
// all of K; its four warps split K. The CTA's rows reach shared memory with one bulk copy per row (TMA engine)
// to a padded pitch, so the lanes' 16-byte reads of 8 rows fall on different banks. The whole grid (768 CTAs for
// N = 6144 at M = 1) is resident at once, so every row of the matrix is requested at the start.
//
// mma.sync m16n8k16 bf16 -> fp32, per 16 inputs of K (k-step t):
//   B[k][n] = 128 + q[n][k]: lane (g, c) turns the two int32 words of row n = g that hold inputs 16t .. 16t+15 into
//     its B registers with one shift and one LOP3 each: (w >> 4c) & 0x000F000F | 0x43004300 is the bf16 pair
//     (128 + q[16t + c], 128 + q[16t + c + 4]) exactly (and 16t + 8 + c, 16t + 12 + c from the second word). So
//     B's k slots (2c, 2c+1, 2c+8, 2c+9) stand for inputs (c, c+4, 8+c, 12+c) of the step.
//   A[m][k] = x[m] in the same input order, staged once per CTA in shared memory as each lane's register pairs.
// The zero point and the 128 offset fold into the group sums:
//   sum_k x_k s (q_k - z) = s (sum_k x_k (128 + q_k) - (128 + z) sum_k x_k),
// with the MMA accumulating the first sum over a group's steps and the second coming from per-step sums of x.
// The warps' partial sums meet in shared memory in a fixed order: results are deterministic.
#include <cooperative_groups.h>

#include "common.cuh"

namespace bpt {
namespace cg = cooperative_groups;
namespace {

constexpr int kMaxRows = 16;  // weight rows per CTA: 8 (one MMA N tile) for M <= 8, 16 (two) above
constexpr int kWarps = 4;   // K split
constexpr int kMaxM = 16;   // x rows per launch (A has 16 rows)
constexpr int kSmemLimit = 110 * 1024;  // two CTAs per SM at least

struct MmaArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  const uint8_t* qweight;  // [N, K/2] bytes
  const __half* scales;    // [N, G]
  const uint32_t* qzeros;  // [N, ZW] or null (symmetric: zero point 8)
  __nv_bfloat16* y;
  int64_t ldy;
  int M, N, K, group, G, ZW;
  int ks;      // CTAs splitting K: one thread-block cluster per row tile
  int Kc;      // inputs per CTA: K / ks
  int T;       // the CTA's k-steps: Kc / 16
  int pitch;   // weight row pitch in shared memory: Kc/2 + 16
  int xpitch;  // staged x row pitch in bytes: 32 T rounded up to 64, + 64 (rows g and g + 1 on other banks)
  int spitch;  // x step-sum row pitch in floats: T rounded up to even, + 2
  int sbytes;  // the CTA's scales: 8 x G f16, rounded up to 16 bytes
  int zbytes;  // the CTA's zero-point words: 8 x ZW u32 (a multiple of 16 bytes)
};

// (not volatile: a pure register operation the compiler may schedule around the loads)
__device__ __forceinline__ void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t offset_codes(uint32_t w, int c) {
  return ((w >> (4 * c)) & 0x000F000Fu) | 0x43004300u;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

template <bool FUSED, int kRows>
__global__ void __launch_bounds__(32 * kWarps, kRows == 8 ? 6 : 4) w4a16_mma_kernel(const MmaArgs a) {
  constexpr int kTiles = kRows / 8;  // 8-row MMA N tiles
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int kr = blockIdx.x % a.ks;                     // this CTA's K slice (its rank in the cluster)
  const int row0 = (blockIdx.x / a.ks) * kRows;
  const int toff = kr * a.T;                            // the slice's first k-step
  const int nrows = min(kRows, a.N - row0);
  const int m0 = blockIdx.y * kMaxM;
  const int mt = min(kMaxM, a.M - m0);
  const int T = a.T;

  // shared memory: weights [8][pitch] | scales [8][G] f16 | zero-point words [8][ZW] | x pairs [mt][xpitch] |
  // x step sums [mt][spitch] f32 | partials [warps][16][8] f32 | mbarrier
  uint8_t* wsm = smem;
  __half* sraw = reinterpret_cast<__half*>(wsm + kRows * a.pitch);
  uint32_t* zraw = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sraw) + a.sbytes);
  uint8_t* xq = reinterpret_cast<uint8_t*>(zraw) + a.zbytes;
  float* xs = reinterpret_cast<float*>(xq + mt * a.xpitch);
  float* red = xs + mt * a.spitch;
  uint64_t* bar = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(red + kWarps * kMaxM * kRows) + 15) &
                                              ~uintptr_t(15));

  const bool whole = nrows == kRows;  // the last CTA may hold fewer rows: its grid comes in by plain loads
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (!whole) {
    for (int i = tid; i < nrows * a.G; i += blockDim.x) sraw[i] = a.scales[int64_t(row0) * a.G + i];
    if (a.qzeros)
      for (int i = tid; i < nrows * a.ZW; i += blockDim.x) zraw[i] = a.qzeros[int64_t(row0) * a.ZW + i];
  }
  __syncthreads();
  const int row_bytes = a.Kc >> 1;
  if (tid == 0) {  // the weights do not depend on the previous kernel: request them before waiting on it
    const uint64_t policy = l2_policy_evict_first();
    const bool zeros = whole && a.qzeros;
    mbar_arrive_expect_tx(bar, uint32_t(nrows * row_bytes + (whole ? a.sbytes : 0) + (zeros ? a.zbytes : 0)));
    for (int r = 0; r < nrows; ++r)
      bulk_g2s_evict_first(wsm + r * a.pitch, a.qweight + int64_t(row0 + r) * (a.K >> 1) + int64_t(kr) * row_bytes,
                           row_bytes, bar, policy);
    if (whole) bulk_g2s(sraw, a.scales + int64_t(row0) * a.G, a.sbytes, bar);
    if (zeros) bulk_g2s(zraw, a.qzeros + int64_t(row0) * a.ZW, a.zbytes, bar);
  }
  pdl_launch_dependents();
  pdl_wait();  // the activations (and the output) belong to the previous kernel until here

  // Each warp works on k-steps [t0, t1) (even bounds) and stages only the x that range needs.
  const int t0 = 2 * (warp * (T / 2) / kWarps), t1 = 2 * ((warp + 1) * (T / 2) / kWarps);
  const int spg = a.group >> 4;  // k-steps per group (even: the group is a multiple of 32)
  // x of step t, row m, lane c: the A pairs (x[16t + c], x[16t + c + 4]) and (x[16t + 8 + c], x[16t + 12 + c]),
  // stored so that a lane reads both of a step pair (t, t + 1) with one 16-byte load; and the step's sum of x.
  const int nt = t1 - t0;
  for (int i = lane; i < mt * nt; i += 32) {
    const int m = i / nt, t = t0 + i % nt;
    const uint4* src = reinterpret_cast<const uint4*>(a.x + int64_t(m0 + m) * a.ldx + 16 * (toff + t));
    const uint4 u0 = src[0], u1 = src[1];  // inputs 0..7 and 8..15 of the step, as bf16 pairs
    const uint32_t lo[4] = {u0.x, u0.y, u0.z, u0.w}, hi[4] = {u1.x, u1.y, u1.z, u1.w};
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      sum += (bf16_bits_to_float(lo[e] & 0xFFFFu) + bf16_bits_to_float(lo[e] >> 16)) +
             (bf16_bits_to_float(hi[e] & 0xFFFFu) + bf16_bits_to_float(hi[e] >> 16));
    uint8_t* row = xq + m * a.xpitch + (t >> 1) * 64 + (t & 1) * 8;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      // input j of the step is half (j & 1) of word j >> 1
      const uint32_t w0 = lo[cc >> 1], w4 = lo[(cc + 4) >> 1], w8 = hi[cc >> 1], w12 = hi[(cc + 4) >> 1];
      const uint32_t sel = (cc & 1) ? 0x7632u : 0x5410u;  // the high or the low halves of the two words
      *reinterpret_cast<uint2*>(row + cc * 16) = make_uint2(__byte_perm(w0, w4, sel), __byte_perm(w8, w12, sel));
    }
    xs[m * a.spitch + t] = sum;
  }
  __syncwarp();

  float total[kTiles][4];  // tile nt: D[m = g, g + 8][n = 8 nt + 2c, 8 nt + 2c + 1]
#pragma unroll
  for (int nt = 0; nt < kTiles; ++nt) total[nt][0] = total[nt][1] = total[nt][2] = total[nt][3] = 0.f;
  int arrived = 0;
  if (lane == 0) arrived = mbar_wait_sleep(bar, 0, 128u) ? 1 : 0;
  arrived = __shfl_sync(0xffffffffu, arrived, 0);
  if (arrived) (void)mbar_try_wait(bar, 0);  // every lane observes the completed phase (acquire)
  if (arrived) {
    const uint8_t* wrow[kTiles];
#pragma unroll
    for (int nt = 0; nt < kTiles; ++nt) wrow[nt] = wsm + (8 * nt + g) * a.pitch;
    // Rows of D at or past mt are never stored, so lanes beyond the x rows read a valid row instead of
    // branching: every load is unconditional.
    const int ga = min(g, mt - 1), gb = min(g + 8, mt - 1);
    const uint8_t* xa = xq + ga * a.xpitch + c * 16;
    const uint8_t* xb = xq + gb * a.xpitch + c * 16;
    const float* sxa = xs + ga * a.spitch;
    const float* sxb = xs + gb * a.spitch;
    const bool two = mt > 8;  // A rows g + 8 carry x (warp-uniform)
    for (int grp = (toff + t0) / spg; grp * spg < toff + t1; ++grp) {  // groups numbered over all of K
      const int ta = max(t0, grp * spg - toff), tb = min(t1, (grp + 1) * spg - toff);  // local, both even
      // per tile two independent chains: the even and the odd step of each pair
      float ae[kTiles][4], ao[kTiles][4];
#pragma unroll
      for (int nt = 0; nt < kTiles; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) ae[nt][e] = ao[nt][e] = 0.f;
      float sa = 0.f, sb = 0.f;  // sums of x over the group's steps here, rows g and g + 8
      int t = ta;
      for (; t + 8 <= tb; t += 8) {  // four step pairs: every load first, then the MMAs
        uint4 wv[4][kTiles], pa[4], pb[4];
        float2 qa[4], qb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int nt = 0; nt < kTiles; ++nt) wv[j][nt] = *reinterpret_cast<const uint4*>(wrow[nt] + 8 * (t + 2 * j));
          pa[j] = *reinterpret_cast<const uint4*>(xa + ((t >> 1) + j) * 64);
          qa[j] = *reinterpret_cast<const float2*>(sxa + t + 2 * j);
          if (two) {
            pb[j] = *reinterpret_cast<const uint4*>(xb + ((t >> 1) + j) * 64);
            qb[j] = *reinterpret_cast<const float2*>(sxb + t + 2 * j);
          } else {
            pb[j] = make_uint4(0u, 0u, 0u, 0u);
            qb[j] = make_float2(0.f, 0.f);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sa += qa[j].x + qa[j].y;
          sb += qb[j].x + qb[j].y;
#pragma unroll
          for (int nt = 0; nt < kTiles; ++nt) {
            mma_bf16(ae[nt], pa[j].x, pb[j].x, pa[j].y, pb[j].y, offset_codes(wv[j][nt].x, c), offset_codes(wv[j][nt].y, c));
            mma_bf16(ao[nt], pa[j].z, pb[j].z, pa[j].w, pb[j].w, offset_codes(wv[j][nt].z, c), offset_codes(wv[j][nt].w, c));
          }
        }
      }
      for (; t < tb; t += 2) {  // the group's remaining pairs (groups of fewer than 8 steps, range edges)
        const uint4 pa = *reinterpret_cast<const uint4*>(xa + (t >> 1) * 64);
        const float2 qa = *reinterpret_cast<const float2*>(sxa + t);
        uint4 pb = make_uint4(0u, 0u, 0u, 0u);
        float2 qb = make_float2(0.f, 0.f);
        if (two) {
          pb = *reinterpret_cast<const uint4*>(xb + (t >> 1) * 64);
          qb = *reinterpret_cast<const float2*>(sxb + t);
        }
        sa += qa.x + qa.y;
        sb += qb.x + qb.y;
#pragma unroll
        for (int nt = 0; nt < kTiles; ++nt) {
          const uint4 wv = *reinterpret_cast<const uint4*>(wrow[nt] + 8 * t);
          mma_bf16(ae[nt], pa.x, pb.x, pa.y, pb.y, offset_codes(wv.x, c), offset_codes(wv.y, c));
          mma_bf16(ao[nt], pa.z, pb.z, pa.w, pb.w, offset_codes(wv.z, c), offset_codes(wv.w, c));
        }
      }
#pragma unroll
      for (int nt = 0; nt < kTiles; ++nt) {
        const int n0 = 8 * nt + 2 * c;
        const float s0 = __half2float(sraw[n0 * a.G + grp]), s1 = __half2float(sraw[(n0 + 1) * a.G + grp]);
        float z0 = 136.f, z1 = 136.f;  // 128 + the zero point (8 when the layout is symmetric)
        if (a.qzeros) {
          z0 = 128.f + float((zraw[n0 * a.ZW + (grp >> 3)] >> (4 * (grp & 7))) & 15u);
          z1 = 128.f + float((zraw[(n0 + 1) * a.ZW + (grp >> 3)] >> (4 * (grp & 7))) & 15u);
        }
        total[nt][0] += s0 * ((ae[nt][0] + ao[nt][0]) - z0 * sa);
        total[nt][1] += s1 * ((ae[nt][1] + ao[nt][1]) - z1 * sa);
        total[nt][2] += s0 * ((ae[nt][2] + ao[nt][2]) - z0 * sb);
        total[nt][3] += s1 * ((ae[nt][3] + ao[nt][3]) - z1 * sb);
      }
    }
  }
  float* rw = red + warp * kMaxM * kRows;
#pragma unroll
  for (int nt = 0; nt < kTiles; ++nt) {
    rw[g * kRows + 8 * nt + 2 * c] = total[nt][0];
    rw[g * kRows + 8 * nt + 2 * c + 1] = total[nt][1];
    rw[(g + 8) * kRows + 8 * nt + 2 * c] = total[nt][2];
    rw[(g + 8) * kRows + 8 * nt + 2 * c + 1] = total[nt][3];
  }
  __syncthreads();
  if (tid == 0) (void)mbar_wait(bar, 0, 50000000ull);  // every copy has landed before the CTA exits (bounded)
  // With K split, the cluster's CTAs (K slices of the same rows) meet in the first one's shared memory: it reads
  // every slice's per-warp partials through distributed shared memory, in a fixed order, and writes y.
  cg::cluster_group cluster = cg::this_cluster();
  if (a.ks > 1) cluster.sync();
  if (kr == 0) {
    auto slice_sum = [&](int m, int n) {
      float sum = 0.f;
      for (int r = 0; r < a.ks; ++r) {
        const float* rr = a.ks > 1 ? cluster.map_shared_rank(red, r) : red;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += rr[(w * kMaxM + m) * kRows + n];
      }
      return sum;
    };
    if constexpr (FUSED) {  // rows 2p, 2p + 1 are gate and up of output row0 / 2 + p
      for (int i = tid; i < mt * (kRows / 2); i += blockDim.x) {
        const int m = i / (kRows / 2), p = i % (kRows / 2);
        if (2 * p + 1 >= nrows) continue;
        const float gs = slice_sum(m, 2 * p), us = slice_sum(m, 2 * p + 1);
        a.y[int64_t(m0 + m) * a.ldy + (row0 >> 1) + p] = __float2bfloat16_rn(silu(gs) * us);
      }
    } else {
      for (int i = tid; i < mt * kRows; i += blockDim.x) {
        const int m = i / kRows, n = i % kRows;
        if (n >= nrows) continue;
        a.y[int64_t(m0 + m) * a.ldy + row0 + n] = __float2bfloat16_rn(slice_sum(m, n));
      }
    }
  }
  if (a.ks > 1) cluster.sync();  // the other slices' shared memory stays until the first CTA has read it
}

int mma_rows(int64_t M) { return M <= 8 ? 8 : 16; }

int mma_smem_bytes(int64_t M, int64_t K, int64_t Kc, int64_t group) {
  const int64_t T = Kc / 16, G = K / group, mt = std::min<int64_t>(M, kMaxM), ZW = (G + 7) / 8;
  const int64_t kRows = mma_rows(M);
  const int64_t bytes = kRows * (Kc / 2 + 16) + ((kRows * G * 2 + 15) / 16) * 16 + kRows * ZW * 4 +
                        mt * (32 * ((T + 1) & ~1) + 64) + mt * (((T + 1) & ~1) + 2) * 4 + kWarps * kMaxM * kRows * 4 +
                        32;
  return int(bytes);
}

// CTAs per row tile along K (a cluster, at most 8): doubled while the grid has fewer CTAs than SMs, or while
// the x staging does not fit; each slice whole groups of at least 256 inputs.
int mma_ksplit(int64_t M, int64_t N, int64_t K, int64_t group) {
  const int rows = mma_rows(M);
  const int64_t tiles = (N + rows - 1) / rows;
  auto fits = [&](int k) { return K % (int64_t(k) * group) == 0 && (K / k) % 32 == 0 && K / k >= 256; };
  int ks = 1;
  while (ks < 8 && fits(2 * ks) &&
         (tiles * ks < num_sms() || mma_smem_bytes(M, K, K / ks, group) > kSmemLimit))
    ks *= 2;
  return ks;
}

}  // namespace

// The tensor-core path takes K a multiple of 16 and of the group (group a multiple of 16), 16-byte aligned rows,
// and shapes whose staging fits two CTAs per SM; M is split into chunks of 16 rows.
bool w4a16_mma_applies(int64_t M, int64_t N, int64_t K, int64_t group) {
  if (K % 32 != 0 || group % 32 != 0 || K / 32 < kWarps) return false;
  const int ks = mma_ksplit(M, N, K, group);
  return mma_smem_bytes(M, K, K / ks, group) <= kSmemLimit;
}

int w4a16_mma(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros, void* y,
              int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags,
              cudaStream_t stream) {
  MmaArgs a;
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
  a.ks = mma_ksplit(M, N, K, group);
  a.Kc = int(K / a.ks);
  a.T = a.Kc / 16;
  a.pitch = a.Kc / 2 + 16;
  a.xpitch = 32 * ((a.T + 1) & ~1) + 64;
  const int rows = mma_rows(M);
  a.sbytes = ((rows * a.G * 2 + 15) / 16) * 16;
  a.zbytes = rows * a.ZW * 4;
  a.spitch = ((a.T + 1) & ~1) + 2;
  const int smem = mma_smem_bytes(M, K, a.Kc, group);
  auto kernel = rows == 8 ? (fused ? w4a16_mma_kernel<true, 8> : w4a16_mma_kernel<false, 8>)
                          : (fused ? w4a16_mma_kernel<true, 16> : w4a16_mma_kernel<false, 16>);
  int st = set_max_smem(reinterpret_cast<const void*>(kernel), smem);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((N + rows - 1) / rows * a.ks), unsigned((M + kMaxM - 1) / kMaxM), 1);
  cfg.blockDim = dim3(32 * kWarps, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(a.ks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = a.ks > 1 ? attr : attr + 1;  // no cluster attribute when K is not split
  cfg.numAttrs = (a.ks > 1 ? 1 : 0) + ((flags & BPT_FLAG_PDL) ? 1 : 0);
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "w4a16 mma launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

}  // namespace bpt
