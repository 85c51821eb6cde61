// W4A16 linear for M >= 32 on the tensor cores: y[M, N] = x[M, K] . (scale * (q - zero))^T as a tiled GEMM.
//
// CTA tile 64 (M) x 32 (N weight rows), K in chunks of 128 through a 3-stage cp.async pipeline:
//   x chunk  [64][128] bf16 (16 KB), 16-byte pieces XOR-swizzled by row so ldmatrix reads are conflict free;
//   W chunk  [32][128] int4 (64 B per row, padded to 80 B so the 8 rows a warp reads fall on distinct banks).
// The tile's scales and zero points (32 rows x K/group; a chunk holds one group of 128 or two of 64) are
// staged once, before the pipeline starts.
// Four warps; warp w owns weight rows 8w .. 8w+7 (the MMA's N) for all four 16-row M tiles, so each weight is
// unpacked once per CTA. mma.sync m16n8k16 bf16 -> fp32:
//   A = x straight from shared memory by ldmatrix (natural k order);
//   B = q - z, exact in bf16: lane (g, c) takes byte c of a code word (inputs 2c, 2c+1 of its 8) with one PRMT
//       (the word and the word >> 4 as sources), masks the two nibbles into bf16 (128 + q) with one LOP3, and
//       subtracts bf16 (128 + z) with one HSUB2.
// Each group's products accumulate in fresh fp32 registers and are scaled into the running sums at the group's
// end (fp32 accumulate, as the reference's dequantize-then-matmul). The gate/up pairs of the fused MLP weight
// are adjacent rows, i.e. the two columns one lane holds: SiLU(gate) * up is taken in registers.
#include <cuda_bf16.h>

#include <cstdlib>

#include "common.cuh"

namespace bpt {
namespace {

constexpr int kBN = 32, kBK = 128;
constexpr int kThreads = 128;
constexpr int kWPitch = 80;               // bytes per weight row in shared memory (64 used)
constexpr int kWBytes = kBN * kWPitch;    // 2560
template <int BM>
constexpr int stage_bytes() { return BM * kBK * 2 + kWBytes; }

struct GemmArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  const uint8_t* qweight;  // [N, K/2] bytes
  const __half* scales;    // [N, G]
  const uint32_t* qzeros;  // [N, ZW] or null (symmetric: zero point 8)
  __nv_bfloat16* y;
  int64_t ldy;
  int M, N, K, group, G, ZW;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  // valid == false copies nothing and fills the 16 bytes with zeros
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* smem) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(smem)));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Inputs 2c and 2c+1 of a code word (its byte c) as the bf16 pair (q - z), given zz = bf16x2 (128 + z).
__device__ __forceinline__ uint32_t codes_minus_zero(uint32_t w, uint32_t sel, uint32_t zz) {
  const uint32_t t = (__byte_perm(w, w >> 4, sel) & 0x000F000Fu) | 0x43004300u;  // bf16 (128 + q_2c, 128 + q_2c+1)
  __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&t);
  const __nv_bfloat162 z = *reinterpret_cast<const __nv_bfloat162*>(&zz);
  v = __hsub2(v, z);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Issue the copies of K chunk `kc` into a stage: the x rows of this M tile and the W rows of this N tile.
template <int BM>
__device__ __forceinline__ void load_chunk(const GemmArgs& a, uint8_t* stage, int kc, int m0, int n0, int tid) {
  uint8_t* xs = stage;
  uint8_t* ws = stage + BM * kBK * 2;
  const int k0 = kc * kBK;
  // x: BM rows x 16 pieces of 16 bytes; piece p of row r lands at piece p ^ (r & 7)
#pragma unroll
  for (int i = 0; i < (BM * 16) / kThreads; ++i) {
    const int idx = tid + i * kThreads;
    const int r = idx >> 4, p = idx & 15;
    const bool ok = m0 + r < a.M;
    const __nv_bfloat16* src = a.x + int64_t(ok ? m0 + r : 0) * a.ldx + k0 + p * 8;
    cp_async16(xs + r * 256 + ((p ^ (r & 7)) * 16), src, ok);
  }
  // W: 32 rows x 4 pieces of 16 bytes
  {
    const int r = tid >> 2, p = tid & 3;
    const bool ok = n0 + r < a.N;
    const uint8_t* src = a.qweight + int64_t(ok ? n0 + r : 0) * (a.K >> 1) + (k0 >> 1) + p * 16;
    cp_async16(ws + r * kWPitch + p * 16, src, ok);
  }
}

template <bool FUSED, int BM, int STAGES>
__global__ void __launch_bounds__(kThreads) w4a16_gemm_kernel(const GemmArgs a) {
  constexpr int MT = BM / 16;  // 16-row M tiles per warp
  constexpr int kStageBytes = stage_bytes<BM>();
  constexpr int kXBytes = BM * kBK * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * BM;
  const int nk = a.K / kBK;
  const int per = kBK / a.group;                     // groups per chunk (1 or 2)
  const int steps_per_group = a.group / 16;          // 8 or 4
  const uint32_t sel = uint32_t(c) | (uint32_t(c) << 4) | ((4u + c) << 8) | ((4u + c) << 12);

  // The grid: scale and bf16x2 (128 + z) per (row, group) of this N tile.
  float* gsc = reinterpret_cast<float*>(smem + STAGES * kStageBytes);
  uint32_t* gzz = reinterpret_cast<uint32_t*>(gsc + kBN * a.G);
  for (int i = tid; i < kBN * a.G; i += kThreads) {
    const int r = i / a.G, gi = i % a.G;
    float sv = 0.f, z = 8.f;
    if (n0 + r < a.N) {
      sv = __half2float(a.scales[int64_t(n0 + r) * a.G + gi]);
      if (a.qzeros) z = float((a.qzeros[int64_t(n0 + r) * a.ZW + (gi >> 3)] >> (4 * (gi & 7))) & 15u);
    }
    gsc[gi * kBN + r] = sv;
    const __nv_bfloat162 zp = __floats2bfloat162_rn(128.f + z, 128.f + z);
    gzz[gi * kBN + r] = *reinterpret_cast<const uint32_t*>(&zp);
  }
  // The weights do not depend on the previous kernel, x does; a chunk is one commit group: wait first.
  pdl_launch_dependents();
  pdl_wait();

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < nk) load_chunk<BM>(a, smem + s * kStageBytes, s, m0, n0, tid);
    cp_async_commit();
  }

  float total[MT][4];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int e = 0; e < 4; ++e) total[mi][e] = 0.f;

  for (int kc = 0; kc < nk; ++kc) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();  // chunk kc is in; every warp is done with the stage about to be refilled
    {
      const int kn = kc + STAGES - 1;
      if (kn < nk) load_chunk<BM>(a, smem + (kn % STAGES) * kStageBytes, kn, m0, n0, tid);
      cp_async_commit();
    }
    const uint8_t* stage = smem + (kc % STAGES) * kStageBytes;
    const uint8_t* xs = stage;
    const uint8_t* wrow = stage + kXBytes + (8 * warp + g) * kWPitch;
    const float* sc = gsc + (kc * per) * kBN;  // [group in chunk][row]
    const uint32_t* zz = gzz + (kc * per) * kBN;
    // ldmatrix row addresses: lane L feeds row (L & 7) + 8 ((L >> 3) & 1) of a 16-row tile, k half L >> 4
    const int lr = (lane & 7) + 8 * ((lane >> 3) & 1), lk = lane >> 4;
    for (int j = 0; j < per; ++j) {
      const uint32_t z0 = zz[j * kBN + 8 * warp + g];  // this lane's row (its B column)
      float acc[MT][4];
#pragma unroll
      for (int mi = 0; mi < MT; ++mi)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mi][e] = 0.f;
#pragma unroll 4
      for (int s = 0; s < steps_per_group; ++s) {
        const int t = j * steps_per_group + s;  // k-step in the chunk
        const uint2 wv = *reinterpret_cast<const uint2*>(wrow + 8 * t);
        const uint32_t b0 = codes_minus_zero(wv.x, sel, z0), b1 = codes_minus_zero(wv.y, sel, z0);
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
          const int r = 16 * mi + lr;
          const int p = (2 * t + lk) ^ (r & 7);
          uint32_t af[4];
          ldmatrix_x4(af, xs + r * 256 + p * 16);
          mma_bf16(acc[mi], af, b0, b1);
        }
      }
      // fold the group: columns 2c, 2c+1 of this warp's tile are rows 8w + 2c, 8w + 2c + 1
      const float s0 = sc[j * kBN + 8 * warp + 2 * c], s1 = sc[j * kBN + 8 * warp + 2 * c + 1];
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        total[mi][0] += s0 * acc[mi][0];
        total[mi][1] += s1 * acc[mi][1];
        total[mi][2] += s0 * acc[mi][2];
        total[mi][3] += s1 * acc[mi][3];
      }
    }
  }
  cp_async_wait<0>();

  // epilogue: lane (g, c) holds D[16 mi + g (+8)][8 w + 2c, 2c + 1]
  const int n = n0 + 8 * warp + 2 * c;
#pragma unroll
  for (int mi = 0; mi < MT; ++mi) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = m0 + 16 * mi + g + 8 * h;
      if (m >= a.M) continue;
      const float v0 = total[mi][2 * h], v1 = total[mi][2 * h + 1];
      if constexpr (FUSED) {
        if (n + 1 < a.N) a.y[int64_t(m) * a.ldy + (n >> 1)] = __float2bfloat16_rn(silu(v0) * v1);
      } else if (n + 1 < a.N && (a.ldy & 1) == 0) {
        *reinterpret_cast<__nv_bfloat162*>(a.y + int64_t(m) * a.ldy + n) = __floats2bfloat162_rn(v0, v1);
      } else {
        if (n < a.N) a.y[int64_t(m) * a.ldy + n] = __float2bfloat16_rn(v0);
        if (n + 1 < a.N) a.y[int64_t(m) * a.ldy + n + 1] = __float2bfloat16_rn(v1);
      }
    }
  }
}

}  // namespace

// The GEMM takes K a multiple of 128, groups of 64 or 128, and 16-byte aligned x rows (checked by the caller).
bool w4a16_gemm_applies(int64_t M, int64_t N, int64_t K, int64_t group) {
  (void)N;
  return M >= 32 && K % kBK == 0 && (group == 64 || group == 128);
}

int w4a16_gemm(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros, void* y,
               int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags,
               cudaStream_t stream) {
  GemmArgs a;
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
  // M tile and pipeline depth: 32-row tiles double the CTAs for M <= 64 (the N tiles alone leave SMs idle); six stages
  // for 32-row tiles, three for 64 (the measured best per tile)
  const int bm = M <= 64 ? 32 : 64;
  const void* kernel = nullptr;
  int smem = 0;
#define BPT_GEMM_PICK(F, B, S)                                                              \
  if (fused == F && bm == B) {                                                              \
    kernel = reinterpret_cast<const void*>(w4a16_gemm_kernel<F, B, S>);                    \
    smem = S * stage_bytes<B>() + kBN * a.G * 8;                                             \
  }
  BPT_GEMM_PICK(false, 32, 6) BPT_GEMM_PICK(false, 64, 3) BPT_GEMM_PICK(true, 32, 6) BPT_GEMM_PICK(true, 64, 3)
#undef BPT_GEMM_PICK
  if (!kernel) return set_error(BPT_ERR_UNSUPPORTED, "w4a16 gemm: no kernel for a %d-row tile", bm);
  int st = set_max_smem(kernel, smem);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((N + kBN - 1) / kBN), unsigned((M + bm - 1) / bm), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BPT_FLAG_PDL) ? 1 : 0;
  void* args[] = {&a};
  cudaError_t err = cudaLaunchKernelExC(&cfg, kernel, args);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "w4a16 gemm launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

}  // namespace bpt
