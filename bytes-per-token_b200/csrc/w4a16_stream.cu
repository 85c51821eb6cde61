// W4A16 linear for M <= 8 tokens as a persistent streaming GEMV: y[M, N] = x[M, K] . (scale * (q - zero))^T.
//
// At most one CTA per SM. CTA b owns the contiguous 16-row weight tiles [b T / P, (b + 1) T / P). Thread 0
// streams each tile (16 code rows, the tile's fp16 scales and zero-point words) into a ring of shared-memory
// stages with bulk copies (TMA engine): the first ring-full right after the CTA lets its dependents launch and
// before the kernel waits on its predecessor (the weights do not depend on it), each later tile as soon as the
// chunk of tiles that held its stage has been reduced. The CTA asks for at most ~113 KB of shared memory and
// ~29 K registers, so under programmatic dependent launch the next call's CTAs sit beside this one's and fetch
// their weights while this one computes. Eight warps split K by whole groups and run each group's x against
// every tile of the chunk. (A dedicated copy warp made nine warps, which capped the registers at 96 per thread
// for two CTAs per SM, and measured slower.) The weights are the MMA's A (the 16 rows of a tile), the tokens its
// B, in one of two forms:
//
// INTEGER form (M <= 2): mma.sync m16n8k32 u8 x s8 -> s32 on the codes q as exact bytes. Each warp first turns
// its group's x into integers: per (token, group) a power-of-two scale 2^S puts the largest |x| in
// [2^20, 2^21), X = round(x 2^S) (one FMA against a magic number whose sum lands X in the low mantissa bits) and
// X = 65536 d0 + 256 d1 + d2 with signed bytes d0 in [-32, 32], d1, d2 in [-128, 127] (byte permutes of the
// FMA's bit pattern), stored in a per-warp buffer with the group sum of X. B's eight columns are two tokens'
// (d0, d1, 0, d2), so lane (g, c) accumulates columns 2c, 2c + 1 of one token and
//   sum_k q_k (256 d0 + d1)_k   (c even)   or   sum_k q_k d2_k   (c odd)
// exactly in int32; subtracting z times the matching part of sum_k X (split at 256) and scaling by
// s 2^-S (256 or 1) gives the lane's share of the group's sum_k x_k (q_k - z) s. The only rounding before the
// fp32 sums is X's: at most 2^-22 of the group's largest |x| per input, so every bf16 input within 2^13 of that
// value is exact. A non-finite x makes its (token, group)'s sum NaN. In a group lane (g, c) owns code words
// cW .. cW + W - 1 (W = group / 32) of rows g and g + 8, read with one 8- or 16-byte load per row; step u takes
// word cW + u: A k slots 4c .. 4c + 3 are its nibbles 0, 2, 4, 6 (w & 0x0F0F0F0F), slots 16 + 4c .. its nibbles
// 1, 3, 5, 7 ((w >> 4) & 0x0F0F0F0F); B holds the digits of the same inputs, stored word by word as (even
// inputs, odd inputs). Three ALU instructions unpack 8 weights and one MMA takes 512 of them. Past two tokens the
// conversion of x (three digit columns per token and group, in every CTA) outweighs that gain.
//
// BF16 form (M <= 8): mma.sync m16n8k16 bf16 -> fp32 with the tokens as B's columns. K is walked in blocks of 64
// inputs (4 k-steps u = 0..3). In a block, lane (g, c) owns code words 2c and 2c + 1 (inputs 16c .. 16c + 15 of
// the block) of rows g and g + 8, read with one 8-byte load per row, and step u takes from them:
//   A k slots (2c, 2c+1)   = (128 + q, as bf16) of inputs 16c + u, 16c + u + 4      (word 2c >> 4u, LOP3 mask)
//   A k slots (2c+8, 2c+9) = inputs 16c + 8 + u, 16c + 12 + u                        (word 2c + 1 >> 4u)
// minus bf16 (128 + z) with one HSUB2: q - z exactly. B holds x at the same inputs (so each lane's B words come
// from the 32 bytes of x at inputs 16c .. 16c + 15, loaded straight from global memory). Over u and c every input
// of the block is used once. The MMA sums x (q - z) over a group in fp32; the group's scale multiplies the sum.
//
// The lane pairs' shares and the warps' partial sums meet in a fixed order: results are deterministic.
#include "common.cuh"

namespace bpt {
namespace {

constexpr int kRows = 16;                        // weight rows per tile (the MMA's M)
constexpr int kConsumers = 8;                    // warps (K split), two per SM sub-partition
constexpr int kThreads = 32 * kConsumers;        // thread 0 also issues the tiles' copies
constexpr int kMaxTok = 8;                       // tokens per launch (the bf16 MMA's N)
constexpr int kIntTok = 2;                       // tokens per launch of the integer form (four B columns each)
constexpr int kChunk = 3;                        // tiles a warp holds partial sums for at once
constexpr int kBudgetShared = 113 * 1024;        // two CTAs per SM (this call's and the next one's)
constexpr int kBudgetAlone = 220 * 1024;         // when two stages do not fit
constexpr uint32_t kMagic = 0x4B408080u;         // bits of 1.5 * 2^23 + 32896: X + 32896 in the low mantissa bits

struct StreamArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  const uint8_t* qweight;  // [N, K/2] bytes
  const __half* scales;    // [N, G]
  const uint32_t* qzeros;  // [N, ZW] or null (symmetric: zero point 8)
  __nv_bfloat16* y;
  int64_t ldy;
  int M, N, K, G, ZW;
  int tiles;   // N / 16
  int pitch;   // bytes per staged code row (stream_pitch)
  int sbytes;  // a tile's scales: 16 G fp16 = 32 G bytes
  int zbytes;  // a tile's zero-point words: 16 ZW u32 (0 without zero points)
  int stage;   // bytes per ring stage: 16 pitch + sbytes + zbytes
  int ns;      // ring stages
};

__host__ __device__ inline bool integer_form(int M) { return M <= kIntTok; }

// A staged code row's pitch: so that the lanes' code reads of a warp's rows fall on distinct banks, K/2 + 32 for
// the bf16 form's 8-byte reads; K/2 rounded up to 128, + 64 (16-byte reads at group 128) or + 32 (8-byte reads
// at group 64) for the integer form's.
__host__ __device__ inline int stream_pitch(int K, int group, bool integer) {
  if (!integer) return K / 2 + 32;
  return ((K / 2 + 127) & ~127) + (group == 128 ? 64 : 32);
}

// A digit column of one group in a warp's buffer: group / 8 words of (even, odd) inputs, 8 bytes each; padded at
// group 128 so that the lanes' 16-byte reads of two neighbouring columns meet no bank twice.
__host__ __device__ constexpr int digit_col_bytes(int group) { return group == 128 ? 144 : group; }

struct StreamLayout {
  int ring, red, digits, warp_digits, bars, total;
};

// ring [ns][stage] | partial sums [2][chunk tiles][warps][16 rows][M] f32 | integer form, per warp: digit columns
// [M][3][col bytes], group sums of X [M] s32, 2^-S [M] f32 | mbarriers full[ns]
__host__ __device__ inline StreamLayout stream_layout(int M, int group, int stage, int ns) {
  StreamLayout l;
  l.ring = 0;
  l.red = ns * stage;
  l.digits = l.red + ((2 * kChunk * kConsumers * kRows * M * 4 + 15) & ~15);
  l.warp_digits = integer_form(M) ? (3 * M * digit_col_bytes(group) + 8 * M + 15) & ~15 : 0;
  l.bars = l.digits + kConsumers * l.warp_digits;
  l.total = l.bars + ns * 8;
  return l;
}

__device__ __forceinline__ void mma_u8s8(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The bf16 pair (q - z) of nibbles u and u + 4 of a code word, given zz = bf16x2 (128 + z): exact.
__device__ __forceinline__ uint32_t codes_minus_zero(uint32_t w, int u, uint32_t zz) {
  const uint32_t t = ((w >> (4 * u)) & 0x000F000Fu) | 0x43004300u;  // bf16 (128 + q_u, 128 + q_u+4)
  __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&t);
  v = __hsub2(v, *reinterpret_cast<const __nv_bfloat162*>(&zz));
  return *reinterpret_cast<const uint32_t*>(&v);
}

// The (d0, d1, d2) byte words of four inputs from their FMA bit patterns t = bits(1.5 * 2^23) + 32896 + X: byte 0
// is d2 + 128, byte 1 is d1 + 128, byte 2 is d0 + 64 (d0 in [-32, 32], so adding 64 per byte carries nowhere).
__device__ __forceinline__ void digits4(uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3, uint32_t& d0,
                                        uint32_t& d1, uint32_t& d2) {
  const uint32_t p01 = __byte_perm(t0, t1, 0x5140), p23 = __byte_perm(t2, t3, 0x5140);
  const uint32_t q01 = __byte_perm(t0, t1, 0x7362), q23 = __byte_perm(t2, t3, 0x7362);
  d2 = __byte_perm(p01, p23, 0x5410) ^ 0x80808080u;
  d1 = __byte_perm(p01, p23, 0x7632) ^ 0x80808080u;
  d0 = (__byte_perm(q01, q23, 0x5410) + 0x40404040u) ^ 0x80808080u;
}

// Digits of the 8 inputs of one code word of x (bf16 words w: inputs 2i, 2i + 1 in the halves of w[i]) at scale f:
// per digit the (even inputs, odd inputs) words, and the sum of the 8 X values.
__device__ __forceinline__ void word_digits(const uint4 w, float f, uint2 (&d)[3], uint32_t& sum) {
  const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
  uint32_t t[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    t[2 * i] = __float_as_uint(fmaf(__uint_as_float(wv[i] << 16), f, __uint_as_float(kMagic)));
    t[2 * i + 1] = __float_as_uint(fmaf(__uint_as_float(wv[i] & 0xFFFF0000u), f, __uint_as_float(kMagic)));
  }
  sum = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) sum += t[i];
  sum -= 8u * kMagic;  // modulo 2^32: the sum of X exactly
  digits4(t[0], t[2], t[4], t[6], d[0].x, d[1].x, d[2].x);
  digits4(t[1], t[3], t[5], t[7], d[0].y, d[1].y, d[2].y);
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumers) : "memory"); }

template <bool FUSED, int GROUP, bool INT>  // INT: the integer form (M <= 2), else the bf16 form (M <= 8)
__global__ void __launch_bounds__(kThreads, 2) w4a16_stream_kernel(const StreamArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = gridDim.x;
  const int tb = int(int64_t(blockIdx.x) * a.tiles / P), te = int(int64_t(blockIdx.x + 1) * a.tiles / P);
  const int nt = te - tb;
  const StreamLayout L = stream_layout(a.M, GROUP, a.stage, a.ns);
  uint8_t* ring = smem + L.ring;
  float* red = reinterpret_cast<float*>(smem + L.red);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);

  // tile j's copies into stage j mod ns, completing on full[stage]
  const uint64_t policy = l2_policy_evict_first();
  auto issue_tile = [&](int j) {
    const int s = j % a.ns;
    const int row_bytes = a.K >> 1;
    uint8_t* st = ring + s * a.stage;
    const int64_t row0 = int64_t(tb + j) * kRows;
    mbar_arrive_expect_tx(&full[s], uint32_t(kRows * row_bytes + a.sbytes + a.zbytes));
    for (int r = 0; r < kRows; ++r)
      bulk_g2s_evict_first(st + r * a.pitch, a.qweight + (row0 + r) * row_bytes, uint32_t(row_bytes), &full[s],
                           policy);
    bulk_g2s(st + kRows * a.pitch, a.scales + row0 * a.G, uint32_t(a.sbytes), &full[s]);
    if (a.zbytes) bulk_g2s(st + kRows * a.pitch + a.sbytes, a.qzeros + row0 * a.ZW, uint32_t(a.zbytes), &full[s]);
  };
  if (tid == 0) {
    for (int s = 0; s < a.ns; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();  // the next call may now place its CTAs beside this one and fetch its weights
  if (tid == 0)  // after the trigger: ~18 copies a tile would otherwise hold back the next call's launch
    for (int j = 0; j < min(nt, a.ns); ++j) issue_tile(j);

  const int cw = warp, ctid = tid;
  const int g = lane >> 2, c = lane & 3;
  const int gb = cw * a.G / kConsumers, ge = (cw + 1) * a.G / kConsumers;  // this warp's groups
  const int chunk = min(kChunk, a.ns);  // tiles resident together
  // The chunk's stages: tile j sits in stage j mod ns, filled for the (j / ns)-th time; every lane waits itself.
  // The first chunk's wait comes before the wait on the previous kernel (the weights do not depend on it).
  auto wait_chunk = [&](int j0, uint32_t* soff) {
    bool ok = true;
#pragma unroll
    for (int jj = 0; jj < kChunk; ++jj) {
      const int j = j0 + jj;
      const int s = j % a.ns;
      soff[jj] = uint32_t(s * a.stage);
      if (j < min(nt, j0 + chunk)) ok = mbar_wait(&full[s], uint32_t((j / a.ns) & 1)) && ok;
    }
    return __all_sync(0xffffffffu, ok);
  };
  uint32_t soff[kChunk];
  bool ok = wait_chunk(0, soff);
  pdl_wait();  // x (and y) belong to the previous kernel until here

  for (int j0 = 0; j0 < nt; j0 += chunk) {
    const int j1 = min(nt, j0 + chunk);
    if (j0 > 0) ok = wait_chunk(j0, soff);
    // the chunk's partials go to red[chunk parity][tile][warp][row][token] (the next chunk uses the other half)
    float* rc = red + ((j0 / chunk) & 1) * (kChunk * kConsumers * kRows * a.M);
    if constexpr (INT) {
      constexpr int W = GROUP / 32;   // code words per lane per row in a group
      constexpr int WPG = GROUP / 8;  // code words per row in a group
      constexpr int CB = digit_col_bytes(GROUP);
      uint8_t* dig = smem + L.digits + warp * L.warp_digits;
      int* xsum = reinterpret_cast<int*>(dig + 3 * a.M * CB);
      float* xmul = reinterpret_cast<float*>(xsum + a.M);
      const int items = a.M * WPG;  // x pieces of a group: piece i is token i / WPG, code word i % WPG
      // B column g: slot g & 3 (d0, d1, zero, d2) of token g >> 2; D columns 2c, 2c + 1: token c >> 1, the
      // (d0, d1) share (c even) or the d2 share (c odd); tokens past M read the last one and are never stored
      const int slot = g & 3;
      const int bcol = (3 * min(g >> 2, a.M - 1) + (slot == 3 ? 2 : slot)) * CB + c * W * 8;
      const int dtok = min(c >> 1, a.M - 1);
      const float xwt = (c & 1) ? 1.0f : 256.0f;
      float tot[kChunk][2] = {};  // per tile: rows g and g + 8, the lane's share of its token
      if (ok) {
        uint4 raw = make_uint4(0u, 0u, 0u, 0u);  // the lane's x piece of a group (16 bytes)
        auto load_raw = [&](int grp) {
          if (lane < items)
            raw = *reinterpret_cast<const uint4*>(a.x + int64_t(lane / WPG) * a.ldx + int64_t(grp) * GROUP +
                                                  8 * (lane % WPG));
        };
        if (gb < ge) load_raw(gb);
        for (int grp = gb; grp < ge; ++grp) {
          // the group's digits into the warp's buffer: a piece's scale is its token's for the group, found by a
          // max over the WPG lanes that hold the token's pieces
          {
            uint32_t mb = 0;
            const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) mb = max(mb, max((wv[q] << 16) & 0x7FFFFFFFu, wv[q] & 0x7FFF0000u));
#pragma unroll
            for (int o = 1; o < WPG; o <<= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
            const int e = int(mb >> 23);       // biased exponent of the largest |x| (255: inf or NaN)
            const int sb = min(274 - e, 253);  // 127 + S with S = 20 - (e - 127), capped at 2^126
            uint2 d[3];
            uint32_t sum;
            word_digits(raw, __uint_as_float(uint32_t(sb) << 23), d, sum);
#pragma unroll
            for (int o = 1; o < WPG; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane < items) {
              const int t = lane / WPG, w = lane % WPG;
#pragma unroll
              for (int k = 0; k < 3; ++k) *reinterpret_cast<uint2*>(dig + (3 * t + k) * CB + 8 * w) = d[k];
              if (w == 0) {
                xsum[t] = int(sum);
                xmul[t] = e == 255 ? __uint_as_float(0x7FC00000u) : __uint_as_float(uint32_t(254 - sb) << 23);
              }
            }
          }
          __syncwarp();
          uint32_t bx[W][2];
          if (slot == 2) {
#pragma unroll
            for (int u = 0; u < W; ++u) bx[u][0] = bx[u][1] = 0u;
          } else if constexpr (W == 4) {
            const uint4 p0 = *reinterpret_cast<const uint4*>(dig + bcol);
            const uint4 p1 = *reinterpret_cast<const uint4*>(dig + bcol + 16);
            bx[0][0] = p0.x; bx[0][1] = p0.y; bx[1][0] = p0.z; bx[1][1] = p0.w;
            bx[2][0] = p1.x; bx[2][1] = p1.y; bx[3][0] = p1.z; bx[3][1] = p1.w;
          } else {
            const uint4 p0 = *reinterpret_cast<const uint4*>(dig + bcol);
            bx[0][0] = p0.x; bx[0][1] = p0.y; bx[1][0] = p0.z; bx[1][1] = p0.w;
          }
          const int xsv = xsum[dtok];
          const int xsl = (c & 1) ? (xsv & 255) : (xsv >> 8);  // the lane's part of the group sum of X
          const float xm = xmul[dtok] * xwt;                    // 2^-S times 256 (c even) or 1 (c odd)
          __syncwarp();  // the buffer is free for the next group
          if (grp + 1 < ge) load_raw(grp + 1);
#pragma unroll
          for (int jj = 0; jj < kChunk; ++jj) {
            const int j = j0 + jj;
            if (j >= j1) break;
            const uint8_t* st = ring + soff[jj];
            const __half* sc = reinterpret_cast<const __half*>(st + kRows * a.pitch);
            const uint32_t* zw = reinterpret_cast<const uint32_t*>(st + kRows * a.pitch + a.sbytes);
            int z0 = 8, z1 = 8;  // symmetric layout: zero point 8
            if (a.zbytes) {
              z0 = int((zw[g * a.ZW + (grp >> 3)] >> (4 * (grp & 7))) & 15u);
              z1 = int((zw[(g + 8) * a.ZW + (grp >> 3)] >> (4 * (grp & 7))) & 15u);
            }
            const float s0 = __half2float(sc[g * a.G + grp]), s1 = __half2float(sc[(g + 8) * a.G + grp]);
            const uint8_t* ra = st + g * a.pitch + grp * (GROUP / 2) + c * W * 4;
            const uint8_t* rb = ra + 8 * a.pitch;
            uint32_t wa[W], wb[W];
            if constexpr (W == 4) {
              const uint4 va = *reinterpret_cast<const uint4*>(ra), vb = *reinterpret_cast<const uint4*>(rb);
              wa[0] = va.x; wa[1] = va.y; wa[2] = va.z; wa[3] = va.w;
              wb[0] = vb.x; wb[1] = vb.y; wb[2] = vb.z; wb[3] = vb.w;
            } else {
              const uint2 va = *reinterpret_cast<const uint2*>(ra), vb = *reinterpret_cast<const uint2*>(rb);
              wa[0] = va.x; wa[1] = va.y;
              wb[0] = vb.x; wb[1] = vb.y;
            }
            int acc[2][4] = {};  // even and odd steps: two dependency chains
#pragma unroll
            for (int u = 0; u < W; ++u)
              mma_u8s8(acc[u & 1], wa[u] & 0x0F0F0F0Fu, wb[u] & 0x0F0F0F0Fu, (wa[u] >> 4) & 0x0F0F0F0Fu,
                       (wb[u] >> 4) & 0x0F0F0F0Fu, bx[u][0], bx[u][1]);
            const int v0 = (acc[0][0] + acc[1][0]) * 256 + acc[0][1] + acc[1][1] - z0 * xsl;
            const int v1 = (acc[0][2] + acc[1][2]) * 256 + acc[0][3] + acc[1][3] - z1 * xsl;
            tot[jj][0] = fmaf(float(v0), s0 * xm, tot[jj][0]);
            tot[jj][1] = fmaf(float(v1), s1 * xm, tot[jj][1]);
          }
        }
      }
      // a lane pair (c, c ^ 1) holds one token's two shares
#pragma unroll
      for (int jj = 0; jj < kChunk; ++jj) {
        if (j0 + jj >= j1) break;
        float* rw = rc + (jj * kConsumers + cw) * kRows * a.M;
        const float y0 = tot[jj][0] + __shfl_xor_sync(0xffffffffu, tot[jj][0], 1);
        const float y1 = tot[jj][1] + __shfl_xor_sync(0xffffffffu, tot[jj][1], 1);
        const int tk = c >> 1;
        if (!(c & 1) && tk < a.M) {
          rw[g * a.M + tk] = y0;
          rw[(g + 8) * a.M + tk] = y1;
        }
      }
    } else {
      constexpr int kBlocks = GROUP / 64;  // 64-input blocks per group
      // B column g is token g (columns past M repeat the last token and are never stored)
      const __nv_bfloat16* xg = a.x + int64_t(min(g, a.M - 1)) * a.ldx + 16 * c;
      float tot[kChunk][4] = {};  // per tile: D[row g][tok 2c, 2c + 1], D[row g + 8][tok 2c, 2c + 1]
      if (ok) {
        // x of the group: lane c's inputs 16c .. 16c + 7 and 16c + 8 .. 16c + 15 of each block (bf16 pairs); the
        // next group's are requested before this group's MMAs
        uint4 xr[kBlocks][2];
        auto load_x = [&](int grp) {
#pragma unroll
          for (int b = 0; b < kBlocks; ++b) {
            const uint4* src = reinterpret_cast<const uint4*>(xg + int64_t(grp) * GROUP + 64 * b);
            xr[b][0] = src[0];
            xr[b][1] = src[1];
          }
        };
        if (gb < ge) load_x(gb);
        for (int grp = gb; grp < ge; ++grp) {
          // this group's B words: block b, step u -> xb[b][2u] (inputs 16c + u, + u + 4), xb[b][2u + 1] (+8, +12)
          uint32_t xb[kBlocks][8];
#pragma unroll
          for (int b = 0; b < kBlocks; ++b) {
            const uint4 lo = xr[b][0], hi = xr[b][1];
            const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const uint32_t sel = (u & 1) ? 0x7632u : 0x5410u;  // input i is half (i & 1) of word i >> 1
              xb[b][2 * u] = __byte_perm(w[u >> 1], w[2 + (u >> 1)], sel);
              xb[b][2 * u + 1] = __byte_perm(w[4 + (u >> 1)], w[6 + (u >> 1)], sel);
            }
          }
          if (grp + 1 < ge) load_x(grp + 1);
#pragma unroll
          for (int jj = 0; jj < kChunk; ++jj) {
            const int j = j0 + jj;
            if (j >= j1) break;
            const uint8_t* st = ring + soff[jj];
            const __half* sc = reinterpret_cast<const __half*>(st + kRows * a.pitch);
            const uint32_t* zw = reinterpret_cast<const uint32_t*>(st + kRows * a.pitch + a.sbytes);
            uint32_t z0 = 8u, z1 = 8u;  // symmetric layout: zero point 8
            if (a.zbytes) {
              z0 = (zw[g * a.ZW + (grp >> 3)] >> (4 * (grp & 7))) & 15u;
              z1 = (zw[(g + 8) * a.ZW + (grp >> 3)] >> (4 * (grp & 7))) & 15u;
            }
            const uint32_t zz0 = (0x4300u | z0) * 0x10001u, zz1 = (0x4300u | z1) * 0x10001u;  // bf16x2 128 + z
            const float s0 = __half2float(sc[g * a.G + grp]), s1 = __half2float(sc[(g + 8) * a.G + grp]);
            const uint8_t* ra = st + g * a.pitch + grp * (GROUP / 2) + 8 * c;
            const uint8_t* rb = ra + 8 * a.pitch;
            float ae[4] = {0.f, 0.f, 0.f, 0.f}, ao[4] = {0.f, 0.f, 0.f, 0.f};  // even and odd steps: two chains
#pragma unroll
            for (int b = 0; b < kBlocks; ++b) {
              const uint2 wa = *reinterpret_cast<const uint2*>(ra + 32 * b);  // row g: words 2c, 2c + 1 of block b
              const uint2 wb = *reinterpret_cast<const uint2*>(rb + 32 * b);  // row g + 8
#pragma unroll
              for (int u = 0; u < 4; ++u)
                mma_bf16((u & 1) ? ao : ae, codes_minus_zero(wa.x, u, zz0), codes_minus_zero(wb.x, u, zz1),
                         codes_minus_zero(wa.y, u, zz0), codes_minus_zero(wb.y, u, zz1), xb[b][2 * u],
                         xb[b][2 * u + 1]);
            }
            tot[jj][0] += s0 * (ae[0] + ao[0]);
            tot[jj][1] += s0 * (ae[1] + ao[1]);
            tot[jj][2] += s1 * (ae[2] + ao[2]);
            tot[jj][3] += s1 * (ae[3] + ao[3]);
          }
        }
      }
#pragma unroll
      for (int jj = 0; jj < kChunk; ++jj) {
        if (j0 + jj >= j1) break;
        float* rw = rc + (jj * kConsumers + cw) * kRows * a.M;
        if (2 * c < a.M) {
          rw[g * a.M + 2 * c] = tot[jj][0];
          rw[(g + 8) * a.M + 2 * c] = tot[jj][2];
        }
        if (2 * c + 1 < a.M) {
          rw[g * a.M + 2 * c + 1] = tot[jj][1];
          rw[(g + 8) * a.M + 2 * c + 1] = tot[jj][3];
        }
      }
    }
    consumers_sync();
    if (tid == 0 && ok)  // every warp is past its reads of the chunk's stages: the tiles ns further on go there
      for (int j = j0 + a.ns; j < min(nt, j1 + a.ns); ++j) issue_tile(j);
    if constexpr (FUSED) {  // rows 2p, 2p + 1 are gate and up of output row0 / 2 + p
      for (int i = ctid; i < (j1 - j0) * a.M * (kRows / 2); i += 32 * kConsumers) {
        const int jj = i / (a.M * (kRows / 2)), rest = i - jj * (a.M * (kRows / 2));
        const int m = rest / (kRows / 2), p = rest % (kRows / 2);
        const float* rr = rc + jj * kConsumers * kRows * a.M;
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w) {
          gs += rr[(w * kRows + 2 * p) * a.M + m];
          us += rr[(w * kRows + 2 * p + 1) * a.M + m];
        }
        const int64_t row0 = int64_t(tb + j0 + jj) * kRows;
        a.y[int64_t(m) * a.ldy + (row0 >> 1) + p] = __float2bfloat16_rn(silu(gs) * us);
      }
    } else {
      for (int i = ctid; i < (j1 - j0) * a.M * kRows; i += 32 * kConsumers) {
        const int jj = i / (a.M * kRows), rest = i - jj * (a.M * kRows);
        const int m = rest / kRows, r = rest % kRows;
        const float* rr = rc + jj * kConsumers * kRows * a.M;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w) v += rr[(w * kRows + r) * a.M + m];
        const int64_t row0 = int64_t(tb + j0 + jj) * kRows;
        a.y[int64_t(m) * a.ldy + row0 + r] = __float2bfloat16_rn(v);
      }
    }
  }
}

struct StreamPlan {
  int grid = 0, ns = 0, stage = 0, smem = 0;
};

StreamPlan stream_plan(int64_t M, int64_t N, int64_t K, int64_t group, bool zeros) {
  StreamPlan p;
  if (M < 1 || M > kMaxTok || N % kRows != 0 || K % 64 != 0 || K % group != 0) return p;
  if (group != 64 && group != 128) return p;
  const int64_t tiles = N / kRows;
  if (tiles < 1 || tiles > (1 << 26)) return p;
  const int G = int(K / group), ZW = (G + 7) / 8;
  p.grid = int(std::min<int64_t>(tiles, num_sms()));
  const int per_cta = int((tiles + p.grid - 1) / p.grid);
  p.stage = kRows * stream_pitch(int(K), int(group), integer_form(int(M))) + 32 * G + (zeros ? kRows * ZW * 4 : 0);
  const int fixed = stream_layout(int(M), int(group), p.stage, 0).total;
  const int need = std::min(per_cta, 2);
  for (int budget : {kBudgetShared, kBudgetAlone}) {
    const int fit = (budget - fixed) / (p.stage + 16);  // each stage adds its two mbarriers too
    p.ns = std::min(per_cta, fit);
    if (p.ns >= need) break;
  }
  if (p.ns < need || p.ns < 1) {
    p.grid = 0;
    return p;
  }
  p.smem = stream_layout(int(M), int(group), p.stage, p.ns).total;
  return p;
}

}  // namespace

// The streaming GEMV takes M <= 8, N a multiple of 16, K a multiple of 64, groups of 64 or 128, and the scales and
// zero points 16-byte aligned (checked by the caller).
bool w4a16_stream_applies(int64_t M, int64_t N, int64_t K, int64_t group, bool zeros) {
  return stream_plan(M, N, K, group, zeros).grid > 0;
}

int w4a16_stream(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros,
                 void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags,
                 cudaStream_t stream) {
  const StreamPlan plan = stream_plan(M, N, K, group, qzeros != nullptr);
  if (!plan.grid) return set_error(BPT_ERR_UNSUPPORTED, "w4a16 stream: unsupported shape");
  StreamArgs a;
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
  a.G = int(K / group);
  a.ZW = (a.G + 7) / 8;
  a.tiles = int(N / kRows);
  a.pitch = stream_pitch(int(K), int(group), integer_form(int(M)));
  a.sbytes = 32 * a.G;
  a.zbytes = qzeros ? kRows * a.ZW * 4 : 0;
  a.stage = plan.stage;
  a.ns = plan.ns;
  const void* kernel = nullptr;
  const bool integer = integer_form(int(M));
#define BPT_STREAM_PICK(G)                                                                                    \
  kernel = fused ? (integer ? reinterpret_cast<const void*>(w4a16_stream_kernel<true, G, true>)               \
                            : reinterpret_cast<const void*>(w4a16_stream_kernel<true, G, false>))             \
                 : (integer ? reinterpret_cast<const void*>(w4a16_stream_kernel<false, G, true>)              \
                            : reinterpret_cast<const void*>(w4a16_stream_kernel<false, G, false>))
  if (group == 64) BPT_STREAM_PICK(64);
  if (group == 128) BPT_STREAM_PICK(128);
#undef BPT_STREAM_PICK
  if (!kernel) return set_error(BPT_ERR_UNSUPPORTED, "w4a16 stream: group %lld", (long long)group);
  int st = set_max_smem(kernel, plan.smem);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(plan.grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BPT_FLAG_PDL) ? 1 : 0;
  void* args[] = {&a};
  cudaError_t err = cudaLaunchKernelExC(&cfg, kernel, args);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "w4a16 stream launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

}  // namespace bpt
