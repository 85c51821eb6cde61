// W4A16 linear for M >= 16 tokens on the 5th-generation tensor cores (tcgen05, sm_100a only):
//   y[M, N] = x[M, K] . W^T,   W[n][k] = bf16(scale[n][g] * (q[n][k] - zero[n][g])),   fp32 accumulation,
// i.e. the dense bf16 weight that the reference's dequantize-then-nn.Linear path multiplies with (one rounding per
// weight), contracted on the tensor cores.
//
// CTA tile: 128 weight rows (the UMMA M) x BN tokens (the UMMA N: 16, 32, 64 or 128) x a slice of K; K is split over a
// thread-block cluster of `ks` CTAs (partial tiles reduced through distributed shared memory) when the row tiles
// alone leave SMs idle. K advances in chunks of 64 inputs (one 128-byte swizzle atom of bf16):
//   two producer warps (one lane each): TMA loads of the chunk's code tile [128 rows][32 B], and of its x
//     tile [BN][64] bf16 (128-byte swizzle, the UMMA K-major canonical layout). The two rings refill
//     independently. The codes do not depend on the previous kernel and are requested before the
//     programmatic-dependent-launch wait (the first ones before anything else); x after it.
//   warps 0-7 (dequantizers, thread = (row r = 32 (warp mod 4) + lane, half h = warp / 4 of the chunk)): the
//     row's 32 inputs of the half become 16 bf16 pairs, stored with one tcgen05.st into the thread's own TMEM lane
//     (A lives in tensor memory: the "TS" MMA form, so the dequantized tile never crosses shared memory). Per
//     pair one PRMT + one LOP3 give bf16 (128 + q) exactly, HSUB2 takes (128 + z) off (exact), and with the fp16
//     scale split as s = s_hi + s_lo (both bf16, exact) HMUL2 + HFMA2 give round_bf16(s (q - z)), one rounding.
//   warp 9 (one lane): tcgen05.mma kind::f16 with A from tensor memory and x from shared memory (bf16 x bf16 ->
//     fp32 in tensor memory), four K=16 steps per chunk, tcgen05.commit releasing the A and x buffers and finally
//     signalling the epilogue.
//   warps 0-3 (epilogue, TMEM lane quadrant = warp): tcgen05.ld of the accumulator rows, bf16 stores (SiLU(gate)
//     * up for the fused gate/up weight, whose rows alternate gate, up), or the split-K reduction.
// Every wait is bounded; on a timeout the kernel records the error, skips the dependent work and still frees its
// tensor memory. No TMA multicast.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"

namespace bpt {
namespace cg = cooperative_groups;
namespace {

constexpr int kTileRows = 128;                    // weight rows per CTA (the UMMA M)
constexpr int kChunkK = 64;                       // inputs per pipeline chunk
constexpr int kDeqWarps = 8;                      // dequantizing warps; 0-3 also run the epilogue
constexpr int kParts = kDeqWarps / 4;             // a row's chunk split over this many threads (one per warp group)
constexpr int kWords = 8 / kParts;                // code words (8 inputs each) per thread per chunk
constexpr int kProducerWarp = kDeqWarps;          // code tiles
constexpr int kMmaWarp = kDeqWarps + 1;
constexpr int kXWarp = kDeqWarps + 2;             // x tiles
constexpr int kThreads = 32 * (kDeqWarps + 3);
static_assert(kWords == 4, "a dequantizing thread takes four code words (32 inputs) of its row per chunk");
constexpr int kACols = kChunkK / 2;              // TMEM columns per A buffer: 64 bf16 of each row, 2 per column
constexpr int kCBytes = kTileRows * kChunkK / 2;  // 4 KB code tile
constexpr int kSmemMax = 227 * 1024;

struct TcArgs {
  __nv_bfloat16* y;
  int64_t ldy;
  const __half* scales;    // [N, G]
  const uint32_t* qzeros;  // [N, ZW] or null (symmetric: zero point 8)
  int M, N, K, G, ZW, group;
  int ks;      // CTAs splitting K (one cluster per row tile and token tile)
  int chunks;  // K chunks per CTA
  int ns;      // code and x ring stages
  int na;      // A ring stages (tensor memory, after the accumulator's BN columns)
  int gc;      // scale-table groups per CTA (an upper bound over the slices)
  int stall;         // BPT_FLAG_TEST_STALL: the first CTA issues no code tile from chunk 1 on (bounded-wait tests)
  uint64_t wait_ns;  // limit of the dequantizers' waits for code tiles
};

struct TcLayout {
  int x, codes, table, bars, slot, total;
};

// x ring | code ring | scale table [gc][128] u32 | mbarriers | TMEM address slot; offsets from a 1024-byte aligned
// base. The split-K partial tile [BN][128] f32 reuses the x and code rings once the main loop is over.
__host__ __device__ inline TcLayout tc_layout(int bn, int ns, int na, int gc) {
  TcLayout l;
  l.x = 0;
  l.codes = l.x + ns * bn * 128;
  l.table = l.codes + ns * kCBytes;
  l.bars = l.table + gc * kTileRows * 4;
  l.slot = l.bars + (4 * ns + 2 * na + 1) * 8;
  l.total = l.slot + 16;
  return l;
}

// ---- tcgen05 / TMA wrappers ----------------------------------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major tile in the 128-byte swizzle layout: rows of 128 bytes, 8-row
// atoms of 1024 bytes (stride-dimension byte offset), version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1), both K-major,
// N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t tc_idesc(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 16 consecutive accumulator columns of this thread's TMEM lane; the wait sits in the same statement, so no
// instruction can read the registers before the asynchronous load has landed.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf162(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

__host__ __device__ inline uint32_t tmem_cols(int bn, int na) {
  uint32_t c = 32;
  while (c < uint32_t(bn + na * kACols)) c <<= 1;
  return c;
}

// This thread's 16 bf16 pairs into 16 consecutive columns of its TMEM lane, waited on in the same statement.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// D (+)= A . B^T with A [128][16] in tensor memory (row m in lane m, two bf16 per column) and B from shared memory.
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t acc) {
  const uint32_t mask = 0u;  // no output lane disabled
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc), "r"(mask), "r"(mask), "r"(mask), "r"(mask)
      : "memory");
}

// A position in a ring of n stages: the stage and the parity of the lap (the phase its full barrier completes).
// Stepped incrementally: no division by the run-time ring size in the loops.
struct Ring {
  int s = 0;
  uint32_t lap = 0;
  __device__ __forceinline__ void next(int n) {
    if (++s == n) {
      s = 0;
      lap ^= 1u;
    }
  }
};

// One 8-input code word -> 8 bf16 weights round(s (q - z)) in input order (16 bytes of an A row).
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t zz, uint32_t shi, uint32_t slo) {
  const uint32_t w4 = w >> 4;
  uint32_t o[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    // byte p of w holds inputs 2p (low nibble) and 2p + 1 (high nibble): as bf16 (128 + q) in the two halves
    const uint32_t sel = uint32_t(p) | (uint32_t(p) << 4) | ((4u + p) << 8) | ((4u + p) << 12);
    const uint32_t t = (__byte_perm(w, w4, sel) & 0x000F000Fu) | 0x43004300u;
    const __nv_bfloat162 qz = __hsub2(bits_bf162(t), bits_bf162(zz));           // q - z, exact
    const __nv_bfloat162 lo = __hmul2(qz, bits_bf162(slo));                      // exact: 4 x 3 significant bits
    o[p] = bf162_bits(__hfma2(qz, bits_bf162(shi), lo));                        // one rounding of s (q - z)
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <bool FUSED, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_x,
                    const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const TcLayout L = tc_layout(BN, a.ns, a.na, a.gc);
  uint8_t* xbuf = smem + L.x;
  uint8_t* cbuf = smem + L.codes;
  uint32_t* table = reinterpret_cast<uint32_t*>(smem + L.table);
  uint64_t* cfull = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* cempty = cfull + a.ns;
  uint64_t* xfull = cempty + a.ns;
  uint64_t* xempty = xfull + a.ns;
  uint64_t* afull = xempty + a.ns;
  uint64_t* aempty = afull + a.na;
  uint64_t* done = aempty + a.na;
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + L.slot);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kr = int(blockIdx.x) % a.ks;               // this CTA's K slice (its rank in the cluster)
  const int n0 = (int(blockIdx.x) / a.ks) * kTileRows;  // first weight row
  const int m0 = int(blockIdx.y) * BN;                 // first token
  const int c0 = kr * a.chunks;                        // first K chunk of the slice
  const int g0 = c0 * kChunkK / a.group;               // first group of the slice
  // tensor memory: the accumulator (BN columns) then the A ring (32 columns per stage), a power of two >= 32
  const uint32_t kCols = tmem_cols(BN, a.na);

  if (tid == 0) {
    for (int s = 0; s < a.ns; ++s) {
      mbar_init(&cfull[s], 1);
      mbar_init(&cempty[s], kDeqWarps);
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < a.na; ++s) {
      mbar_init(&afull[s], kDeqWarps);
      mbar_init(&aempty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {  // the accumulator: 128 lanes x BN fp32 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();  // the barriers are initialised
  const uint64_t policy = l2_policy_evict_first();
  // (producer lane) the code tile of chunk c into stage rc.s; a refill (c >= ns) first waits for the release of
  // the stage's previous lap
  Ring rc;
  const bool stall_here = a.stall && blockIdx.x == 0 && blockIdx.y == 0;
  auto issue_codes = [&](int c) {
    // BPT_FLAG_TEST_STALL: the first CTA stops before chunk 1 (chunk 0 when it has one). The dequantizers await
    // every tile issued before it, in order, so no copy is left in flight; their waits for the rest run out.
    if (stall_here && c >= min(1, a.chunks - 1)) return false;
    if (c >= a.ns && !mbar_wait_sleep(&cempty[rc.s], rc.lap ^ 1u, 32u)) return false;
    mbar_arrive_expect_tx(&cfull[rc.s], kCBytes);
    tma_load_2d_hint(cbuf + rc.s * kCBytes, &tm_codes, (c0 + c) * (kChunkK / 8), n0, &cfull[rc.s], policy);
    rc.next(a.ns);
    return true;
  };
  const int pre = min(a.ns, a.chunks);
  if (warp == kProducerWarp && lane == 0)
    for (int c = 0; c < pre; ++c) (void)issue_codes(c);
  // The slice's scales and zero points, one u32 per (group, row): fp16 scale bits << 16 | zero point. Weights side:
  // no dependence on the previous kernel.
  // Loads are issued in batches of 8 per thread before any store, so the fill costs one memory round trip per
  // batch rather than one per entry.
  const int ng = min(a.gc, a.G - g0);
  for (int i0 = tid; i0 < ng * kTileRows; i0 += 8 * kThreads) {
    uint32_t sb[8], zw[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kThreads, gl = i / kTileRows, n = n0 + (i - gl * kTileRows);
      sb[u] = 0u;  // rows past N: scale 0, zero point 8
      zw[u] = 0x88888888u;
      if (i < ng * kTileRows && n < a.N) {
        sb[u] = __half_as_ushort(a.scales[int64_t(n) * a.G + g0 + gl]);
        if (a.qzeros) zw[u] = a.qzeros[int64_t(n) * a.ZW + ((g0 + gl) >> 3)];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kThreads, gl = i / kTileRows;
      if (i < ng * kTileRows) table[i] = (sb[u] << 16) | ((zw[u] >> (4 * ((g0 + gl) & 7))) & 15u);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  // Every CTA of this grid holds its tensor memory before any dependent CTA can start (and allocate).
  pdl_launch_dependents();

  bool ok = true;
  if (warp == kProducerWarp) {
    if (lane == 0)
      for (int c = pre; c < a.chunks && ok; ++c) ok = issue_codes(c);
  } else if (warp == kXWarp) {
    if (lane == 0) {
      pdl_wait();  // x belongs to the previous kernel until here
      Ring rx;
      for (int c = 0; c < a.chunks; ++c, rx.next(a.ns)) {
        if (c >= a.ns && !mbar_wait_sleep(&xempty[rx.s], rx.lap ^ 1u, 32u)) break;
        mbar_arrive_expect_tx(&xfull[rx.s], BN * 128);
        tma_load_2d(xbuf + rx.s * (BN * 128), &tm_x, (c0 + c) * kChunkK, m0, &xfull[rx.s]);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc_idesc(kTileRows, BN);
      Ring rx, ra;
      for (int c = 0; c < a.chunks && ok; ++c, rx.next(a.ns), ra.next(a.na)) {
        ok = mbar_wait(&afull[ra.s], ra.lap) && mbar_wait(&xfull[rx.s], rx.lap);
        if (!ok) break;
        tc_fence_after();
        const uint32_t at = tmem + uint32_t(BN + ra.s * kACols);
        const uint64_t bd = sw128_desc(smem_u32(xbuf + rx.s * (BN * 128)));
#pragma unroll
        for (int kk = 0; kk < kChunkK / 16; ++kk)  // K = 16 per MMA: 8 A columns, 32 bytes along the x rows
          tc_mma_ts(tmem, at + uint32_t(8 * kk), bd + 2 * kk, idesc, (c > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&aempty[ra.s]);
        tc_commit(&xempty[rx.s]);
      }
      tc_commit(done);  // arrives once every MMA issued above has completed (also on a timeout)
    }
  } else {  // dequantizers: thread -> row r, half h of the chunk (code words 4h .. 4h + 3)
    const int r = tid & (kTileRows - 1), h = tid >> 7;
    // this thread's A columns: its TMEM lane (row r), inputs 32h .. 32h + 31 of the chunk (2 per column)
    const uint32_t alane = tmem + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(BN + 16 * h);
    int gl_cur = -1;
    uint32_t zz = 0, shi = 0, slo = 0;
    const int cpg = a.group / kChunkK;                   // chunks per group (1 or 2)
    int gl = 0, sub = (c0 * kChunkK % a.group) / kChunkK;  // the chunk's group (table row) and place in it
    Ring rc, ra;
    for (int c = 0; c < a.chunks; ++c, rc.next(a.ns), ra.next(a.na)) {
      ok = mbar_wait(&cfull[rc.s], rc.lap, a.wait_ns) && ok;
      const uint4 w = *reinterpret_cast<const uint4*>(cbuf + rc.s * kCBytes + r * 32 + 16 * h);
      __syncwarp();
      if (lane == 0) mbar_arrive(&cempty[rc.s]);
      if (gl != gl_cur) {  // a new group: its zero point and split scale for this row
        gl_cur = gl;
        const uint32_t e = table[gl * kTileRows + r];
        zz = (0x4300u | (e & 15u)) * 0x10001u;  // bf16x2 (128 + z)
        const float sf = __half2float(__ushort_as_half(static_cast<unsigned short>(e >> 16)));
        const __nv_bfloat16 hi = __float2bfloat16_rn(sf);
        const __nv_bfloat16 lo = __float2bfloat16_rn(sf - __bfloat162float(hi));  // exact: s has 11 bits
        shi = bf162_bits(__halves2bfloat162(hi, hi));
        slo = bf162_bits(__halves2bfloat162(lo, lo));
      }
      if (++sub == cpg) {
        sub = 0;
        ++gl;
      }
      const uint32_t ws[kWords] = {w.x, w.y, w.z, w.w};
      uint32_t v[4 * kWords];  // inputs 32h .. 32h + 31 of the chunk as bf16 pairs, in order
#pragma unroll
      for (int i = 0; i < kWords; ++i) {
        const uint4 d = dequant_word(ws[i], zz, shi, slo);
        v[4 * i] = d.x;
        v[4 * i + 1] = d.y;
        v[4 * i + 2] = d.z;
        v[4 * i + 3] = d.w;
      }
      ok = mbar_wait(&aempty[ra.s], ra.lap ^ 1u) && ok;
      tc_fence_after();
      tmem_st16(alane + uint32_t(ra.s * kACols), v);
      tc_fence_before();  // the stores are complete; the MMA thread orders itself after this warp's arrival
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[ra.s]);
    }
  }

  // Epilogue: warps 0-3 read the accumulator rows 32 w .. 32 w + 31 (their TMEM lane quadrant).
  const int r = 32 * warp + lane;  // weight row in the tile (warps 0-3)
  float* part = reinterpret_cast<float*>(smem);  // split-K partials [BN][128], over the x and code rings
  if (warp < 4) {
    const bool fin = __all_sync(0xffffffffu, mbar_wait(done, 0u));
    tc_fence_after();
    pdl_wait();  // (already satisfied: the MMAs consumed x) y belongs to this kernel from here
    if (fin) {
#pragma unroll 1
      for (int j = 0; j < BN / 16; ++j) {
        uint32_t v[16];
        tmem_ld16(tmem + (uint32_t(32 * warp) << 16) + uint32_t(16 * j), v);
        if (a.ks > 1) {
#pragma unroll
          for (int i = 0; i < 16; ++i) part[(16 * j + i) * kTileRows + r] = __uint_as_float(v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int m = m0 + 16 * j + i;
            const float val = __uint_as_float(v[i]);
            if constexpr (FUSED) {  // rows 2p, 2p + 1 (adjacent lanes) are gate and up of output (n0 + r) / 2
              const float up = __shfl_xor_sync(0xffffffffu, val, 1);
              if (m < a.M && (r & 1) == 0 && n0 + r + 1 < a.N)
                a.y[int64_t(m) * a.ldy + ((n0 + r) >> 1)] = __float2bfloat16_rn(silu(val) * up);
            } else {
              if (m < a.M && n0 + r < a.N) a.y[int64_t(m) * a.ldy + n0 + r] = __float2bfloat16_rn(val);
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (a.ks > 1) {
    // the cluster's K slices of this tile: rank kr reduces tokens [kr BN / ks, (kr + 1) BN / ks) over the ranks'
    // partials (fixed order) and stores them
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    pdl_wait();
    const int t0 = kr * BN / a.ks, t1 = (kr + 1) * BN / a.ks;
    // Four consecutive rows of a token per item, every rank's partial requested before any is added (the ranks'
    // shared-memory windows mapped once): distributed shared-memory loads are long-latency, so they go wide.
    constexpr int kMaxKs = 8;
    const float4* pr[kMaxKs];
#pragma unroll
    for (int q = 0; q < kMaxKs; ++q)
      pr[q] = reinterpret_cast<const float4*>(cluster.map_shared_rank(part, q < a.ks ? q : 0));
    for (int i = tid; i < (t1 - t0) * (kTileRows / 4); i += kThreads) {
      const int t = t0 + i / (kTileRows / 4), r4 = i % (kTileRows / 4);
      float4 w[kMaxKs];
#pragma unroll
      for (int q = 0; q < kMaxKs; ++q)
        if (q < a.ks) w[q] = pr[q][t * (kTileRows / 4) + r4];
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < kMaxKs; ++q)  // the ranks in order: the sums do not depend on the timing
        if (q < a.ks) {
          v[0] += w[q].x;
          v[1] += w[q].y;
          v[2] += w[q].z;
          v[3] += w[q].w;
        }
      const int m = m0 + t;
      if (m >= a.M) continue;
      const int rr = 4 * r4;  // rows rr .. rr + 3 of the tile
      if constexpr (FUSED) {  // rows 2p, 2p + 1 are gate and up of output (n0 >> 1) + p
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (n0 + rr + 2 * e + 1 < a.N)
            a.y[int64_t(m) * a.ldy + (n0 >> 1) + (rr >> 1) + e] = __float2bfloat16_rn(silu(v[2 * e]) * v[2 * e + 1]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n0 + rr + e < a.N) a.y[int64_t(m) * a.ldy + n0 + rr + e] = __float2bfloat16_rn(v[e]);
      }
    }
    cluster.sync();  // the other slices' shared memory stays until every rank has read it
  }
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols)
                 : "memory");
  }
}

// ---- host ------------------------------------------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
}

struct TcPlan {
  int bn = 0, ks = 1, chunks = 0, ns = 0, na = 0, gc = 0, smem = 0, token_tiles = 0, row_tiles = 0;
};

TcPlan tc_plan(int64_t M, int64_t N, int64_t K, int64_t group) {
  TcPlan p;
  if (M < 16 || N < 1 || K % kChunkK != 0 || K < 2 * kChunkK || (group != 64 && group != 128) || K % group != 0)
    return p;
  if (M >= (1ll << 31) || N >= (1ll << 31)) return p;
  // tokens per tile: M rounded up to 16 / 32 / 64 / 128; more tokens take more tiles (each CTA pair per SM then
  // gets its own tiles, which beats one 256-token tile per SM)
  p.bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  p.token_tiles = int((M + p.bn - 1) / p.bn);
  p.row_tiles = int((N + kTileRows - 1) / kTileRows);
  p.na = 3;  // A stages in tensor memory
  // Up to 128 tokens a CTA fits in half an SM (<= 113 KB of shared memory, <= 256 TMEM columns): two run side by
  // side, each latency bound, so the K split aims at two CTAs per SM.
  const bool pair = p.bn <= 128;
  const int per_sm = pair ? 2 : 1;
  const int budget = pair ? 113 * 1024 : kSmemMax;
  const int64_t ctas = int64_t(p.row_tiles) * p.token_tiles;
  const int sms = num_sms();
  while (p.ks < 8 && ctas * p.ks * 2 <= int64_t(per_sm) * sms && K % (int64_t(kChunkK) * p.ks * 2) == 0 &&
         K / (p.ks * 2) >= 2 * kChunkK)
    p.ks *= 2;
  p.chunks = int(K / (kChunkK * p.ks));
  p.gc = int((int64_t(p.chunks) * kChunkK + group - 1) / group) + 1;
  for (p.ns = 8; p.ns >= 2; --p.ns)
    if (tc_layout(p.bn, p.ns, p.na, p.gc).total + 1024 <= budget) break;
  // the split-K partial tile [BN][128] f32 goes over the x and code rings
  if (p.ns < 2 || tmem_cols(p.bn, p.na) > uint32_t(512 / per_sm) ||
      (p.ks > 1 && p.bn * kTileRows * 4 > tc_layout(p.bn, p.ns, p.na, p.gc).table)) {
    p.bn = 0;
    return p;
  }
  p.smem = tc_layout(p.bn, p.ns, p.na, p.gc).total + 1024;
  return p;
}

}  // namespace

// The tcgen05 path takes M >= 16, K a multiple of 64 (at least 128), groups of 64 or 128; x and qweight 16-byte
// aligned with ldx a multiple of 8 (checked by the caller), and a driver that provides the tensor-map encoder.
bool w4a16_tc_applies(int64_t M, int64_t N, int64_t K, int64_t group) {
  return tc_plan(M, N, K, group).bn > 0 && encode_fn() != nullptr;
}

int w4a16_tc(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const int32_t* qzeros, void* y,
             int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group, bool fused, int flags, cudaStream_t stream) {
  const TcPlan plan = tc_plan(M, N, K, group);
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  if (!plan.bn || !encode) return set_error(BPT_ERR_UNSUPPORTED, "w4a16 tc: unsupported shape or driver");
  CUtensorMap tm_codes, tm_x;
  std::memset(&tm_codes, 0, sizeof(tm_codes));
  std::memset(&tm_x, 0, sizeof(tm_x));
  {  // codes: [N rows][K/8 words] u32, box 8 words x 128 rows, no swizzle; rows past N read as zero
    const cuuint64_t dims[2] = {cuuint64_t(K / 8), cuuint64_t(N)};
    const cuuint64_t strides[1] = {cuuint64_t(K / 2)};
    const cuuint32_t box[2] = {cuuint32_t(kChunkK / 8), cuuint32_t(kTileRows)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<int32_t*>(qweight), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(BPT_ERR_CUDA, "w4a16 tc: code tensor map (%d)", int(r));
  }
  {  // x: [M rows][K] bf16 (row pitch ldx), box 64 inputs x BN tokens, 128-byte swizzle; tokens past M read as zero
    const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(M)};
    const cuuint64_t strides[1] = {cuuint64_t(ldx * 2)};
    const cuuint32_t box[2] = {cuuint32_t(kChunkK), cuuint32_t(plan.bn)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(BPT_ERR_CUDA, "w4a16 tc: x tensor map (%d)", int(r));
  }
  TcArgs a;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.scales = static_cast<const __half*>(scales);
  a.qzeros = reinterpret_cast<const uint32_t*>(qzeros);
  a.M = int(M);
  a.N = int(N);
  a.K = int(K);
  a.group = int(group);
  a.G = int(K / group);
  a.ZW = (a.G + 7) / 8;
  a.ks = plan.ks;
  a.chunks = plan.chunks;
  a.ns = plan.ns;
  a.na = plan.na;
  a.gc = plan.gc;
  a.stall = (flags & BPT_FLAG_TEST_STALL) ? 1 : 0;
  a.wait_ns = a.stall ? kTestWaitNs : kWaitNs;
  const void* kernel = nullptr;
#define BPT_TC_PICK(F, B) \
  if (fused == F && plan.bn == B) kernel = reinterpret_cast<const void*>(w4a16_tc_kernel<F, B>);
  BPT_TC_PICK(false, 16) BPT_TC_PICK(false, 32) BPT_TC_PICK(false, 64) BPT_TC_PICK(false, 128)
  BPT_TC_PICK(true, 16) BPT_TC_PICK(true, 32) BPT_TC_PICK(true, 64) BPT_TC_PICK(true, 128)
#undef BPT_TC_PICK
  if (!kernel) return set_error(BPT_ERR_UNSUPPORTED, "w4a16 tc: no kernel for %d tokens", plan.bn);
  int st = set_max_smem(kernel, plan.smem);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(plan.row_tiles * plan.ks), unsigned(plan.token_tiles), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (plan.ks > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = unsigned(plan.ks);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (flags & BPT_FLAG_PDL) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  void* args[] = {&tm_codes, &tm_x, &a};
  cudaError_t err = cudaLaunchKernelExC(&cfg, kernel, args);
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "w4a16 tc launch: %s", cudaGetErrorString(err));
  return BPT_OK;
}

}  // namespace bpt
