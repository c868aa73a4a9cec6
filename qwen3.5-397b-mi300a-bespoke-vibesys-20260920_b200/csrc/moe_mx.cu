// Routed MXFP4 experts on the block-scaled tensor-core MMA (tcgen05.mma kind::mxf8f6f4).
//
// Weights: the packed e2m1 codes go from HBM to shared memory by TMA with the 16U4_ALIGN16B data
// type, which places every 16 codes in a 16-byte slot (the operand layout the MMA reads for 4-bit
// types), under the 128-byte swizzle. Their e8m0 block scales (one per 32 K) are applied by the
// MMA itself from tensor memory. No weight is decoded by any thread and none reaches HBM in a
// wider type.
//
// Activations: every bf16 activation x is written as two e4m3 terms with per-32 e8m0 scales,
//   x = 2^E * hi + 2^(E-4) * lo,   E = floor(log2(block max)) - 7,
// hi = x / 2^E truncated to e4m3, lo = the remainder * 16 truncated to e4m3. A bf16 value has 8
// significant bits; hi takes the top 4 and lo the next 4, so the split is exact whenever hi is a
// normal e4m3 (|x| >= 2^(E-6), which holds for every element within 2^13 of its block maximum);
// smaller ones keep an error below 2^-20 of the block maximum.
// e2m1 x e4m3 products are exact, so the two MMAs per K-block (hi then lo, same fp32 accumulator)
// reproduce the bf16 reference's products, as the f16 path does.
//
// Scale factors in tensor memory: for 128 rows and 4 consecutive K-blocks, one 512-byte chunk
// (32 lines of 16 bytes; line r holds the 4 scales of rows r, r+32, r+64, r+96) is copied by
// tcgen05.cp .32x128b.warpx4 into 4 columns of all four lane quarters; the MMA of K-block j of
// the chunk selects byte j (bits 30-31 of the scale address and the sf-id fields of the
// instruction descriptor). Weight chunks are arranged once at load time; activation chunks are
// written by the quantisation kernel per token tile.
//
// Kernel roles (256 threads, one CTA per SM, persistent over work units = (token tile, 128-row
// weight tile), weight tile fastest):
//   warp 0      TMA producer: fp4 tile (128 rows x 128 K), hi/lo token tiles, three scale chunks
//   warp 1      TMEM allocator + MMA issuer (tcgen05.cp of the chunks, then 8 MMAs per stage)
//   warps 4..7  epilogue (TMEM lane quarters 0..3): SiLU(gate) * up or plain, bf16 out
//
// Reference behaviour: `prefill_moe.py` (grouped expert GEMM over expert-sorted rows),
// `mxfp4_gemv.py` (MXFP4 layout: low nibble = even K, e8m0 per 32), `moe_hip.hip`.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "numerics.cuh"

#include <cstdlib>

namespace qb {

using bf16 = __nv_bfloat16;

constexpr int MX_THREADS = 256;
constexpr int MX_SK = 128;            // K per stage: one 128-byte swizzle atom of each operand
constexpr int MX_CHUNK = 512;         // bytes of one scale chunk (128 rows x 4 K-blocks)
constexpr int MX_MAX_EXPERTS = 512;  // experts per rank (the model has 512)

// W: the wide path (tiled codes, one box per operand, one hi|lo MMA operand, two scale chunks
// per stage: weight and activation); else three chunks (weight, hi, lo).
// KA (wide path only): 128-K atoms per pipeline stage. Two halve the copies, barrier round trips
// and scale copies per byte (one 256-row weight box, the two atoms' scale chunks in one bulk copy
// each) for the same bytes in flight.
template <int BN, bool W, int KA = 1>
struct MxCfg {
  static constexpr int A = 128 * MX_SK;          // fp4 tile, one byte per code in shared memory
  static constexpr int B = BN * MX_SK;           // one e4m3 token tile (hi or lo)
  static constexpr int STAGE = KA * (A + 2 * B);  // multiple of 1024: KA weight atoms, then KA hi|lo tiles
  static constexpr int SF = KA * (W ? 2 : 3) * MX_CHUNK;  // scale chunks per stage
  static constexpr int SF_COLS = KA * (W ? 8 : 12);       // their tensor-memory columns
  static constexpr int STAGING = BN * 128 * 2;   // one output tile (bf16)
  // token-tile prefix, counts and offsets of the experts in shared memory (16-byte multiple: the
  // mbarriers after it stay aligned)
  static constexpr int PREFIX = (4 * (3 * MX_MAX_EXPERTS + 1) + 15) / 16 * 16;
  static constexpr int BUDGET = (W ? 222 : 210) * 1024 - STAGING - PREFIX;
  static constexpr int STAGES = BUDGET / (STAGE + SF) > 12 ? 12 : BUDGET / (STAGE + SF);
  static constexpr int SMEM = 1024 + STAGES * STAGE + STAGES * SF + STAGING + PREFIX + 1024;
  // TMEM: two accumulators of ACC columns (2 BN: the hi and lo products side by side when BN <= 64),
  // then 12 scale columns per stage
  static constexpr int ACC = BN <= 64 ? 2 * BN : BN;
  static constexpr int SF_COL = 2 * ACC;
  static constexpr int TMEM_COLS = 512;
  static_assert(SF_COL + SF_COLS * STAGES <= TMEM_COLS, "tensor memory overflow");
  static_assert(SMEM <= 232448, "shared memory per block");
  static_assert((STAGES * (STAGE + SF) + STAGING + PREFIX) % 16 == 0, "mbarriers must stay aligned");
};

struct MxArgs {
  const uint8_t* sfa;      // weight scale chunks [E][n_tiles][K/128][512]
  const uint8_t* sfb_hi;   // activation scale chunks [tiles][K/128][512]
  const uint8_t* sfb_lo;
  const int* offsets;
  const int* counts;
  const int* tstart;       // [count + 1] first token tile of every expert
  void* out;
  int out_cols;
  int n_rows;
  int K;
  int count;
  int act;
  int* err;
  int tiled;               // weights re-laid so that every (128-row tile, K stage) block is contiguous
  int wide;                // tiled only: one 128-row weight box and one BN-row box per token tile
  int probe;               // diagnostics: accumulate the roles' wait cycles into g_mx_probe
};

// Diagnostic cycle counters (QB_MX_PROBE=1): [0] producer waiting for a free stage, [1] producer
// total, [2] MMA issuer waiting for a full stage, [3] MMA issuer total, [4] MMA waiting for the
// epilogue to free an accumulator, [5] producer cycles issuing a stage's copies, [6] MMA issuer
// cycles issuing a stage's scale copies and MMAs, [7] stages. Summed over CTAs; read (and
// cleared) by mx_probe_read.
__device__ unsigned long long g_mx_probe[8];

// e8m0 x e2m1 (A) x e4m3 (B), fp32 accumulate, M = 128, N = n, K-major operands.
__host__ __device__ constexpr uint32_t idesc_mxf8f6f4(int n) {
  return (5u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                       uint32_t sfb, bool acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)acc), "r"(sfa), "r"(sfb));
}

// 512 contiguous bytes (32 rows of 16 bytes) -> 4 columns x 32 lanes, repeated in all 4 lane quarters.
__device__ __forceinline__ void tmem_cp_chunk(uint32_t taddr, uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)(128 >> 4) << 16;  // leading byte offset (one 16-byte column: unused)
  d |= (uint64_t)(128 >> 4) << 32;  // stride byte offset: 8 rows x 16 bytes
  d |= (uint64_t)1 << 46;           // descriptor version
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(d) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <int BN>
__device__ __forceinline__ int mx_cols(int rest) {
  const int n = (rest + 15) & ~15;
  return n < BN ? n : BN;
}

// Wide path: the hi|lo planes of a token tile by boxes of exactly the tile's rows rounded up to
// 16 (m[i] loads 16 (i + 1) rows of each plane), so a tile of an expert with fewer tokens than BN
// moves and multiplies only those rows.
struct MxPlanes {
  CUtensorMap m[4];
};

template <int BN, bool W, int KA = 1>
__global__ void __launch_bounds__(MX_THREADS, 1)
    moe_mx_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmH,
                  const __grid_constant__ CUtensorMap tmL, const __grid_constant__ MxPlanes pl, MxArgs a) {
  using C = MxCfg<BN, W, KA>;
  static_assert(KA == 1 || W, "two-atom stages: wide path only");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* sfs = smem + C::STAGES * C::STAGE;                    // [STAGES][3][512]
  uint16_t* staging = reinterpret_cast<uint16_t*>(sfs + C::STAGES * C::SF);
  int* tstart = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(staging) + C::STAGING);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(tstart) + C::PREFIX);
  uint64_t* full = bars;
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_p = const_cast<int*>(abort_flag) + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_tiles = a.n_rows / 128;
  const int kstages = a.K / MX_SK;
  const bool gu = a.act == 1;

  int* cnts = tstart + MX_MAX_EXPERTS + 1;
  int* offs = cnts + MX_MAX_EXPERTS;
  for (int i = threadIdx.x; i <= a.count; i += blockDim.x) tstart[i] = a.tstart[i];
  for (int i = threadIdx.x; i < a.count; i += blockDim.x) {
    cnts[i] = a.counts[i];
    offs[i] = a.offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *issued_p = 0;
    fence_barrier_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmH);
    prefetch_tmap(&tmL);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int units = tstart[a.count] * n_tiles;
  // unit u -> (expert e, weight tile nt, token tile tt). Each role walks its units in increasing
  // order, so e (the last expert whose first token tile is <= tt) only moves forward from the
  // caller's previous value.
  auto unit = [&](int u, int& e, int& nt, int& tt) {
    tt = u / n_tiles;
    nt = u % n_tiles;
    while (e + 1 < a.count && tstart[e + 1] <= tt) ++e;
  };
  auto wrow = [&](int nt, int r) -> int {
    return gu ? (r < 64 ? nt * 64 + r : a.n_rows / 2 + nt * 64 + (r - 64)) : nt * 128 + r;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (W && elect_one()) {
      // stage ring in 32-bit shared addresses; stage index and barrier parity advanced, not divided
      const uint32_t st0 = smem_u32(stages), sf0 = smem_u32(sfs), full0 = smem_u32(full), empty0 = smem_u32(empty);
      int it = 0, s = 0;
      uint32_t ph = 1;  // parity of the empty barrier a first-round stage waits on (passes at once)
      long long pw = 0, pi = 0, w1 = 0;
      const long long p0 = clock64();
      int e = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int nt, tt;
        unit(u, e, nt, tt);
        const int m0 = (tt - tstart[e]) * BN;
        const int row_b = offs[e] + m0;
        const int ne = mx_cols<BN>(cnts[e] - m0);  // the tile's rows, rounded up to 16
        const CUtensorMap* tmP = &pl.m[ne / 16 - 1];
        const uint32_t TX = KA * (C::A / 2 + 2 * ne * MX_SK + 2 * MX_CHUNK);
        const int wtile = e * n_tiles + nt;
        int trow = wtile * kstages * 128;  // < 2^31: 512 experts x 32 tiles x 32 stages x 128
        const uint8_t* sfw = a.sfa + (long)wtile * kstages * MX_CHUNK;
        const uint8_t* sfb = a.sfb_hi + (long)tt * kstages * MX_CHUNK;
        for (int kx = 0; kx < kstages * MX_SK; kx += KA * MX_SK, ++it) {
          const long long w0 = a.probe ? clock64() : 0;
          if (!mbar_wait_s(empty0 + 8 * s, ph, a.err, ERR_TMA_WAIT, abort_flag)) goto prod_done_w;
          if (a.probe) {
            w1 = clock64();
            pw += w1 - w0;
          }
          const uint32_t fb = full0 + 8 * s, st = st0 + s * C::STAGE, sf = sf0 + s * C::SF;
          mbar_expect_tx_s(fb, TX);
          tma_load_2d_s(st, &tmW, fb, 0, trow);  // KA consecutive 128-row blocks of the tile
#pragma unroll
          for (int j = 0; j < KA; ++j)  // atom j: ne hi rows, then ne lo rows
            tma_load_3d_s(st + KA * C::A + j * 2 * ne * MX_SK, tmP, fb, kx + j * MX_SK, row_b, 0);
          bulk_g2s_s(sf, sfw, KA * MX_CHUNK, fb);  // the atoms' chunks are consecutive in memory
          bulk_g2s_s(sf + KA * MX_CHUNK, sfb, KA * MX_CHUNK, fb);
          trow += KA * 128;
          sfw += KA * MX_CHUNK;
          sfb += KA * MX_CHUNK;
          *issued_p = it + 1;
          if (a.probe) pi += clock64() - w1;
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    prod_done_w:
      if (a.probe) {
        atomicAdd(&g_mx_probe[0], (unsigned long long)pw);
        atomicAdd(&g_mx_probe[1], (unsigned long long)(clock64() - p0));
        atomicAdd(&g_mx_probe[5], (unsigned long long)pi);
        atomicAdd(&g_mx_probe[7], (unsigned long long)it);
      }
    } else if (!W && elect_one()) {
      int it = 0;
      long long pw = 0, pi = 0, w1 = 0;
      const long long p0 = clock64();
      int e = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int nt, tt;
        unit(u, e, nt, tt);
        const int m0 = (tt - tstart[e]) * BN;
        const int ne = mx_cols<BN>(cnts[e] - m0);
        const int row_b = offs[e] + m0;
        const long erow = (long)e * a.n_rows;
        const uint8_t* sfa_u = a.sfa + ((long)e * n_tiles + nt) * kstages * MX_CHUNK;
        const uint8_t* sfh_u = a.sfb_hi + (long)tt * kstages * MX_CHUNK;
        const uint8_t* sfl_u = a.sfb_lo + (long)tt * kstages * MX_CHUNK;
        for (int ks = 0; ks < kstages; ++ks, ++it) {
          const int s = it % C::STAGES;
          const long long w0 = a.probe ? clock64() : 0;
          if (!mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1, a.err, ERR_TMA_WAIT, abort_flag)) goto prod_done;
          if (a.probe) {
            w1 = clock64();
            pw += w1 - w0;
          }
          uint8_t* st = stages + s * C::STAGE;
          uint8_t* sf = sfs + s * C::SF;
          // the fp4 tile counts its global (packed) bytes: half of its shared-memory footprint
          if (W) {  // one box per operand: the 8 KB weight block, BN token rows of hi and lo
            mbar_expect_tx(&full[s], C::A / 2 + 2 * BN * MX_SK + 2 * MX_CHUNK);
            const int trow = (int)((((long)e * n_tiles + nt) * kstages + ks) * 128);
            tma_load_2d(st, &tmW, &full[s], 0, trow);
            tma_load_3d(st + C::A, &tmH, &full[s], ks * MX_SK, row_b, 0);  // hi then lo plane
            bulk_g2s(sf, sfa_u + ks * MX_CHUNK, MX_CHUNK, &full[s]);
            bulk_g2s(sf + MX_CHUNK, a.sfb_hi + ((long)tt * kstages + ks) * MX_CHUNK, MX_CHUNK, &full[s]);
          } else {
            mbar_expect_tx(&full[s], C::A / 2 + 2 * ne * MX_SK + 3 * MX_CHUNK);
          }
          if (W) {
          } else if (a.tiled) {  // one contiguous 8 KB block: rows (tile, stage, 0..127) of 64 bytes
            const int trow = (int)((((long)e * n_tiles + nt) * kstages + ks) * 128);
            tma_load_2d(st, &tmW, &full[s], 0, trow);
            tma_load_2d(st + 64 * MX_SK, &tmW, &full[s], 0, trow + 64);
          } else {
            tma_load_2d(st, &tmW, &full[s], ks * MX_SK, (int)(erow + wrow(nt, 0)));
            tma_load_2d(st + 64 * MX_SK, &tmW, &full[s], ks * MX_SK, (int)(erow + wrow(nt, 64)));
          }
          for (int t = 0; !W && t < ne; t += 16) {
            tma_load_2d(st + C::A + t * MX_SK, &tmH, &full[s], ks * MX_SK, row_b + t);
            tma_load_2d(st + C::A + C::B + t * MX_SK, &tmL, &full[s], ks * MX_SK, row_b + t);
          }
          if (!W) {
            bulk_g2s(sf, sfa_u + ks * MX_CHUNK, MX_CHUNK, &full[s]);
            bulk_g2s(sf + MX_CHUNK, sfh_u + ks * MX_CHUNK, MX_CHUNK, &full[s]);
            bulk_g2s(sf + 2 * MX_CHUNK, sfl_u + ks * MX_CHUNK, MX_CHUNK, &full[s]);
          }
          *issued_p = it + 1;
          if (a.probe) pi += clock64() - w1;
        }
      }
    prod_done:
      if (a.probe) {
        atomicAdd(&g_mx_probe[0], (unsigned long long)pw);
        atomicAdd(&g_mx_probe[1], (unsigned long long)(clock64() - p0));
        atomicAdd(&g_mx_probe[5], (unsigned long long)pi);
        atomicAdd(&g_mx_probe[7], (unsigned long long)it);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (W && elect_one()) {
      const uint32_t full0 = smem_u32(full), empty0 = smem_u32(empty), accf0 = smem_u32(acc_full),
                     acce0 = smem_u32(acc_empty);
      const uint64_t da0 = desc_sw128(smem_u32(stages));
      const uint32_t sf_s0 = smem_u32(sfs);
      int s = 0, ti = 0, e = 0;
      uint32_t ph = 0;
      bool ok = true;
      long long mw = 0, aw = 0, mi = 0, m1 = 0;
      const long long m0c = clock64();
      for (int u = blockIdx.x; u < units && ok && !*abort_flag; u += gridDim.x, ++ti) {
        int nt, tt;
        unit(u, e, nt, tt);
        // hi | lo rows of the tile: one N = 2 ne operand (lo products in columns [ne, 2 ne))
        const int ne = mx_cols<BN>(cnts[e] - (tt - tstart[e]) * BN);
        const uint32_t idesc = idesc_mxf8f6f4(2 * ne);
        const int acc = ti & 1;
        const long long a0 = a.probe ? clock64() : 0;
        if (!mbar_wait_s(acce0 + 8 * acc, ((ti >> 1) & 1) ^ 1, a.err, ERR_ACC_WAIT, abort_flag)) break;
        if (a.probe) aw += clock64() - a0;
        tc_fence_after();
        const uint32_t d = tmem + acc * C::ACC;
        for (int ks = 0; ks < kstages; ks += KA) {
          const long long w0 = a.probe ? clock64() : 0;
          if (!mbar_wait_s(full0 + 8 * s, ph, a.err, ERR_MMA_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          if (a.probe) {
            m1 = clock64();
            mw += m1 - w0;
          }
          tc_fence_after();
          const uint32_t sf_t = tmem + C::SF_COL + s * C::SF_COLS, sf_s = sf_s0 + s * C::SF;
          const uint64_t so = (uint64_t)((s * C::STAGE) >> 4);  // descriptor address field: bytes / 16
          const uint64_t da = da0 + so, dh = da0 + so + (uint64_t)((KA * C::A) >> 4);
          // KA weight scale chunks, then KA activation chunks: 4 tensor-memory columns each
#pragma unroll
          for (int c = 0; c < 2 * KA; ++c) tmem_cp_chunk(sf_t + 4 * c, sf_s + c * MX_CHUNK);
#pragma unroll
          for (int at = 0; at < KA; ++at) {
            const uint64_t dat = da + (uint64_t)((at * C::A) >> 4), dht = dh + (uint64_t)((at * 2 * ne * MX_SK) >> 4);
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // K-block j: hi | lo products into accumulator columns [0, 2 ne)
              const uint32_t id_j = idesc | ((uint32_t)j << 29) | ((uint32_t)j << 4);
              const uint32_t bsel = (uint32_t)j << 30;
              mma_mx(d, dat + 2 * j, dht + 2 * j, id_j, (sf_t + 4 * at) | bsel, (sf_t + 4 * KA + 4 * at) | bsel,
                     (ks | at | j) != 0);
            }
          }
          mma_commit_s(empty0 + 8 * s);
          if (a.probe) mi += clock64() - m1;
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_s(accf0 + 8 * acc);
      }
      if (a.probe) {
        atomicAdd(&g_mx_probe[2], (unsigned long long)mw);
        atomicAdd(&g_mx_probe[3], (unsigned long long)(clock64() - m0c));
        atomicAdd(&g_mx_probe[4], (unsigned long long)aw);
        atomicAdd(&g_mx_probe[6], (unsigned long long)mi);
      }
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_DRAIN, nullptr);
    } else if (!W && elect_one()) {
      int it = 0, ti = 0;
      bool ok = true;
      long long mw = 0, aw = 0, mi = 0, m1 = 0;
      const long long m0c = clock64();
      int e = 0;
      for (int u = blockIdx.x; u < units && ok && !*abort_flag; u += gridDim.x, ++ti) {
        // wide: hi and lo token rows form one N = 2 BN operand (all BN rows of each: the lo rows start
        // at BN); else one MMA per term with N = the tile's valid rows
        uint32_t idesc = idesc_mxf8f6f4(2 * BN);
        if (!W) {
          int nt, tt;
          unit(u, e, nt, tt);
          idesc = idesc_mxf8f6f4(mx_cols<BN>(cnts[e] - (tt - tstart[e]) * BN));
        }
        const int acc = ti & 1;
        const long long a0 = a.probe ? clock64() : 0;
        if (!mbar_wait(&acc_empty[acc], ((ti >> 1) & 1) ^ 1, a.err, ERR_ACC_WAIT, abort_flag)) break;
        if (a.probe) aw += clock64() - a0;
        tc_fence_after();
        const uint32_t d = tmem + acc * C::ACC;
        for (int ks = 0; ks < kstages; ++ks, ++it) {
          const int s = it % C::STAGES;
          const long long w0 = a.probe ? clock64() : 0;
          if (!mbar_wait(&full[s], (it / C::STAGES) & 1, a.err, ERR_MMA_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          if (a.probe) {
            m1 = clock64();
            mw += m1 - w0;
          }
          tc_fence_after();
          const uint32_t sf_t = tmem + C::SF_COL + s * C::SF_COLS;
          const uint32_t sf_s = smem_u32(sfs + s * C::SF);
          const uint32_t sbase = smem_u32(stages + s * C::STAGE);
          const uint64_t da = desc_sw128(sbase), dh = desc_sw128(sbase + C::A), dl = desc_sw128(sbase + C::A + C::B);
          if (W) {
            tmem_cp_chunk(sf_t, sf_s);
            tmem_cp_chunk(sf_t + 4, sf_s + MX_CHUNK);
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // K-block j: hi | lo products into accumulator columns [0, 2 BN)
              const uint32_t id_j = idesc | ((uint32_t)j << 29) | ((uint32_t)j << 4);
              const uint32_t bsel = (uint32_t)j << 30;
              mma_mx(d, da + 2 * j, dh + 2 * j, id_j, (sf_t) | bsel, (sf_t + 4) | bsel, (ks | j) != 0);
            }
          } else {
            tmem_cp_chunk(sf_t, sf_s);
            tmem_cp_chunk(sf_t + 4, sf_s + MX_CHUNK);
            tmem_cp_chunk(sf_t + 8, sf_s + 2 * MX_CHUNK);
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // K-block j of the stage: 32 codes = 32 shared-memory bytes
              const uint32_t id_j = idesc | ((uint32_t)j << 29) | ((uint32_t)j << 4);
              const uint32_t bsel = (uint32_t)j << 30;
              mma_mx(d, da + 2 * j, dh + 2 * j, id_j, (sf_t) | bsel, (sf_t + 4) | bsel, (ks | j) != 0);
              mma_mx(d, da + 2 * j, dl + 2 * j, id_j, (sf_t) | bsel, (sf_t + 8) | bsel, true);
            }
          }
          mma_commit(&empty[s]);
          if (a.probe) mi += clock64() - m1;
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
      }
      if (a.probe) {
        atomicAdd(&g_mx_probe[2], (unsigned long long)mw);
        atomicAdd(&g_mx_probe[3], (unsigned long long)(clock64() - m0c));
        atomicAdd(&g_mx_probe[4], (unsigned long long)aw);
        atomicAdd(&g_mx_probe[6], (unsigned long long)mi);
      }
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_DRAIN, nullptr);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- epilogue
    const int ew = warp & 3;
    const int row = ew * 32 + lane;
    const int et = threadIdx.x - 128;
    int ti = 0;
    int e = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++ti) {
      int nt, tt;
      unit(u, e, nt, tt);
      const int m0 = (tt - tstart[e]) * BN;
      const int cnt = cnts[e];
      const int row_b = offs[e] + m0;
      const int acc = ti & 1;
      if (!mbar_wait(&acc_full[acc], (ti >> 1) & 1, a.err, ERR_EPI_WAIT, abort_flag)) break;
      tc_fence_after();
      const int ne = mx_cols<BN>(cnt - m0);
      for (int c0 = 0; c0 < ne; c0 += 16) {
        float v[16];
        const uint32_t ta = tmem + acc * C::ACC + c0 + ((uint32_t)(ew * 32) << 16);
        tmem_ld16(ta, v);
        if (W) {  // hi products in columns [0, ne), lo products in [ne, 2 ne)
          float vl[16];
          tmem_ld16(ta + ne, vl);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += vl[j];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          bf16 o = __float2bfloat16(v[j]);
          staging[(c0 + j) * 128 + row] = *reinterpret_cast<uint16_t*>(&o);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int nvalid = min(ne, cnt - m0);
      bf16* Y = reinterpret_cast<bf16*>(a.out);
      if (gu) {
        for (int idx = et; idx < nvalid * 64; idx += 128) {
          const int j = idx / 64, r = idx % 64;
          uint16_t gb = staging[j * 128 + r], ub = staging[j * 128 + 64 + r];
          const float g = __bfloat162float(*reinterpret_cast<bf16*>(&gb));
          const float uu = __bfloat162float(*reinterpret_cast<bf16*>(&ub));
          const float sg = __bfloat162float(__float2bfloat16(g / (1.f + expf(-g))));
          Y[(long)(row_b + j) * a.out_cols + nt * 64 + r] = __float2bfloat16(sg * uu);
        }
      } else {
        for (int idx = et; idx < nvalid * 16; idx += 128) {
          const int j = idx / 16, q = idx % 16;
          const uint4 val = *reinterpret_cast<const uint4*>(&staging[j * 128 + q * 8]);
          *reinterpret_cast<uint4*>(Y + (long)(row_b + j) * a.out_cols + nt * 128 + q * 8) = val;
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
  }

  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    const int n = *issued_p;
    for (int i = n - C::STAGES < 0 ? 0 : n - C::STAGES; i < n; ++i)
      mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, a.err, ERR_DRAIN, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ activation split
// Rows of the token tile holding row r_e of expert e (tiles of BN rows from the expert's first
// row), rounded up to 16: the tile's hi | lo MMA operand is 2 x this many rows.
__device__ __forceinline__ int mx_tile_rows(const int* offsets, int count, int n_rows, int e, int r_e, int BN) {
  const int cnt = (e + 1 < count ? offsets[e + 1] : n_rows) - offsets[e];
  const int m0 = r_e / BN * BN;
  const int n = (cnt - m0 + 15) & ~15;
  return n < BN ? n : BN;
}

// One warp per row: rows `a < *n_rows` of x (row a read from x[perm[a]] when perm is given) ->
// hi / lo e4m3 bytes [cap, K] and their scales, written straight into the per-tile chunks (the
// token tile of row a is the tile of its expert's run; tiles of BN rows). Each lane holds 8
// consecutive elements, so 4 lanes form one 32-element block.
__global__ void mx_quant_kernel(const bf16* x, const int* perm, const int* n_rows, int K, int wpr, const int* offsets,
                                const int* tstart, int count, int BN, uint8_t* hi, uint8_t* lo, uint8_t* sf_hi,
                                uint8_t* sf_lo, int cstride, int lo_rows) {
  const int lane = threadIdx.x % 32;
  const int w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int a = w / wpr, part = w % wpr;  // `wpr` warps share a row when there are few rows
  if (a >= *n_rows) return;
  const int kseg = K / wpr, kbeg = part * kseg, kend = kbeg + kseg;
  // expert of assignment row a: the last expert whose first row is <= a (an empty expert shares
  // its offset with the next one, so the last such expert is never empty); then its token tile
  int lo_e = 0, hi_e = count - 1;
  while (lo_e < hi_e) {
    const int mid = (lo_e + hi_e + 1) >> 1;
    if (offsets[mid] <= a) lo_e = mid; else hi_e = mid - 1;
  }
  const int r_e = a - offsets[lo_e];
  const int tt = tstart[lo_e] + r_e / BN, rr = r_e % BN;
  // merged layout: the lo scales follow the tile's own rows (rounded up to 16), the rows of its
  // one hi | lo MMA operand
  const int lo_off = lo_rows ? mx_tile_rows(offsets, count, *n_rows, lo_e, r_e, BN) : 0;
  const bf16* src = x + (long)(perm ? perm[a] : a) * K;
  uint8_t* hrow = hi + (long)a * K;
  uint8_t* lrow = lo + (long)a * K;
  const long sf_tile = (long)tt * (K / MX_SK) * cstride;  // cstride: bytes from one chunk to the next
  for (int kbase = kbeg; kbase < kend; kbase += 256) {  // warp-uniform trip count (shuffles below)
    const int k0 = kbase + lane * 8;
    const bool valid = k0 < kend;                       // segments are multiples of 128, not always of 256
    const uint4 raw = valid ? *reinterpret_cast<const uint4*>(src + k0) : make_uint4(0, 0, 0, 0);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(p2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
    uint32_t mb = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) mb = max(mb, __float_as_uint(fabsf(v[i])));
    mb = max(mb, __shfl_xor_sync(0xffffffff, mb, 1));
    mb = max(mb, __shfl_xor_sync(0xffffffff, mb, 2));  // max over the 4 lanes of the block
    const int E = mx_block_exponent(mb);  // block max / 2^E in [128, 256)
    uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint8_t ch, cl;
      mx_split(v[i], E, ch, cl);
      hw[i / 4] |= (uint32_t)ch << (8 * (i % 4));
      lw[i / 4] |= (uint32_t)cl << (8 * (i % 4));
    }
    if (!valid) continue;
    *reinterpret_cast<uint2*>(hrow + k0) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(lrow + k0) = make_uint2(lw[0], lw[1]);
    if ((lane & 3) == 0) {
      const int kb = k0 / 32;
      const long cb = sf_tile + (long)(kb / 4) * cstride;
      sf_hi[cb + mx_chunk_offset(rr, kb % 4)] = (uint8_t)(E + 127);
      sf_lo[cb + mx_chunk_offset(rr + lo_off, kb % 4)] = (uint8_t)(E - 4 + 127);
    }
  }
}

// Each token once: rows of x [T, K] -> hi / lo e4m3 bytes [T, K] and one exponent byte (E + 127)
// per 32-element block [T, K/32], with the same per-lane code as mx_quant_kernel (identical
// bytes). mx_expand_kernel then places every (token, expert) assignment's row and scales into the
// expert-sorted tiles: the routed MoE input is quantised T times instead of T x k times.
__global__ void mx_quant_rows_kernel(const bf16* x, int T, int K, int wpr, uint8_t* hi, uint8_t* lo,
                                     uint8_t* exps, const int* ids, int k) {
  const int lane = threadIdx.x % 32;
  const int w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int a = w / wpr, part = w % wpr;
  if (a >= T) return;
  if (ids && ids[(long)a * k] < 0) return;  // a row routed nowhere (unused receive-area row)
  const int kseg = K / wpr, kbeg = part * kseg, kend = kbeg + kseg;
  const bf16* src = x + (long)a * K;
  for (int kbase = kbeg; kbase < kend; kbase += 256) {
    const int k0 = kbase + lane * 8;
    const bool valid = k0 < kend;
    const uint4 raw = valid ? *reinterpret_cast<const uint4*>(src + k0) : make_uint4(0, 0, 0, 0);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(p2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
    uint32_t mb = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) mb = max(mb, __float_as_uint(fabsf(v[i])));
    mb = max(mb, __shfl_xor_sync(0xffffffff, mb, 1));
    mb = max(mb, __shfl_xor_sync(0xffffffff, mb, 2));
    const int E = mx_block_exponent(mb);
    uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint8_t ch, cl;
      mx_split(v[i], E, ch, cl);
      hw[i / 4] |= (uint32_t)ch << (8 * (i % 4));
      lw[i / 4] |= (uint32_t)cl << (8 * (i % 4));
    }
    if (!valid) continue;
    *reinterpret_cast<uint2*>(hi + (long)a * K + k0) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(lo + (long)a * K + k0) = make_uint2(lw[0], lw[1]);
    if ((lane & 3) == 0) exps[(long)a * (K / 32) + k0 / 32] = (uint8_t)(E + 127);
  }
}

// One warp per assignment row a < *n_rows: the hi / lo bytes of token perm[a] and its block
// exponents, into row a and the chunk of row a's token tile (as mx_quant_kernel writes them).
__global__ void mx_expand_kernel(const uint8_t* qhi, const uint8_t* qlo, const uint8_t* exps, const int* perm,
                                 const int* n_rows, int K, const int* offsets, const int* tstart, int count, int BN,
                                 uint8_t* hi, uint8_t* lo, uint8_t* sf_hi, uint8_t* sf_lo, int cstride, int lo_rows) {
  const int lane = threadIdx.x % 32;
  const int a = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (a >= *n_rows) return;
  int lo_e = 0, hi_e = count - 1;
  while (lo_e < hi_e) {
    const int mid = (lo_e + hi_e + 1) >> 1;
    if (offsets[mid] <= a) lo_e = mid; else hi_e = mid - 1;
  }
  const int r_e = a - offsets[lo_e];
  const int tt = tstart[lo_e] + r_e / BN, rr = r_e % BN;
  const int lo_off = lo_rows ? mx_tile_rows(offsets, count, *n_rows, lo_e, r_e, BN) : 0;
  const long src = perm[a];
  const uint4* sh = reinterpret_cast<const uint4*>(qhi + src * K);
  const uint4* sl = reinterpret_cast<const uint4*>(qlo + src * K);
  uint4* dh = reinterpret_cast<uint4*>(hi + (long)a * K);
  uint4* dl = reinterpret_cast<uint4*>(lo + (long)a * K);
  // eight 16-byte loads in flight per lane before their stores (the rows come from L2)
  const int nv = K / 16;
  int v = lane;
  for (; v + 96 < nv; v += 128) {
    uint4 h[4], l[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      h[u] = sh[v + 32 * u];
      l[u] = sl[v + 32 * u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      dh[v + 32 * u] = h[u];
      dl[v + 32 * u] = l[u];
    }
  }
  for (; v < nv; v += 32) {
    dh[v] = sh[v];
    dl[v] = sl[v];
  }
  const long sf_tile = (long)tt * (K / MX_SK) * cstride;
  for (int kb = lane; kb < K / 32; kb += 32) {
    const uint8_t eb = exps[src * (K / 32) + kb];
    const long cb = sf_tile + (long)(kb / 4) * cstride;
    sf_hi[cb + mx_chunk_offset(rr, kb % 4)] = eb;
    sf_lo[cb + mx_chunk_offset(rr + lo_off, kb % 4)] = (uint8_t)(eb - 4);
  }
}

// tstart[e] = sum over e' < e of ceil(counts[e'] / BN), tstart[count] = total token tiles.
__global__ void mx_tile_prefix_kernel(const int* counts, int count, int BN, int* tstart) {
  const int lane = threadIdx.x;
  int run = 0;
  for (int base = 0; base < count; base += 32) {
    const int e = base + lane;
    const int t = e < count ? (counts[e] + BN - 1) / BN : 0;
    int incl = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffff, incl, o);
      if (lane >= o) incl += v;
    }
    if (e < count) tstart[e] = run + incl - t;
    run += __shfl_sync(0xffffffff, incl, 31);
  }
  if (lane == 0) tstart[count] = run;
}

// ------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 mx_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D map [rows][cols] with a (128 elements x box_rows) box and the 128-byte swizzle; fp4 = packed
// e2m1 codes unpacked to one code per shared-memory byte (16U4_ALIGN16B), else one byte per element.
static int mx_tmap(CUtensorMap* m, const void* base, long rows, long cols, long row_bytes, int box_rows, bool fp4) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = mx_encode()(m, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                           const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

// 3-D map of the hi and lo activation planes [2][rows][cols] (bytes), box (128, box_rows, 2):
// one load brings a token tile's hi rows followed by its lo rows.
static int mx_tmap_planes(CUtensorMap* m, const void* base, long rows, long cols, long plane_bytes, int box_rows) {
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, 2};
  cuuint64_t strides[2] = {(cuuint64_t)cols, (cuuint64_t)plane_bytes};
  cuuint32_t box[3] = {128, (cuuint32_t)box_rows, 2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = mx_encode()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

int mx_probe_read(unsigned long long* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_mx_probe, sizeof(g_mx_probe));
  if (e != cudaSuccess) return (int)e;
  static const unsigned long long zero[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  return (int)cudaMemcpyToSymbol(g_mx_probe, zero, sizeof(zero));
}

// Merged activation layout (wide boxes over tiled codes, token tiles of at most 64): the lo plane
// right after the hi plane, and one scale chunk per (token tile, K stage) holding the hi scales in
// rows [0, n) and the lo scales in rows [n, 2 n), n = the tile's rows rounded up to 16: the rows of
// its one N = 2 n MMA operand.
bool mx_merged(bool tiled, int BN) {
  static const bool wide_env = !getenv("QB_MX_WIDE") || atoi(getenv("QB_MX_WIDE")) != 0;
  return tiled && wide_env && BN <= 64;
}

static int mx_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool W, int KA = 1>
static int mx_launch(const CUtensorMap& tw, const CUtensorMap& th, const CUtensorMap& tl, const MxPlanes& pl,
                     const MxArgs& a, cudaStream_t st) {
  using C = MxCfg<BN, W, KA>;
  auto k = moe_mx_kernel<BN, W, KA>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr = true;
  }
  k<<<mx_sms(), MX_THREADS, C::SMEM, st>>>(tw, th, tl, pl, a);
  return (int)cudaGetLastError();
}

// Token-tile width: about 1.5x the mean tokens per expert (routing is uneven), at most 64 so that
// the pipeline keeps at least 5 stages (QB_MX_BN_MAX overrides the cap). Wider tiles only save
// re-reads of an expert's weights, which the unit order serves from L2 (an expert's token tiles
// are scheduled side by side); narrower tiles buy pipeline depth, which HBM streaming needs more.
int mx_token_tile(int cap, int count) {
  static const int bn_max = getenv("QB_MX_BN_MAX") ? atoi(getenv("QB_MX_BN_MAX")) : 64;
  const int avg = (cap + count - 1) / (count > 0 ? count : 1);
  const int want = avg + avg / 2 + 2;
  const int bn = want <= 16 ? 16 : want <= 32 ? 32 : want <= 64 ? 64 : 128;
  return bn > bn_max ? (bn_max >= 64 ? 64 : bn_max >= 32 ? 32 : 16) : bn;
}

int mx_tile_prefix(const int* counts, int count, int BN, int* tstart, cudaStream_t s) {
  mx_tile_prefix_kernel<<<1, 32, 0, s>>>(counts, count, BN, tstart);
  return (int)cudaGetLastError();
}

int mx_quant(const void* x, const int* perm, const int* n_rows, int cap, int K, const int* offsets, const int* counts,
             const int* tstart, int count, int BN, uint8_t* hi, uint8_t* lo, uint8_t* sf_hi, uint8_t* sf_lo,
             cudaStream_t s, bool merged) {
  if (!cap) return 0;
  if (K % MX_SK) return -1;
  (void)counts;
  // warps per row: enough warps in flight for small batches (at least 256 elements per warp)
  int wpr = 1;
  while ((long)cap * wpr < 2048 && (K / (wpr * 2)) % 256 == 0) wpr *= 2;
  const long warps = (long)cap * wpr;
  mx_quant_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>((const bf16*)x, perm, n_rows, K, wpr, offsets, tstart,
                                                               count, BN, hi, lo, sf_hi, sf_lo, MX_CHUNK,
                                                               merged ? BN : 0);
  return (int)cudaGetLastError();
}

int mx_quant_expand(const void* x, int T, const int* perm, const int* n_rows, int cap, int K, const int* offsets,
                    const int* tstart, int count, int BN, uint8_t* qscratch, uint8_t* hi, uint8_t* lo, uint8_t* sf_hi,
                    uint8_t* sf_lo, cudaStream_t s, bool merged, const int* skip_ids, int k) {
  if (!cap || !T) return 0;
  if (K % MX_SK) return -1;
  uint8_t* qhi = qscratch;
  uint8_t* qlo = qhi + (long)T * K;
  uint8_t* exps = qlo + (long)T * K;
  int wpr = 1;
  while ((long)T * wpr < 2048 && (K / (wpr * 2)) % 256 == 0) wpr *= 2;
  const long warps = (long)T * wpr;
  mx_quant_rows_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>((const bf16*)x, T, K, wpr, qhi, qlo, exps,
                                                                   skip_ids, k);
  mx_expand_kernel<<<(unsigned)((cap + 7) / 8), 256, 0, s>>>(qhi, qlo, exps, perm, n_rows, K, offsets, tstart, count,
                                                             BN, hi, lo, sf_hi, sf_lo, MX_CHUNK, merged ? BN : 0);
  return (int)cudaGetLastError();
}

int moe_mx_gemm(const uint8_t* hi, const uint8_t* lo, const uint8_t* sf_hi, const uint8_t* sf_lo, int cap,
                const uint8_t* wq, const uint8_t* sfa, int n_rows, int K, const int* offsets, const int* counts,
                const int* tstart, int count, int BN, int act, void* out, int out_cols, int* err, cudaStream_t s,
                bool tiled) {
  if (!cap || !count) return 0;
  if (n_rows % 128 || K % MX_SK || count > MX_MAX_EXPERTS) return -1;
  if ((reinterpret_cast<uintptr_t>(wq) & 31) || (reinterpret_cast<uintptr_t>(hi) & 15) ||
      (reinterpret_cast<uintptr_t>(lo) & 15))
    return -2;
  CUtensorMap tw, th, tl;
  // row-major codes [count * n_rows][K/2 bytes], or tiled: [count * n_rows * K/128][64 bytes]
  const bool wide = mx_merged(tiled, BN);
  if (wide && (lo <= hi || ((lo - hi) & 15))) return -3;
  // two 128-K atoms per stage for token tiles of at most 32 rows (wide path, an even number of
  // atoms): measured 7 % faster at 32 tokens, 3 % at 800; at 2048 tokens (64-row tiles) the
  // pipeline is short of bytes in flight, not of issue slots, and the longer stages lose 4 %.
  // QB_MX_K2=0 / 1 forces one or two atoms per stage.
  static const int k2_env = getenv("QB_MX_K2") ? atoi(getenv("QB_MX_K2")) : -1;
  const bool k2 = k2_env < 0 ? BN <= 32 : k2_env != 0;
  const int ka = (wide && k2 && (K / MX_SK) % 2 == 0) ? 2 : 1;
  int r = tiled ? mx_tmap(&tw, wq, (long)count * n_rows * (K / MX_SK), MX_SK, MX_SK / 2, wide ? 128 * ka : 64, true)
                : mx_tmap(&tw, wq, (long)count * n_rows, K, K / 2, 64, true);
  if (r) return 1000 + r;
  r = wide ? mx_tmap_planes(&th, hi, cap, K, lo - hi, BN) : mx_tmap(&th, hi, cap, K, K, 16, false);
  if (r) return 2000 + r;
  r = mx_tmap(&tl, lo, cap, K, K, 16, false);
  if (r) return 3000 + r;
  MxPlanes pl{};
  for (int i = 0; wide && i < BN / 16; ++i) {
    r = mx_tmap_planes(&pl.m[i], hi, cap, K, lo - hi, 16 * (i + 1));
    if (r) return 4000 + r;
  }
  static const int probe = getenv("QB_MX_PROBE") ? atoi(getenv("QB_MX_PROBE")) : 0;
  MxArgs a{sfa, sf_hi, sf_lo, offsets, counts, tstart, out, out_cols, n_rows, K, count, act, err, tiled ? 1 : 0,
           wide ? 1 : 0, probe};
  switch (BN) {
    case 16: return !wide ? mx_launch<16, false>(tw, th, tl, pl, a, s)
                 : ka == 2 ? mx_launch<16, true, 2>(tw, th, tl, pl, a, s) : mx_launch<16, true>(tw, th, tl, pl, a, s);
    case 32: return !wide ? mx_launch<32, false>(tw, th, tl, pl, a, s)
                 : ka == 2 ? mx_launch<32, true, 2>(tw, th, tl, pl, a, s) : mx_launch<32, true>(tw, th, tl, pl, a, s);
    case 64: return !wide ? mx_launch<64, false>(tw, th, tl, pl, a, s)
                 : ka == 2 ? mx_launch<64, true, 2>(tw, th, tl, pl, a, s) : mx_launch<64, true>(tw, th, tl, pl, a, s);
    default: return mx_launch<128, false>(tw, th, tl, pl, a, s);
  }
}

}  // namespace qb
