// Routed experts: dispatch metadata, token gather, grouped expert GEMMs on tcgen05 with the
// MXFP4 weights decoded inside shared memory, and the weighted combine.
//
// MXFP4 -> tensor core: the packed e2m1 codes (two per byte, low nibble = even K) are brought
// into shared memory by TMA exactly as stored (no dequantised weight ever touches HBM). Four
// converter warps turn each 64-wide K slice of the 128-row weight tile into f16 with the
// sm_100a hardware conversion `cvt.rn.f16x2.e2m1x2`, multiply by the block's e8m0 scale
// (a power of two, exact in f16), and store it in the 128-byte-swizzled K-major layout the MMA
// reads. Activations are gathered once per layer into an f16 copy (bf16 -> f16 is exact for
// the normalised activations), so every product equals the bf16 reference product
// `x_bf16 * dequant(w)`: `kind::f16` needs both operands in the same type.
//
// Warp roles (320 threads, one persistent CTA per SM):
//   warp 0      TMA producer (raw fp4 tile, f16 token tile; e8m0 scales by bulk copy per unit)
//   warp 1      TMEM allocator + MMA issuer
//   warps 2..5  epilogue (silu(gate)*up for the gate_up GEMM, plain for down)
//   warps 6..13 fp4 -> f16 converters (two threads per weight row, one 32-element block each)
// Work unit = (local expert, 128-row weight tile); each unit loops over its expert's token
// tiles. For the gate_up GEMM a weight tile is 64 gate rows + the matching 64 up rows, so the
// epilogue sees both halves of silu(g)*u in one accumulator.
#include "common.cuh"
#include "kernels.h"
#include "numerics.cuh"

#include <cstdlib>
#include <type_traits>

namespace qb {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------ dispatch metadata
// Counting sort of the (token, slot) assignments that hit local experts [first, first+count).
__global__ void moe_dispatch_kernel(const int* topi, int T, int k, int first, int count, int* counts, int* offsets,
                                    int* perm_tok, int* perm_slot, int* inv, int* n_assign, int tile, int* tstart) {
  extern __shared__ int sh[];  // count counters + count cursors
  int* cnt = sh;
  int* cur = sh + count;
  for (int e = threadIdx.x; e < count; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int n = T * k;
  for (int a = threadIdx.x; a < n; a += blockDim.x) {
    const int e = topi[a] - first;
    if (e >= 0 && e < count) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // exclusive prefix over experts (token rows, and token tiles of `tile` rows): block-wide scan,
  // one expert per thread per round of blockDim.x experts
  __shared__ int warp_tot[2][32];
  __shared__ int carry[2];
  if (threadIdx.x == 0) carry[0] = carry[1] = 0;
  const int lane = threadIdx.x % 32, wid = threadIdx.x / 32, nw = blockDim.x / 32;
  for (int base = 0; base < count; base += blockDim.x) {
    __syncthreads();
    const int e = base + threadIdx.x;
    const int c = e < count ? cnt[e] : 0;
    const int t = (e < count && tstart) ? (c + tile - 1) / tile : 0;
    int ic = c, itl = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int vc = __shfl_up_sync(0xffffffff, ic, o), vt = __shfl_up_sync(0xffffffff, itl, o);
      if (lane >= o) {
        ic += vc;
        itl += vt;
      }
    }
    if (lane == 31) {
      warp_tot[0][wid] = ic;
      warp_tot[1][wid] = itl;
    }
    __syncthreads();
    if (wid == 0) {
      int wc = lane < nw ? warp_tot[0][lane] : 0, wt = lane < nw ? warp_tot[1][lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int vc = __shfl_up_sync(0xffffffff, wc, o), vt = __shfl_up_sync(0xffffffff, wt, o);
        if (lane >= o) {
          wc += vc;
          wt += vt;
        }
      }
      if (lane < nw) {  // exclusive warp offsets
        warp_tot[0][lane] = wc - warp_tot[0][lane];
        warp_tot[1][lane] = wt - warp_tot[1][lane];
      }
    }
    __syncthreads();
    const int ex_c = carry[0] + warp_tot[0][wid] + ic - c, ex_t = carry[1] + warp_tot[1][wid] + itl - t;
    if (e < count) {
      cur[e] = ex_c;
      offsets[e] = ex_c;
      counts[e] = c;
      if (tstart) tstart[e] = ex_t;
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) {  // running totals for the next round of experts
      carry[0] = ex_c + c;
      carry[1] = ex_t + t;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *n_assign = carry[0];
    if (tstart) tstart[count] = carry[1];
  }
  __syncthreads();
  for (int a = threadIdx.x; a < n; a += blockDim.x) {
    const int e = topi[a] - first;
    if (e >= 0 && e < count) {
      const int p = atomicAdd(&cur[e], 1);
      perm_tok[p] = a / k;
      perm_slot[p] = a % k;
      inv[a] = p;
    } else {
      inv[a] = -1;
    }
  }
}

int moe_dispatch(const int* topi, int T, int k, int first, int count, int* counts, int* offsets, int* perm_tok,
                 int* perm_slot, int* inv, int* n_assign, cudaStream_t s, int tile, int* tstart) {
  moe_dispatch_kernel<<<1, 1024, 2 * count * sizeof(int), s>>>(topi, T, k, first, count, counts, offsets, perm_tok,
                                                                perm_slot, inv, n_assign, tile, tstart);
  return (int)cudaGetLastError();
}

// xh[a, :] = h[perm_tok[a], :] (bf16 -> f16, or bf16 copy when OUT_BF16)
template <bool OUT_BF16>
__global__ void moe_gather_kernel(const bf16* h, const int* perm_tok, const int* n_assign, int H, void* xh) {
  const int a = blockIdx.x;
  if (a >= *n_assign) return;
  const bf16* src = h + (long)perm_tok[a] * H;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(src + i);
    if (OUT_BF16) {
      *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(xh) + (long)a * H + i) = raw;
    } else {
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
      uint4 o;
      __half* oe = reinterpret_cast<__half*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) oe[j] = __float2half_rn(__bfloat162float(e[j]));
      *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(xh) + (long)a * H + i) = o;
    }
  }
}

int moe_gather_f16(const void* h, const int* perm_tok, const int* n_assign, int cap, int H, void* xh,
                   cudaStream_t s) {
  if (!cap) return 0;
  moe_gather_kernel<false><<<cap, 128, 0, s>>>((const bf16*)h, perm_tok, n_assign, H, xh);
  return (int)cudaGetLastError();
}

int moe_gather_bf16(const void* h, const int* perm_tok, const int* n_assign, int cap, int H, void* xh,
                    cudaStream_t s) {
  if (!cap) return 0;
  moe_gather_kernel<true><<<cap, 128, 0, s>>>((const bf16*)h, perm_tok, n_assign, H, xh);
  return (int)cudaGetLastError();
}

// out[t, :] = sum_j topw[t, j] * y2[inv[t, j], :] over local assignments (fp32, rounded once)
// shared (optional): the shared expert's output rows and their gate logits (gl, ldgl apart): the
// row becomes bf16(routed) + bf16(bf16(sigmoid(gate)) * shared), the same bits as
// shared_gate_combine after the routed sum, without the extra pass over the rows.
__global__ void moe_combine_kernel(const bf16* y2, const int* inv, const float* topw, int k, int H, bf16* out,
                                   bool skip_empty, const bf16* shared, const bf16* gl, long ldgl) {
  const long t = blockIdx.x;
  if (skip_empty) {  // rows no expert of this rank serves are left unwritten (nobody reads them)
    bool any = false;
    for (int j = 0; j < k; ++j) any |= inv[t * k + j] >= 0;
    if (!any) return;
  }
  // blockIdx.y splits the row so that small batches still spread over the SMs
  const int per = (H + gridDim.y - 1) / gridDim.y;
  const int i0 = blockIdx.y * per, i1 = min(H, i0 + per);
  for (int i = i0 + threadIdx.x * 8; i < i1; i += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < k; ++j) {
      const int a = inv[t * k + j];
      if (a < 0) continue;
      const float w = topw[t * k + j];
      const uint4 raw = *reinterpret_cast<const uint4*>(y2 + (long)a * H + i);
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] += w * __bfloat162float(e[u]);
    }
    uint4 o;
    bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
    for (int u = 0; u < 8; ++u) oe[u] = __float2bfloat16(acc[u]);
    if (shared != nullptr) {
      const float g = __bfloat162float(gl[t * ldgl]);
      const float sg = __bfloat162float(__float2bfloat16(1.f / (1.f + expf(-g))));
      const uint4 sr = *reinterpret_cast<const uint4*>(shared + t * H + i);
      const bf16* se = reinterpret_cast<const bf16*>(&sr);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float sh = __bfloat162float(__float2bfloat16(sg * __bfloat162float(se[u])));
        oe[u] = __float2bfloat16(__bfloat162float(oe[u]) + sh);
      }
    }
    *reinterpret_cast<uint4*>(out + t * H + i) = o;
  }
}

int moe_combine(const void* y2, const int* inv, const float* topw, int T, int k, int H, void* out, cudaStream_t s,
                bool skip_empty, const void* shared, const void* gl, long ldgl) {
  if (!T) return 0;
  int split = 1;  // row chunks of at least 1024 columns (multiples of 8) until ~2 blocks per SM
  while (T * split < 296 && H / (split * 2) >= 1024 && (H / (split * 2)) % 8 == 0) split *= 2;
  moe_combine_kernel<<<dim3(T, split), 128, 0, s>>>((const bf16*)y2, inv, topw, k, H, (bf16*)out, skip_empty,
                                                     (const bf16*)shared, (const bf16*)gl, ldgl);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ grouped expert GEMM
constexpr int MOE_THREADS = 448;
constexpr int MBK = 64;

template <int BN, bool FP4>
struct MoeCfg {
  static constexpr int RAW = FP4 ? 128 * MBK / 2 : 0;   // packed fp4 codes of the A tile
  static constexpr int A = 128 * MBK * 2;                // f16/bf16 A tile (converted or TMA)
  static constexpr int B = BN * MBK * 2;
  static constexpr int STAGE = A + B + RAW;              // A first: keeps 1024-byte alignment
  static constexpr int SCALE_MAX = 128 * 128;            // 128 rows x (K/32 <= 128) bytes
  static constexpr int STAGING = 32 * 128 * 2;
  static constexpr int BUDGET = 210 * 1024 - STAGING - (FP4 ? 2 * SCALE_MAX : 0);
  static constexpr int STAGES = BUDGET / STAGE > 10 ? 10 : BUDGET / STAGE;
  static constexpr int TMEM_COLS = (2 * BN) < 32 ? 32 : 2 * BN;
  static constexpr int SMEM = 1024 + STAGES * STAGE + STAGING + (FP4 ? 2 * SCALE_MAX : 0) + 512;
};

struct MoeArgs {
  const uint8_t* scales;  // [E_local * n_rows, K/32] (FP4 only)
  const int* offsets;
  const int* counts;
  void* out;
  int out_cols;
  int n_rows;  // weight rows per expert (2I for gate_up, H for down)
  int K;
  int count;   // local experts
  int act;
  int* err;
};

// Two e2m1 codes (one byte) -> f16x2; the low nibble becomes the low half.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{\n .reg .b8 b;\n cvt.u8.u32 b, %1;\n cvt.rn.f16x2.e2m1x2 %0, b;\n}" : "=r"(r) : "r"(byte));
  return r;
}

template <int BN, bool FP4>
__global__ void __launch_bounds__(MOE_THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, MoeArgs a,
                    uint32_t idesc) {
  using C = MoeCfg<BN, FP4>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint16_t* staging = reinterpret_cast<uint16_t*>(smem + C::STAGES * C::STAGE);
  uint8_t* sbuf = smem + C::STAGES * C::STAGE + C::STAGING;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbuf + (FP4 ? 2 * C::SCALE_MAX : 0));
  uint64_t* full = bars;
  uint64_t* conv = full + C::STAGES;
  uint64_t* empty = conv + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* sc_full = acc_empty + 2;
  uint64_t* sc_empty = sc_full + 2;
  uint64_t* drain = sc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_p = const_cast<int*>(abort_flag) + 1;
  int* consumed_p = issued_p + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_tiles = a.n_rows / 128;
  const int units = a.count * n_tiles;
  const int kblocks = a.K / MBK;
  const int srow = a.K / 32;  // scale bytes per weight row
  const bool gu = a.act == 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 256);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
      mbar_init(&sc_full[i], 1);
      mbar_init(&sc_empty[i], 256);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *issued_p = 0;
    *consumed_p = 0;
    fence_barrier_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // weight row (within the expert) of A-tile row r for tile nt
  auto wrow = [&](int nt, int r) -> int {
    return gu ? (r < 64 ? nt * 64 + r : a.n_rows / 2 + nt * 64 + (r - 64)) : nt * 128 + r;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one()) {
      int it = 0, ui = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const int e = u / n_tiles, nt = u % n_tiles;
        const int cnt = a.counts[e];
        if (cnt == 0) continue;
        const int off = a.offsets[e];
        const long erow = (long)e * a.n_rows;
        if (FP4) {
          const int sb = ui & 1;
          if (!mbar_wait(&sc_empty[sb], ((ui >> 1) & 1) ^ 1, a.err, ERR_TMA_WAIT, abort_flag)) break;
          uint8_t* dst = sbuf + sb * C::SCALE_MAX;
          const uint32_t half = 64 * srow;
          mbar_expect_tx(&sc_full[sb], 2 * half);
          const uint8_t* s0 = a.scales + (erow + wrow(nt, 0)) * srow;
          const uint8_t* s1 = a.scales + (erow + wrow(nt, 64)) * srow;
          asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                           smem_u32(dst)),
                       "l"(s0), "r"(half), "r"(smem_u32(&sc_full[sb]))
                       : "memory");
          asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                           smem_u32(dst + half)),
                       "l"(s1), "r"(half), "r"(smem_u32(&sc_full[sb]))
                       : "memory");
        }
        ++ui;
        for (int m0 = 0; m0 < cnt; m0 += BN) {
          for (int kb = 0; kb < kblocks; ++kb, ++it) {
            const int s = it % C::STAGES;
            if (!mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1, a.err, ERR_TMA_WAIT, abort_flag)) goto prod_done;
            uint8_t* st = stages + s * C::STAGE;
            if (FP4) {
              mbar_expect_tx(&full[s], C::RAW + C::B);
              tma_load_2d(st + C::A + C::B, &tmW, &full[s], kb * MBK / 2, (int)(erow + wrow(nt, 0)));
              tma_load_2d(st + C::A + C::B + C::RAW / 2, &tmW, &full[s], kb * MBK / 2, (int)(erow + wrow(nt, 64)));
            } else {
              mbar_expect_tx(&full[s], C::A + C::B);
              tma_load_2d(st, &tmW, &full[s], kb * MBK, (int)(erow + wrow(nt, 0)));
              tma_load_2d(st + C::A / 2, &tmW, &full[s], kb * MBK, (int)(erow + wrow(nt, 64)));
            }
            tma_load_2d(st + C::A, &tmX, &full[s], kb * MBK, off + m0);
            *issued_p = it + 1;
          }
        }
      }
    prod_done:;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      int it = 0, ti = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok && !*abort_flag; u += gridDim.x) {
        const int e = u / n_tiles;
        const int cnt = a.counts[e];
        for (int m0 = 0; m0 < cnt && ok; m0 += BN, ++ti) {
          const int acc = ti & 1;
          if (!mbar_wait(&acc_empty[acc], ((ti >> 1) & 1) ^ 1, a.err, ERR_ACC_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + acc * BN;
          for (int kb = 0; kb < kblocks; ++kb, ++it) {
            const int s = it % C::STAGES;
            uint64_t* ready = FP4 ? &conv[s] : &full[s];
            if (!mbar_wait(ready, (it / C::STAGES) & 1, a.err, ERR_MMA_WAIT, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(stages + s * C::STAGE);
            const uint64_t da = desc_sw128(sa), db = desc_sw128(sa + C::A);
#pragma unroll
            for (int kk = 0; kk < MBK / 16; ++kk) mma_f16_ss(d, da + 2 * kk, db + 2 * kk, idesc, (kb | kk) != 0);
            mma_commit(&empty[s]);
            *consumed_p = it + 1;
          }
          if (!ok) break;
          mma_commit(&acc_full[acc]);
        }
      }
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_DRAIN, nullptr);
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- epilogue
    const int ew = warp & 3;
    const int row = ew * 32 + lane;
    const int et = threadIdx.x - 64;
    int ti = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int e = u / n_tiles, nt = u % n_tiles;
      const int cnt = a.counts[e];
      const int off = a.offsets[e];
      bool stop = false;
      for (int m0 = 0; m0 < cnt; m0 += BN, ++ti) {
        const int acc = ti & 1;
        if (!mbar_wait(&acc_full[acc], (ti >> 1) & 1, a.err, ERR_EPI_WAIT, abort_flag)) {
          stop = true;
          break;
        }
        tc_fence_after();
        constexpr int CH = BN < 32 ? BN : 32;
        for (int c0 = 0; c0 < BN; c0 += CH) {
          float v[32];
          const uint32_t taddr = tmem + acc * BN + c0 + ((uint32_t)(ew * 32) << 16);
          if constexpr (CH == 32) tmem_ld32(taddr, v); else tmem_ld16(taddr, v);
          // staging holds the fp32 accumulator rounded to bf16 (the reference rounding point)
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            bf16 o = __float2bfloat16(v[j]);
            staging[j * 128 + row] = *reinterpret_cast<uint16_t*>(&o);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          const int nvalid = min(CH, cnt - m0 - c0);
          if (gu) {
            // the intermediate feeds the down GEMM: f16 for the fp4 path, bf16 for bf16 experts
            using IT = typename std::conditional<FP4, __half, bf16>::type;
            IT* Y = reinterpret_cast<IT*>(a.out);
            for (int idx = et; idx < CH * 64; idx += 128) {
              const int j = idx / 64, r = idx % 64;
              if (j < nvalid) {
                uint16_t gb = staging[j * 128 + r], ub = staging[j * 128 + 64 + r];
                const float g = __bfloat162float(*reinterpret_cast<bf16*>(&gb));
                const float uu = __bfloat162float(*reinterpret_cast<bf16*>(&ub));
                const float sg = __bfloat162float(__float2bfloat16(g / (1.f + expf(-g))));
                const float y = __bfloat162float(__float2bfloat16(sg * uu));
                Y[(long)(off + m0 + c0 + j) * a.out_cols + nt * 64 + r] = from_f<IT>(y);
              }
            }
          } else {
            bf16* Y = reinterpret_cast<bf16*>(a.out);
            for (int idx = et; idx < CH * 16; idx += 128) {
              const int j = idx / 16, q = idx % 16;
              if (j < nvalid) {
                const uint4 val = *reinterpret_cast<const uint4*>(&staging[j * 128 + q * 8]);
                *reinterpret_cast<uint4*>(Y + (long)(off + m0 + c0 + j) * a.out_cols + nt * 128 + q * 8) = val;
              }
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
      }
      if (stop) break;
    }
  } else if (FP4) {
    // ---------------------------------------------------------------- fp4 -> f16 converters
    const int ct = threadIdx.x - 192;  // 0..255
    const int r = ct & 127;            // weight-tile row
    const int blk = ct >> 7;           // which 32-element scale block of the 64-wide K slice
    int it = 0, ui = 0;
    bool stop = false;
    for (int u = blockIdx.x; u < units && !stop; u += gridDim.x) {
      const int e = u / n_tiles;
      const int cnt = a.counts[e];
      if (cnt == 0) continue;
      const int sb = ui & 1;
      if (!mbar_wait(&sc_full[sb], (ui >> 1) & 1, a.err, ERR_MMA_WAIT, abort_flag)) break;
      const uint8_t* srw = sbuf + sb * C::SCALE_MAX + r * srow;
      for (int m0 = 0; m0 < cnt && !stop; m0 += BN) {
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(&full[s], (it / C::STAGES) & 1, a.err, ERR_MMA_WAIT, abort_flag)) {
            stop = true;
            break;
          }
          uint8_t* st = stages + s * C::STAGE;
          // 32 codes of this thread's block: 16 bytes
          const uint4 c = *reinterpret_cast<const uint4*>(st + C::A + C::B + r * (MBK / 2) + blk * 16);
          const uint32_t words[4] = {c.x, c.y, c.z, c.w};
          const int sexp = (int)srw[kb * 2 + blk] - 127;
          // f16 bit pattern of 2**sexp (normal range [-14, 15], subnormal down to -24)
          const bool in_range = sexp >= -24 && sexp <= 15;
          const uint16_t sbits = sexp >= -14 ? (uint16_t)((sexp + 15) << 10) : (uint16_t)(1u << (sexp + 24));
          __half2 sc2;
          {
            const uint32_t sw = (uint32_t)sbits | ((uint32_t)sbits << 16);
            sc2 = *reinterpret_cast<const __half2*>(&sw);
          }
          const float scf = exp2f((float)sexp);
          uint8_t* arow = st + r * 128;  // SW128 row r: 16-byte chunk j stored at j ^ (r & 7)
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // chunk = 8 codes = 8 f16
            uint32_t outw[4];
#pragma unroll
            for (int b2 = 0; b2 < 4; ++b2) {
              uint32_t h2 = e2m1x2_to_f16x2((words[q] >> (8 * b2)) & 0xff);
              __half2 v = *reinterpret_cast<__half2*>(&h2);
              if (in_range) {
                v = __hmul2(v, sc2);
              } else {
                const float2 f = __half22float2(v);
                v = __floats2half2_rn(f.x * scf, f.y * scf);
              }
              outw[b2] = *reinterpret_cast<uint32_t*>(&v);
            }
            const int chunk = blk * 4 + q;
            *reinterpret_cast<uint4*>(arow + ((chunk ^ (r & 7)) * 16)) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
          }
          // make the generic-proxy shared-memory writes visible to the tensor core (async proxy)
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(&conv[s]);
        }
      }
      mbar_arrive(&sc_empty[sb]);
      ++ui;
    }
  }

  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    for (int it = *consumed_p; it < *issued_p; ++it)
      mbar_wait(&full[it % C::STAGES], (it / C::STAGES) & 1, a.err, ERR_DRAIN, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}


// ------------------------------------------------------------------ grouped MXFP4 GEMM, A in TMEM
// Same work decomposition as moe_gemm_kernel, but the converted f16 weight tile is written to
// tensor memory (tcgen05.st) and the MMA reads its A operand from there. Shared memory only
// carries the packed fp4 codes and the token tiles. One pipeline stage covers 256 K elements:
// the fp4 tile arrives as 128 rows x 128 bytes (128-byte swizzled, so the per-row reads of the
// converters are bank-conflict free) and the token tile as four 64-wide swizzle atoms.
//   warp 0       TMA producer (codes, token tile; e8m0 scales by bulk copy per tile)
//   warp 1       TMEM allocator
//   warps 2..5   epilogue
//   warps 6..21  four converter groups of four warps (warp w covers TMEM lane quarter w % 4).
//                Group g decodes sub-block g of every stage and one of its threads issues that
//                sub-block's MMAs into the group's own accumulator, so MMA issue is spread over
//                four threads that already run at the converters' pace (a single issuer thread
//                sharing its scheduler with four ALU-bound converter warps fell behind), and the
//                four accumulators form independent chains. The epilogue adds them.
constexpr int MT_THREADS = 704;
constexpr int MT_NA = 8;          // A ring depth in TMEM (32 columns = 64 K elements each)
constexpr int MT_ABASE = 256;     // first TMEM column of the A ring; accumulators below it
constexpr int MT_SK = 256;        // K elements per stage
constexpr int MT_MAX_EXPERTS = 1024;  // local experts per launch (tile prefix lives in shared memory)

// Columns (tokens) of one tile: the rest of the expert's tokens, rounded up to 16, at most BN.
template <int BN>
__device__ __forceinline__ int tile_cols(int rest) {
  const int n = (rest + 15) & ~15;
  return n < BN ? n : BN;
}

template <int BN>
struct MoeTmCfg {
  static constexpr int ACC_COLS = 4 * BN;                        // one tile: 4 group accumulators
  static constexpr int NBUF = MT_ABASE / ACC_COLS >= 2 ? 2 : 1;  // tile buffers below the A ring
  static constexpr int B_ATOM = BN * 64 * 2;   // one 64-wide swizzled token tile
  static constexpr int B = 4 * B_ATOM;
  static constexpr int RAW = 128 * MT_SK / 2;   // 16 KB of packed codes
  static constexpr int STAGE = B + RAW;         // multiple of 1024
  static constexpr int SCALE_MAX = 128 * 128;
  static constexpr int STAGING = BN * 128 * 2;  // one whole output tile (bf16)
  static constexpr int PREFIX = 4 * (MT_MAX_EXPERTS + 1);
  static constexpr int BUDGET = 212 * 1024 - STAGING - 2 * SCALE_MAX - PREFIX;
  static constexpr int STAGES = BUDGET / STAGE > 12 ? 12 : BUDGET / STAGE;
  static constexpr int SMEM = 1024 + STAGES * STAGE + STAGING + 2 * SCALE_MAX + 1024 + PREFIX;
};

template <int BN>
__global__ void __launch_bounds__(MT_THREADS, 1)
    moe_fp4_tmem_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, MoeArgs a,
                        uint32_t idesc) {
  using C = MoeTmCfg<BN>;
  static_assert(C::STAGE % 1024 == 0, "stage must keep the token tiles 1024-byte aligned");
  static_assert(C::NBUF * C::ACC_COLS <= MT_ABASE, "accumulators overlap the A ring");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint16_t* staging = reinterpret_cast<uint16_t*>(smem + C::STAGES * C::STAGE);
  uint8_t* sbuf = smem + C::STAGES * C::STAGE + C::STAGING;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbuf + 2 * C::SCALE_MAX);
  uint64_t* full = bars;
  uint64_t* empty = full + C::STAGES;
  uint64_t* a_full = empty + C::STAGES;
  uint64_t* a_empty = a_full + MT_NA;
  uint64_t* acc_full = a_empty + MT_NA;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* sc_full = acc_empty + 2;
  uint64_t* sc_empty = sc_full + 2;
  uint64_t* drain = sc_empty + 2;  // [4], one per issuing group
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_p = const_cast<int*>(abort_flag) + 1;
  int* tstart = reinterpret_cast<int*>(sbuf + 2 * C::SCALE_MAX + 1024);  // [count + 1]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_tiles = a.n_rows / 128;
  const int ksub = a.K / MBK;                        // 64-wide sub-blocks in K
  const int kstages = (a.K + MT_SK - 1) / MT_SK;     // stages per tile
  const int srow = a.K / 32;
  const bool gu = a.act == 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);  // one commit (or plain arrive) per converter group
    }
    for (int i = 0; i < MT_NA; ++i) {
      mbar_init(&a_full[i], 128);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 4);
      mbar_init(&acc_empty[i], 128);
      mbar_init(&sc_full[i], 1);
      mbar_init(&sc_empty[i], 512);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&drain[i], 1);
    *abort_flag = 0;
    *issued_p = 0;
    fence_barrier_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 2) {
    // exclusive prefix of token tiles per expert: tstart[e] = sum over e' < e of ceil(counts[e'] / BN)
    int run = 0;
    for (int base = 0; base < a.count; base += 32) {
      const int e = base + lane;
      const int t = e < a.count ? (a.counts[e] + BN - 1) / BN : 0;
      int incl = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffff, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < a.count) tstart[e] = run + incl - t;
      run += __shfl_sync(0xffffffff, incl, 31);
    }
    if (lane == 0) tstart[a.count] = run;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Work unit = (token tile, 128-row weight tile), weight tile fastest: one hot expert's token
  // tiles spread over many CTAs, and CTAs working on one token tile run side by side (the tile
  // stays in L2).
  const int units = tstart[a.count] * n_tiles;
  auto unit = [&](int u, int& e, int& nt, int& m0) {
    const int tt = u / n_tiles;
    nt = u % n_tiles;
    int lo = 0, hi = a.count - 1;  // last expert whose first tile is <= tt (empty experts share starts)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tstart[mid] <= tt) lo = mid; else hi = mid - 1;
    }
    e = lo;
    m0 = (tt - tstart[e]) * BN;
  };
  auto wrow = [&](int nt, int r) -> int {
    return gu ? (r < 64 ? nt * 64 + r : a.n_rows / 2 + nt * 64 + (r - 64)) : nt * 128 + r;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one()) {
      int it = 0, ui = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int e, nt, m0;
        unit(u, e, nt, m0);
        const int cnt = a.counts[e];
        const int off = a.offsets[e];
        const long erow = (long)e * a.n_rows;
        const int sb = ui & 1;
        if (!mbar_wait(&sc_empty[sb], ((ui >> 1) & 1) ^ 1, a.err, ERR_TMA_WAIT, abort_flag)) break;
        uint8_t* dst = sbuf + sb * C::SCALE_MAX;
        const uint32_t half = 64 * srow;
        mbar_expect_tx(&sc_full[sb], 2 * half);
        const uint8_t* s0 = a.scales + (erow + wrow(nt, 0)) * srow;
        const uint8_t* s1 = a.scales + (erow + wrow(nt, 64)) * srow;
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_u32(dst)),
                     "l"(s0), "r"(half), "r"(smem_u32(&sc_full[sb]))
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_u32(dst + half)),
                     "l"(s1), "r"(half), "r"(smem_u32(&sc_full[sb]))
                     : "memory");
        ++ui;
        const int ne = tile_cols<BN>(cnt - m0);
        for (int ks = 0; ks < kstages; ++ks, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1, a.err, ERR_TMA_WAIT, abort_flag)) goto prod_done;
          uint8_t* st = stages + s * C::STAGE;
          mbar_expect_tx(&full[s], 4 * ne * 128 + C::RAW);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            for (int t = 0; t < ne; t += 16)
              tma_load_2d(st + j * C::B_ATOM + t * 128, &tmX, &full[s], ks * MT_SK + j * 64, off + m0 + t);
          tma_load_2d(st + C::B, &tmW, &full[s], ks * MT_SK / 2, (int)(erow + wrow(nt, 0)));
          tma_load_2d(st + C::B + C::RAW / 2, &tmW, &full[s], ks * MT_SK / 2, (int)(erow + wrow(nt, 64)));
          *issued_p = it + 1;
        }
      }
    prod_done:;
    }
  } else if (warp >= 2 && warp < 6) {
    // ---------------------------------------------------------------- epilogue
    const int ew = warp & 3;
    const int row = ew * 32 + lane;
    const int et = threadIdx.x - 64;
    const int nacc = ksub < 4 ? ksub : 4;  // group accumulators written (group g owns sub-blocks g mod 4)
    int ti = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++ti) {
      int e, nt, m0;
      unit(u, e, nt, m0);
      const int cnt = a.counts[e];
      const int off = a.offsets[e];
      const int ab = ti % C::NBUF;
      if (!mbar_wait(&acc_full[ab], (ti / C::NBUF) & 1, a.err, ERR_EPI_WAIT, abort_flag)) break;
      tc_fence_after();
      const int ne = tile_cols<BN>(cnt - m0);
      // TMEM -> registers (sum of the group accumulators) -> bf16 staging; then free the buffer
      for (int c0 = 0; c0 < ne; c0 += 16) {
        float v[16];
        const uint32_t taddr = tmem + ab * C::ACC_COLS + c0 + ((uint32_t)(ew * 32) << 16);
        tmem_ld16(taddr, v);
        for (int g = 1; g < nacc; ++g) {
          float w[16];
          tmem_ld16(taddr + g * BN, w);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += w[j];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          bf16 o = __float2bfloat16(v[j]);
          staging[(c0 + j) * 128 + row] = *reinterpret_cast<uint16_t*>(&o);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int nvalid = min(ne, cnt - m0);
      if (gu) {
        __half* Y = reinterpret_cast<__half*>(a.out);
        for (int idx = et; idx < nvalid * 64; idx += 128) {
          const int j = idx / 64, r = idx % 64;
          uint16_t gb = staging[j * 128 + r], ub = staging[j * 128 + 64 + r];
          const float g = __bfloat162float(*reinterpret_cast<bf16*>(&gb));
          const float uu = __bfloat162float(*reinterpret_cast<bf16*>(&ub));
          const float sg = __bfloat162float(__float2bfloat16(g / (1.f + expf(-g))));
          const float y = __bfloat162float(__float2bfloat16(sg * uu));
          Y[(long)(off + m0 + j) * a.out_cols + nt * 64 + r] = __float2half_rn(y);
        }
      } else {
        bf16* Y = reinterpret_cast<bf16*>(a.out);
        for (int idx = et; idx < nvalid * 16; idx += 128) {
          const int j = idx / 16, q = idx % 16;
          const uint4 val = *reinterpret_cast<const uint4*>(&staging[j * 128 + q * 8]);
          *reinterpret_cast<uint4*>(Y + (long)(off + m0 + j) * a.out_cols + nt * 128 + q * 8) = val;
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------------- converters + MMA issue
    const int cw = warp - 6;   // 0..15
    const int grp = cw >> 2;   // sub-block of every stage this group decodes
    const int q = warp & 3;    // TMEM lane quarter
    const int r = q * 32 + lane;
    // the issuing warp of the group (one per SMSP); it waits as a whole warp so that it stays
    // converged for the warp-collective tcgen05.st, and its lane 0 issues the MMAs and commits
    const bool iwarp = q == grp;
    int it = 0, ui = 0, sit0 = 0, ti = 0;
    bool stop = false;
    for (int u = blockIdx.x; u < units && !stop; u += gridDim.x, ++ti) {
      int e, nt, m0;
      unit(u, e, nt, m0);
      const int ab = ti % C::NBUF;
      const uint32_t dacc = tmem + ab * C::ACC_COLS + grp * BN;
      const uint32_t id_t = (idesc & ~(0x3Fu << 17)) | ((uint32_t)(tile_cols<BN>(a.counts[e] - m0) >> 3) << 17);
      const int sb = ui & 1;
      if (!mbar_wait(&sc_full[sb], (ui >> 1) & 1, a.err, ERR_MMA_WAIT, abort_flag)) break;
      const uint8_t* srw = sbuf + sb * C::SCALE_MAX + r * srow;
      // the group's last stage with a sub-block in this tile (its acc_full commit follows it)
      const int last_ks = grp < ksub ? (ksub - 1 - grp) / 4 : -1;
      if (iwarp) {
        // the tile buffer must be free of the epilogue before the group's first MMA into it
        if (!mbar_wait(&acc_empty[ab], ((ti / C::NBUF) & 1) ^ 1, a.err, ERR_ACC_WAIT, abort_flag)) stop = true;
        tc_fence_after();
        if (last_ks < 0 && !stop && lane == 0) mbar_arrive(&acc_full[ab]);  // nothing to add for this group
        __syncwarp();
      }
      uint4 scw = make_uint4(0, 0, 0, 0);  // this row's scale bytes of two stages (16-byte rows only)
      for (int ks = 0; ks < kstages && !stop; ++ks, ++it) {
        const int nsub = min(4, ksub - ks * 4);
        const int sit = sit0 + grp;
        sit0 += nsub;
        const int s = it % C::STAGES;
        if (!mbar_wait(&full[s], (it / C::STAGES) & 1, a.err, ERR_MMA_WAIT, abort_flag)) {
          stop = true;
          break;
        }
        if (grp >= nsub) {  // no sub-block for this group in this stage
          if (iwarp && lane == 0) mbar_arrive(&empty[s]);
          continue;
        }
        const int ai = sit % MT_NA;
        if (!mbar_wait(&a_empty[ai], ((sit / MT_NA) & 1) ^ 1, a.err, ERR_MMA_WAIT, abort_flag)) {
          stop = true;
          break;
        }
        const int kb = ks * 4 + grp;  // 64-wide K sub-block index
        // the fp4 tile is 128-byte swizzled: 16-byte chunk c of row r sits at chunk c ^ (r & 7)
        const uint8_t* rrow = stages + s * C::STAGE + C::B + r * (MT_SK / 2);
        const uint4 c0 = *reinterpret_cast<const uint4*>(rrow + (((2 * grp) ^ (r & 7)) << 4));
        const uint4 c1 = *reinterpret_cast<const uint4*>(rrow + (((2 * grp + 1) ^ (r & 7)) << 4));
        const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        uint32_t sc16;  // the two block exponents of this sub-block, low byte first
        if (srow % 16 == 0) {
          if ((ks & 1) == 0) scw = *reinterpret_cast<const uint4*>(srw + ks * 8);
          const uint32_t wsel = (ks & 1) ? ((grp & 2) ? scw.w : scw.z) : ((grp & 2) ? scw.y : scw.x);
          sc16 = (wsel >> ((grp & 1) * 16)) & 0xffff;
        } else {
          sc16 = srw[kb * 2] | ((uint32_t)srw[kb * 2 + 1] << 8);
        }
        uint32_t outw[32];
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          const int sexp = (int)((sc16 >> (8 * blk)) & 0xff) - 127;
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) e2m1x8_placed(words[blk * 4 + w4], outw + blk * 16 + w4 * 4);
          if (sexp >= -23 && sexp <= 1) {  // 2^(14 + sexp) is a normal f16 and every product is exact
            const uint32_t sb16 = (uint32_t)(sexp + 29) << 10;
            const uint32_t sw = sb16 | (sb16 << 16);
            const __half2 sc2 = *reinterpret_cast<const __half2*>(&sw);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              __half2 v = __hmul2(*reinterpret_cast<const __half2*>(&outw[blk * 16 + j]), sc2);
              outw[blk * 16 + j] = *reinterpret_cast<uint32_t*>(&v);
            }
          } else {  // large or tiny scales: scale in fp32, round once to f16
            const float scf = exp2f((float)(sexp + 14));
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&outw[blk * 16 + j]));
              __half2 v = __floats2half2_rn(f.x * scf, f.y * scf);
              outw[blk * 16 + j] = *reinterpret_cast<uint32_t*>(&v);
            }
          }
        }
        tmem_st32(tmem + MT_ABASE + ai * 32 + ((uint32_t)(q * 32) << 16), outw);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&a_full[ai]);
        if (iwarp) {
          // all four warps of the group have stored their lane quarters of this sub-block
          if (!mbar_wait(&a_full[ai], (sit / MT_NA) & 1, a.err, ERR_MMA_WAIT, abort_flag)) {
            stop = true;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint64_t db = desc_sw128(smem_u32(stages + s * C::STAGE + grp * C::B_ATOM));
            const uint32_t at = tmem + MT_ABASE + ai * 32;
#pragma unroll
            for (int kk = 0; kk < MBK / 16; ++kk)
              mma_f16_ts(dacc, at + kk * 8, db + 2 * kk, id_t, (ks | kk) != 0);
            mma_commit(&a_empty[ai]);
            mma_commit(&empty[s]);
            if (ks == last_ks) mma_commit(&acc_full[ab]);
          }
          __syncwarp();
        }
      }
      mbar_arrive(&sc_empty[sb]);
      ++ui;
    }
    if (iwarp && lane == 0) {  // every MMA of this thread completes before TMEM is released
      mma_commit(&drain[grp]);
      mbar_wait(&drain[grp], 0, a.err, ERR_DRAIN, nullptr);
    }
  }

  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // TMA copies may still be in flight for the last issued stages: wait for each of them
    const int n = *issued_p;
    for (int i = n - C::STAGES < 0 ? 0 : n - C::STAGES; i < n; ++i)
      mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, a.err, ERR_DRAIN, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int BN>
static int moe_tm_launch(const CUtensorMap& tw, const CUtensorMap& tx, const MoeArgs& a, int max_ctas,
                         cudaStream_t st) {
  using C = MoeTmCfg<BN>;
  auto k = moe_fp4_tmem_kernel<BN>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr = true;
  }
  const int units = a.count * (a.n_rows / 128);
  int grid = units < max_ctas ? units : max_ctas;
  if (grid < 1) grid = 1;
  k<<<grid, MT_THREADS, C::SMEM, st>>>(tw, tx, a, idesc_f16(128, BN, false));
  return (int)cudaGetLastError();
}

static int moe_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool FP4>
static int moe_launch(const CUtensorMap& tw, const CUtensorMap& tx, const MoeArgs& a, int max_ctas,
                      cudaStream_t st) {
  using C = MoeCfg<BN, FP4>;
  auto k = moe_gemm_kernel<BN, FP4>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr = true;
  }
  const int units = a.count * (a.n_rows / 128);
  int grid = units < max_ctas ? units : max_ctas;
  if (grid < 1) grid = 1;
  k<<<grid, MOE_THREADS, C::SMEM, st>>>(tw, tx, a, idesc_f16(128, BN, !FP4));
  return (int)cudaGetLastError();
}

// Token-tile width: an expert with more tokens than one tile converts its weight tile once per
// tile, so size the tile for about twice the mean load (routing is uneven) rather than the mean.
static int pick_bn(int cap, int count) {
  const int avg = (cap + count - 1) / (count > 0 ? count : 1);
  const int want = 2 * avg + 2;
  return want <= 16 ? 16 : want <= 32 ? 32 : want <= 64 ? 64 : 128;
}

int moe_expert_gemm(const void* xin, int in_cols, const uint8_t* wq, const uint8_t* ws, int n_rows, int k_cols,
                    long w_expert_stride, long s_expert_stride, const int* offsets, const int* counts, int count,
                    int cap, int act, void* out, int out_cols, int* err, cudaStream_t s, int max_ctas) {
  if (!cap || !count) return 0;
  if (n_rows % 128 || k_cols % MBK || k_cols / 32 > 128) return -1;
  (void)w_expert_stride;
  (void)s_expert_stride;
  const int BN = pick_bn(cap, count);
  CUtensorMap tw, tx;
  MoeArgs a{ws, offsets, counts, out, out_cols, n_rows, k_cols, count, act, err};
  if (max_ctas <= 0) max_ctas = moe_sms();
  static const bool smem_a = getenv("QB_MOE_SMEM_A") && getenv("QB_MOE_SMEM_A")[0] == '1';
  int r;
  if (!smem_a) {
    if (count > MT_MAX_EXPERTS) return -2;
    static const int bn_max = getenv("QB_MOE_BN_MAX") ? atoi(getenv("QB_MOE_BN_MAX")) : 64;
    const int bn = BN > bn_max ? bn_max : BN;
    r = make_tmap_2d(&tw, wq, 1, (long)count * n_rows, k_cols / 2, k_cols / 2, 64, MT_SK / 2, true);
    if (r) return 1000 + r;
    r = make_tmap_2d(&tx, xin, 2, cap, k_cols, in_cols, 16, MBK, true);  // 16-token boxes
    if (r) return 2000 + r;
    switch (bn) {
      case 16: return moe_tm_launch<16>(tw, tx, a, max_ctas, s);
      case 32: return moe_tm_launch<32>(tw, tx, a, max_ctas, s);
      default: return moe_tm_launch<64>(tw, tx, a, max_ctas, s);
    }
  }
  r = make_tmap_2d(&tw, wq, 1, (long)count * n_rows, k_cols / 2, k_cols / 2, 64, MBK / 2, false);
  if (r) return 1000 + r;
  r = make_tmap_2d(&tx, xin, 2, cap, k_cols, in_cols, BN, MBK, true);
  if (r) return 2000 + r;
  {  // converted tile in shared memory (A/B comparison path)
    switch (BN) {
      case 16: return moe_launch<16, true>(tw, tx, a, max_ctas, s);
      case 32: return moe_launch<32, true>(tw, tx, a, max_ctas, s);
      case 64: return moe_launch<64, true>(tw, tx, a, max_ctas, s);
      default: return moe_launch<128, true>(tw, tx, a, max_ctas, s);
    }
  }
}

int moe_expert_gemm_bf16(const void* xin, int in_cols, const void* w, int n_rows, int k_cols, long w_expert_stride,
                         const int* offsets, const int* counts, int count, int cap, int act, void* out, int out_cols,
                         cudaStream_t s) {
  if (!cap || !count) return 0;
  if (n_rows % 128 || k_cols % MBK) return -1;
  (void)w_expert_stride;
  const int BN = pick_bn(cap, count);
  CUtensorMap tw, tx;
  int r = make_tmap_2d(&tw, w, 2, (long)count * n_rows, k_cols, k_cols, 64, MBK, true);
  if (r) return 1000 + r;
  r = make_tmap_2d(&tx, xin, 2, cap, k_cols, in_cols, BN, MBK, true);
  if (r) return 2000 + r;
  MoeArgs a{nullptr, offsets, counts, out, out_cols, n_rows, k_cols, count, act, nullptr};
  const int mc = moe_sms();
  switch (BN) {
    case 16: return moe_launch<16, false>(tw, tx, a, mc, s);
    case 32: return moe_launch<32, false>(tw, tx, a, mc, s);
    case 64: return moe_launch<64, false>(tw, tx, a, mc, s);
    default: return moe_launch<128, false>(tw, tx, a, mc, s);
  }
}

}  // namespace qb
