// Prefill flash attention on the 5th-generation tensor cores (causal, GQA, paged KV).
//
// CTA = (query tile, kv head). The 128 MMA rows are (128/G tokens) x (G query heads of the kv
// head), token-major, so every query head sharing a kv head reuses one K/V tile. Per 64-key tile:
//   S = Q K^T         tcgen05.mma kind::f16, M=128, N=64, K=head_dim; Q and K K-major (SW128)
//   softmax           4 warps, one row per thread: causal mask from the row's absolute position,
//                     online max/sum in the exp2 domain, P rounded to bf16 into shared memory,
//                     O rescaled in TMEM (tcgen05.ld / st) when the running max moves
//   O += P V          M=128, N=head_dim, K=64; V is the MN-major B operand straight from the cache
// S is double buffered in TMEM (cols 0..127) so the next QK^T overlaps this tile's softmax; O
// lives in TMEM (cols 256..256+head_dim). K and V pages (16 tokens) arrive by 3-D TMA boxes,
// two stages. Warp 0 = TMA producer, warp 1 = MMA issuer, warps 2..5 = softmax + epilogue.
// All waits are bounded (common.cuh).
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace qb {

using bf16 = __nv_bfloat16;

constexpr int FA_KT = 64;        // keys per tile
constexpr int FA_THREADS = 192;
constexpr int FA_S_COL = 0;      // S buffers: cols [0, 64) and [64, 128)
constexpr int FA_O_COL = 256;    // O accumulator
constexpr int FA_WS_HEAD = 4;    // partial record: max, sum, 2 pad words, then O (16-byte aligned)

// K-major SW128 descriptor is desc_sw128; MN-major SW128 needs explicit LBO (MN-atom stride) and
// SBO (8-row K-group stride).
__device__ __forceinline__ uint64_t desc_sw128_mn(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_st_col32(uint32_t taddr, const float* v) {
  uint32_t r[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
  tmem_st32(taddr, r);
}

template <int HD>
struct FaCfg {
  static constexpr int ATOMS = HD / 64;
  static constexpr int Q_BYTES = ATOMS * 128 * 128;      // 128 rows x HD bf16
  static constexpr int KV_ATOM = FA_KT * 128;            // 64 keys x 128 B
  static constexpr int K_BYTES = ATOMS * KV_ATOM;
  static constexpr int STAGE = 2 * K_BYTES;              // K then V
  static constexpr int P_BYTES = 128 * 128;              // 128 rows x 64 keys bf16
  static constexpr int SMEM = 1024 + Q_BYTES + 2 * STAGE + P_BYTES + 256;
};

struct FaArgs {
  const int* tiles;  // [n_tiles][3]: segment, first row, rows
  const int* pos;    // [T] absolute positions
  const int* seg_lane;
  const int* table;  // [lanes, max_blocks]
  int max_blocks;
  int G;             // query heads per kv head
  int QT;            // tokens per tile = 128 / G
  int nq;
  bf16* out;         // [T, nq, HD]
  float scale_log2;  // head_dim**-0.5 * log2(e)
  int* err;
  int splits;        // key-range splits per tile (grid z); > 1 writes partial results to ws
  float* ws;         // [T * nq][splits][4 + HD]: running max (log2 units), sum, 2 pad, unnormalised O
};

template <int HD>
__global__ void __launch_bounds__(FA_THREADS, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, FaArgs a) {
  using C = FaCfg<HD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* kv = qs + C::Q_BYTES;
  uint8_t* ps = kv + 2 * C::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ps + C::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;   // [2]
  uint64_t* kv_empty = kv_full + 2; // [2]
  uint64_t* s_full = kv_empty + 2;  // [2]
  uint64_t* s_free = s_full + 2;    // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tile = blockIdx.x, g = blockIdx.y;
  const int seg = a.tiles[tile * 3], row0 = a.tiles[tile * 3 + 1], nrows = a.tiles[tile * 3 + 2];
  const int lane_id = a.seg_lane[seg];
  const int last_pos = a.pos[row0 + nrows - 1];
  // key tiles [kt0, kt1) of this split (all tiles up to the tile's last position when unsplit)
  const int n_all = (last_pos + FA_KT) / FA_KT;
  int kt0 = 0, kt1 = n_all;
  if (a.splits > 1) {
    const int per = (n_all + a.splits - 1) / a.splits;
    kt0 = blockIdx.z * per;
    kt1 = min(n_all, kt0 + per);
    if (kt0 >= kt1) {  // nothing to read: an empty partial (the combine skips it)
      if (threadIdx.x < 128 && threadIdx.x / a.G < nrows) {
        const int r = threadIdx.x;
        float* w = a.ws + (((long)(row0 + r / a.G) * a.nq + (long)g * a.G + r % a.G) * a.splits + blockIdx.z) * (HD + FA_WS_HEAD);
        w[0] = -INFINITY;
        w[1] = 0.f;
      }
      return;
    }
  }
  const int n_kt = kt1 - kt0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (elect_one()) {
      mbar_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int j = 0; j < C::ATOMS; ++j) tma_load_3d(qs + j * 16384, &tmQ, q_full, 64 * j, g * a.G, row0);
      const int* tab = a.table + (long)lane_id * a.max_blocks;
      for (int i = 0; i < n_kt && !*abort_flag; ++i) {
        const int st = i & 1;
        if (!mbar_wait(&kv_empty[st], ((i >> 1) & 1) ^ 1, a.err, ERR_TMA_WAIT, abort_flag)) break;
        uint8_t* kb = kv + st * C::STAGE;
        uint8_t* vb = kb + C::K_BYTES;
        mbar_expect_tx(&kv_full[st], C::STAGE);
#pragma unroll
        for (int p = 0; p < FA_KT / 16; ++p) {
          const int blk = ((kt0 + i) * FA_KT) / 16 + p;
          const int page = blk < a.max_blocks ? tab[blk] : 0;
#pragma unroll
          for (int j = 0; j < C::ATOMS; ++j) {
            tma_load_3d(kb + j * C::KV_ATOM + p * 2048, &tmK, &kv_full[st], 64 * j, g, page * 16);
            tma_load_3d(vb + j * C::KV_ATOM + p * 2048, &tmV, &kv_full[st], 64 * j, g, page * 16);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      const uint32_t idesc_s = idesc_f16(128, FA_KT, true);
      const uint32_t idesc_o = idesc_f16(128, HD, true) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, a.err, ERR_MMA_WAIT, abort_flag);
      const uint32_t qa = smem_u32(qs);
      auto pv = [&](int t) -> bool {
        // O += P V for tile t (P written by the softmax warps for tile t)
        if (!mbar_wait(p_full, t & 1, a.err, ERR_MMA_WAIT, abort_flag)) return false;
        tc_fence_after();
        const uint32_t vb = smem_u32(kv + (t & 1) * C::STAGE + C::K_BYTES);
        const uint64_t dp = desc_sw128(smem_u32(ps));
#pragma unroll
        for (int kk = 0; kk < FA_KT / 16; ++kk)
          mma_f16_ss(tmem + FA_O_COL, dp + 2 * kk, desc_sw128_mn(vb + kk * 2048, C::KV_ATOM, 1024), idesc_o,
                     (t | kk) != 0);
        mma_commit(o_done);
        mma_commit(&kv_empty[t & 1]);
        return true;
      };
      for (int i = 0; i < n_kt && ok; ++i) {
        const int st = i & 1;
        if (!mbar_wait(&kv_full[st], (i >> 1) & 1, a.err, ERR_MMA_WAIT, abort_flag) ||
            !mbar_wait(&s_free[st], ((i >> 1) & 1) ^ 1, a.err, ERR_MMA_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kb = smem_u32(kv + st * C::STAGE);
#pragma unroll
        for (int j = 0; j < C::ATOMS; ++j)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ss(tmem + FA_S_COL + st * FA_KT, desc_sw128(qa + j * 16384) + 2 * kk,
                       desc_sw128(kb + j * C::KV_ATOM) + 2 * kk, idesc_s, (j | kk) != 0);
        mma_commit(&s_full[st]);
        if (i > 0 && !pv(i - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) pv(n_kt - 1);
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_DRAIN, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;          // tile row = (token r / G, head r % G)
    const int tok = r / a.G;
    const bool valid = tok < nrows;
    const int qpos = valid ? a.pos[row0 + tok] : -1;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    uint8_t* prow = ps + r * 128;
    for (int i = 0; i < n_kt && ok; ++i) {
      const int st = i & 1;
      if (!mbar_wait(&s_full[st], (i >> 1) & 1, a.err, ERR_EPI_WAIT, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[64];
      tmem_ld32(tmem + lane_off + FA_S_COL + st * FA_KT, sv);
      tmem_ld32(tmem + lane_off + FA_S_COL + st * FA_KT + 32, sv + 32);
      tc_fence_before();
      mbar_arrive(&s_free[st]);
      const int k0 = (kt0 + i) * FA_KT;
      float mx = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < 64; ++jj) {
        const bool keep = valid && (k0 + jj) <= qpos;
        sv[jj] = keep ? sv[jj] * a.scale_log2 : -INFINITY;
        mx = fmaxf(mx, sv[jj]);
      }
      const float m_new = fmaxf(m, mx);
      const float corr = (m == -INFINITY) ? (m_new == -INFINITY ? 1.f : 0.f) : exp2f(m - m_new);
      float sum = 0.f;
      uint32_t pw[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const float p0 = m_new == -INFINITY ? 0.f : exp2f(sv[2 * u] - m_new);
        const float p1 = m_new == -INFINITY ? 0.f : exp2f(sv[2 * u + 1] - m_new);
        const __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
        sum += __bfloat162float(pb.x) + __bfloat162float(pb.y);
        pw[u] = *reinterpret_cast<const uint32_t*>(&pb);
      }
      l = l * corr + sum;
      m = m_new;
      if (i > 0) {
        // P.V of tile i-1 must finish before P is overwritten and before O is rescaled
        if (!mbar_wait(o_done, (i - 1) & 1, a.err, ERR_EPI_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffff, corr != 1.f)) {  // tcgen05.ld/st are warp-collective
#pragma unroll 1
          for (int c0 = 0; c0 < HD; c0 += 32) {
            float ov[32];
            tmem_ld32(tmem + lane_off + FA_O_COL + c0, ov);
#pragma unroll
            for (int u = 0; u < 32; ++u) ov[u] *= corr;
            tmem_st_col32(tmem + lane_off + FA_O_COL + c0, ov);
          }
          tmem_wait_st();
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) * 16)) =
            make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(o_done, (n_kt - 1) & 1, a.err, ERR_EPI_WAIT, abort_flag)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const long orow = (long)(valid ? row0 + tok : 0) * a.nq + (long)g * a.G + (r % a.G);
      bf16* dst = a.out + orow * HD;
      float* wsr = a.splits > 1 ? a.ws + (orow * a.splits + blockIdx.z) * (HD + FA_WS_HEAD) : nullptr;
      if (wsr && valid) {
        wsr[0] = m;
        wsr[1] = l;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < HD; c0 += 32) {
        float ov[32];
        tmem_ld32(tmem + lane_off + FA_O_COL + c0, ov);  // every lane: the load is warp-collective
        if (wsr && valid) {
#pragma unroll
          for (int u = 0; u < 32; u += 4)
            *reinterpret_cast<float4*>(wsr + FA_WS_HEAD + c0 + u) = make_float4(ov[u], ov[u + 1], ov[u + 2], ov[u + 3]);
        } else if (valid) {
          uint32_t w[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const __nv_bfloat162 pb = __floats2bfloat162_rn(ov[2 * u] * inv, ov[2 * u + 1] * inv);
            w[u] = *reinterpret_cast<const uint32_t*>(&pb);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(dst + c0 + u * 8) = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
        }
      }
    }
  }

  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // drain stages whose TMA loads may still be in flight
    for (int i = 0; i < 2; ++i) mbar_wait(&kv_full[i], 0, a.err, ERR_DRAIN, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Merge the key-range partials of every (row, head): O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.
template <int HD>
__global__ void fa_combine_kernel(const float* ws, int splits, bf16* out) {
  const long th = blockIdx.x;  // row * nq + head
  const float* base = ws + th * splits * (HD + FA_WS_HEAD);
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, base[s * (HD + FA_WS_HEAD)]);
  float L = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float mm = base[s * (HD + FA_WS_HEAD)];
    if (mm > -INFINITY) L += exp2f(mm - M) * base[s * (HD + FA_WS_HEAD) + 1];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float mm = base[s * (HD + FA_WS_HEAD)];
      if (mm > -INFINITY) acc += exp2f(mm - M) * base[s * (HD + FA_WS_HEAD) + FA_WS_HEAD + d];
    }
    out[th * HD + d] = __float2bfloat16(acc * inv);
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 fa_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D bf16 tensor [d2][d1][d0] (d0 innermost), box (64, b1, b2), 128-byte swizzle.
static int tmap3(CUtensorMap* m, const void* base, long d0, long d1, long d2, int b1, int b2) {
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)(d0 * 2), (cuuint64_t)(d0 * d1 * 2)};
  cuuint32_t box[3] = {64, (cuuint32_t)b1, (cuuint32_t)b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fa_encode()(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

int fa_prefill(const void* q, const void* kc, const void* vc, long cache_rows, const int* table, int max_blocks,
               const int* pos, const int* seg_lane, const int* tiles, int n_tiles, int T, int nq, int nkv, int hd,
               int block_size, int splits, float* ws, void* out, int* err, cudaStream_t s) {
  const int G = nq / nkv;
  if (splits < 1 || (splits > 1 && !ws)) return -1;
  if (block_size != 16 || nq % nkv || 128 % G || (hd != 64 && hd != 128 && hd != 256)) return -1;
  if (!n_tiles) return 0;
  CUtensorMap tq, tk, tv;
  int r = tmap3(&tq, q, hd, nq, T, G, 128 / G);
  if (r) return 1000 + r;
  r = tmap3(&tk, kc, hd, nkv, cache_rows, 1, 16);
  if (r) return 2000 + r;
  r = tmap3(&tv, vc, hd, nkv, cache_rows, 1, 16);
  if (r) return 3000 + r;
  FaArgs a{tiles, pos, seg_lane, table, max_blocks, G, 128 / G, nq, (bf16*)out,
           (float)(1.4426950408889634 / sqrt((double)hd)), err, splits, ws};
  dim3 grid(n_tiles, nkv, splits);
#define QB_FA(H)                                                                                          \
  {                                                                                                       \
    static bool attr = false;                                                                             \
    if (!attr) {                                                                                          \
      cudaFuncSetAttribute(fa_prefill_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize, FaCfg<H>::SMEM); \
      attr = true;                                                                                        \
    }                                                                                                     \
    fa_prefill_kernel<H><<<grid, FA_THREADS, FaCfg<H>::SMEM, s>>>(tq, tk, tv, a);                          \
    if (splits > 1) fa_combine_kernel<H><<<(long)T * nq, 64, 0, s>>>(ws, splits, (bf16*)out);             \
  }
  if (hd == 256) QB_FA(256) else if (hd == 128) QB_FA(128) else QB_FA(64)
#undef QB_FA
  return (int)cudaGetLastError();
}

}  // namespace qb
