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
constexpr float FA_RESCALE_LOG2 = 8.f;  // running-max slack before O is rescaled (log2 units)

// 2^x by the hardware's approximate base-2 exponential (MUFU; relative error ~2^-22, far below
// the bf16 rounding P gets next); -inf gives 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

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

// 64 consecutive fp32 columns of this warp's 32 TMEM lanes, one load and one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
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
      tmem_ld64(tmem + lane_off + FA_S_COL + st * FA_KT, sv);
      tc_fence_before();
      mbar_arrive(&s_free[st]);
      const int k0 = (kt0 + i) * FA_KT;
      // keys past the row's position (the diagonal tiles) and rows past the tile are masked; the
      // softmax scale is applied inside the exponent (one FFMA per score)
      if (!valid || k0 + FA_KT - 1 > qpos) {
#pragma unroll
        for (int jj = 0; jj < 64; ++jj)
          if (k0 + jj > qpos) sv[jj] = -INFINITY;  // qpos = -1 on invalid rows masks every key
      }
      // row max as eight independent chains (one dependent chain of 64 would expose its latency:
      // a softmax warp is alone on its sub-partition)
      float mx8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx8[u] = sv[u];
#pragma unroll
      for (int jj = 8; jj < 64; ++jj) mx8[jj & 7] = fmaxf(mx8[jj & 7], sv[jj]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * a.scale_log2;
      // lazy rescale: the running max m moves only when a tile's max passes it by more than
      // FA_RESCALE_LOG2, so O is rescaled in TMEM rarely; in between, p = 2^(s - m) <= 2^8, which
      // fp32 and bf16 hold with full relative precision, and O and l stay relative to the same m
      const float m_new = (mx > m + FA_RESCALE_LOG2) ? mx : m;
      const float corr = (m_new == m) ? 1.f : (m == -INFINITY ? 0.f : ex2_approx(m - m_new));
      const float nm = m_new == -INFINITY ? 0.f : -m_new;  // every score is -inf while m_new is
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pw[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const float p0 = ex2_approx(fmaf(sv[2 * u], a.scale_log2, nm));
        const float p1 = ex2_approx(fmaf(sv[2 * u + 1], a.scale_log2, nm));
        const __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
        s4[u & 3] += __bfloat162float(pb.x) + __bfloat162float(pb.y);
        pw[u] = *reinterpret_cast<const uint32_t*>(&pb);
      }
      const float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
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
