// Dense GEMM on the 5th-generation tensor cores: Y[T, N] = X[T, K] @ W[N, K]^T.
//
// Weight-stationary orientation ("swap AB"): the weight tile is the 128-row MMA A operand and
// the token tile is the N operand (16..256 wide). Decode batches (T <= 64) then use a narrow N
// instead of padding tokens to 128, and every weight byte is streamed exactly once per tile.
//
// One persistent CTA per SM, 6 warps:
//   warp 0      TMA producer: 128x64 weight tile + BNx64 token tile per stage (128B swizzle)
//   warp 1      TMEM allocator and MMA issuer (one elected lane, tcgen05.mma kind::f16)
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator, optional fused activation,
//               transpose through shared memory, 16-byte coalesced stores of Y rows
// The accumulator is double buffered in TMEM (2 x BN columns), so the epilogue of one tile
// overlaps the MMAs of the next. All waits are bounded (see common.cuh).
//
// Stream-K for decode shapes (token tile <= 64): when the output's 128-row tiles do not divide
// evenly over the CTAs (N = 4096 projections are 32 tiles, N = 20608 is 161), every CTA takes an
// equal contiguous share of the (tile, K-block) space instead of whole tiles. A CTA's first and
// last segment may cover part of a tile's K range: it writes that fp32 partial to its own
// workspace slot and bumps the tile's counter (one releasing thread after a barrier); the CTA
// that arrives last adds the tile's partials (a handful, loaded two at a time) and runs the
// normal epilogue, then re-arms the counter. Segments in between cover whole tiles and take the
// normal epilogue directly.
//
// GEMM -> reduce-scatter (``push``): for a row-parallel projection followed by the
// sequence-parallel all-reduce, the epilogue stores each output row straight into the symmetric
// region of the rank that owns the row (rows [o per, (o+1) per) belong to rank o), at row
// rank * per + (t - o per) of the owner's partial slot; the slot is (device epoch + 1) & 1, read
// at entry. The transfer over NVLink thus runs tile by tile under the MMAs of the next tiles,
// and the reduce kernel that follows (comm.cu) reads only local memory.
#include "common.cuh"
#include "kernels.h"
#include <cudaTypedefs.h>

#include <algorithm>

namespace qb {

constexpr int GEMM_THREADS = 192;

__device__ __forceinline__ int ld_acquire_sys_g(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
constexpr int BK = 64;  // K elements per stage (one 128-byte swizzle atom of 16-bit values)

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGING = 32 * 128 * 2;  // 32 token columns x 128 weight rows, 16-bit
  // at most 8 stages in 200 KB (more stages measured no faster on the decode shapes)
  static constexpr int STAGES = (200 * 1024 - STAGING) / STAGE > 8 ? 8 : (200 * 1024 - STAGING) / STAGE;
  static constexpr int TMEM_COLS = (2 * BN) < 32 ? 32 : 2 * BN;
  static constexpr int SMEM = 1024 + STAGES * STAGE + STAGING + 256;
  static_assert(SMEM <= 232448, "shared memory per block");
};

struct GemmArgs {
  void* y;
  long ldy;
  int T, N, K;
  int act;  // 0: none, 1: silu(g)*u over row pairs (g rows [0,64), u rows [64,128) of each tile)
  int* err;
  int bn;      // token columns per tile actually used (<= BN, a multiple of 16): prefill token
               // counts are split evenly over the tiles instead of filling all but the last
  int ctas;    // stream-K: CTAs sharing the (tile, K-block) space (0: whole tiles per CTA)
  float* ws;   // stream-K: [ctas][2][128][BN] fp32 partials (a CTA's first and last segment)
  int* cnt;    // stream-K: [tiles] arrival counters, zero between calls
  GemmPush push;  // push.world > 0: rows go to the owner ranks' slots instead of y
  GemmGather gather;  // the all-gather -> GEMM kernel only: owners of the token rows
};

// Token tile `tt` -> its rows [t0, tend). Plain GEMM: tiles of bn rows over [0, T). All-gather
// GEMM: ceil(per / bn) tiles per owner, so no tile spans two owners; a tile of an owner with fewer
// rows may be empty (tend <= t0: computed from whatever the area holds, never stored).
struct TokTiles {
  int bn, T, per, tpo;
  bool g;
  __device__ TokTiles(const GemmArgs& a, bool gather) : bn(a.bn), T(a.T), per(a.gather.per), g(gather) {
    tpo = g ? (per + bn - 1) / bn : 0;
  }
  __device__ int count(int world) const { return g ? world * tpo : (T + bn - 1) / bn; }
  __device__ void rows(int tt, int& t0, int& tend, int& owner) const {
    if (!g) {
      owner = -1;
      t0 = tt * bn;
      tend = min(T, t0 + bn);
      return;
    }
    owner = tt / tpo;
    t0 = owner * per + (tt % tpo) * bn;
    tend = min(min(T, (owner + 1) * per), t0 + bn);
  }
};

// The sequence of (tile, K-block range) segments one CTA works through, identical for its
// producer, MMA and epilogue roles.
struct SegIter {
  long pos, end;  // stream-K: position in the (tile, K-block) space
  int u, step;    // whole tiles: next tile, stride
  int tiles, kblocks;
  bool sk;
  __device__ SegIter(int cta, int ctas, int grid, int tiles_, int kblocks_)
      : tiles(tiles_), kblocks(kblocks_), sk(ctas > 0) {
    const long W = (long)tiles_ * kblocks_;
    pos = sk ? (long)cta * W / ctas : 0;
    end = sk ? (long)(cta + 1) * W / ctas : 0;
    u = cta;
    step = grid;
  }
  __device__ bool next(int& tile, int& k0, int& k1) {
    if (sk) {
      if (pos >= end) return false;
      tile = (int)(pos / kblocks);
      k0 = (int)(pos % kblocks);
      k1 = (int)min((long)kblocks, k0 + (end - pos));
      pos += k1 - k0;
      return true;
    }
    if (u >= tiles) return false;
    tile = u;
    k0 = 0;
    k1 = kblocks;
    u += step;
    return true;
  }
};

// Stream-K: the CTA whose share contains position p of the (tile, K-block) space of size W.
__device__ __forceinline__ int sk_owner(long p, long W, int ctas) { return (int)(((p + 1) * ctas - 1) / W); }

struct GatherMaps {
  CUtensorMap m[8];  // owner o's gather area: 3-D [slot][row][K] boxes of BK x bn x 1
};

template <int BN, typename OutT, bool G>
__device__ __forceinline__ void gemm_ws_body(const CUtensorMap* tmW, const CUtensorMap* tmX, const CUtensorMap* gmaps,
                                             const GemmArgs& a, uint32_t idesc) {
  using C = GemmCfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint16_t* staging = reinterpret_cast<uint16_t*>(smem + C::STAGES * C::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE + C::STAGING);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_p = const_cast<int*>(abort_flag) + 1;
  int* consumed_p = issued_p + 1;
  volatile int* last_p = consumed_p + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_tiles = (a.N + 127) / 128;
  const TokTiles tokt(a, G);
  const int t_tiles = tokt.count(a.gather.world);
  const int tiles = n_tiles * t_tiles;
  const int kblocks = (a.K + BK - 1) / BK;

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
    *consumed_p = 0;
    fence_barrier_init();
    prefetch_tmap(tmW);
    if constexpr (G) {
      for (int o = 0; o < a.gather.world; ++o) prefetch_tmap(gmaps + o);
    } else {
      prefetch_tmap(tmX);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one()) {
      // launched as a programmatic dependent, everything above overlapped the previous kernel;
      // its results (the activations) are read from here on, and every write of this grid (the
      // epilogue's, after the MMAs on these loads) comes later still
      pdl_wait();
      int it = 0;
      SegIter sg(blockIdx.x, a.ctas, gridDim.x, tiles, kblocks);
      int tile, k0, k1;
      // stage ring in 32-bit shared addresses; stage index and parity advanced, not divided
      const uint32_t st0 = smem_u32(stages), full0 = smem_u32(full), empty0 = smem_u32(empty);
      int s = 0;
      uint32_t ph = 1;  // a first-round stage waits on the parity that passes at once
      int e_src = 0, ready_mask = 0;
      if constexpr (G) {
        e_src = *reinterpret_cast<volatile const int*>(a.gather.epoch);
        ready_mask = 1 << a.gather.rank;  // own rows: written by the previous kernel on this stream
      }
      while (!*abort_flag && sg.next(tile, k0, k1)) {
        const int n0 = (tile / t_tiles) * 128;
        int t0, tend, owner;
        tokt.rows(tile % t_tiles, t0, tend, owner);
        if constexpr (G) {
          if (!((ready_mask >> owner) & 1)) {
            // owner's rows for this call are complete once its ready word reaches the epoch
            // (system-scope acquire); then order the async-proxy (TMA) reads after it
            const int* f = a.gather.ready[owner];
            const uint64_t w0 = globaltimer();
            bool got = true;
            while (ld_acquire_sys_g(f) < e_src) {
              if (globaltimer() - w0 > a.gather.timeout_ns) {
                atomicCAS(a.err, 0, ERR_PEER_WAIT);
                *abort_flag = 1;
                got = false;
                break;
              }
            }
            if (!got) break;
            asm volatile("fence.proxy.async.global;" ::: "memory");
            ready_mask |= 1 << owner;
          }
        }
        bool ok = true;
        for (int kx = k0 * BK; kx < k1 * BK; kx += BK, ++it) {
          if (!mbar_wait_s(empty0 + 8 * s, ph, a.err, ERR_TMA_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t st = st0 + s * C::STAGE, fb = full0 + 8 * s;
          mbar_expect_tx_s(fb, C::A_BYTES + a.bn * BK * 2);
          tma_load_2d_s(st, tmW, fb, kx, n0);
          if constexpr (G)
            tma_load_3d_s(st + C::A_BYTES, gmaps + owner, fb, kx, t0, e_src & 1);
          else
            tma_load_2d_s(st + C::A_BYTES, tmX, fb, kx, t0);
          *issued_p = it + 1;
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      int it = 0, ti = 0;
      SegIter sg(blockIdx.x, a.ctas, gridDim.x, tiles, kblocks);
      int tile, k0, k1;
      const uint32_t full0 = smem_u32(full), empty0 = smem_u32(empty), accf0 = smem_u32(acc_full),
                     acce0 = smem_u32(acc_empty);
      const uint64_t da0 = desc_sw128(smem_u32(stages)), db0 = desc_sw128(smem_u32(stages) + C::A_BYTES);
      int s = 0;
      uint32_t ph = 0;
      for (; !*abort_flag && sg.next(tile, k0, k1); ++ti) {
        const int acc = ti & 1;
        if (!mbar_wait_s(acce0 + 8 * acc, ((ti >> 1) & 1) ^ 1, a.err, ERR_ACC_WAIT, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        bool ok = true;
        for (int kb = k0; kb < k1; ++kb, ++it) {
          if (!mbar_wait_s(full0 + 8 * s, ph, a.err, ERR_MMA_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t so = (uint64_t)((s * C::STAGE) >> 4);  // descriptor address field: bytes / 16
          const uint64_t da = da0 + so, db = db0 + so;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // +32 bytes per 16-element K step inside the swizzle atom (>>4 in the descriptor)
            mma_f16_ss(d, da + 2 * kk, db + 2 * kk, idesc, (kb != k0) || kk != 0);
          }
          mma_commit_s(empty0 + 8 * s);
          *consumed_p = it + 1;
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_s(accf0 + 8 * acc);
      }
      // make sure no MMA is still writing TMEM when the CTA tears down
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_DRAIN, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (128 threads)
    const int ew = warp & 3;             // TMEM lane quarter this warp may access
    const int row = ew * 32 + lane;      // accumulator row = weight row within the tile
    const int et = threadIdx.x - 64;     // 0..127
    OutT* Y = reinterpret_cast<OutT*>(a.y);
    const bool push = a.push.world > 0;
    const long push_off = push ? (long)((*reinterpret_cast<volatile const int*>(a.push.epoch) + 1) & 1) *
                                     a.push.slot_stride : 0;
    constexpr int CH = BN < 32 ? BN : 32;
    // stage one chunk of CH token columns (fp32 values of this thread's weight row) and store it
    auto emit = [&](int n0, int t0, int tend, int c0, const float* v) {
#pragma unroll
      for (int j = 0; j < CH; ++j) {  // staging[j][row]: token column j, weight row `row`
        OutT o = from_f<OutT>(v[j]);
        staging[j * 128 + row] = *reinterpret_cast<uint16_t*>(&o);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (a.act == 1) {
        // silu(gate) * up: rows [0,64) are gate rows, [64,128) the matching up rows;
        // output columns are n0/2 .. n0/2 + 64
        for (int idx = et; idx < CH * 64; idx += 128) {
          const int j = idx / 64, r = idx % 64;
          const int t = t0 + c0 + j, n = n0 / 2 + r;
          if (t < tend && n < a.N / 2) {
            uint16_t gb = staging[j * 128 + r], ub = staging[j * 128 + 64 + r];
            float g = to_f<OutT>(*reinterpret_cast<OutT*>(&gb)), u = to_f<OutT>(*reinterpret_cast<OutT*>(&ub));
            Y[(long)t * a.ldy + n] = from_f<OutT>(silu(g) * u);
          }
        }
      } else {
        // 16-byte vectors: each token row of the chunk is 128 outputs = 16 vectors
        for (int idx = et; idx < CH * 16; idx += 128) {
          const int j = idx / 16, q = idx % 16;
          const int t = t0 + c0 + j, n = n0 + q * 8;
          if (t < tend) {
            const uint4 val = *reinterpret_cast<const uint4*>(&staging[j * 128 + q * 8]);
            OutT* dst;
            if (push) {
              const int o = t / a.push.per;
              dst = reinterpret_cast<OutT*>(a.push.base[o]) + push_off +
                    (long)(a.push.rank * a.push.per + t - o * a.push.per) * a.ldy + n;
            } else {
              dst = Y + (long)t * a.ldy + n;
            }
            if (n + 8 <= a.N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
              *reinterpret_cast<uint4*>(dst) = val;
            } else {
              const uint16_t* e = reinterpret_cast<const uint16_t*>(&val);
              for (int u = 0; u < 8 && n + u < a.N; ++u) reinterpret_cast<uint16_t*>(dst)[u] = e[u];
            }
          }
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    };
    int ti = 0;
    SegIter sg(blockIdx.x, a.ctas, gridDim.x, tiles, kblocks);
    const long W = (long)tiles * kblocks;
    const int first_tile = a.ctas ? (int)(sg.pos / kblocks) : -1;  // tile of this CTA's first segment
    int tile, k0, k1;
    for (; sg.next(tile, k0, k1); ++ti) {
      const int n0 = (tile / t_tiles) * 128;
      int t0, tend, owner;
      tokt.rows(tile % t_tiles, t0, tend, owner);
      const int acc = ti & 1;
      if (!mbar_wait(&acc_full[acc], (ti >> 1) & 1, a.err, ERR_EPI_WAIT, abort_flag)) break;
      tc_fence_after();
      if (k0 == 0 && k1 == kblocks) {  // a whole tile
        for (int c0 = 0; c0 < a.bn; c0 += CH) {
          float v[32];
          const uint32_t taddr = tmem + acc * BN + c0 + ((uint32_t)(ew * 32) << 16);
          if constexpr (CH == 32) tmem_ld32(taddr, v); else tmem_ld16(taddr, v);
          emit(n0, t0, tend, c0, v);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        continue;
      }
      // part of a tile's K range: fp32 partial -> this CTA's slot; the last arriver adds them up
      const int slot = tile == first_tile ? 0 : 1;
      float* part = a.ws + (((long)blockIdx.x * 2 + slot) * 128 + row) * BN;
      for (int c0 = 0; c0 < BN; c0 += CH) {
        float v[32];
        const uint32_t taddr = tmem + acc * BN + c0 + ((uint32_t)(ew * 32) << 16);
        if constexpr (CH == 32) tmem_ld32(taddr, v); else tmem_ld16(taddr, v);
#pragma unroll
        for (int j = 0; j < CH; j += 4)
          *reinterpret_cast<float4*>(part + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      const long p0 = (long)tile * kblocks;
      const int cf = sk_owner(p0, W, a.ctas), cl = sk_owner(p0 + kblocks - 1, W, a.ctas);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (et == 0) {
        // release this CTA's partial (ordered before by the barrier), count it, acquire the others
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        const bool last = atomicAdd(&a.cnt[tile], 1) == cl - cf;
        if (last) asm volatile("fence.acq_rel.gpu;" ::: "memory");
        *last_p = last;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (!*last_p) continue;
      for (int c0 = 0; c0 < BN; c0 += CH) {
        float v[32];
#pragma unroll
        for (int j = 0; j < CH; ++j) v[j] = 0.f;
        for (int c = cf; c <= cl; c += 2) {  // two partials' loads in flight together
          const int s0 = (int)(((long)c * W / a.ctas) / kblocks) == tile ? 0 : 1;
          const float* p0p = a.ws + (((long)c * 2 + s0) * 128 + row) * BN + c0;
          const bool two = c + 1 <= cl;
          const int s1 = two && (int)(((long)(c + 1) * W / a.ctas) / kblocks) == tile ? 0 : 1;
          const float* p1p = a.ws + (((long)(two ? c + 1 : c) * 2 + s1) * 128 + row) * BN + c0;
          float4 f0[CH / 4], f1[CH / 4];
#pragma unroll
          for (int j = 0; j < CH / 4; ++j) {
            f0[j] = __ldcg(reinterpret_cast<const float4*>(p0p) + j);
            f1[j] = two ? __ldcg(reinterpret_cast<const float4*>(p1p) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int j = 0; j < CH / 4; ++j) {
            v[4 * j] += f0[j].x + f1[j].x;
            v[4 * j + 1] += f0[j].y + f1[j].y;
            v[4 * j + 2] += f0[j].z + f1[j].z;
            v[4 * j + 3] += f0[j].w + f1[j].w;
          }
        }
        emit(n0, t0, tend, c0, v);
      }
      if (et == 0) a.cnt[tile] = 0;  // re-armed for the next call on this stream
    }
  }

  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // drain TMA loads issued but never consumed before the shared memory goes away
    for (int it = *consumed_p; it < *issued_p; ++it)
      mbar_wait(&full[it % C::STAGES], (it / C::STAGES) & 1, a.err, ERR_DRAIN, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int BN, typename OutT>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_ws_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, GemmArgs a,
                   uint32_t idesc) {
  gemm_ws_body<BN, OutT, false>(&tmW, &tmX, nullptr, a, idesc);
}

// all-gather -> GEMM: token tiles from the owners' gather areas (bf16)
template <int BN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_ag_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ GatherMaps gm, GemmArgs a,
                   uint32_t idesc) {
  gemm_ws_body<BN, __nv_bfloat16, true>(&tmW, nullptr, gm.m, a, idesc);
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D row-major [rows, cols] tensor of 16-bit (or 8-bit) elements, box [box_rows, box_cols].
int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, long rows, long cols, long ld_elems,
                 int box_rows, int box_cols, bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld_elems * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// QB_PDL (default 1): dense GEMMs are launched as programmatic dependents of the previous kernel.
static bool gemm_pdl() {
  static const int on = getenv("QB_PDL") ? atoi(getenv("QB_PDL")) : 1;
  return on != 0;
}

template <int BN, typename OutT>
static int launch_bn(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a, bool bf16, int max_ctas,
                     cudaStream_t st) {
  using C = GemmCfg<BN>;
  auto k = gemm_ws_kernel<BN, OutT>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr = true;
  }
  const int tiles = ((a.N + 127) / 128) * ((a.T + a.bn - 1) / a.bn);
  int grid = a.ctas ? a.ctas : tiles < max_ctas ? tiles : max_ctas;
  if (grid < 1) grid = 1;
  const uint32_t idesc = idesc_f16(128, a.bn, bf16);
  if (gemm_pdl()) {  // programmatic dependent: the prologue overlaps the previous kernel's tail
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, k, tw, tx, a, idesc);
  } else {
    k<<<grid, GEMM_THREADS, C::SMEM, st>>>(tw, tx, a, idesc);
  }
  return (int)cudaGetLastError();
}

static int gemm_bn(int T) { return T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256; }

// Stream-K CTAs for a GEMM (0: whole tiles per CTA). Decode shapes only (token tile <= 64): they
// stream weights and their 128 x BN fp32 partials are small next to the weights, while a prefill
// GEMM is compute bound with wide partials. Each CTA keeps at least 8 K-blocks so that its
// pipeline fills. Chosen when the longest CTA's K-blocks, plus the partial write and fixup
// (measured at about 15 % plus 8 K-blocks), beat whole tiles: N = 4096 (32 tiles) and N = 20608
// (161 tiles, a ragged second wave) split; 136 tiles on 148 SMs stay whole.
int gemm_streamk_ctas(int T, int N, int K) {
  const int BN = gemm_bn(T);
  const long tiles = (long)((N + 127) / 128) * ((T + BN - 1) / BN);
  const long kblocks = (K + BK - 1) / BK;
  const int sms = num_sms();
  if (BN > 64 || kblocks < 16 || tiles % sms == 0) return 0;
  const long ctas = std::min<long>(sms, tiles * kblocks / 8);
  const double whole = (double)((tiles + sms - 1) / sms) * kblocks;
  const double split = (double)tiles * kblocks / ctas * 1.15 + 8.0;
  return split < whole ? (int)ctas : 0;
}

// Token-tile width (a multiple of 16, at most 256) for more than 128 tokens. The tokens split
// evenly over tt tiles; every (weight tile, token tile) pair is one work tile of the persistent
// grid, so a step costs about waves(tt) x (bn + c0) token columns, c0 being a tile's fixed cost
// (pipeline fill, epilogue), about 32 columns at K = 4096 and relatively more for shorter K.
// Narrower tiles pay when the weight tiles alone leave the last wave ragged: 21 weight tiles x 8
// tiles of 256 tokens = 168 tiles on 148 SMs run as two full-length waves, 21 x 13 tiles of 160
// as two waves of shorter tiles. The cheapest width is taken only when the model has it 10 %
// under the widest one: measured, 2048 tokens x 2576 x 4096 went 52.4 -> 45.8 us (160 wide), but
// 800 x 20608 x 4096 lost 8 % at 160 wide for a modelled 4 % gain (with many waves the ragged last
// one matters less than the narrower MMAs). QB_GEMM_BN_FIT=0: the widest width only (the tokens
// split evenly over ceil(T / 256) tiles).
int gemm_token_tile(int T, int N, int K) {
  const int tt0 = (T + 255) / 256;
  const int widest = ((T + tt0 - 1) / tt0 + 15) / 16 * 16;
  static const int fit = getenv("QB_GEMM_BN_FIT") ? atoi(getenv("QB_GEMM_BN_FIT")) : 1;
  if (!fit) return widest;
  const int sms = num_sms();
  const long wt = (N + 127) / 128;
  const double c0 = 32.0 * 4096.0 / (K > 128 ? K : 128);
  int best = widest;
  double best_cost = 1e300, widest_cost = 0.0;
  for (int tt = tt0;; ++tt) {
    const int bn = ((T + tt - 1) / tt + 15) / 16 * 16;
    const long tiles = wt * tt;
    const double cost = (double)((tiles + sms - 1) / sms) * (bn + c0);
    if (tt == tt0) widest_cost = cost;
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
    if (bn <= 64) break;
  }
  return best_cost < 0.9 * widest_cost ? best : widest;
}

long gemm_split_ws_floats(int T, int N, int K) {
  const int c = gemm_streamk_ctas(T, N, K);
  return c ? (long)c * 2 * 128 * gemm_bn(T) : 0;
}

int gemm_ws(const void* x, long ldx, const void* w, long ldw, void* y, long ldy, int T, int N, int K, bool bf16,
            int act, int* err, cudaStream_t stream, int max_ctas, float* ws, int* cnt, const GemmPush* push) {
  if (T <= 0 || N <= 0) return 0;
  if (push && (act || push->world < 1 || push->world > 8 || push->per < 1 || ldy != N)) return -1;
  int BN = gemm_bn(T);
  // the widest tile: the tokens split evenly over its tile count (800 -> 4 x 208, not 3 x 256 + 32)
  int bn = BN;
  if (BN == 256) bn = gemm_token_tile(T, N, K);
  CUtensorMap tw, tx;
  int r = make_tmap_2d(&tw, w, 2, N, K, ldw, 128, BK, true);
  if (r) return 1000 + r;
  r = make_tmap_2d(&tx, x, 2, T, K, ldx, bn, BK, true);
  if (r) return 2000 + r;
  const int ctas = (ws && cnt) ? gemm_streamk_ctas(T, N, K) : 0;
  GemmArgs a{y, ldy, T, N, K, act, err, bn, ctas, ws, cnt, push ? *push : GemmPush{}};
  if (max_ctas <= 0) max_ctas = num_sms();
  switch (BN) {
    case 16: return bf16 ? launch_bn<16, __nv_bfloat16>(tw, tx, a, bf16, max_ctas, stream)
                         : launch_bn<16, __half>(tw, tx, a, bf16, max_ctas, stream);
    case 32: return bf16 ? launch_bn<32, __nv_bfloat16>(tw, tx, a, bf16, max_ctas, stream)
                         : launch_bn<32, __half>(tw, tx, a, bf16, max_ctas, stream);
    case 64: return bf16 ? launch_bn<64, __nv_bfloat16>(tw, tx, a, bf16, max_ctas, stream)
                         : launch_bn<64, __half>(tw, tx, a, bf16, max_ctas, stream);
    case 128: return bf16 ? launch_bn<128, __nv_bfloat16>(tw, tx, a, bf16, max_ctas, stream)
                          : launch_bn<128, __half>(tw, tx, a, bf16, max_ctas, stream);
    default: return bf16 ? launch_bn<256, __nv_bfloat16>(tw, tx, a, bf16, max_ctas, stream)
                         : launch_bn<256, __half>(tw, tx, a, bf16, max_ctas, stream);
  }
}

// 3-D [2 slots][rows][K] view of one owner's gather area (16-bit elements), box [1][bn][BK]
static int make_tmap_gather(CUtensorMap* map, const void* base, long rows, long K, long ld_elems, long slot_elems,
                            int bn) {
  auto fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, 2};
  cuuint64_t strides[2] = {(cuuint64_t)(ld_elems * 2), (cuuint64_t)(slot_elems * 2)};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)bn, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

template <int BN>
static int launch_ag(const CUtensorMap& tw, const GatherMaps& gm, const GemmArgs& a, cudaStream_t st) {
  using C = GemmCfg<BN>;
  auto k = gemm_ag_kernel<BN>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr = true;
  }
  const int tpo = (a.gather.per + a.bn - 1) / a.bn;
  const int tiles = ((a.N + 127) / 128) * a.gather.world * tpo;
  const int grid = std::max(1, std::min(tiles, num_sms()));
  k<<<grid, GEMM_THREADS, C::SMEM, st>>>(tw, gm, a, idesc_f16(128, a.bn, true));
  return (int)cudaGetLastError();
}

int gemm_ag(const void* const* src, long src_ld, long slot_stride, const void* w, long ldw, void* y, long ldy, int T,
            int N, int K, const GemmGather& g, int* err, cudaStream_t stream) {
  if (T <= 0 || N <= 0) return 0;
  if (g.world < 1 || g.world > 8 || g.rank < 0 || g.rank >= g.world || g.per < 1 || (long)g.per * g.world < T ||
      K % BK)
    return -1;
  // token tiles per owner: its `per` rows split evenly (as the plain GEMM splits T)
  const int BN = gemm_bn(g.per);
  int bn = BN;
  if (BN == 256) {
    const int tt = (g.per + 255) / 256;
    bn = ((g.per + tt - 1) / tt + 15) / 16 * 16;
  }
  CUtensorMap tw;
  int r = make_tmap_2d(&tw, w, 2, N, K, ldw, 128, BK, true);
  if (r) return 1000 + r;
  GatherMaps gm{};
  for (int o = 0; o < g.world; ++o) {
    r = make_tmap_gather(&gm.m[o], src[o], (long)g.per * g.world, K, src_ld, slot_stride, bn);
    if (r) return 2000 + r;
  }
  GemmArgs a{y, ldy, T, N, K, 0, err, bn, 0, nullptr, nullptr, GemmPush{}, g};
  switch (BN) {
    case 16: return launch_ag<16>(tw, gm, a, stream);
    case 32: return launch_ag<32>(tw, gm, a, stream);
    case 64: return launch_ag<64>(tw, gm, a, stream);
    case 128: return launch_ag<128>(tw, gm, a, stream);
    default: return launch_ag<256>(tw, gm, a, stream);
  }
}

}  // namespace qb
