// Fused all-reduce + residual add + RMSNorm over NVLink peer memory (one-shot), and the
// symmetric-buffer plumbing it needs (IPC export/import of one cudaMalloc'd region per rank).
//
// Every rank owns a symmetric region: two data slots of [max_rows, H] bf16 (double buffering
// across consecutive calls) and two flag arrays of [max_blocks] int. A call with epoch e uses
// slot s = e & 1. Block b of every rank
//   1. copies its row chunk of the local partial sum into its own slot s,
//   2. publishes flag[s][b] = e with a system-scope release,
//   3. waits (bounded) until every peer's flag[s][b] == e (system-scope acquire, peer loads; one
//      thread per peer, so the remote round trips overlap),
//   4. sums the W partial rows in rank order (fp32, so every rank gets identical bits), rounds
//      to bf16, adds the residual, writes the new residual and its RMSNorm.
// A rank reaching call e+2 overwrites slot s only after it saw every peer's flag for e+1, and a
// peer's kernel for e+1 starts only after its kernel for e finished: no peer still reads slot s.
// The epoch lives in device memory (read by every block at entry, advanced by the last block to
// finish), so the kernel can be captured in a CUDA graph and replayed.
// Waits are bounded by `timeout_ns` (%globaltimer); on expiry the kernel records ERR_PEER_WAIT in
// the status word, skips the reduction and returns. Reference counterpart: the one-shot IPC
// all-reduce family of allreduce_custom.py (its watchdog traps; this one never does).
#include "common.cuh"
#include "kernels.h"

namespace qb {

using bf16 = __nv_bfloat16;

struct SymmPtrs {
  void* data[8];   // per-rank region bases (peer-mapped; own entry is local)
  int world;
  int rank;
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int AR_THREADS = 256;

__global__ void __launch_bounds__(AR_THREADS) ar_add_rmsnorm_kernel(
    SymmPtrs ptrs, const bf16* partial, long ldp, bf16* res, const float* w1p, bf16* out, int rows, int H,
    float eps, long slot_elems, int max_blocks, int* epoch, int* done, int* err, unsigned long long timeout_ns) {
  pdl_launch_dependents();  // the next projection (launched as a dependent) may start its prologue
  __shared__ float red[32];
  __shared__ int s_epoch;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile int*>(epoch) + 1;
  __syncthreads();
  const int e = s_epoch;
  const int slot = e & 1;
  const int W = ptrs.world, me = ptrs.rank;
  auto flags_of = [&](int r) -> int* {
    return reinterpret_cast<int*>(reinterpret_cast<bf16*>(ptrs.data[r]) + 2 * slot_elems) + slot * max_blocks;
  };
  bf16* mine = reinterpret_cast<bf16*>(ptrs.data[me]) + slot * slot_elems;
  const int b = blockIdx.x;
  // 1. stage this block's rows of the local partial
  for (int r = b; r < rows; r += gridDim.x)
    for (int i = threadIdx.x * 8; i < H; i += AR_THREADS * 8)
      *reinterpret_cast<uint4*>(mine + (long)r * H + i) = *reinterpret_cast<const uint4*>(partial + (long)r * ldp + i);
  __syncthreads();
  // 2. publish
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(flags_of(me) + b, e);
  }
  // 3. wait for every peer's chunk (bounded); thread p polls peer p, so the W - 1 remote
  //    round trips overlap instead of following one another
  int ok = 1;
  if (threadIdx.x < W && threadIdx.x != me) {
    const int* f = flags_of(threadIdx.x) + b;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(f) < e) {
      if (globaltimer() - t0 > timeout_ns) {
        atomicCAS(err, 0, ERR_PEER_WAIT);
        ok = 0;
        break;
      }
    }
  }
  if (__syncthreads_and(ok)) {
    // 4. reduce in rank order, add residual, RMSNorm
    for (int r = b; r < rows; r += gridDim.x) {
      float acc[16];
      float ss = 0.f;
      const int nper = (H + AR_THREADS * 8 - 1) / (AR_THREADS * 8);  // chunks of 8 per thread (<= 2)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int i = (threadIdx.x + c * AR_THREADS) * 8;
        if (c < nper && i < H) {
          float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          uint4 raw[8];  // every rank's chunk in flight at once, then summed in rank order
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            if (p < W) {
              const bf16* src = reinterpret_cast<const bf16*>(ptrs.data[p]) + slot * slot_elems + (long)r * H + i;
              raw[p] = __ldcv(reinterpret_cast<const uint4*>(src));  // bypass L1: slots are reused
            }
          }
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            if (p < W) {
              const bf16* ev = reinterpret_cast<const bf16*>(&raw[p]);
#pragma unroll
              for (int u = 0; u < 8; ++u) sum[u] += __bfloat162float(ev[u]);
            }
          }
          const uint4 rr = *reinterpret_cast<const uint4*>(res + (long)r * H + i);
          const bf16* rv = reinterpret_cast<const bf16*>(&rr);
          uint4 nr;
          bf16* nv = reinterpret_cast<bf16*>(&nr);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float sb = __bfloat162float(__float2bfloat16(sum[u]));
            nv[u] = __float2bfloat16(__bfloat162float(rv[u]) + sb);
            acc[c * 8 + u] = __bfloat162float(nv[u]);
            ss += acc[c * 8 + u] * acc[c * 8 + u];
          }
          *reinterpret_cast<uint4*>(res + (long)r * H + i) = nr;
        }
      }
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
      __syncthreads();
      if (threadIdx.x < 32) {
        float t = threadIdx.x < AR_THREADS / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
      }
      __syncthreads();
      const float inv = rsqrtf(red[0] / H + eps);
      __syncthreads();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int i = (threadIdx.x + c * AR_THREADS) * 8;
        if (c < nper && i < H) {
          uint4 o;
          bf16* ov = reinterpret_cast<bf16*>(&o);
#pragma unroll
          for (int u = 0; u < 8; ++u) ov[u] = __float2bfloat16(acc[c * 8 + u] * inv * w1p[i + u]);
          *reinterpret_cast<uint4*>(out + (long)r * H + i) = o;
        }
      }
    }
  }
  // the last block to finish advances the epoch (every block already read it at entry)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int d = atomicAdd(done, 1);
    if (d == (int)gridDim.x - 1) {
      *done = 0;
      __threadfence();
      atomicExch(epoch, e);
    }
  }
}

// ------------------------------------------------------------------ sequence-parallel variant
// Reduce-scatter + residual add + RMSNorm + all-gather, for prefill-sized messages. Rank o owns
// rows [o per, (o+1) per) with per = ceil(R / W) (the last ranks may own fewer or none); inside
// every rank's range, block b handles rows b, b + G, ... (the same (rank, block) units on every
// rank). Region per rank and slot: the partial slot [W per, H], where rank p's rows of the
// owner's range sit at rows p per + (t - o per), and the results [R_max, 2H] (new residual row,
// normed row); then phase-A and phase-B flags [2 slots][max_blocks] each.
//   A. block b stores, for every owner rank, its unit's rows of the local partial into the
//      owner's partial slot (posted stores over NVLink); flag A[b] = e
//   B. block b waits for flag A[b] of every peer (one thread per peer), then for its own unit:
//      rank-order fp32 sum of the W partial rows, bf16 round, + residual, RMSNorm; writes the
//      results to the local tensors and stores them into every peer's result area (stores are
//      posted, so the all-gather costs no round trips); flag B[b] = e
//   C. block b waits for flag B[b] of every peer and copies the peers' units' result rows, now
//      in its own result area, into the local tensors.
// Slot reuse: rank o writes rank p's result area of slot s for call e + 2 only after its block b
// saw p's flag A[b] for e + 2, which p's block b raised after p's whole kernel for call e ended.
// Same bits as the one-shot kernel (and as NCCL all-reduce + add + RMSNorm); each rank moves
// about 3 (W-1)/W of the bf16 payload over NVLink instead of (W-1) copies of it.
// PUSHED: the projection GEMM before this kernel already stored its rows into the owners' slots
// (gemm.cu, GemmPush), so phase A only publishes (the GEMM's stores completed with that kernel).
// Either way phase B reads local memory only.
// res_local (runtime): the residual stays sequence-parallel: phase B stores only the normed rows
// into the peers' result areas and phase C copies only those, so every rank's `res` holds the new
// residual on its own range only (the next sequence-parallel call reads and writes only that
// range); half the gather traffic. The caller keeps it off for the last call of a forward, whose
// residual rows are read elsewhere.
// OWN (all-gather left to the next GEMM): phase B writes the new residual and normed rows of this
// rank's range to the local tensors only, and the normed rows also into this rank's own result
// area; there is no phase C. The last block to finish raises this rank's ready word to e (after
// every block's system-scope fence), and the next projection's GEMM (gemm.cu, gemm_ag) pulls each
// owner's normed rows from that owner's result area once its ready word reaches e. The rows of
// `res` outside this rank's range keep stale values: the next sequence-parallel call reads and
// writes only this rank's range of them. Slot reuse is as above: the result area of slot s is
// written again at call e + 2 only after every peer's flag A of e + 2, which each peer raised
// after its gathering GEMM of call e had ended (stream order).
__device__ __forceinline__ bool wait_peers(const SymmPtrs& ptrs, long flag_off, int b, int e, int* err,
                                           unsigned long long timeout_ns) {
  int ok = 1;
  if (threadIdx.x < ptrs.world && threadIdx.x != ptrs.rank) {
    const int* f = reinterpret_cast<const int*>(reinterpret_cast<const char*>(ptrs.data[threadIdx.x]) + flag_off) + b;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(f) < e) {
      if (globaltimer() - t0 > timeout_ns) {
        atomicCAS(err, 0, ERR_PEER_WAIT);
        ok = 0;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

template <bool PUSHED, bool OWN>
__global__ void __launch_bounds__(AR_THREADS) sp_ar_add_rmsnorm_kernel(
    SymmPtrs ptrs, const bf16* partial, long ldp, bf16* res, const float* w1p, bf16* out, int rows, int H,
    float eps, long slot_elems, int max_blocks, int* epoch, int* done, int* err, unsigned long long timeout_ns,
    int per, bool res_local) {
  __shared__ float red[32];
  __shared__ int s_epoch;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile int*>(epoch) + 1;
  __syncthreads();
  const int e = s_epoch, slot = e & 1;
  const int W = ptrs.world, me = ptrs.rank, b = blockIdx.x, G = gridDim.x;
  const long slot_stride = 3 * slot_elems;                          // elements per slot
  const long flags_base = 2 * slot_stride * (long)sizeof(bf16);     // bytes
  const long flagA = flags_base + (long)slot * max_blocks * 4;
  const long flagB = flags_base + (2L + slot) * max_blocks * 4;
  auto part_of = [&](int r) { return reinterpret_cast<bf16*>(ptrs.data[r]) + slot * slot_stride; };
  auto result_of = [&](int r) { return reinterpret_cast<bf16*>(ptrs.data[r]) + slot * slot_stride + slot_elems; };
  auto range = [&](int r, int& r0, int& r1) {
    r0 = min(rows, r * per);
    r1 = min(rows, (r + 1) * per);
  };
  auto publish = [&](long off) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      st_release_sys(reinterpret_cast<int*>(reinterpret_cast<char*>(ptrs.data[me]) + off) + b, e);
    }
  };
  // A. store this block's rows of every owner's range into the owner's partial slot
  bf16* mine = part_of(me);
  for (int r = 0; r < (PUSHED ? 0 : W); ++r) {
    int r0, r1;
    range(r, r0, r1);
    bf16* dst = part_of(r) + (long)me * per * H;
    for (int row = r0 + b; row < r1; row += G)
      for (int i = threadIdx.x * 8; i < H; i += AR_THREADS * 8)
        *reinterpret_cast<uint4*>(dst + (long)(row - r0) * H + i) =
            *reinterpret_cast<const uint4*>(partial + (long)row * ldp + i);
  }
  publish(flagA);
  // B. reduce + add + norm for this block's unit of my range
  if (wait_peers(ptrs, flagA, b, e, err, timeout_ns)) {
    int r0, r1;
    range(me, r0, r1);
    bf16* peer_res[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) peer_res[p] = p < W ? result_of(p) : nullptr;
    const int nper = (H + AR_THREADS * 8 - 1) / (AR_THREADS * 8);  // chunks of 8 per thread (<= 2)
    for (int row = r0 + b; row < r1; row += G) {
      float acc[16];
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int i = (threadIdx.x + c * AR_THREADS) * 8;
        if (c < nper && i < H) {
          float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          uint4 raw[8];
#pragma unroll
          for (int p = 0; p < 8; ++p)
            if (p < W) raw[p] = __ldcv(reinterpret_cast<const uint4*>(mine + ((long)p * per + row - r0) * H + i));
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            if (p < W) {
              const bf16* ev = reinterpret_cast<const bf16*>(&raw[p]);
#pragma unroll
              for (int u = 0; u < 8; ++u) sum[u] += __bfloat162float(ev[u]);
            }
          }
          const uint4 rr = *reinterpret_cast<const uint4*>(res + (long)row * H + i);
          const bf16* rv = reinterpret_cast<const bf16*>(&rr);
          uint4 nr;
          bf16* nv = reinterpret_cast<bf16*>(&nr);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float sb = __bfloat162float(__float2bfloat16(sum[u]));
            nv[u] = __float2bfloat16(__bfloat162float(rv[u]) + sb);
            acc[c * 8 + u] = __bfloat162float(nv[u]);
            ss += acc[c * 8 + u] * acc[c * 8 + u];
          }
          *reinterpret_cast<uint4*>(res + (long)row * H + i) = nr;
          if (!OWN && !res_local) {
#pragma unroll
            for (int p = 0; p < 8; ++p)
              if (p < W && p != me) *reinterpret_cast<uint4*>(peer_res[p] + (long)row * 2 * H + i) = nr;
          }
        }
      }
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
      __syncthreads();
      if (threadIdx.x < 32) {
        float t = threadIdx.x < AR_THREADS / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
      }
      __syncthreads();
      const float inv = rsqrtf(red[0] / H + eps);
      __syncthreads();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int i = (threadIdx.x + c * AR_THREADS) * 8;
        if (c < nper && i < H) {
          uint4 o;
          bf16* ov = reinterpret_cast<bf16*>(&o);
#pragma unroll
          for (int u = 0; u < 8; ++u) ov[u] = __float2bfloat16(acc[c * 8 + u] * inv * w1p[i + u]);
          *reinterpret_cast<uint4*>(out + (long)row * H + i) = o;
          if (OWN) {
            *reinterpret_cast<uint4*>(peer_res[me] + (long)row * 2 * H + H + i) = o;
          } else {
#pragma unroll
            for (int p = 0; p < 8; ++p)
              if (p < W && p != me) *reinterpret_cast<uint4*>(peer_res[p] + (long)row * 2 * H + H + i) = o;
          }
        }
      }
    }
    if (!OWN) publish(flagB);
    // C. the peers' result rows of this block's units, stored into this rank's result area
    if (!OWN && wait_peers(ptrs, flagB, b, e, err, timeout_ns)) {
      const bf16* pr = result_of(me);
      for (int p = 0; p < W; ++p) {
        if (p == me) continue;
        int q0, q1;
        range(p, q0, q1);
        for (int row = q0 + b; row < q1; row += G) {
          uint4 nr[2], o[2];  // every load of the row in flight before the stores
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int i = (threadIdx.x + c * AR_THREADS) * 8;
            if (i < H) {
              if (!res_local) nr[c] = __ldcv(reinterpret_cast<const uint4*>(pr + (long)row * 2 * H + i));
              o[c] = __ldcv(reinterpret_cast<const uint4*>(pr + (long)row * 2 * H + H + i));
            }
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int i = (threadIdx.x + c * AR_THREADS) * 8;
            if (i < H) {
              if (!res_local) *reinterpret_cast<uint4*>(res + (long)row * H + i) = nr[c];
              *reinterpret_cast<uint4*>(out + (long)row * H + i) = o[c];
            }
          }
        }
      }
    }
  }
  // the last block to finish advances the epoch (every block already read it at entry)
  __syncthreads();
  if (threadIdx.x == 0) {
    if (OWN)
      __threadfence_system();  // this block's result rows before the ready word (below)
    else
      __threadfence();
    const int d = atomicAdd(done, 1);
    if (d == (int)gridDim.x - 1) {
      *done = 0;
      __threadfence_system();
      if (OWN) st_release_sys(reinterpret_cast<int*>(reinterpret_cast<char*>(ptrs.data[me]) + flags_base +
                                                     4L * max_blocks * 4), e);
      atomicExch(epoch, e);
    }
  }
}

int symm_sp_ar_add_rmsnorm(void* const* bases, int world, int rank, const void* partial, long ldp, void* res,
                           const float* w1p, void* out, int rows, int H, float eps, long slot_elems, int max_blocks,
                           int* epoch, int* done, int* err, unsigned long long timeout_ns, cudaStream_t s, bool own,
                           bool res_local) {
  const int per = (rows + world - 1) / world;  // rows of one rank's range: one block per row, up to max_blocks
  if (world > 8 || H % 8 || H > 2 * AR_THREADS * 8 || (long)per * world * H > slot_elems) return -1;
  SymmPtrs p{};
  for (int r = 0; r < world; ++r) p.data[r] = bases[r];
  p.world = world;
  p.rank = rank;
  int grid = per < max_blocks ? per : max_blocks;
  if (grid < 1) grid = 1;
  if (own)
    sp_ar_add_rmsnorm_kernel<false, true><<<grid, AR_THREADS, 0, s>>>(p, (const bf16*)partial, ldp, (bf16*)res, w1p,
                                                                     (bf16*)out, rows, H, eps, slot_elems, max_blocks,
                                                                     epoch, done, err, timeout_ns, per, true);
  else
    sp_ar_add_rmsnorm_kernel<false, false><<<grid, AR_THREADS, 0, s>>>(p, (const bf16*)partial, ldp, (bf16*)res,
                                                                      w1p, (bf16*)out, rows, H, eps, slot_elems,
                                                                      max_blocks, epoch, done, err, timeout_ns, per,
                                                                      res_local);
  return (int)cudaGetLastError();
}

int symm_sp_rs_add_rmsnorm(void* const* bases, int world, int rank, int per, void* res, const float* w1p, void* out,
                           int rows, int H, float eps, long slot_elems, int max_blocks, int* epoch, int* done,
                           int* err, unsigned long long timeout_ns, cudaStream_t s, bool res_local) {
  if (world > 8 || H % 8 || H > 2 * AR_THREADS * 8 || per < 1 || (long)per * world < rows ||
      (long)per * world * H > slot_elems)
    return -1;
  SymmPtrs p{};
  for (int r = 0; r < world; ++r) p.data[r] = bases[r];
  p.world = world;
  p.rank = rank;
  int grid = per < max_blocks ? per : max_blocks;
  if (grid < 1) grid = 1;
  sp_ar_add_rmsnorm_kernel<true, false><<<grid, AR_THREADS, 0, s>>>(p, nullptr, 0, (bf16*)res, w1p, (bf16*)out, rows, H,
                                                             eps, slot_elems, max_blocks, epoch, done, err,
                                                             timeout_ns, per, res_local);
  return (int)cudaGetLastError();
}

int symm_ar_add_rmsnorm(void* const* bases, int world, int rank, const void* partial, long ldp, void* res,
                        const float* w1p, void* out, int rows, int H, float eps, long slot_elems, int max_blocks,
                        int* epoch, int* done, int* err, unsigned long long timeout_ns, cudaStream_t s) {
  if (world > 8 || H % 8 || H > 2 * AR_THREADS * 8 || (long)rows * H > slot_elems) return -1;
  SymmPtrs p{};
  for (int r = 0; r < world; ++r) p.data[r] = bases[r];
  p.world = world;
  p.rank = rank;
  int grid = rows < max_blocks ? rows : max_blocks;
  if (grid < 1) grid = 1;
  ar_add_rmsnorm_kernel<<<grid, AR_THREADS, 0, s>>>(p, (const bf16*)partial, ldp, (bf16*)res, w1p, (bf16*)out, rows,
                                                    H, eps, slot_elems, max_blocks, epoch, done, err, timeout_ns);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// NVLS (NVLink SHARP) all-reduce + residual add + RMSNorm for large messages.
//
// The region is one symmetric allocation bound to an NVSwitch multicast object: `uc` is this
// rank's own (unicast) mapping, `mc` the multicast address of the same bytes on every rank.
// Layout: two slots (call parity) of [partial | x], each [rows_cap, H] bf16, then two
// monotonically increasing u32 arrival counters. A call with index e (device epoch + 1):
//   A. every CTA copies its rows of the local partial into slot e&1 (unicast stores), then one
//      thread adds 1 to counter 0 on EVERY rank at once (multimem.red.release) and waits,
//      bounded, until its local copy reaches e * world * grid (all ranks' CTAs arrived);
//   B. rank r owns rows [r*per, (r+1)*per): for each, multimem.ld_reduce makes the switch return
//      the sum over all ranks (fp32 accumulation, one bf16 rounding), the kernel adds the
//      residual and multimem.st writes the new residual row into every rank's x area with one
//      store;
//   C. counter 1 the same way, then every CTA takes rows from the local x area: the new
//      residual, and its RMSNorm computed locally.
// Each row is reduced by one rank only, so every rank ends with identical bits, and the norm is
// recomputed from those bits rather than sent (NVLink carries the partials once and x once). The counters wrap safely (signed distance). Slot e&1 is rewritten at call
// e+2, after every rank passed counter 1 of call e+1, so no rank still reads it. Accesses
// through the multicast and unicast addresses of the same memory are ordered with
// fence.proxy.alias. No TMA and no cluster multicast are involved.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mc_red_add_release(unsigned* mc_addr, unsigned v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }
__device__ __forceinline__ uint4 mc_ld_reduce_bf16x8(const void* mc_addr) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc_addr)
               : "memory");
  return r;
}
__device__ __forceinline__ void mc_st_16(void* mc_addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}

// One thread per CTA: arrive on every rank's counter `c`, then wait until this rank's copy shows
// all `target` arrivals. Returns false (and records ERR_PEER_WAIT) when the wait runs out.
__device__ __forceinline__ bool nvls_barrier(unsigned* mc_cnt, const unsigned* uc_cnt, unsigned target, int* err,
                                             unsigned long long timeout_ns) {
  __threadfence_system();
  fence_proxy_alias();
  mc_red_add_release(mc_cnt, 1u);
  const uint64_t t0 = globaltimer();
  while ((int)(ld_acquire_sys_u32(uc_cnt) - target) < 0) {
    if (globaltimer() - t0 > timeout_ns) {
      atomicCAS(err, 0, ERR_PEER_WAIT);
      return false;
    }
  }
  fence_proxy_alias();
  return true;
}

__global__ void __launch_bounds__(AR_THREADS) nvls_ar_add_rmsnorm_kernel(
    char* uc, char* mc, int world, int rank, const bf16* partial, long ldp, bf16* res, const float* w1p, bf16* out,
    int rows, int H, float eps, long slot_elems, int* epoch, int* done, int* err, unsigned long long timeout_ns) {
  __shared__ float red[32];
  __shared__ int s_epoch, s_ok;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile int*>(epoch) + 1;
  __syncthreads();
  const int e = s_epoch;
  const int slot = e & 1;
  const long slot_bytes = 2 * slot_elems * 2;
  bf16* part_uc = reinterpret_cast<bf16*>(uc + slot * slot_bytes);
  bf16* part_mc = reinterpret_cast<bf16*>(mc + slot * slot_bytes);
  const bf16* x_uc = part_uc + slot_elems;
  bf16* x_mc = part_mc + slot_elems;
  unsigned* cnt_uc = reinterpret_cast<unsigned*>(uc + 2 * slot_bytes);
  unsigned* cnt_mc = reinterpret_cast<unsigned*>(mc + 2 * slot_bytes);
  const unsigned target = (unsigned)e * (unsigned)world * gridDim.x;
  const int G = gridDim.x, b = blockIdx.x;
  // A. stage the local partial (all rows: every rank's slice is read by its owner via the switch)
  for (int r = b; r < rows; r += G)
    for (int i = threadIdx.x * 8; i < H; i += AR_THREADS * 8)
      *reinterpret_cast<uint4*>(part_uc + (long)r * H + i) = *reinterpret_cast<const uint4*>(partial + (long)r * ldp + i);
  __syncthreads();
  if (threadIdx.x == 0) s_ok = nvls_barrier(cnt_mc, cnt_uc, target, err, timeout_ns);
  __syncthreads();
  if (s_ok) {
    // B. this rank's rows: switch-reduced sum (one bf16 rounding), residual add, and the new
    //    residual row multicast into every rank's x area
    const int per = (rows + world - 1) / world;
    const int r0 = rank * per, r1 = min(rows, r0 + per);
    for (int r = r0 + b; r < r1; r += G)
      for (int i = threadIdx.x * 8; i < H; i += AR_THREADS * 8) {
        const uint4 sm = mc_ld_reduce_bf16x8(part_mc + (long)r * H + i);
        const uint4 rr = *reinterpret_cast<const uint4*>(res + (long)r * H + i);
        const bf16* sv = reinterpret_cast<const bf16*>(&sm);
        const bf16* rv = reinterpret_cast<const bf16*>(&rr);
        uint4 nr;
        bf16* nv = reinterpret_cast<bf16*>(&nr);
#pragma unroll
        for (int u = 0; u < 8; ++u) nv[u] = __float2bfloat16(__bfloat162float(rv[u]) + __bfloat162float(sv[u]));
        mc_st_16(x_mc + (long)r * H + i, nr);
      }
    __syncthreads();
    if (threadIdx.x == 0) s_ok = nvls_barrier(cnt_mc + 1, cnt_uc + 1, target, err, timeout_ns);
    __syncthreads();
    // C. every row from this rank's own copy of the x area: the new residual and its RMSNorm
    //    (each rank normalises locally from identical bits, so the norms agree too)
    if (s_ok) {
      for (int r = b; r < rows; r += G) {
        uint4 xv[2];
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int i = (threadIdx.x + c * AR_THREADS) * 8;
          if (i < H) {
            xv[c] = __ldcv(reinterpret_cast<const uint4*>(x_uc + (long)r * H + i));
            const bf16* v = reinterpret_cast<const bf16*>(&xv[c]);
#pragma unroll
            for (int u = 0; u < 8; ++u) ss += __bfloat162float(v[u]) * __bfloat162float(v[u]);
            *reinterpret_cast<uint4*>(res + (long)r * H + i) = xv[c];
          }
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
        __syncthreads();
        if (threadIdx.x < 32) {
          float t = threadIdx.x < AR_THREADS / 32 ? red[threadIdx.x] : 0.f;
          t = warp_sum(t);
          if (threadIdx.x == 0) red[0] = t;
        }
        __syncthreads();
        const float inv = rsqrtf(red[0] / H + eps);
        __syncthreads();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int i = (threadIdx.x + c * AR_THREADS) * 8;
          if (i < H) {
            const bf16* v = reinterpret_cast<const bf16*>(&xv[c]);
            uint4 o;
            bf16* ov = reinterpret_cast<bf16*>(&o);
#pragma unroll
            for (int u = 0; u < 8; ++u) ov[u] = __float2bfloat16(__bfloat162float(v[u]) * inv * w1p[i + u]);
            *reinterpret_cast<uint4*>(out + (long)r * H + i) = o;
          }
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int d = atomicAdd(done, 1);
    if (d == (int)gridDim.x - 1) {
      *done = 0;
      __threadfence();
      atomicExch(epoch, e);
    }
  }
}

long nvls_region_bytes(long slot_elems) { return 2 * 2 * slot_elems * 2 + 256; }

int nvls_ar_add_rmsnorm(void* uc, void* mc, int world, int rank, const void* partial, long ldp, void* res,
                        const float* w1p, void* out, int rows, int H, float eps, long slot_elems, int grid,
                        int* epoch, int* done, int* err, unsigned long long timeout_ns, cudaStream_t s) {
  if (world < 1 || world > 8 || H % 8 || H > 2 * AR_THREADS * 8 || (long)rows * H > slot_elems || grid < 1 ||
      (reinterpret_cast<uintptr_t>(uc) | reinterpret_cast<uintptr_t>(mc)) % 16)
    return -1;
  nvls_ar_add_rmsnorm_kernel<<<grid, AR_THREADS, 0, s>>>((char*)uc, (char*)mc, world, rank, (const bf16*)partial, ldp,
                                                         (bf16*)res, w1p, (bf16*)out, rows, H, eps, slot_elems, epoch,
                                                         done, err, timeout_ns);
  return (int)cudaGetLastError();
}

}  // namespace qb
