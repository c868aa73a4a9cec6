// Expert-parallel MoE over NVLink peer memory: dispatch of token rows into the ranks that own
// their experts, the grouped block-scaled expert GEMMs on each rank's received rows, and the
// combine of the routing-weighted partial outputs back at the tokens' owners.
//
// Each rank owns a symmetric region (one cudaMalloc, IPC-mapped by every peer) with two parity
// halves p = epoch & 1, each holding per source rank s a receive area of `cap` rows:
//   x[p][s][cap][H] bf16    token rows sent by s          (written by s with peer stores)
//   i[p][s][cap][k] int32   their expert ids              (-1 marks an unused row)
//   w[p][s][cap][k] fp32    their routing weights
//   y[p][s][cap][H] bf16    this rank's weighted expert sum for each received row (read by s)
//   flags: disp[p][8] (epoch of s's dispatch), cnt[p][8] (rows s sent), done[p] (y is ready)
// One call (epoch e):
//   route     slots[t][d] = position of token t in rank d's area for this rank (-1: not sent),
//             deterministic (prefix over tokens), and counts[d]
//   dispatch  every token row goes to each distinct rank owning one of its experts, straight into
//             that rank's x/i/w area (16-byte peer stores); the last block publishes cnt and
//             disp = e to every rank with a system-scope release
//   recv      waits (bounded) for disp = e from every rank, marks the rows past each count unused
//   experts   the block-scaled grouped GEMMs (moe_mx.cu) over all received rows; expert ids
//             outside this rank's range are skipped by the expert dispatch, so each row's output
//             is the weighted sum over this rank's experts, written into y[p]
//   done      done[p] = e (release)
//   combine   waits (bounded) for done = e from every rank, then each token's output is the sum
//             over ranks (in rank order, fp32) of y rows at its slots, read with peer loads
// Reuse of a parity half at e + 2 is safe without acknowledgements: a rank dispatches for e + 2
// only after its own combine of e + 1, and every rank's experts for e + 1 waited for that rank's
// dispatch of e + 1, which follows its combine of e. The epoch lives in device memory (graph
// replay safe). Waits give up after `timeout_ns` and record ERR_PEER_WAIT (no trap).
// Reference counterpart: the reference keeps activations replicated and folds the routed sum into
// the tensor-parallel all-reduce (model.py:2770-2790); this is the expert-parallel form.
#include "common.cuh"
#include "kernels.h"

namespace qb {

using bf16 = __nv_bfloat16;

struct EpPtrs {
  char* base[8];  // every rank's region (peer-mapped; own entry local)
  int world, rank;
};

struct EpLayout {
  long x[2], y[2], i[2], w[2];  // byte offsets of the parity halves
  long flags;                   // int disp[2][8], cnt[2][8], done[2]
  int cap, H, k;
};

static long align256(long v) { return (v + 255) / 256 * 256; }

static EpLayout ep_layout(int world, int cap, int H, int k) {
  EpLayout L{};
  long o = 0;
  const long xb = align256((long)world * cap * H * 2), ib = align256((long)world * cap * k * 4);
  for (int p = 0; p < 2; ++p) { L.x[p] = o; o += xb; }
  for (int p = 0; p < 2; ++p) { L.y[p] = o; o += xb; }
  for (int p = 0; p < 2; ++p) { L.i[p] = o; o += ib; }
  for (int p = 0; p < 2; ++p) { L.w[p] = o; o += ib; }
  L.flags = o;
  L.cap = cap;
  L.H = H;
  L.k = k;
  return L;
}

long ep_region_bytes(int world, int cap, int H, int k) { return ep_layout(world, cap, H, k).flags + 64 * 4; }

__device__ __forceinline__ void ep_st_release(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ep_ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int* ep_flags(const EpPtrs& P, const EpLayout& L, int r) {
  return reinterpret_cast<int*>(P.base[r] + L.flags);
}
// flags: disp[p][s] at 0 + p * 8 + s, cnt[p][s] at 16 + p * 8 + s, done[p] at 32 + p

// ------------------------------------------------------------------ route (one CTA)
// state[0] = epoch (advanced here), state[1] = dispatch blocks finished
__global__ void __launch_bounds__(1024) ep_route_kernel(const int* topi, int T, int k, int per_rank, int world,
                                                        int* slots, int* counts, int* state) {
  __shared__ int wsum[32];
  __shared__ int base_d;
  const int tid = threadIdx.x, lane = tid % 32, wid = tid / 32;
  const int ipt = (T + blockDim.x - 1) / blockDim.x;  // tokens per thread, contiguous
  const int t0 = tid * ipt, t1 = min(T, t0 + ipt);
  for (int d = 0; d < world; ++d) {
    int c = 0;
    for (int t = t0; t < t1; ++t) {
      bool hit = false;
      for (int j = 0; j < k; ++j) {
        const int e = topi[(long)t * k + j];
        hit |= e >= 0 && e / per_rank == d;  // id -1: no expert
      }
      c += hit;
    }
    // exclusive block scan of c
    int v = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffff, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) wsum[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int s = lane < (int)(blockDim.x / 32) ? wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffff, s, o);
        if (lane >= o) s += n;
      }
      wsum[lane] = s;  // inclusive prefix of warp sums
      if (lane == 31) base_d = s;
    }
    __syncthreads();
    int pos = v - c + (wid > 0 ? wsum[wid - 1] : 0);
    for (int t = t0; t < t1; ++t) {
      bool hit = false;
      for (int j = 0; j < k; ++j) {
        const int e = topi[(long)t * k + j];
        hit |= e >= 0 && e / per_rank == d;
      }
      slots[(long)t * world + d] = hit ? pos++ : -1;
    }
    if (tid == 0) counts[d] = base_d;
    __syncthreads();
  }
  if (tid == 0) {
    state[0] += 1;
    state[1] = 0;
  }
}

// ------------------------------------------------------------------ dispatch
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpPtrs P, EpLayout L, const bf16* x, long ldx,
                                                          const int* topi, const float* topw, const int* slots,
                                                          const int* counts, int T, int* state) {
  const int e = *reinterpret_cast<volatile int*>(state);
  const int par = e & 1, W = P.world, me = P.rank, H = L.H, k = L.k;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (long)t * ldx);
    for (int d = 0; d < W; ++d) {
      const int sl = slots[(long)t * W + d];
      if (sl < 0) continue;
      const long row = (long)me * L.cap + sl;
      uint4* dx = reinterpret_cast<uint4*>(P.base[d] + L.x[par]) + row * (H / 8);
      for (int v = threadIdx.x; v < H / 8; v += blockDim.x) dx[v] = src[v];
      if (threadIdx.x < k) {
        reinterpret_cast<int*>(P.base[d] + L.i[par])[row * k + threadIdx.x] = topi[(long)t * k + threadIdx.x];
        reinterpret_cast<float*>(P.base[d] + L.w[par])[row * k + threadIdx.x] = topw[(long)t * k + threadIdx.x];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const bool last = atomicAdd(&state[1], 1) == (int)gridDim.x - 1;
    if (last) {  // every block's rows are out: publish counts, then the epoch
      __threadfence_system();
      for (int d = 0; d < W; ++d) {
        int* f = ep_flags(P, L, d);
        *reinterpret_cast<volatile int*>(f + 16 + par * 8 + me) = counts[d];
      }
      __threadfence_system();
      for (int d = 0; d < W; ++d) ep_st_release(ep_flags(P, L, d) + par * 8 + me, e);
    }
  }
}

// ------------------------------------------------------------------ receive (one CTA)
__global__ void __launch_bounds__(256) ep_recv_kernel(EpPtrs P, EpLayout L, const int* state, int* err,
                                                      unsigned long long timeout_ns) {
  __shared__ int cnt[8];
  const int e = *reinterpret_cast<volatile const int*>(state);
  const int par = e & 1, W = P.world, me = P.rank;
  int* f = ep_flags(P, L, me);
  if (threadIdx.x < W) {
    const uint64_t t0 = globaltimer();
    int n = 0;
    while (true) {
      if (ep_ld_acquire(f + par * 8 + threadIdx.x) >= e) {
        n = *reinterpret_cast<volatile int*>(f + 16 + par * 8 + threadIdx.x);
        break;
      }
      if (globaltimer() - t0 > timeout_ns) {  // no data from this rank: its rows stay unused
        atomicCAS(err, 0, ERR_PEER_WAIT);
        break;
      }
    }
    cnt[threadIdx.x] = n;
  }
  __syncthreads();
  int* ids = reinterpret_cast<int*>(P.base[me] + L.i[par]);
  for (int s = 0; s < W; ++s)
    for (long r = (long)cnt[s] * L.k + threadIdx.x; r < (long)L.cap * L.k; r += blockDim.x)
      ids[(long)s * L.cap * L.k + r] = -1;
}

// ------------------------------------------------------------------ done (one thread)
__global__ void ep_done_kernel(EpPtrs P, EpLayout L, const int* state) {
  const int e = *reinterpret_cast<volatile const int*>(state);
  __threadfence_system();
  ep_st_release(ep_flags(P, L, P.rank) + 32 + (e & 1), e);
}

// ------------------------------------------------------------------ combine
__global__ void __launch_bounds__(256) ep_combine_kernel(EpPtrs P, EpLayout L, const int* slots, int T, bf16* out,
                                                         long ldo, const int* state, int* err,
                                                         unsigned long long timeout_ns) {
  __shared__ int ok_s;
  const int e = *reinterpret_cast<volatile const int*>(state);
  const int par = e & 1, W = P.world, me = P.rank, H = L.H;
  if (threadIdx.x == 0) ok_s = 1;
  __syncthreads();
  if (threadIdx.x < W) {  // every rank's expert outputs for this epoch (one poller per rank)
    const int* f = ep_flags(P, L, threadIdx.x) + 32 + par;
    const uint64_t t0 = globaltimer();
    while (ep_ld_acquire(f) < e) {
      if (globaltimer() - t0 > timeout_ns) {
        atomicCAS(err, 0, ERR_PEER_WAIT);
        ok_s = 0;
        break;
      }
    }
  }
  __syncthreads();
  const bool ok = ok_s;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int d = 0; d < W && ok; ++d) {  // rank order: identical bits whatever the arrival order
        const int sl = slots[(long)t * W + d];
        if (sl < 0) continue;
        const uint4 q = reinterpret_cast<const uint4*>(P.base[d] + L.y[par])[((long)me * L.cap + sl) * (H / 8) + v];
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f2 = __bfloat1622float2(h2[j]);
          acc[2 * j] += f2.x;
          acc[2 * j + 1] += f2.y;
        }
      }
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) o2[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
      reinterpret_cast<uint4*>(out + (long)t * ldo)[v] = o;
    }
  }
}

// ------------------------------------------------------------------ host
static EpPtrs ep_ptrs(void* const* bases, int world, int rank) {
  EpPtrs P{};
  for (int r = 0; r < world; ++r) P.base[r] = static_cast<char*>(bases[r]);
  P.world = world;
  P.rank = rank;
  return P;
}

int ep_dispatch(void* const* bases, int world, int rank, int cap, int H, int k, int experts_per_rank, const void* x,
                long ldx, const int* topi, const float* topw, int T, int* slots, int* counts, int* state,
                unsigned long long timeout_ns, int* err, cudaStream_t s) {
  if (world < 1 || world > 8 || H % 8 || k > 32 || T > cap) return -1;
  const EpLayout L = ep_layout(world, cap, H, k);
  const EpPtrs P = ep_ptrs(bases, world, rank);
  ep_route_kernel<<<1, 1024, 0, s>>>(topi, T, k, experts_per_rank, world, slots, counts, state);
  const int grid = T < 296 ? (T > 0 ? T : 1) : 296;
  ep_dispatch_kernel<<<grid, 256, 0, s>>>(P, L, (const bf16*)x, ldx, topi, topw, slots, counts, T, state);
  ep_recv_kernel<<<1, 256, 0, s>>>(P, L, state, err, timeout_ns);
  return (int)cudaGetLastError();
}

int ep_combine(void* const* bases, int world, int rank, int cap, int H, int k, const int* slots, int T, void* out,
               long ldo, const int* state, unsigned long long timeout_ns, int* err, cudaStream_t s) {
  if (world < 1 || world > 8 || H % 8) return -1;
  const EpLayout L = ep_layout(world, cap, H, k);
  const EpPtrs P = ep_ptrs(bases, world, rank);
  ep_done_kernel<<<1, 32, 0, s>>>(P, L, state);
  const int grid = T < 296 ? (T > 0 ? T : 1) : 296;
  ep_combine_kernel<<<grid, 256, 0, s>>>(P, L, slots, T, (bf16*)out, ldo, state, err, timeout_ns);
  return (int)cudaGetLastError();
}

// byte offsets of this rank's receive areas for the expert GEMMs: x, i, w, y of parity `par`
void ep_offsets(int world, int cap, int H, int k, int par, long* x, long* i, long* w, long* y) {
  const EpLayout L = ep_layout(world, cap, H, k);
  *x = L.x[par];
  *i = L.i[par];
  *w = L.w[par];
  *y = L.y[par];
}

}  // namespace qb
