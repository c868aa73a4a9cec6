// Sequence kernels over varlen batches of segments (a segment = consecutive rows of one lane):
//   causal_conv_varlen   depthwise causal conv (kernel 4) + SiLU, continuing the lane's window
//   gated_delta_varlen   gated delta rule with the DeltaNet glue fused in (beta, g, q/k l2norm,
//                        key-head repeat), continuing and updating the lane's fp32 state
//   attention_varlen     causal GQA attention over the paged KV cache, split-K (flash-decoding)
// Rounding follows the HuggingFace modeling code (see elementwise.cu).
#include "common.cuh"
#include "kernels.h"

namespace qb {

using bf16 = __nv_bfloat16;
__device__ __forceinline__ float rbf2(float x) { return __bfloat162float(__float2bfloat16(x)); }

__device__ __forceinline__ int seg_of(const int* cu, int S, int t) {
  int lo = 0, hi = S - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) / 2;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ------------------------------------------------------------------ causal conv
template <int K>
__global__ void conv_kernel(const bf16* x, long ldx, bf16* state, long lane_stride, const bf16* w,
                            const int* seg_lane, const int* cu, int C, bf16* out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int s = blockIdx.y;
  if (c >= C) return;
  const int lane = seg_lane[s];
  bf16* st = state + (long)lane * lane_stride + (long)c * (K - 1);
  float win[K - 1], wt[K];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = __bfloat162float(st[j]);
#pragma unroll
  for (int j = 0; j < K; ++j) wt[j] = __bfloat162float(w[(long)c * K + j]);
  for (int t = cu[s]; t < cu[s + 1]; ++t) {
    const float xt = __bfloat162float(x[(long)t * ldx + c]);
    float acc = wt[K - 1] * xt;
#pragma unroll
    for (int j = 0; j < K - 1; ++j) acc += wt[j] * win[j];
    const float a = rbf2(acc);
    out[(long)t * C + c] = __float2bfloat16(a / (1.f + expf(-a)));
#pragma unroll
    for (int j = 0; j < K - 2; ++j) win[j] = win[j + 1];
    win[K - 2] = xt;
  }
#pragma unroll
  for (int j = 0; j < K - 1; ++j) st[j] = __float2bfloat16(win[j]);
}

int causal_conv_varlen(const void* x, long ldx, void* state, long lane_stride, const void* w, const int* seg_lane,
                       const int* cu, int S, int C, int K, void* out, cudaStream_t s) {
  if (!S) return 0;
  if (K != 4) return -1;
  dim3 grid((C + 127) / 128, S);
  conv_kernel<4><<<grid, 128, 0, s>>>((const bf16*)x, ldx, (bf16*)state, lane_stride, (const bf16*)w, seg_lane, cu,
                                      C, (bf16*)out);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ gated delta rule
// One CTA per (value head, segment), DV threads; thread j owns state column j (DK fp32 values
// in registers) so the recurrence needs no cross-thread reduction:
//   S *= exp(g);  delta_j = (v_j - sum_i S_ij k_i) * beta;  S_ij += k_i delta_j;  o_j = sum_i S_ij q_i
template <int DK>
__global__ void __launch_bounds__(128) delta_kernel(const bf16* qkv, long ldqkv, const bf16* ab, long ldab,
                                                    const float* a_log, const float* dt_bias, float* state,
                                                    long lane_stride, const int* seg_lane, const int* cu, int nk,
                                                    int nv, int dv, bf16* out) {
  __shared__ float qs[DK], ks[DK], red[8], gb[2];
  const int h = blockIdx.x, s = blockIdx.y, j = threadIdx.x;
  const int lane = seg_lane[s];
  const int hk = h / (nv / nk);
  float* st = state + (long)lane * lane_stride + (long)h * DK * dv;
  float S[DK];
  if (j < dv) {
#pragma unroll
    for (int i = 0; i < DK; ++i) S[i] = st[(long)i * dv + j];
  }
  const float A = -expf(a_log[h]);
  const float dtb = dt_bias[h];
  const float scale = rsqrtf((float)DK);
  const int nw = (blockDim.x + 31) / 32;
  for (int t = cu[s]; t < cu[s + 1]; ++t) {
    const bf16* row = qkv + (long)t * ldqkv;
    // l2norm of q and k in bf16 arithmetic (HF applies it to the bf16 tensors)
    float qv = 0.f, kv = 0.f, qq = 0.f, kk = 0.f;
    if (j < DK) {
      qv = __bfloat162float(row[(long)hk * DK + j]);
      kv = __bfloat162float(row[(long)nk * DK + (long)hk * DK + j]);
      qq = rbf2(qv * qv);
      kk = rbf2(kv * kv);
    }
    qq = warp_sum(qq);
    kk = warp_sum(kk);
    if ((j & 31) == 0) {
      red[j / 32] = qq;
      red[4 + j / 32] = kk;
    }
    if (j == 0) {
      const float b = __bfloat162float(ab[(long)t * ldab + h]);
      const float a = __bfloat162float(ab[(long)t * ldab + nv + h]);
      gb[0] = A * softplus(a + dtb);   // log decay (fp32)
      gb[1] = rbf2(1.f / (1.f + expf(-b)));  // beta, rounded like the bf16 sigmoid
    }
    __syncthreads();
    if (j < DK) {
      float sq = 0.f, sk = 0.f;
      for (int w = 0; w < nw && w < 4; ++w) {
        sq += red[w];
        sk += red[4 + w];
      }
      const float iq = rbf2(rsqrtf(rbf2(rbf2(sq) + 1e-6f)));
      const float ik = rbf2(rsqrtf(rbf2(rbf2(sk) + 1e-6f)));
      qs[j] = rbf2(qv * iq) * scale;
      ks[j] = rbf2(kv * ik);
    }
    __syncthreads();
    if (j < dv) {
      const float decay = expf(gb[0]), beta = gb[1];
      const float v = __bfloat162float(row[2L * nk * DK + (long)h * dv + j]);
      float kvm = 0.f;
#pragma unroll
      for (int i = 0; i < DK; ++i) {
        S[i] *= decay;
        kvm += S[i] * ks[i];
      }
      const float delta = (v - kvm) * beta;
      float o = 0.f;
#pragma unroll
      for (int i = 0; i < DK; ++i) {
        S[i] += ks[i] * delta;
        o += S[i] * qs[i];
      }
      out[((long)t * nv + h) * dv + j] = __float2bfloat16(o);
    }
    __syncthreads();
  }
  if (j < dv) {
#pragma unroll
    for (int i = 0; i < DK; ++i) st[(long)i * dv + j] = S[i];
  }
}

int gated_delta_varlen(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log,
                       const float* dt_bias, float* state, long lane_stride, const int* seg_lane, const int* cu,
                       int S, int nk, int nv, int dk, int dv, void* out, cudaStream_t s) {
  if (!S) return 0;
  if (dv > 128 || dk > 128) return -1;
  const int threads = ((dv > dk ? dv : dk) + 31) / 32 * 32;
  dim3 grid(nv, S);
#define QB_DELTA(DKV)                                                                                        \
  delta_kernel<DKV><<<grid, threads, 0, s>>>((const bf16*)qkv, ldqkv, (const bf16*)ab, ldab, a_log, dt_bias, \
                                             state, lane_stride, seg_lane, cu, nk, nv, dv, (bf16*)out)
  if (dk == 128) QB_DELTA(128);
  else if (dk == 64) QB_DELTA(64);
  else if (dk == 32) QB_DELTA(32);
  else return -1;
#undef QB_DELTA
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ paged attention
// Grid (splits, kv heads, query rows). Each CTA streams 32-key tiles of its split of the
// row's causal context from the paged cache into shared memory; lane j scores key j of the
// tile for each of the warp's query heads, then the warp accumulates P.V with each lane owning
// HD/32 output dims. Partial (max, sum, o) per split go to `ws`; a second kernel combines.
constexpr int ATT_WARPS = 4;
constexpr int ATT_KT = 32;

template <int HD>
__global__ void __launch_bounds__(ATT_WARPS * 32)
    attn_split_kernel(const bf16* q, const bf16* kc, const bf16* vc, const int* table, int max_blocks, const int* pos,
                      const int* seg_lane, const int* cu, int S, int nq, int nkv, int bs, int splits, float* ws,
                      bf16* out) {
  constexpr int KST = HD + 8;  // padded K row (bf16 elements): conflict-free 16B lane reads
  constexpr int PER = HD / 32;
  __shared__ __align__(16) bf16 Ks[ATT_KT * KST];
  __shared__ __align__(16) bf16 Vs[ATT_KT * HD];
  __shared__ float Ps[ATT_WARPS][ATT_KT];
  const int split = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int G = nq / nkv;
  const int lanei = seg_lane[seg_of(cu, S, t)];
  const int ctx = pos[t] + 1;
  int chunk = (ctx + splits - 1) / splits;
  chunk = (chunk + ATT_KT - 1) / ATT_KT * ATT_KT;
  const int k0 = split * chunk, k1 = min(ctx, k0 + chunk);
  const float scale = rsqrtf((float)HD);
  const int* tab = table + (long)lanei * max_blocks;
  // per-warp heads: h = w, w + ATT_WARPS, ... (< G); at most 4 per warp
  constexpr int MAXH = 4;
  float m[MAXH], l[MAXH], o[MAXH][PER];
  float qr[MAXH][HD / 8 > 0 ? 1 : 1];
  (void)qr;
#pragma unroll
  for (int a = 0; a < MAXH; ++a) {
    m[a] = -INFINITY;
    l[a] = 0.f;
#pragma unroll
    for (int d = 0; d < PER; ++d) o[a][d] = 0.f;
  }
  for (int kt = k0; kt < k1; kt += ATT_KT) {
    __syncthreads();
    // load up to 32 keys/values (16B vectors)
    for (int idx = threadIdx.x; idx < ATT_KT * HD / 8; idx += blockDim.x) {
      const int r = idx / (HD / 8), c = idx % (HD / 8);
      const int p = kt + r;
      uint4 kvv = make_uint4(0, 0, 0, 0), vvv = make_uint4(0, 0, 0, 0);
      if (p < k1) {
        const long prow = (long)tab[p / bs] * bs + p % bs;
        kvv = *reinterpret_cast<const uint4*>(kc + (prow * nkv + g) * HD + c * 8);
        vvv = *reinterpret_cast<const uint4*>(vc + (prow * nkv + g) * HD + c * 8);
      }
      *reinterpret_cast<uint4*>(&Ks[r * KST + c * 8]) = kvv;
      *reinterpret_cast<uint4*>(&Vs[r * HD + c * 8]) = vvv;
    }
    __syncthreads();
    const int nvalid = min(ATT_KT, k1 - kt);
#pragma unroll
    for (int a = 0; a < MAXH; ++a) {
      const int hh = w + a * ATT_WARPS;
      if (hh >= G) break;
      const bf16* qrow = q + ((long)t * nq + (long)g * G + hh) * HD;
      // lane = key index within the tile: full dot product over HD
      float sc = -INFINITY;
      if (lane < nvalid) {
        float acc = 0.f;
        for (int c = 0; c < HD / 8; ++c) {
          const uint4 kk = *reinterpret_cast<const uint4*>(&Ks[lane * KST + c * 8]);
          const uint4 qq = *reinterpret_cast<const uint4*>(qrow + c * 8);
          const bf16* ke = reinterpret_cast<const bf16*>(&kk);
          const bf16* qe = reinterpret_cast<const bf16*>(&qq);
#pragma unroll
          for (int u = 0; u < 8; ++u) acc += __bfloat162float(qe[u]) * __bfloat162float(ke[u]);
        }
        sc = acc * scale;
      }
      const float mt = warp_max(sc);
      const float mn = fmaxf(m[a], mt);
      const float p = lane < nvalid ? expf(sc - mn) : 0.f;
      const float corr = expf(m[a] - mn);
      l[a] = l[a] * corr + warp_sum(p);
      m[a] = mn;
      Ps[w][lane] = p;
      __syncwarp();
#pragma unroll
      for (int d = 0; d < PER; ++d) o[a][d] *= corr;
      for (int jj = 0; jj < nvalid; ++jj) {
        const float pj = Ps[w][jj];
#pragma unroll
        for (int d = 0; d < PER; ++d) o[a][d] += pj * __bfloat162float(Vs[jj * HD + lane * PER + d]);
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int a = 0; a < MAXH; ++a) {
    const int hh = w + a * ATT_WARPS;
    if (hh >= G) break;
    const int head = g * G + hh;
    if (splits == 1) {
      const float inv = l[a] > 0.f ? 1.f / l[a] : 0.f;
#pragma unroll
      for (int d = 0; d < PER; ++d) out[((long)t * nq + head) * HD + lane * PER + d] = __float2bfloat16(o[a][d] * inv);
    } else {
      float* wsr = ws + (((long)t * nq + head) * splits + split) * (HD + 2);
#pragma unroll
      for (int d = 0; d < PER; ++d) wsr[2 + lane * PER + d] = o[a][d];
      if (lane == 0) {
        wsr[0] = m[a];
        wsr[1] = l[a];
      }
    }
  }
}

template <int HD>
__global__ void attn_combine_kernel(const float* ws, int splits, int nq, bf16* out) {
  const long th = blockIdx.x;  // t * nq + head
  const float* base = ws + th * splits * (HD + 2);
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, base[s * (HD + 2)]);
  float L = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float mm = base[s * (HD + 2)];
    if (mm > -INFINITY) L += expf(mm - M) * base[s * (HD + 2) + 1];
  }
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float mm = base[s * (HD + 2)];
      if (mm > -INFINITY) acc += expf(mm - M) * base[s * (HD + 2) + 2 + d];
    }
    out[th * HD + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
  }
}

int attention_varlen(const void* q, const void* kc, const void* vc, const int* table, int max_blocks, const int* pos,
                     const int* seg_lane, const int* cu, int S, int T, int nq, int nkv, int hd, int block_size,
                     int splits, float* ws, void* out, cudaStream_t s) {
  if (!T) return 0;
  if (nq / nkv > ATT_WARPS * 4) return -1;
  dim3 grid(splits, nkv, T);
#define QB_ATT(H)                                                                                                   \
  attn_split_kernel<H><<<grid, ATT_WARPS * 32, 0, s>>>((const bf16*)q, (const bf16*)kc, (const bf16*)vc, table,    \
                                                       max_blocks, pos, seg_lane, cu, S, nq, nkv, block_size, splits, \
                                                       ws, (bf16*)out);                                             \
  if (splits > 1) attn_combine_kernel<H><<<T * nq, 128, 0, s>>>(ws, splits, nq, (bf16*)out)
  if (hd == 256) { QB_ATT(256); }
  else if (hd == 128) { QB_ATT(128); }
  else if (hd == 64) { QB_ATT(64); }
  else return -1;
#undef QB_ATT
  return (int)cudaGetLastError();
}

}  // namespace qb

// ------------------------------------------------------------------ allocation-free entry point
// See noalloc.h: the split-K scratch of the attention kernels above lives in this file-scope
// device array, so callers that cannot allocate device memory can still run the kernel.
#include <mutex>

#include "noalloc.h"

static __device__ __align__(256) float g_attn_noalloc_scratch[QB_ATTN_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device (looked up once per device).
int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return QB_NOALLOC_ERR_ARGS;
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return QB_NOALLOC_ERR_SYMBOL;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return QB_NOALLOC_OK;
}
}  // namespace

extern "C" __attribute__((visibility("default"))) size_t qb_attention_noalloc_scratch_bytes(void) {
  return QB_ATTN_NOALLOC_SCRATCH_BYTES;
}

extern "C" __attribute__((visibility("default"))) int qb_attention_varlen_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* block_table, int max_blocks,
    const int* positions, const int* seg_lane, const int* cu, int num_segments, int num_rows, int nq, int nkv,
    int head_dim, int block_size, int splits, void* out, cudaStream_t stream) {
  if (num_rows < 0 || num_segments <= 0 || nq <= 0 || nkv <= 0 || splits < 1 || splits > 64 || block_size <= 0 ||
      nq % nkv != 0 || (head_dim != 64 && head_dim != 128 && head_dim != 256))
    return QB_NOALLOC_ERR_ARGS;
  if (num_rows == 0) return QB_NOALLOC_OK;
  const size_t need = (size_t)num_rows * nq * splits * (head_dim + 2) * sizeof(float);
  if (splits > 1 && need > QB_ATTN_NOALLOC_SCRATCH_BYTES) return QB_NOALLOC_ERR_TOO_LARGE;
  float* ws = nullptr;
  const int rc = noalloc_scratch(&ws);
  if (rc != QB_NOALLOC_OK) return rc;
  // the split kernel writes every (row, head, split) slot it owns before the combine reads it,
  // so the scratch needs no clearing between calls
  return qb::attention_varlen(q, k_cache, v_cache, block_table, max_blocks, positions, seg_lane, cu, num_segments,
                              num_rows, nq, nkv, head_dim, block_size, splits, ws, out, stream);
}
