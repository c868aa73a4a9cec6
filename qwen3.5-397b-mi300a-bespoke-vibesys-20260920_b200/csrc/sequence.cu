// Sequence kernels over varlen batches of segments (a segment = consecutive rows of one lane):
//   causal_conv_varlen   depthwise causal conv (kernel 4) + SiLU, continuing the lane's window
//   gated_delta_varlen   gated delta rule with the DeltaNet glue fused in (beta, g, q/k l2norm,
//                        key-head repeat), continuing and updating the lane's fp32 state
//   attention_varlen     causal GQA attention over the paged KV cache, split-K (flash-decoding)
// Rounding follows the HuggingFace modeling code (see elementwise.cu).
#include "common.cuh"
#include "bounds.cuh"
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
// Output kernel: one thread per (channel, run of CONV_RUN consecutive tokens); the thread keeps
// the K-1 previous inputs in registers, so every input is read once, and takes the K-1 inputs
// before a segment's first token from the lane's saved window. State kernel (launched after): the
// window becomes the last K-1 inputs of the segment (old window entries when the segment is
// shorter).
constexpr int CONV_RUN = 16;

template <int K>
__global__ void conv_out_kernel(const bf16* x, long ldx, const bf16* state, long lane_stride, const bf16* w,
                                const int* seg_lane, const int* cu, int S, int C, bf16* out, int lanes) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int T = cu[S];
  const int tb = blockIdx.y * CONV_RUN;
  if (c >= C || tb >= T) return;  // rows past the last segment: padding of a fixed-size batch
  const int te = min(T, tb + CONV_RUN);
  float wk[K];
#pragma unroll
  for (int j = 0; j < K; ++j) wk[j] = __bfloat162float(w[(long)c * K + j]);
  int s = seg_of(cu, S, tb);
  int t0 = cu[s], t1 = cu[s + 1];
  // win[i]: the input at row t - (K-1) + i for the current t
  float win[K - 1];
  auto load_window = [&](int t) -> bool {
    const int ln = seg_lane[s];
    if (!bounds_ok(BS_LANE, ln, lanes)) return false;
    const bf16* st = state + (long)ln * lane_stride + (long)c * (K - 1);
#pragma unroll
    for (int i = 0; i < K - 1; ++i) {
      const int src = t - (K - 1) + i;
      win[i] = src >= t0 ? __bfloat162float(x[(long)src * ldx + c]) : __bfloat162float(st[src - t0 + K - 1]);
    }
    return true;
  };
  if (!load_window(tb)) return;
  // every input of the run in flight at once (the loop below then only waits for the first)
  float xs[CONV_RUN];
#pragma unroll
  for (int i = 0; i < CONV_RUN; ++i) xs[i] = tb + i < te ? __bfloat162float(x[(long)(tb + i) * ldx + c]) : 0.f;
#pragma unroll
  for (int i = 0; i < CONV_RUN; ++i) {
    const int t = tb + i;
    if (t >= te) break;
    if (t >= t1) {  // the next (non-empty) segment starts: its window comes from its lane's state
      while (t >= t1) {
        ++s;
        t0 = t1;
        t1 = cu[s + 1];
      }
      if (!load_window(t)) return;
    }
    const float xt = xs[i];
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < K - 1; ++j) acc += wk[j] * win[j];
    acc += wk[K - 1] * xt;
    const float a = rbf2(acc);
    out[(long)t * C + c] = __float2bfloat16(a / (1.f + expf(-a)));
#pragma unroll
    for (int q = 0; q < K - 2; ++q) win[q] = win[q + 1];
    win[K - 2] = xt;
  }
}

template <int K>
__global__ void conv_state_kernel(const bf16* x, long ldx, bf16* state, long lane_stride, const int* seg_lane,
                                  const int* cu, int C, int lanes) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int s = blockIdx.y;
  if (c >= C) return;
  if (!bounds_ok(BS_LANE, seg_lane[s], lanes)) return;
  const int t0 = cu[s], len = cu[s + 1] - cu[s];
  bf16* st = state + (long)seg_lane[s] * lane_stride + (long)c * (K - 1);
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {  // ascending: reads index len + i > i before it is overwritten
    const int src = len + i;       // position in [window(K-1) | segment(len)]
    st[i] = src < K - 1 ? st[src] : x[(long)(t0 + src - (K - 1)) * ldx + c];
  }
}

int causal_conv_varlen_t(const void* x, long ldx, void* state, long lane_stride, const void* w, const int* seg_lane,
                         const int* cu, int S, int T, int C, int K, void* out, bool commit, int lanes,
                         cudaStream_t s) {
  if (!S || !T) return 0;
  if (K != 4) return -1;
  conv_out_kernel<4><<<dim3((C + 127) / 128, (T + CONV_RUN - 1) / CONV_RUN), 128, 0, s>>>(
      (const bf16*)x, ldx, (const bf16*)state, lane_stride, (const bf16*)w, seg_lane, cu, S, C, (bf16*)out, lanes);
  if (commit)
    conv_state_kernel<4><<<dim3((C + 127) / 128, S), 128, 0, s>>>((const bf16*)x, ldx, (bf16*)state, lane_stride,
                                                                   seg_lane, cu, C, lanes);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ gated delta rule
// Prep kernel (parallel over tokens): per key head the l2-normalised q (times dk**-0.5) and k in
// fp32, computed with the bf16 rounding points of the HF code; per value head the decay
// exp(g) and beta. Recurrence kernel: grid (value head, segment, column block of 32); four
// threads share one state column (32 rows each), so per token a thread does ~32-wide dot
// products and two 2-step shuffle reductions. Tokens are staged in shared memory in chunks.
__global__ void __launch_bounds__(256) delta_prep_kernel(const bf16* qkv, long ldqkv, const bf16* ab, long ldab, const float* a_log,
                                  const float* dt_bias, int nk, int nv, int dk, float* qn, float* kn, float* gb) {
  const int t = blockIdx.x;
  const int warps = blockDim.x / 32, w = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bf16* row = qkv + (long)t * ldqkv;
  const float scale = rsqrtf((float)dk);
  for (int hh = w; hh < 2 * nk; hh += warps) {  // q heads then k heads
    const bool isq = hh < nk;
    const int h = isq ? hh : hh - nk;
    const bf16* src = row + (isq ? 0 : (long)nk * dk) + (long)h * dk;
    float ss = 0.f;
    for (int i = lane; i < dk; i += 32) {
      const float v = __bfloat162float(src[i]);
      ss += rbf2(v * v);
    }
    ss = warp_sum(ss);
    const float inv = rbf2(rsqrtf(rbf2(rbf2(ss) + 1e-6f)));
    float* dst = (isq ? qn : kn) + ((long)t * nk + h) * dk;
    for (int i = lane; i < dk; i += 32) {
      const float v = rbf2(__bfloat162float(src[i]) * inv);
      dst[i] = isq ? v * scale : v;
    }
  }
  for (int h = threadIdx.x; h < nv; h += blockDim.x) {  // per value head: (decay, beta, log decay, 0)
    const float b = __bfloat162float(ab[(long)t * ldab + h]);
    const float a = __bfloat162float(ab[(long)t * ldab + nv + h]);
    const float g = -expf(a_log[h]) * softplus(a + dt_bias[h]);
    *reinterpret_cast<float4*>(gb + ((long)t * nv + h) * 4) = make_float4(expf(g), rbf2(1.f / (1.f + expf(-b))), g, 0.f);
  }
}

constexpr int DR_CT = 16;  // tokens staged per chunk
constexpr int DR_TPC = 4;  // threads per state column

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Token recurrence. Tokens are staged in chunks of DR_CT through two shared-memory buffers filled
// by 16-byte cp.async copies: chunk c+1 is in flight while chunk c is computed.
template <int DK>
__global__ void __launch_bounds__(128) delta_rec_kernel(const float* qn, const float* kn, const float* gb,
                                                        const bf16* qkv, long ldqkv, float* state, long lane_stride,
                                                        const int* seg_lane, const int* cu, int nk, int nv, int dv,
                                                        bf16* out, int commit) {
  constexpr int COLS = 128 / DR_TPC;  // state columns per CTA
  constexpr int PART = DK / DR_TPC;   // rows per thread
  constexpr int PST = PART + 4;       // padded part stride (floats; 16-byte multiple): parts in different banks
  static_assert((PST * 4) % 16 == 0 && PART % 4 == 0, "16-byte staging");
  __shared__ __align__(16) float qs[2][DR_CT][DR_TPC * PST];
  __shared__ __align__(16) float ks[2][DR_CT][DR_TPC * PST];
  __shared__ __align__(16) bf16 vs[2][DR_CT][COLS];
  __shared__ __align__(16) float gs[2][DR_CT][4];
  const int h = blockIdx.x, s = blockIdx.y, cb = blockIdx.z;
  const int tid = threadIdx.x;
  const int col = tid / DR_TPC, part = tid % DR_TPC;
  const int j = cb * COLS + col;  // state column (value dim)
  const int lane = seg_lane[s];
  const int hk = h / (nv / nk);
  float* st = state + (long)lane * lane_stride + (long)h * DK * dv;
  const bool active = j < dv;
  // v rows by 16-byte cp.async when the column block is whole and the rows are 16-byte aligned
  const bool vfull = cb * COLS + COLS <= dv && (ldqkv % 8) == 0 && (reinterpret_cast<uintptr_t>(qkv) % 16) == 0;
  float S[PART];
#pragma unroll
  for (int i = 0; i < PART; ++i) S[i] = active ? st[(long)(part * PART + i) * dv + j] : 0.f;
  const int t0 = cu[s], t1 = cu[s + 1];
  auto stage = [&](int buf, int c0) {  // issue the copies of tokens [c0, c0 + n) into buffer `buf`
    const int n = min(DR_CT, t1 - c0);
    constexpr int QV = DK / 4;  // 16-byte pieces per q (or k) row
    for (int idx = tid; idx < n * QV; idx += blockDim.x) {
      const int tt = idx / QV, i4 = (idx % QV) * 4;
      const long base = ((long)(c0 + tt) * nk + hk) * DK + i4;
      const int off = (i4 / PART) * PST + i4 % PART;
      cp_async16(&qs[buf][tt][off], qn + base);
      cp_async16(&ks[buf][tt][off], kn + base);
    }
    if (vfull) {
      constexpr int VV = COLS / 8;  // 16-byte pieces of one token's v slice
      for (int idx = tid; idx < n * VV; idx += blockDim.x) {
        const int tt = idx / VV, c8 = (idx % VV) * 8;
        cp_async16(&vs[buf][tt][c8], qkv + (long)(c0 + tt) * ldqkv + 2L * nk * DK + (long)h * dv + cb * COLS + c8);
      }
    } else {
      for (int idx = tid; idx < n * COLS; idx += blockDim.x) {
        const int tt = idx / COLS, cc = idx % COLS;
        const int jj = cb * COLS + cc;
        vs[buf][tt][cc] = jj < dv ? qkv[(long)(c0 + tt) * ldqkv + 2L * nk * DK + (long)h * dv + jj]
                                  : __float2bfloat16(0.f);
      }
    }
    for (int tt = tid; tt < n; tt += blockDim.x) cp_async16(&gs[buf][tt][0], gb + ((long)(c0 + tt) * nv + h) * 4);
    cp_async_commit();
  };
  if (t0 < t1) stage(0, t0);
  int buf = 0;
  for (int c0 = t0; c0 < t1; c0 += DR_CT, buf ^= 1) {
    const int n = min(DR_CT, t1 - c0);
    if (c0 + DR_CT < t1) {
      stage(buf ^ 1, c0 + DR_CT);  // the next chunk lands while this one is computed
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    for (int tt = 0; tt < n; ++tt) {
      const float* kp = &ks[buf][tt][part * PST];
      const float* qp = &qs[buf][tt][part * PST];
      const float decay = gs[buf][tt][0], beta = gs[buf][tt][1];
      float kv4[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums: short dependency chains
#pragma unroll
      for (int i = 0; i < PART; i += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(kp + i);
        kv4[0] += S[i] * k4.x;
        kv4[1] += S[i + 1] * k4.y;
        kv4[2] += S[i + 2] * k4.z;
        kv4[3] += S[i + 3] * k4.w;
      }
      float kv = (kv4[0] + kv4[1]) + (kv4[2] + kv4[3]);
#pragma unroll
      for (int o = 1; o < DR_TPC; o <<= 1) kv += __shfl_xor_sync(0xffffffff, kv, o);
      const float delta = (__bfloat162float(vs[buf][tt][col]) - decay * kv) * beta;
      float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < PART; i += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(kp + i);
        const float4 q4 = *reinterpret_cast<const float4*>(qp + i);
        S[i] = S[i] * decay + k4.x * delta;
        S[i + 1] = S[i + 1] * decay + k4.y * delta;
        S[i + 2] = S[i + 2] * decay + k4.z * delta;
        S[i + 3] = S[i + 3] * decay + k4.w * delta;
        o4[0] += S[i] * q4.x;
        o4[1] += S[i + 1] * q4.y;
        o4[2] += S[i + 2] * q4.z;
        o4[3] += S[i + 3] * q4.w;
      }
      float o = (o4[0] + o4[1]) + (o4[2] + o4[3]);
#pragma unroll
      for (int of = 1; of < DR_TPC; of <<= 1) o += __shfl_xor_sync(0xffffffff, o, of);
      if (part == 0 && active) out[((long)(c0 + tt) * nv + h) * dv + j] = __float2bfloat16(o);
    }
    __syncthreads();  // buffer `buf` is refilled two chunks later
  }
  if (active && commit) {
#pragma unroll
    for (int i = 0; i < PART; ++i) st[(long)(part * PART + i) * dv + j] = S[i];
  }
}

int delta_prep(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log, const float* dt_bias,
               int T, int nk, int nv, int dk, float* qn, float* kn, float* gb, cudaStream_t s) {
  delta_prep_kernel<<<T, 256, 0, s>>>((const bf16*)qkv, ldqkv, (const bf16*)ab, ldab, a_log, dt_bias, nk, nv, dk,
                                      qn, kn, gb);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ DeltaNet decode (one token per lane)
// The whole token mixer of a DeltaNet layer between its two projections, for a batch in which
// every lane brings one token: causal conv + SiLU of the token's q/k/v channels (continuing and
// shifting the lane's conv window), q/k l2norm, decay and beta, the gated delta step on the fp32
// state, and the gated RMSNorm of the head's output. One CTA per (value head, token), 8 warps;
// warp w holds state rows w, w+8, ... and lane l columns 4l..4l+3 (one float4 per row), so the
// state streams in and out as whole 512-byte rows. The state loads are issued first and overlap
// the conv. The value heads of one key head form a thread-block cluster: all of them read the
// key head's q/k conv window, and after a cluster barrier the first one writes it shifted.
// Rounding points are those of the separate conv, prep, recurrence and norm kernels.
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

template <int DK, int DV>
__global__ void __launch_bounds__(256, 2)
    delta_decode_kernel(const bf16* proj, long ldp, bf16* cstate, long cls, const bf16* cw, const float* a_log,
                        const float* dt_bias, float* state, long sls, const bf16* norm_w, const int* seg_lane, int nk,
                        int nv, float eps, bf16* out) {
  pdl_launch_dependents();  // the next projection (launched as a dependent) may start its prologue
  constexpr int K = 4, RPW = DK / 8;
  static_assert(DV == 128 && DK % 32 == 0, "one float4 of columns per lane");
  __shared__ float qs[DK], ks[DK], vs[DV], os[DV];
  __shared__ __align__(16) float red_kv[8][DV];
  __shared__ __align__(16) float red_o[8][DV];
  __shared__ float gsh[2];
  const int h = blockIdx.x, t = blockIdx.y;  // value head, token (one token = one lane's segment)
  const int lane_id = seg_lane[t];
  const int warp = threadIdx.x / 32, l = threadIdx.x % 32;
  const int hk = h / (nv / nk);
  const bool qk_owner = cluster_ctarank() == 0;  // the cluster is this key head's value heads
  float* st = state + (long)lane_id * sls + (long)h * DK * DV;
  float4 S[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) S[r] = *reinterpret_cast<const float4*>(st + (long)(warp + 8 * r) * DV + 4 * l);

  const bf16* row = proj + (long)t * ldp;
  bf16* cs = cstate + (long)lane_id * cls;
  const int C = 2 * nk * DK + nv * DV;
  // causal conv (K = 4) of channel c: the K-1 saved inputs then this token, SiLU of the bf16 sum
  auto conv = [&](int c, bf16 (&win)[K]) -> float {
    const bf16* sc = cs + (long)c * (K - 1);
    const bf16* wc = cw + (long)c * K;
    win[0] = sc[0];
    win[1] = sc[1];
    win[2] = sc[2];
    win[3] = row[c];
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) acc += __bfloat162float(wc[j]) * __bfloat162float(win[j]);
    const float a = rbf2(acc);
    return __bfloat162float(__float2bfloat16(a / (1.f + expf(-a))));
  };
  bf16 qkwin[DK / 32][K];  // warps 0/1: this lane's q/k channels' windows (written by the owner)
  bf16 vwin[K];
  if (warp < 2) {  // l2-normalised q (times dk^-0.5) or k of key head hk
    const bool isq = warp == 0;
    const int c0 = (isq ? 0 : nk * DK) + hk * DK;
    float v[DK / 32], ss = 0.f;
#pragma unroll
    for (int m = 0; m < DK / 32; ++m) {
      v[m] = conv(c0 + l + 32 * m, qkwin[m]);
      ss += rbf2(v[m] * v[m]);
    }
    ss = warp_sum(ss);
    const float inv = rbf2(rsqrtf(rbf2(rbf2(ss) + 1e-6f)));
    const float scale = rsqrtf((float)DK);
#pragma unroll
    for (int m = 0; m < DK / 32; ++m) {
      const float y = rbf2(v[m] * inv);
      if (isq) qs[l + 32 * m] = y * scale; else ks[l + 32 * m] = y;
    }
  } else if (warp < 6) {  // v channels of value head h
    const int j = (warp - 2) * 32 + l;
    vs[j] = conv(2 * nk * DK + h * DV + j, vwin);
  } else if (warp == 6 && l == 0) {
    const float b = __bfloat162float(row[C + nv * DV + h]);
    const float a = __bfloat162float(row[C + nv * DV + nv + h]);
    const float g = -expf(a_log[h]) * softplus(a + dt_bias[h]);
    gsh[0] = expf(g);
    gsh[1] = rbf2(1.f / (1.f + expf(-b)));
  }
  cluster_arrive_release();  // this CTA has read the shared q/k windows
  __syncthreads();
  const float decay = gsh[0], beta = gsh[1];
  // kv = S^T k over this warp's rows, then across warps
  float4 kp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const float k = ks[warp + 8 * r];
    kp.x += S[r].x * k;
    kp.y += S[r].y * k;
    kp.z += S[r].z * k;
    kp.w += S[r].w * k;
  }
  *reinterpret_cast<float4*>(&red_kv[warp][4 * l]) = kp;
  __syncthreads();
  float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const float4 p = *reinterpret_cast<const float4*>(&red_kv[w][4 * l]);
    kv.x += p.x;
    kv.y += p.y;
    kv.z += p.z;
    kv.w += p.w;
  }
  const float4 vv = *reinterpret_cast<const float4*>(&vs[4 * l]);
  const float4 dl = make_float4((vv.x - decay * kv.x) * beta, (vv.y - decay * kv.y) * beta,
                                (vv.z - decay * kv.z) * beta, (vv.w - decay * kv.w) * beta);
  float4 op = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const float k = ks[warp + 8 * r], q = qs[warp + 8 * r];
    S[r].x = S[r].x * decay + k * dl.x;
    S[r].y = S[r].y * decay + k * dl.y;
    S[r].z = S[r].z * decay + k * dl.z;
    S[r].w = S[r].w * decay + k * dl.w;
    op.x += S[r].x * q;
    op.y += S[r].y * q;
    op.z += S[r].z * q;
    op.w += S[r].w * q;
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) *reinterpret_cast<float4*>(st + (long)(warp + 8 * r) * DV + 4 * l) = S[r];
  *reinterpret_cast<float4*>(&red_o[warp][4 * l]) = op;
  __syncthreads();
  if (warp == 0) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float4 p = *reinterpret_cast<const float4*>(&red_o[w][4 * l]);
      o.x += p.x;
      o.y += p.y;
      o.z += p.z;
      o.w += p.w;
    }
    os[4 * l] = rbf2(o.x);  // the recurrence's output is bf16
    os[4 * l + 1] = rbf2(o.y);
    os[4 * l + 2] = rbf2(o.z);
    os[4 * l + 3] = rbf2(o.w);
    __syncwarp();
    // gated RMSNorm over the head (same order as the separate norm kernel)
    float ss = 0.f;
    for (int i = l; i < DV; i += 32) ss += os[i] * os[i];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / DV + eps);
    const bf16* zr = row + C + (long)h * DV;
    bf16* orow = out + ((long)t * nv + h) * DV;
    for (int i = l; i < DV; i += 32) {
      float y = rbf2(os[i] * inv);
      y = rbf2(__bfloat162float(norm_w[i]) * y);
      const float zz = __bfloat162float(zr[i]);
      orow[i] = __float2bfloat16(y * (zz / (1.f + expf(-zz))));
    }
  }
  // conv windows shift by this token: v channels by their own head, q/k after every head of the
  // cluster has read them
  if (warp >= 2 && warp < 6) {
    bf16* sc = cs + (long)(2 * nk * DK + h * DV + (warp - 2) * 32 + l) * (K - 1);
    sc[0] = vwin[1];
    sc[1] = vwin[2];
    sc[2] = vwin[3];
  }
  cluster_wait_acquire();
  if (warp < 2 && qk_owner) {
    const int c0 = (warp == 0 ? 0 : nk * DK) + hk * DK;
#pragma unroll
    for (int m = 0; m < DK / 32; ++m) {
      bf16* sc = cs + (long)(c0 + l + 32 * m) * (K - 1);
      sc[0] = qkwin[m][1];
      sc[1] = qkwin[m][2];
      sc[2] = qkwin[m][3];
    }
  }
}

template <int DK, int DV>
__global__ void __launch_bounds__(256, 3)
    delta_decode_sm_kernel(const bf16* proj, long ldp, bf16* cstate, long cls, const bf16* cw, const float* a_log,
                        const float* dt_bias, float* state, long sls, const bf16* norm_w, const int* seg_lane, int nk,
                        int nv, float eps, bf16* out, int* err) {
  pdl_launch_dependents();  // the next projection (launched as a dependent) may start its prologue
  constexpr int K = 4, RPW = DK / 8;
  static_assert(DV == 128 && DK % 32 == 0, "one float4 of columns per lane");
  __shared__ float qs[DK], ks[DK], vs[DV], os[DV];
  __shared__ __align__(16) float red_kv[8][DV];
  __shared__ __align__(16) float red_o[8][DV];
  __shared__ float gsh[2];
  const int h = blockIdx.x, t = blockIdx.y;  // value head, token (one token = one lane's segment)
  const int lane_id = seg_lane[t];
  const int warp = threadIdx.x / 32, l = threadIdx.x % 32;
  const int hk = h / (nv / nk);
  const bool qk_owner = cluster_ctarank() == 0;  // the cluster is this key head's value heads
  float* st = state + (long)lane_id * sls + (long)h * DK * DV;
  // the state [DK][DV] fp32 comes into shared memory by one bulk copy that overlaps the conv
  extern __shared__ __align__(128) uint8_t dsm[];
  float4* S4 = reinterpret_cast<float4*>(dsm);
  __shared__ __align__(8) uint64_t sbar;
  constexpr uint32_t SBYTES = DK * DV * 4;
  if (threadIdx.x == 0) {
    mbar_init(&sbar, 1);
    fence_barrier_init();
    mbar_expect_tx(&sbar, SBYTES);
    bulk_g2s_s(smem_u32(dsm), st, SBYTES, smem_u32(&sbar));
  }

  const bf16* row = proj + (long)t * ldp;
  bf16* cs = cstate + (long)lane_id * cls;
  const int C = 2 * nk * DK + nv * DV;
  // causal conv (K = 4) of channel c: the K-1 saved inputs then this token, SiLU of the bf16 sum
  auto conv = [&](int c, bf16 (&win)[K]) -> float {
    const bf16* sc = cs + (long)c * (K - 1);
    const bf16* wc = cw + (long)c * K;
    win[0] = sc[0];
    win[1] = sc[1];
    win[2] = sc[2];
    win[3] = row[c];
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) acc += __bfloat162float(wc[j]) * __bfloat162float(win[j]);
    const float a = rbf2(acc);
    return __bfloat162float(__float2bfloat16(a / (1.f + expf(-a))));
  };
  bf16 qkwin[DK / 32][K];  // warps 0/1: this lane's q/k channels' windows (written by the owner)
  bf16 vwin[K];
  if (warp < 2) {  // l2-normalised q (times dk^-0.5) or k of key head hk
    const bool isq = warp == 0;
    const int c0 = (isq ? 0 : nk * DK) + hk * DK;
    float v[DK / 32], ss = 0.f;
#pragma unroll
    for (int m = 0; m < DK / 32; ++m) {
      v[m] = conv(c0 + l + 32 * m, qkwin[m]);
      ss += rbf2(v[m] * v[m]);
    }
    ss = warp_sum(ss);
    const float inv = rbf2(rsqrtf(rbf2(rbf2(ss) + 1e-6f)));
    const float scale = rsqrtf((float)DK);
#pragma unroll
    for (int m = 0; m < DK / 32; ++m) {
      const float y = rbf2(v[m] * inv);
      if (isq) qs[l + 32 * m] = y * scale; else ks[l + 32 * m] = y;
    }
  } else if (warp < 6) {  // v channels of value head h
    const int j = (warp - 2) * 32 + l;
    vs[j] = conv(2 * nk * DK + h * DV + j, vwin);
  } else if (warp == 6 && l == 0) {
    const float b = __bfloat162float(row[C + nv * DV + h]);
    const float a = __bfloat162float(row[C + nv * DV + nv + h]);
    const float g = -expf(a_log[h]) * softplus(a + dt_bias[h]);
    gsh[0] = expf(g);
    gsh[1] = rbf2(1.f / (1.f + expf(-b)));
  }
  cluster_arrive_release();  // this CTA has read the shared q/k windows
  __syncthreads();  // also makes the barrier's initialisation visible before anyone waits on it
  const bool have = mbar_wait(&sbar, 0, err, ERR_TMA_WAIT, nullptr);  // the state has arrived
  const float decay = gsh[0], beta = gsh[1];
  // kv = S^T k over this warp's rows, then across warps
  float4 kp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const float k = ks[warp + 8 * r];
    const float4 sv = S4[(warp + 8 * r) * (DV / 4) + l];
    kp.x += sv.x * k;
    kp.y += sv.y * k;
    kp.z += sv.z * k;
    kp.w += sv.w * k;
  }
  *reinterpret_cast<float4*>(&red_kv[warp][4 * l]) = kp;
  __syncthreads();
  float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const float4 p = *reinterpret_cast<const float4*>(&red_kv[w][4 * l]);
    kv.x += p.x;
    kv.y += p.y;
    kv.z += p.z;
    kv.w += p.w;
  }
  const float4 vv = *reinterpret_cast<const float4*>(&vs[4 * l]);
  const float4 dl = make_float4((vv.x - decay * kv.x) * beta, (vv.y - decay * kv.y) * beta,
                                (vv.z - decay * kv.z) * beta, (vv.w - decay * kv.w) * beta);
  float4 op = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const float k = ks[warp + 8 * r], q = qs[warp + 8 * r];
    float4 sv = S4[(warp + 8 * r) * (DV / 4) + l];
    sv.x = sv.x * decay + k * dl.x;
    sv.y = sv.y * decay + k * dl.y;
    sv.z = sv.z * decay + k * dl.z;
    sv.w = sv.w * decay + k * dl.w;
    S4[(warp + 8 * r) * (DV / 4) + l] = sv;
    op.x += sv.x * q;
    op.y += sv.y * q;
    op.z += sv.z * q;
    op.w += sv.w * q;
  }
  // the updated state goes back by one bulk store (generic-proxy writes made visible to it first)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  *reinterpret_cast<float4*>(&red_o[warp][4 * l]) = op;
  __syncthreads();
  if (threadIdx.x == 0 && have) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(st), "r"(smem_u32(dsm)),
                 "r"(SBYTES)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
  if (warp == 0) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float4 p = *reinterpret_cast<const float4*>(&red_o[w][4 * l]);
      o.x += p.x;
      o.y += p.y;
      o.z += p.z;
      o.w += p.w;
    }
    os[4 * l] = rbf2(o.x);  // the recurrence's output is bf16
    os[4 * l + 1] = rbf2(o.y);
    os[4 * l + 2] = rbf2(o.z);
    os[4 * l + 3] = rbf2(o.w);
    __syncwarp();
    // gated RMSNorm over the head (same order as the separate norm kernel)
    float ss = 0.f;
    for (int i = l; i < DV; i += 32) ss += os[i] * os[i];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / DV + eps);
    const bf16* zr = row + C + (long)h * DV;
    bf16* orow = out + ((long)t * nv + h) * DV;
    for (int i = l; i < DV; i += 32) {
      float y = rbf2(os[i] * inv);
      y = rbf2(__bfloat162float(norm_w[i]) * y);
      const float zz = __bfloat162float(zr[i]);
      orow[i] = __float2bfloat16(y * (zz / (1.f + expf(-zz))));
    }
  }
  // conv windows shift by this token: v channels by their own head, q/k after every head of the
  // cluster has read them
  if (warp >= 2 && warp < 6) {
    bf16* sc = cs + (long)(2 * nk * DK + h * DV + (warp - 2) * 32 + l) * (K - 1);
    sc[0] = vwin[1];
    sc[1] = vwin[2];
    sc[2] = vwin[3];
  }
  if (threadIdx.x == 0 && have) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  cluster_wait_acquire();
  if (warp < 2 && qk_owner) {
    const int c0 = (warp == 0 ? 0 : nk * DK) + hk * DK;
#pragma unroll
    for (int m = 0; m < DK / 32; ++m) {
      bf16* sc = cs + (long)(c0 + l + 32 * m) * (K - 1);
      sc[0] = qkwin[m][1];
      sc[1] = qkwin[m][2];
      sc[2] = qkwin[m][3];
    }
  }
}

int deltanet_decode(const void* proj, long ldp, void* conv_state, long cls, const void* conv_w, const float* a_log,
                    const float* dt_bias, float* state, long sls, const void* norm_w, const int* seg_lane, int T,
                    int nk, int nv, int dk, int dv, int K, float eps, void* out, cudaStream_t s, int* err) {
  if (!T) return 0;
  const int rep = nk > 0 ? nv / nk : 0;
  if (dk != 128 || dv != 128 || K != 4 || rep < 1 || rep > 8 || nv % nk) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nv, T);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = rep;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // state path: shared memory by bulk copies from 16 lanes up (3 CTAs per SM keep more state in
  // flight: 0.070 vs 0.079 ms at 32 lanes), registers below (fewer CTAs than slots: the register
  // form's shorter per-CTA latency wins, 0.024 vs 0.027 ms at 8 lanes); QB_DN_DECODE=reg|sm forces
  static const char* mode = getenv("QB_DN_DECODE");
  const bool sm = mode && mode[0] ? mode[0] == 's' : T >= 16;
  if (sm) {
    auto k = delta_decode_sm_kernel<128, 128>;
    static bool attr_set = false;
    if (!attr_set) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 128 * 4);
      attr_set = true;
    }
    cfg.dynamicSmemBytes = 128 * 128 * 4;
    return (int)cudaLaunchKernelEx(&cfg, k, (const bf16*)proj, ldp, (bf16*)conv_state, cls, (const bf16*)conv_w,
                                   a_log, dt_bias, state, sls, (const bf16*)norm_w, seg_lane, nk, nv, eps,
                                   (bf16*)out, err);
  }
  return (int)cudaLaunchKernelEx(&cfg, delta_decode_kernel<128, 128>, (const bf16*)proj, ldp, (bf16*)conv_state, cls,
                                 (const bf16*)conv_w, a_log, dt_bias, state, sls, (const bf16*)norm_w, seg_lane, nk,
                                 nv, eps, (bf16*)out);
}

int gated_delta_varlen_t(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log,
                         const float* dt_bias, float* state, long lane_stride, const int* seg_lane, const int* cu,
                         int S, int T, int nk, int nv, int dk, int dv, float* scratch, void* out, bool commit,
                         cudaStream_t s) {
  if (!S || !T) return 0;
  if (dk % (4 * DR_TPC) || dk > 128) return -1;
  float* qn = scratch;
  float* kn = qn + (long)T * nk * dk;
  float* gb = kn + (long)T * nk * dk;
  delta_prep_kernel<<<T, 256, 0, s>>>((const bf16*)qkv, ldqkv, (const bf16*)ab, ldab, a_log, dt_bias, nk, nv, dk,
                                      qn, kn, gb);
  dim3 grid(nv, S, (dv + 128 / DR_TPC - 1) / (128 / DR_TPC));
#define QB_DREC(DKV)                                                                                          \
  delta_rec_kernel<DKV><<<grid, 128, 0, s>>>(qn, kn, gb, (const bf16*)qkv, ldqkv, state, lane_stride, seg_lane, \
                                             cu, nk, nv, dv, (bf16*)out, commit ? 1 : 0)
  if (dk == 128) QB_DREC(128);
  else if (dk == 64) QB_DREC(64);
  else if (dk == 32) QB_DREC(32);
  else return -1;
#undef QB_DREC
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

namespace qb {
QB_BOUNDS_INSTALL(bounds_install_sequence)
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
      nq % nkv != 0 || nq / nkv > QB_NOALLOC_MAX_GQA_GROUP || (head_dim != 64 && head_dim != 128 && head_dim != 256))
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
