// Chunked gated delta rule for prefill segments (fp32), the chunkwise WY form of Yang et al.,
// "Parallelizing Linear Transformers with the Delta Rule over Sequence Length" (NeurIPS 2024) and
// "Gated Delta Networks" (ICLR 2025).
//
// Recurrence per value head (state S [dk, dv], token t with log decay g_t and beta_t):
//   S~ = exp(g_t) S;  delta_t = beta_t (v_t - S~^T k_t);  S = S~ + k_t delta_t^T;  o_t = S^T q_t.
// With G_t the cumulative log decay inside a chunk of C tokens and S0 the state entering it:
//   (I + A) [U | W] = [diag(beta) V | diag(beta exp(G)) K],  A_ts = beta_t (k_t . k_s) e^(G_t-G_s) (s<t)
//   Delta = U - W S0                      (the chunk's delta_t rows)
//   O     = diag(exp(G)) Q S0 + M Delta,  M_ts = (q_t . k_s) e^(G_t-G_s) (s<=t)
//   S     = exp(G_last) S0 + (diag(exp(G_last - G)) K)^T Delta
// (identities obtained by unrolling the recurrence over the chunk; the forward substitution
// solves the lower-triangular system row by row).
//
// Two kernels: `dn_chunk_prep` (grid: chunk x value head, all chunks at once) builds U, W, M,
// Q exp(G), K exp(G_last - G) and exp(G_last) into a scratch record per (chunk, head);
// `dn_chunk_state` (grid: segment x value head x 32-column slice of the state) walks the
// segment's chunks in order with its state slice in registers. Serial depth: C rows of forward
// substitution (per chunk, in parallel) + T / C state steps, instead of T token steps.
// All arithmetic is fp32 FFMA, as the fp32 reference recurrence.
//
// Reference behaviour: `deltanet_prefill_chunked.py` (the reference's chunked prefill, same
// published algorithm), `model.delta_rule_chunked`.
#include "common.cuh"
#include "kernels.h"

namespace qb {

using bf16 = __nv_bfloat16;

constexpr int DC = 64;  // tokens per chunk

template <int DK, int DV>
struct DcRec {  // scratch record per (chunk, value head), floats
  static constexpr int U = 0;
  static constexpr int W = U + DC * DV;
  static constexpr int QG = W + DC * DK;
  static constexpr int KG = QG + DC * DK;
  static constexpr int M = KG + DC * DK;
  static constexpr int GL = M + DC * DC;
  static constexpr int SIZE = (GL + 1 + 3) / 4 * 4;
};

template <int DK, int DV>
__global__ void __launch_bounds__(256) dn_chunk_prep_kernel(const float* qn, const float* kn, const float* gb,
                                                            const bf16* qkv, long ldqkv, const int* chunks, int nk,
                                                            int nv, float* rec) {
  using R = DcRec<DK, DV>;
  constexpr int KP = DK + 1, XP = DV + DK + 1, AP = DC + 1;
  extern __shared__ float sm[];
  float* Ks = sm;                 // [DC][KP]
  float* Qs = Ks + DC * KP;       // [DC][KP]
  float* X = Qs + DC * KP;        // [DC][XP]: right-hand side, then [U | W]
  float* A = X + DC * XP;         // [DC][AP]
  float* Ms = A + DC * AP;        // [DC][AP]
  float* G = Ms + DC * AP;        // [DC]
  float* beta = G + DC;           // [DC]
  const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int row0 = chunks[c * 3 + 1], rows = chunks[c * 3 + 2];
  const int hk = h / (nv / nk);
  // ---- load the chunk (rows >= `rows` are zero: they change nothing)
  for (int idx = tid; idx < DC * DK; idx += blockDim.x) {
    const int t = idx / DK, i = idx % DK;
    const bool ok = t < rows;
    const long base = ((long)(row0 + t) * nk + hk) * DK + i;
    Ks[t * KP + i] = ok ? kn[base] : 0.f;
    Qs[t * KP + i] = ok ? qn[base] : 0.f;
  }
  if (tid < DC) {
    const bool ok = tid < rows;
    const float4 gr = ok ? *reinterpret_cast<const float4*>(gb + ((long)(row0 + tid) * nv + h) * 4)
                         : make_float4(1.f, 0.f, 0.f, 0.f);
    beta[tid] = gr.y;
    G[tid] = gr.z;
  }
  __syncthreads();
  if (tid == 0) {  // cumulative log decay
    float run = 0.f;
    for (int t = 0; t < DC; ++t) {
      run += G[t];
      G[t] = run;
    }
  }
  __syncthreads();
  // right-hand side [beta_t v_t | beta_t exp(G_t) k_t]
  for (int idx = tid; idx < DC * DV; idx += blockDim.x) {
    const int t = idx / DV, j = idx % DV;
    const float v = t < rows ? __bfloat162float(qkv[(long)(row0 + t) * ldqkv + 2L * nk * DK + (long)h * DV + j]) : 0.f;
    X[t * XP + j] = beta[t] * v;
  }
  for (int idx = tid; idx < DC * DK; idx += blockDim.x) {
    const int t = idx / DK, i = idx % DK;
    X[t * XP + DV + i] = beta[t] * __expf(G[t]) * Ks[t * KP + i];
  }
  // A (strictly lower) and M (lower incl. diagonal): 2 x DC x DC dot products over DK
  for (int idx = tid; idx < DC * DC; idx += blockDim.x) {
    const int t = idx / DC, s = idx % DC;
    float a = 0.f, m = 0.f;
    if (s <= t) {
      const float* kt = Ks + t * KP;
      const float* ks = Ks + s * KP;
      const float* qt = Qs + t * KP;
#pragma unroll 8
      for (int i = 0; i < DK; ++i) {
        a += kt[i] * ks[i];
        m += qt[i] * ks[i];
      }
      const float dec = __expf(G[t] - G[s]);
      a = s < t ? beta[t] * a * dec : 0.f;
      m *= dec;
    }
    A[t * AP + s] = a;
    Ms[t * AP + s] = m;
  }
  __syncthreads();
  // forward substitution, one column of [U | W] per thread: X_t -= sum_{s<t} A_ts X_s
  for (int j = tid; j < DV + DK; j += blockDim.x) {
    for (int t = 1; t < DC; ++t) {
      float x = X[t * XP + j];
      for (int s2 = 0; s2 < t; ++s2) x -= A[t * AP + s2] * X[s2 * XP + j];
      X[t * XP + j] = x;
    }
  }
  __syncthreads();
  // ---- record
  float* r = rec + ((long)c * nv + h) * R::SIZE;
  const int last = rows > 0 ? rows - 1 : 0;
  const float Gl = G[last];
  for (int idx = tid; idx < DC * DV; idx += blockDim.x) r[R::U + idx] = X[(idx / DV) * XP + idx % DV];
  for (int idx = tid; idx < DC * DK; idx += blockDim.x) {
    const int t = idx / DK, i = idx % DK;
    r[R::W + idx] = X[t * XP + DV + i];
    r[R::QG + idx] = Qs[t * KP + i] * __expf(G[t]);
    r[R::KG + idx] = Ks[t * KP + i] * __expf(Gl - G[t]);
  }
  for (int idx = tid; idx < DC * DC; idx += blockDim.x) r[R::M + idx] = Ms[(idx / DC) * AP + idx % DC];
  if (tid == 0) r[R::GL] = __expf(Gl);
}

// One CTA per (segment, value head, VB-column slice of the state). 256 threads: thread (i, hf)
// owns state row i (of DK = 128) for VB/2 columns. Per chunk: Delta = U - W S, O = QG S + M Delta,
// S = gl S + KG^T Delta, with S staged in shared memory for the row-times-state products.
template <int DK, int DV, int VB>
__global__ void __launch_bounds__(256) dn_chunk_state_kernel(const float* rec, const int* chunks,
                                                             const int* seg_chunk0, const int* seg_lane,
                                                             float* state, long lane_stride, int nv, bf16* out,
                                                             int commit) {
  using R = DcRec<DK, DV>;
  static_assert(DK == 128, "two threads per state row");
  constexpr int HALF = VB / 2;
  constexpr int SP = VB + 1;
  __shared__ float Ss[DK * SP];
  __shared__ float Ds[DC * SP];
  const int seg = blockIdx.x, h = blockIdx.y, vb = blockIdx.z;
  const int tid = threadIdx.x;
  const int i = tid >> 1, hf = tid & 1;  // state row, column half
  const int c0 = hf * HALF;
  float* st = state + (long)seg_lane[seg] * lane_stride + (long)h * DK * DV + vb * VB;
  float S[HALF];
#pragma unroll
  for (int j = 0; j < HALF; ++j) S[j] = st[(long)i * DV + c0 + j];
  // output mapping for the [DC x VB] products: thread -> chunk row t, 8 columns
  const int ot = tid % DC, oc = (tid / DC) * (VB / 4);
  for (int c = seg_chunk0[seg]; c < seg_chunk0[seg + 1]; ++c) {
    const float* r = rec + ((long)c * nv + h) * R::SIZE;
    const int row0 = chunks[c * 3 + 1], rows = chunks[c * 3 + 2];
    __syncthreads();
#pragma unroll
    for (int j = 0; j < HALF; ++j) Ss[i * SP + c0 + j] = S[j];
    __syncthreads();
    // Delta[t][:] = U[t][vb cols] - W[t] . S
    {
      float acc[VB / 4];
#pragma unroll
      for (int j = 0; j < VB / 4; ++j) acc[j] = r[R::U + ot * DV + vb * VB + oc + j];
      const float* w = r + R::W + ot * DK;
      for (int k = 0; k < DK; ++k) {
        const float wk = __ldg(w + k);
#pragma unroll
        for (int j = 0; j < VB / 4; ++j) acc[j] -= wk * Ss[k * SP + oc + j];
      }
#pragma unroll
      for (int j = 0; j < VB / 4; ++j) Ds[ot * SP + oc + j] = acc[j];
    }
    __syncthreads();
    // O[t][:] = QG[t] . S + sum_{s<=t} M[t][s] Delta[s]
    {
      float acc[VB / 4];
#pragma unroll
      for (int j = 0; j < VB / 4; ++j) acc[j] = 0.f;
      const float* q = r + R::QG + ot * DK;
      for (int k = 0; k < DK; ++k) {
        const float qk = __ldg(q + k);
#pragma unroll
        for (int j = 0; j < VB / 4; ++j) acc[j] += qk * Ss[k * SP + oc + j];
      }
      const float* m = r + R::M + ot * DC;
      for (int s2 = 0; s2 <= ot; ++s2) {
        const float ms = __ldg(m + s2);
#pragma unroll
        for (int j = 0; j < VB / 4; ++j) acc[j] += ms * Ds[s2 * SP + oc + j];
      }
      if (ot < rows) {
        bf16* o = out + ((long)(row0 + ot) * nv + h) * DV + vb * VB + oc;
#pragma unroll
        for (int j = 0; j < VB / 4; ++j) o[j] = __float2bfloat16(acc[j]);
      }
    }
    // S[i][:] = gl S[i][:] + sum_t KG[t][i] Delta[t][:]
    {
      const float gl = __ldg(r + R::GL);
#pragma unroll
      for (int j = 0; j < HALF; ++j) S[j] *= gl;
      const float* kg = r + R::KG + i;
      for (int t = 0; t < DC; ++t) {
        const float kt = __ldg(kg + t * DK);
#pragma unroll
        for (int j = 0; j < HALF; ++j) S[j] += kt * Ds[t * SP + c0 + j];
      }
    }
  }
  if (commit) {
#pragma unroll
    for (int j = 0; j < HALF; ++j) st[(long)i * DV + c0 + j] = S[j];
  }
}

int gated_delta_chunked(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log,
                        const float* dt_bias, float* state, long lane_stride, const int* seg_lane,
                        const int* chunks, int n_chunks, const int* seg_chunk0, int S, int T, int nk, int nv, int dk,
                        int dv, float* scratch, void* out, bool commit, cudaStream_t s) {
  if (!S || !T) return 0;
  if (dk != 128 || dv != 128) return -1;
  using R = DcRec<128, 128>;
  float* qn = scratch;
  float* kn = qn + (long)T * nk * dk;
  float* gb = kn + (long)T * nk * dk;
  float* rec = gb + (long)T * nv * 4;
  int r = delta_prep(qkv, ldqkv, ab, ldab, a_log, dt_bias, T, nk, nv, dk, qn, kn, gb, s);
  if (r) return r;
  constexpr int KP = 129, XP = 257, AP = DC + 1;
  const int smem = (2 * DC * KP + DC * XP + 2 * DC * AP + 2 * DC) * (int)sizeof(float);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(dn_chunk_prep_kernel<128, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  dn_chunk_prep_kernel<128, 128><<<dim3(n_chunks, nv), 256, smem, s>>>(qn, kn, gb, (const bf16*)qkv, ldqkv, chunks,
                                                                       nk, nv, rec);
  dn_chunk_state_kernel<128, 128, 32><<<dim3(S, nv, dv / 32), 256, 0, s>>>(rec, chunks, seg_chunk0, seg_lane, state,
                                                                          lane_stride, nv, (bf16*)out, commit ? 1 : 0);
  (void)R::SIZE;
  return (int)cudaGetLastError();
}

long gated_delta_chunked_scratch(int T, int n_chunks, int nk, int nv, int dk) {
  return (long)T * (2L * nk * dk + 4L * nv) + (long)n_chunks * nv * DcRec<128, 128>::SIZE;
}

}  // namespace qb
