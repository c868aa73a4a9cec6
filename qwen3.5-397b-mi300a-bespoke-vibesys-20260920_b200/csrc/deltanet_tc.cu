// Chunked gated delta rule for prefill segments with the state on the 5th-generation tensor
// cores (tcgen05 + TMEM), for key/value head size 128.
//
// Same chunkwise (WY) identities as deltanet.cu (Yang et al., "Parallelizing Linear Transformers
// with the Delta Rule over Sequence Length", NeurIPS 2024; "Gated Delta Networks", ICLR 2025):
// with G the cumulative log decay inside a chunk of C = 64 tokens and S0 [dk, dv] the state
// entering it,
//   T = (I + A)^-1,  A_ts = beta_t (k_t . k_s) e^(G_t - G_s)  (s < t)
//   U = T diag(beta) V,  W = T diag(beta e^G) K
//   Delta = U - W S0
//   O     = diag(e^G) Q S0 + Mq Delta,     Mq_ts = (q_t . k_s) e^(G_t - G_s)  (s <= t)
//   S     = e^(G_last) S0 + (diag(e^(G_last - G)) K)^T Delta
//
// dn_tc_prep (grid: chunk x key head, every chunk at once, CUDA cores in fp32): the two 64x64
// Gram products once per key head, then for each value head sharing it the decays, the unit
// lower-triangular inverse T in 16 x 16 blocks (diagonal blocks by substitution from registers,
// then three block rows of small products), U and W,
// and a per-(chunk, value head) record in exactly the shared-memory image the
// state kernel's MMAs read: U fp32, then W, Q e^G, Mq (bf16, K-major, 128-byte swizzle) and
// K e^(G_last - G) (bf16, M-major), and e^(G_last).
//
// dn_tc_state (grid: segment x value head x value-column half, 128 threads): walks the segment's chunks in order with
// the fp32 state S in tensor memory (lane = key row, 128 columns). Per chunk, once the chunk's record
// has landed (bulk copies in three parts, each requested for the next chunk as soon as this
// chunk has used its shared-memory region): S is read once (tcgen05.ld) to a bf16 MN-major operand and written back scaled
// by e^(G_last); MMA  D1 = W S;  threads form Delta = U - D1 (bf16 operand);  MMAs
// D2 = (Q e^G) S + Mq Delta  and  S += (K e^(G_last-G))^T Delta  (accumulating in TMEM); threads
// write O = D2. All MMAs are kind::f16 (bf16 operands, fp32 accumulate), M = 128 (the 64-token
// operands are padded with zero rows), N = 128. The serial depth of a segment is its number of
// chunks instead of its number of tokens. Waits are bounded (common.cuh) and every wait is
// followed by a block-wide vote, so all threads leave the chunk loop together and TMEM is
// released on every path (a wait that runs out only leaves the status word set). Any
// copies or MMAs still in flight after such a give-up are drained before the release.
//
// Reference behaviour: `deltanet_prefill_chunked.py` (the reference's chunked prefill, same
// published algorithm, fp32 Triton dots), `model.delta_rule_chunked`.
#include "common.cuh"
#include "kernels.h"

namespace qb {

using bf16 = __nv_bfloat16;

namespace dntc {
constexpr int C = 64;      // tokens per chunk
constexpr int D = 128;     // key and value head size
constexpr int KP = 132;    // fp32 row pitch of the prep kernel's operand tiles
constexpr int AP = 65;     // fp32 row pitch of its 64 x 64 tiles
// record of one (chunk, value head), bytes
constexpr int R_U = 0;            // [64][128] fp32
constexpr int R_EGL = 32768;      // e^(G_last), 16 bytes
constexpr int R_W = 32784;        // 2 K-atoms x [64 rows][128 B]
constexpr int R_QG = R_W + 16384;
constexpr int R_M = R_QG + 16384;  // 1 K-atom x [64 rows][128 B]
constexpr int R_KG = R_M + 8192;   // 2 M-atoms x [64 K-rows][128 B]
constexpr int R_END = R_KG + 16384;
constexpr int REC = (R_END + 127) / 128 * 128;
// state kernel shared memory (offsets from a 1024-byte aligned base)
constexpr int S_W = 0;            // 2 x 16 KB (128-row K-atoms, rows 64..127 zero)
constexpr int S_QG = 32768;
constexpr int S_M = 65536;        // 16 KB (rows 64..127 zero)
constexpr int S_KG = 81920;       // 16 KB
constexpr int S_U = 98304;        // U fp32 + e^(G_last)
constexpr int S_S = 132096;       // S as bf16 MN-major B operand: 2 N-atoms x [128 K-rows][128 B]
constexpr int S_D = 164864;       // Delta as bf16 MN-major B operand: 2 N-atoms x [64 K-rows][128 B]
constexpr int S_BAR = 181248;
constexpr int S_BYTES = S_BAR + 64 + 1024;
constexpr int PP = 3 * 16 + 1;     // fp32 row pitch of the inverse's block-row partial products
constexpr int PREP_SMEM = (3 * C * KP + 4 * C * AP + 3 * C + 16 * PP) * 4;
constexpr int TM_S = 0, TM_D1 = 128, TM_D2 = 256;
}  // namespace dntc

__device__ __forceinline__ uint64_t desc_sw128_mn_dn(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 r;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return r;
}

// byte offset of element chunk `ch` (8 bf16) of row `r` in a 128-byte swizzled atom
__device__ __forceinline__ int swz(int r, int ch) { return r * 128 + ((ch ^ (r & 7)) << 4); }

__global__ void __launch_bounds__(256) dn_tc_prep_kernel(const float* qn, const float* kn, const float* gb,
                                                         const bf16* qkv, long ldqkv, const int* chunks, int nk,
                                                         int nv, int hpc, uint8_t* rec_all) {
  // one CTA per (chunk, key head, group of hpc value heads): the Gram products K K^T and Q K^T
  // depend on the key head only and are computed once for the value heads of the group (all
  // nv / nk of them when the grid has enough CTAs, one per CTA when it would not fill the GPU)
  using namespace dntc;
  extern __shared__ float sm[];
  float* Ks = sm;              // [64][KP]
  float* Qs = Ks + C * KP;     // [64][KP]
  float* Vs = Qs + C * KP;     // [64][KP] (one value head at a time)
  float* Kg = Vs + C * KP;     // [64][AP] raw k_t . k_s
  float* Qg = Kg + C * AP;     // [64][AP] raw q_t . k_s
  float* A = Qg + C * AP;      // [64][AP]
  float* Tm = A + C * AP;      // [64][AP]
  float* G = Tm + C * AP;
  float* Bt = G + C;
  float* EG = Bt + C;
  float* Pb = EG + C;          // [16][PP] block-row partial products of the inverse
  const int c = blockIdx.x, hk = blockIdx.y, tid = threadIdx.x;
  const int row0 = chunks[c * 3 + 1], rows = chunks[c * 3 + 2];
  const int R = nv / nk;
  const int h0 = hk * R + blockIdx.z * hpc;
  // ---- K and Q of the key head (rows >= `rows` are zero: they change nothing); all loads of a
  // thread are issued before its shared-memory stores
  {
    float4 kv[8], qv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = tid + u * 256, t = idx >> 5, i = (idx & 31) * 4;
      kv[u] = qv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t < rows) {
        const long base = ((long)(row0 + t) * nk + hk) * D + i;
        kv[u] = *reinterpret_cast<const float4*>(kn + base);
        qv[u] = *reinterpret_cast<const float4*>(qn + base);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = tid + u * 256, t = idx >> 5, i = (idx & 31) * 4;
      *reinterpret_cast<float4*>(Ks + t * KP + i) = kv[u];
      *reinterpret_cast<float4*>(Qs + t * KP + i) = qv[u];
    }
  }
  __syncthreads();
  // ---- raw Gram products, 4 x 4 outputs per thread
  const int ty = tid >> 4, tx = tid & 15;
  {
    float aa[4][4], mm[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int s = 0; s < 4; ++s) aa[r][s] = mm[r][s] = 0.f;
    for (int i = 0; i < D; i += 4) {
      float4 kt[4], qt[4], ks[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        kt[r] = *reinterpret_cast<const float4*>(Ks + (4 * ty + r) * KP + i);
        qt[r] = *reinterpret_cast<const float4*>(Qs + (4 * ty + r) * KP + i);
        // key rows tx + 16 r: the 8 threads of a quarter warp read 8 distinct 4-bank groups
        ks[r] = *reinterpret_cast<const float4*>(Ks + (tx + 16 * r) * KP + i);
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          aa[r][s] += kt[r].x * ks[s].x + kt[r].y * ks[s].y + kt[r].z * ks[s].z + kt[r].w * ks[s].w;
          mm[r][s] += qt[r].x * ks[s].x + qt[r].y * ks[s].y + qt[r].z * ks[s].z + qt[r].w * ks[s].w;
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        Kg[(4 * ty + r) * AP + tx + 16 * s] = aa[r][s];
        Qg[(4 * ty + r) * AP + tx + 16 * s] = mm[r][s];
      }
  }
  const int last = rows > 0 ? rows - 1 : 0;
  for (int rr = 0; rr < hpc; ++rr) {
    const int h = h0 + rr;
    uint8_t* rec = rec_all + ((long)c * nv + h) * REC;
    __syncthreads();  // the previous value head is done with Vs, A, Tm, G
    // ---- V of this value head, gates
    {
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = tid + u * 256, t = idx >> 4, j = (idx & 15) * 8;
        raw[u] = make_uint4(0, 0, 0, 0);
        if (t < rows)
          raw[u] = *reinterpret_cast<const uint4*>(qkv + (long)(row0 + t) * ldqkv + 2L * nk * D + (long)h * D + j);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = tid + u * 256, t = idx >> 4, j = (idx & 15) * 8;
        const bf16* e = reinterpret_cast<const bf16*>(&raw[u]);
        *reinterpret_cast<float4*>(Vs + t * KP + j) = make_float4(__bfloat162float(e[0]), __bfloat162float(e[1]),
                                                                  __bfloat162float(e[2]), __bfloat162float(e[3]));
        *reinterpret_cast<float4*>(Vs + t * KP + j + 4) = make_float4(__bfloat162float(e[4]), __bfloat162float(e[5]),
                                                                      __bfloat162float(e[6]), __bfloat162float(e[7]));
      }
    }
    if (tid < C) {
      const float4 g4 = tid < rows ? *reinterpret_cast<const float4*>(gb + ((long)(row0 + tid) * nv + h) * 4)
                                   : make_float4(1.f, 0.f, 0.f, 0.f);
      Bt[tid] = g4.y;
      G[tid] = g4.z;
    }
    __syncthreads();
    if (tid < 32) {  // inclusive scan of the log decays, two per lane
      const float a0 = G[2 * tid], a1 = G[2 * tid + 1];
      float s = a0 + a1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, s, o);
        if (tid >= o) s += n;
      }
      const float ex = s - (a0 + a1);
      G[2 * tid] = ex + a0;
      G[2 * tid + 1] = s;
    }
    __syncthreads();
    if (tid < C) EG[tid] = expf(G[tid]);
    // ---- A (strictly lower) into shared memory; Mq (lower incl. diagonal) straight to the record
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = 4 * ty + r;
      float m4[4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int u = 4 * tx + s;
        const float dec = u <= t ? expf(G[t] - G[u]) : 0.f;
        A[t * AP + u] = u < t ? Bt[t] * Kg[t * AP + u] * dec : 0.f;
        m4[s] = u <= t ? Qg[t * AP + u] * dec : 0.f;
      }
      __nv_bfloat162 p0 = __floats2bfloat162_rn(m4[0], m4[1]), p1 = __floats2bfloat162_rn(m4[2], m4[3]);
      uint2 w;
      w.x = *reinterpret_cast<uint32_t*>(&p0);
      w.y = *reinterpret_cast<uint32_t*>(&p1);
      const int u0 = 4 * tx;
      *reinterpret_cast<uint2*>(rec + R_M + swz(t, u0 >> 3) + (u0 & 7) * 2) = w;
    }
    __syncthreads();
    // ---- T = (I + A)^-1 (A strictly lower triangular) in 16 x 16 blocks T_ij:
    //   (1) diagonal blocks D_i = (I + A_ii)^-1 by forward substitution, one thread per (block,
    //       column) holding its column in registers: no barrier inside, depth 15;
    //   (2) block rows i = 1, 2, 3 in order: P_ij = sum_{k=j}^{i-1} A_ik T_kj, then T_ij = -D_i P_ij
    //       (from (I + A) T = I restricted to block row i). Blocks above the diagonal are zero.
    {
      if (tid < 64) {
        const int o = (tid >> 4) * 16, cc = tid & 15;
        float col[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          float acc = t == cc ? 1.f : 0.f;
#pragma unroll
          for (int u = 0; u < t; ++u) acc -= A[(o + t) * AP + o + u] * col[u];
          col[t] = t < cc ? 0.f : acc;
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) Tm[(o + t) * AP + o + cc] = col[t];
      } else {
        // the six blocks above the diagonal: (0,1..3), (1,2..3), (2,3)
        for (int e = tid - 64; e < 6 * 256; e += 192) {
          const int b = e >> 8, r = (e >> 4) & 15, q = e & 15;
          const int bi = b < 3 ? 0 : (b < 5 ? 1 : 2);
          const int bj = b < 3 ? b + 1 : (b < 5 ? b - 1 : 3);
          Tm[(16 * bi + r) * AP + 16 * bj + q] = 0.f;
        }
      }
      const int r = tid >> 4, q = tid & 15;
      for (int bi = 1; bi < 4; ++bi) {
        __syncthreads();  // block rows < bi of T (and the diagonal blocks) are complete
        for (int bj = 0; bj < bi; ++bj) {
          float acc = 0.f;
          for (int k = bj; k < bi; ++k) {
#pragma unroll
            for (int u = 0; u < 16; ++u)
              acc += A[(16 * bi + r) * AP + 16 * k + u] * Tm[(16 * k + u) * AP + 16 * bj + q];
          }
          Pb[r * PP + 16 * bj + q] = acc;
        }
        __syncthreads();
        for (int bj = 0; bj < bi; ++bj) {
          float acc = 0.f;
#pragma unroll
          for (int u = 0; u < 16; ++u) acc += Tm[(16 * bi + r) * AP + 16 * bi + u] * Pb[u * PP + 16 * bj + q];
          Tm[(16 * bi + r) * AP + 16 * bj + q] = -acc;
        }
      }
    }
    __syncthreads();
    // ---- U = T diag(beta) V (fp32 record), W = T diag(beta e^G) K (bf16 K-major image): 8 x 8 per thread
    {
      const int gy = tid >> 5, gx = tid & 31;
      const bool isU = gx < 16;
      const float* src = isU ? Vs + gx * 8 : Ks + (gx - 16) * 8;
      float acc[8][8];
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[r][e] = 0.f;
      for (int s = 0; s < C; ++s) {
        const float sc = isU ? Bt[s] : Bt[s] * EG[s];
        const float4 r0 = *reinterpret_cast<const float4*>(src + s * KP);
        const float4 r1 = *reinterpret_cast<const float4*>(src + s * KP + 4);
        const float rv[8] = {r0.x * sc, r0.y * sc, r0.z * sc, r0.w * sc, r1.x * sc, r1.y * sc, r1.z * sc, r1.w * sc};
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float tv = Tm[(8 * gy + r) * AP + s];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[r][e] += tv * rv[e];
        }
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int t = 8 * gy + r;
        if (isU) {
          float* u = reinterpret_cast<float*>(rec + R_U) + t * D + gx * 8;
          *reinterpret_cast<float4*>(u) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
          *reinterpret_cast<float4*>(u + 4) = make_float4(acc[r][4], acc[r][5], acc[r][6], acc[r][7]);
        } else {
          const int i = (gx - 16) * 8;
          *reinterpret_cast<uint4*>(rec + R_W + (i >> 6) * 8192 + swz(t, (i & 63) >> 3)) = pack8(acc[r]);
        }
      }
    }
    // ---- Q e^G (K-major), K e^(G_last - G) (M-major: the same byte image), e^G_last
    const float Gl = G[last];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = tid + u * 256, t = idx >> 4, ch = idx & 15;
      const float eg = EG[t], ekg = t < rows ? expf(Gl - G[t]) : 0.f;
      float q8[8], k8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        q8[e] = Qs[t * KP + ch * 8 + e] * eg;
        k8[e] = Ks[t * KP + ch * 8 + e] * ekg;
      }
      const int off = (ch >> 3) * 8192 + swz(t, ch & 7);
      *reinterpret_cast<uint4*>(rec + R_QG + off) = pack8(q8);
      *reinterpret_cast<uint4*>(rec + R_KG + off) = pack8(k8);
    }
    if (tid == 0) *reinterpret_cast<float4*>(rec + R_EGL) = make_float4(expf(Gl), 0.f, 0.f, 0.f);
  }
}

template <int NS>
__global__ void __launch_bounds__(128, 1) dn_tc_state_kernel(const uint8_t* rec_all, const int* chunks,
                                                             const int* seg_chunk0, const int* seg_lane, float* state,
                                                             long lane_stride, int nv, bf16* out, int commit, int* err) {
  using namespace dntc;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u - smem_u32(smem_raw));
  // the chunk record arrives in three parts, each with its barrier, so that the next chunk's part
  // is requested as soon as this chunk has used its shared-memory region: W after the first MMA,
  // U and e^(G_last) after Delta, the rest (Q e^G, Mq, K e^(G_last - G)) after the last MMAs
  uint64_t* bar_w = reinterpret_cast<uint64_t*>(base + S_BAR);
  uint64_t* bar_u = bar_w + 1;
  uint64_t* bar_r = bar_w + 2;
  uint64_t* bar_mma = bar_w + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_w + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_w + 5);
  // NS value columns of the state per CTA (blockIdx.z picks which): the columns evolve
  // independently (Delta, O and the update are column-wise in V), so a head can be split over
  // CTAs by value columns; 64 columns are exactly one N-atom of the MN-major operands
  constexpr int NQ = NS / 32;
  const int seg = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5;
  const int col0 = blockIdx.z * NS;
  const int c_begin = seg_chunk0[seg], c_end = seg_chunk0[seg + 1];
  if (c_begin >= c_end) return;
  // zero the pad rows (64..127) of the 64-token A operands, once
  for (int i = tid; i < 8192 / 16; i += 128) {
    const uint4 z = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(base + S_W + 8192)[i] = z;
    reinterpret_cast<uint4*>(base + S_W + 16384 + 8192)[i] = z;
    reinterpret_cast<uint4*>(base + S_QG + 8192)[i] = z;
    reinterpret_cast<uint4*>(base + S_QG + 16384 + 8192)[i] = z;
    reinterpret_cast<uint4*>(base + S_M + 8192)[i] = z;
  }
  if (tid == 0) {
    mbar_init(bar_w, 1);
    mbar_init(bar_u, 1);
    mbar_init(bar_r, 1);
    mbar_init(bar_mma, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_t = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's TMEM lanes
  // ---- initial state: thread tid = key row
  float* st = state + (long)seg_lane[seg] * lane_stride + (long)h * D * D + (long)tid * D + col0;
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(st + 32 * q + i);
      r[i] = __float_as_uint(v.x);
      r[i + 1] = __float_as_uint(v.y);
      r[i + 2] = __float_as_uint(v.z);
      r[i + 3] = __float_as_uint(v.w);
    }
    tmem_st32(lane_t + TM_S + 32 * q, r);
  }
  tmem_wait_st();
  auto rec_of = [&](int c) { return rec_all + ((long)c * nv + h) * REC; };
  auto load_w = [&](int c) {
    const uint32_t bar = smem_u32(bar_w);
    mbar_expect_tx_s(bar, 16384u);
    bulk_g2s_s(base_u + S_W, rec_of(c) + R_W, 8192, bar);
    bulk_g2s_s(base_u + S_W + 16384, rec_of(c) + R_W + 8192, 8192, bar);
  };
  auto load_u = [&](int c) {  // U, then e^(G_last)
    const uint32_t bar = smem_u32(bar_u);
    mbar_expect_tx_s(bar, 32784u);
    bulk_g2s_s(base_u + S_U, rec_of(c) + R_U, 32784, bar);
  };
  auto load_r = [&](int c) {
    const uint32_t bar = smem_u32(bar_r);
    mbar_expect_tx_s(bar, 40960u);
    bulk_g2s_s(base_u + S_QG, rec_of(c) + R_QG, 8192, bar);
    bulk_g2s_s(base_u + S_QG + 16384, rec_of(c) + R_QG + 8192, 8192, bar);
    bulk_g2s_s(base_u + S_M, rec_of(c) + R_M, 8192, bar);
    bulk_g2s_s(base_u + S_KG, rec_of(c) + R_KG, 16384, bar);
  };
  // issue counts (kept by thread 0, which issues every copy and MMA): copies of each record part,
  // MMA groups; `*_done` counts the completions every thread has waited for
  int w_issued = 0, u_issued = 0, r_issued = 0, w_done = 0, u_done = 0, r_done = 0, mma_issued = 0, mma_done = 0;
  if (tid == 0) {
    fence_proxy_async_smem();
    load_u(c_begin);
    load_w(c_begin);
    load_r(c_begin);
    ++u_issued, ++w_issued, ++r_issued;
  }
  const uint32_t idesc = idesc_f16(128, NS, true) | (1u << 16);  // A K-major, B MN-major
  const uint32_t idesc_mn = idesc | (1u << 15);                    // A MN-major too
  uint32_t ph_w = 0, ph_u = 0, ph_r = 0, ph_mma = 0;
  bool ok = true;
  for (int c = c_begin; c < c_end && ok; ++c) {
    const int row0 = chunks[c * 3 + 1], rows = chunks[c * 3 + 2];
    const bool more = c + 1 < c_end;
    // 1. U and e^(G_last) of this chunk have landed
    if (!__syncthreads_and(mbar_wait(bar_u, ph_u, err, ERR_TMA_WAIT, abort_flag))) { ok = false; break; }
    ph_u ^= 1;
    ++u_done;
    // 2. S -> bf16 MN-major operand (row tid), and S *= e^(G_last) in place
    {
      const float egl = *reinterpret_cast<const float*>(base + S_U + R_EGL);
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        float v[32];
        tmem_ld32(lane_t + TM_S + 32 * q, v);
        uint8_t* row = base + S_S + (q >> 1) * 16384 + tid * 128;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int ch = (q & 1) * 4 + k;
          *reinterpret_cast<uint4*>(row + ((ch ^ (tid & 7)) << 4)) = pack8(v + 8 * k);
        }
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i] * egl);
        tmem_st32(lane_t + TM_S + 32 * q, r);
      }
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // 3. D1 = W S (once W has landed)
    if (!__syncthreads_and(mbar_wait(bar_w, ph_w, err, ERR_TMA_WAIT, abort_flag))) { ok = false; break; }
    ph_w ^= 1;
    ++w_done;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + TM_D1, desc_sw128(base_u + S_W + a * 16384) + 2 * kk,
                     desc_sw128_mn_dn(base_u + S_S + (a * 4 + kk) * 2048, 16384), idesc, (a | kk) != 0);
      mma_commit(bar_mma);
      ++mma_issued;
    }
    if (!__syncthreads_and(mbar_wait(bar_mma, ph_mma, err, ERR_MMA_WAIT, abort_flag))) { ok = false; break; }
    ph_mma ^= 1;
    ++mma_done;
    tc_fence_after();
    if (tid == 0 && more) {  // W has been read: the next chunk's W streams in from here on
      fence_proxy_async_smem();
      load_w(c + 1);
      ++w_issued;
    }
    // 4. Delta = U - D1 (token rows 0..63: warps 0 and 1) -> bf16 MN-major operand
    if (warp < 2) {
      const float* u = reinterpret_cast<const float*>(base + S_U) + tid * D + col0;
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        float v[32];
        tmem_ld32(lane_t + TM_D1 + 32 * q, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = u[32 * q + i] - v[i];
        uint8_t* row = base + S_D + (q >> 1) * 8192 + tid * 128;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int ch = (q & 1) * 4 + k;
          *reinterpret_cast<uint4*>(row + ((ch ^ (tid & 7)) << 4)) = pack8(v + 8 * k);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && more) {  // U has been read (every thread passed the barrier): the next U
      fence_proxy_async_smem();
      load_u(c + 1);
      ++u_issued;
    }
    // 5. D2 = (Q e^G) S + Mq Delta;  S += (K e^(G_last - G))^T Delta (once the rest has landed)
    if (!__syncthreads_and(mbar_wait(bar_r, ph_r, err, ERR_TMA_WAIT, abort_flag))) { ok = false; break; }
    ph_r ^= 1;
    ++r_done;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + TM_D2, desc_sw128(base_u + S_QG + a * 16384) + 2 * kk,
                     desc_sw128_mn_dn(base_u + S_S + (a * 4 + kk) * 2048, 16384), idesc, (a | kk) != 0);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss(tmem + TM_D2, desc_sw128(base_u + S_M) + 2 * kk,
                   desc_sw128_mn_dn(base_u + S_D + kk * 2048, 8192), idesc, 1);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss(tmem + TM_S, desc_sw128_mn_dn(base_u + S_KG + kk * 2048, 8192),
                   desc_sw128_mn_dn(base_u + S_D + kk * 2048, 8192), idesc_mn, 1);
      mma_commit(bar_mma);
      ++mma_issued;
    }
    if (!__syncthreads_and(mbar_wait(bar_mma, ph_mma, err, ERR_MMA_WAIT, abort_flag))) { ok = false; break; }
    ph_mma ^= 1;
    ++mma_done;
    tc_fence_after();
    // 6. the rest of the next record streams in while the outputs of this chunk go out
    if (tid == 0 && more) {
      fence_proxy_async_smem();
      load_r(c + 1);
      ++r_issued;
    }
    if (warp < 2) {  // whole warps: tcgen05.ld is warp-collective; only the stores are per row
      bf16* o = out + ((long)(row0 + tid) * nv + h) * D + col0;
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        float v[32];
        tmem_ld32(lane_t + TM_D2 + 32 * q, v);
        if (tid < rows) {
#pragma unroll
          for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4*>(o + 32 * q + 8 * k) = pack8(v + 8 * k);
        }
      }
    }
  }
  // ---- after a give-up: let this CTA's own copies and MMAs in flight finish (bounded) before
  // its shared memory and tensor memory are released
  if (!ok && tid == 0) {
    for (; u_done < u_issued; ++u_done, ph_u ^= 1)
      if (!mbar_wait(bar_u, ph_u, err, ERR_DRAIN, nullptr)) break;
    for (; w_done < w_issued; ++w_done, ph_w ^= 1)
      if (!mbar_wait(bar_w, ph_w, err, ERR_DRAIN, nullptr)) break;
    for (; r_done < r_issued; ++r_done, ph_r ^= 1)
      if (!mbar_wait(bar_r, ph_r, err, ERR_DRAIN, nullptr)) break;
    for (; mma_done < mma_issued; ++mma_done, ph_mma ^= 1)
      if (!mbar_wait(bar_mma, ph_mma, err, ERR_DRAIN, nullptr)) break;
  }
  // ---- final state (fp32) back to the lane
  if (ok && commit) {
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      float v[32];
      tmem_ld32(lane_t + TM_S + 32 * q, v);
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(st + 32 * q + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

long gated_delta_tc_scratch(int T, int n_chunks, int nk, int nv) {
  // floats: qn, kn, gate record, then 128-byte aligned chunk records
  return (long)T * (2L * nk * dntc::D + 4L * nv) + 32 + (long)n_chunks * nv * dntc::REC / 4;
}

int gated_delta_tc(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log, const float* dt_bias,
                   float* state, long lane_stride, const int* seg_lane, const int* chunks, int n_chunks,
                   const int* seg_chunk0, int S, int T, int nk, int nv, int dk, int dv, float* scratch, void* out,
                   bool commit, int* err, cudaStream_t s) {
  using namespace dntc;
  if (!S || !T || !n_chunks) return 0;
  if (dk != D || dv != D || nv % nk || ldqkv % 8) return -1;
  float* qn = scratch;
  float* kn = qn + (long)T * nk * D;
  float* gb = kn + (long)T * nk * D;
  uint8_t* rec = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gb + (long)T * nv * 4) + 127) & ~uintptr_t(127));
  int r = delta_prep(qkv, ldqkv, ab, ldab, a_log, dt_bias, T, nk, nv, dk, qn, kn, gb, s);
  if (r) return r;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(dn_tc_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM);
    cudaFuncSetAttribute(dn_tc_state_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, S_BYTES);
    cudaFuncSetAttribute(dn_tc_state_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, S_BYTES);
    attr = true;
  }
  // value heads per prep CTA: a key head's whole group while that still gives a full wave of
  // CTAs (the Gram products are shared), else one (more CTAs in flight for short segments)
  const int R = nv / nk;
  const int hpc = (long)n_chunks * nk >= 148 ? R : 1;
  dn_tc_prep_kernel<<<dim3(n_chunks, nk, R / hpc), 256, PREP_SMEM, s>>>(qn, kn, gb, (const bf16*)qkv, ldqkv, chunks,
                                                                       nk, nv, hpc, rec);
  // state CTAs: one per (segment, value head), or two per head on 64 value columns each when that
  // packs the waves better (few heads per rank, few segments: the serial chunk walk is latency
  // bound, so half the columns per CTA is close to half the time). QB_DN_VSPLIT = 1 / 2 forces.
  const char* vs_env = getenv("QB_DN_VSPLIT");
  int vsplit = vs_env ? atoi(vs_env) : 0;
  if (vsplit != 1 && vsplit != 2) {
    const long ctas = (long)S * nv, w1 = (ctas + 147) / 148, w2 = (2 * ctas + 147) / 148;
    vsplit = w2 < 2 * w1 ? 2 : 1;
  }
  if (vsplit == 2)
    dn_tc_state_kernel<64><<<dim3(S, nv, 2), 128, S_BYTES, s>>>(rec, chunks, seg_chunk0, seg_lane, state, lane_stride,
                                                                nv, (bf16*)out, commit ? 1 : 0, err);
  else
    dn_tc_state_kernel<128><<<dim3(S, nv, 1), 128, S_BYTES, s>>>(rec, chunks, seg_chunk0, seg_lane, state,
                                                                 lane_stride, nv, (bf16*)out, commit ? 1 : 0, err);
  return (int)cudaGetLastError();
}

}  // namespace qb
