// Norms, activations, embedding, greedy argmax, router top-k and the attention prologue
// (q/k RMSNorm + partial RoPE + paged KV write). Activations are bf16; every kernel keeps the
// rounding points of the HuggingFace modeling code (an op whose PyTorch statement produces a
// bf16 tensor rounds to bf16 at the same place here), so greedy decoding agrees with it.
#include "common.cuh"
#include "bounds.cuh"
#include "kernels.h"

namespace qb {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16(x)); }

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < NT / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  t = red[0];
  __syncthreads();
  return t;
}

// ------------------------------------------------------------------ rmsnorm / add_rmsnorm
constexpr int NORM_T = 256;
constexpr int NORM_MAXV = 4;  // up to 4 x 8 elements per thread (H <= 8192)

template <bool ADD>
__global__ void __launch_bounds__(NORM_T) norm_kernel(const bf16* x, long ldx, bf16* res, long ldr, const float* w1p,
                                                      bf16* out, long ldo, int H, float eps) {
  pdl_launch_dependents();  // the next projection (launched as a dependent) may start its prologue
  __shared__ float red[32];
  const long r = blockIdx.x;
  const bf16* xr = x + r * ldx;
  bf16* rr = ADD ? res + r * ldr : nullptr;
  float v[NORM_MAXV][8];
  float ss = 0.f;
  const int nvec = H / 8;
#pragma unroll
  for (int i = 0; i < NORM_MAXV; ++i) {
    const int vi = threadIdx.x + i * NORM_T;
    if (vi < nvec) {
      uint4 raw = *reinterpret_cast<const uint4*>(xr + vi * 8);
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
      if (ADD) {
        uint4 rraw = *reinterpret_cast<const uint4*>(rr + vi * 8);
        const bf16* re = reinterpret_cast<const bf16*>(&rraw);
        uint4 o;
        bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          oe[j] = __float2bfloat16(__bfloat162float(re[j]) + __bfloat162float(e[j]));
          v[i][j] = __bfloat162float(oe[j]);
        }
        *reinterpret_cast<uint4*>(rr + vi * 8) = o;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(e[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  const float tot = block_sum<NORM_T>(ss, red);
  const float inv = rsqrtf(tot / H + eps);
  bf16* orow = out + r * ldo;
#pragma unroll
  for (int i = 0; i < NORM_MAXV; ++i) {
    const int vi = threadIdx.x + i * NORM_T;
    if (vi < nvec) {
      uint4 o;
      bf16* oe = reinterpret_cast<bf16*>(&o);
      const float4 w0 = *reinterpret_cast<const float4*>(w1p + vi * 8);
      const float4 w1 = *reinterpret_cast<const float4*>(w1p + vi * 8 + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) oe[j] = __float2bfloat16(v[i][j] * inv * wv[j]);
      *reinterpret_cast<uint4*>(orow + vi * 8) = o;
    }
  }
}

int rmsnorm(const void* x, long ldx, const float* w1p, void* out, long ldo, int rows, int H, float eps,
            cudaStream_t s) {
  if (H % 8 || H > NORM_T * NORM_MAXV * 8) return -1;
  if (rows == 0) return 0;
  norm_kernel<false><<<rows, NORM_T, 0, s>>>((const bf16*)x, ldx, nullptr, 0, w1p, (bf16*)out, ldo, H, eps);
  return (int)cudaGetLastError();
}

int add_rmsnorm(const void* x, long ldx, void* res, long ldr, const float* w1p, void* out, long ldo, int rows, int H,
                float eps, cudaStream_t s) {
  if (H % 8 || H > NORM_T * NORM_MAXV * 8) return -1;
  if (rows == 0) return 0;
  norm_kernel<true><<<rows, NORM_T, 0, s>>>((const bf16*)x, ldx, (bf16*)res, ldr, w1p, (bf16*)out, ldo, H, eps);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ gated rmsnorm (DeltaNet)
// One warp per (token, head): y = bf16(w * bf16(norm(x))) * silu(z), rounded to bf16.
__global__ void gated_rmsnorm_kernel(const bf16* core, const bf16* z, long ldz, const bf16* w, bf16* out, int T,
                                     int heads, int dv, float eps) {
  pdl_launch_dependents();  // the next projection (launched as a dependent) may start its prologue
  const long gw = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= (long)T * heads) return;
  const long t = gw / heads;
  const int h = gw % heads;
  const bf16* xr = core + gw * dv;
  const bf16* zr = z + t * ldz + (long)h * dv;
  float ss = 0.f;
  for (int i = lane; i < dv; i += 32) {
    float v = __bfloat162float(xr[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / dv + eps);
  bf16* orow = out + gw * dv;
  for (int i = lane; i < dv; i += 32) {
    float y = rbf(__bfloat162float(xr[i]) * inv);
    y = rbf(__bfloat162float(w[i]) * y);
    float zz = __bfloat162float(zr[i]);
    orow[i] = __float2bfloat16(y * (zz / (1.f + expf(-zz))));
  }
}

int gated_rmsnorm(const void* core, const void* z, long ldz_row, const void* w, void* out, int T, int heads, int dv,
                  float eps, cudaStream_t s) {
  const long warps = (long)T * heads;
  if (!warps) return 0;
  gated_rmsnorm_kernel<<<(warps + 7) / 8, 256, 0, s>>>((const bf16*)core, (const bf16*)z, ldz_row, (const bf16*)w,
                                                       (bf16*)out, T, heads, dv, eps);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ small elementwise ops
__global__ void silu_mul_kernel(const bf16* gu, long ldg, bf16* out, long ldo, int T, int n) {
  pdl_launch_dependents();  // the next projection (launched as a dependent) may start its prologue
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * n) return;
  const long t = i / n;
  const int c = i % n;
  const float g = __bfloat162float(gu[t * ldg + c]), u = __bfloat162float(gu[t * ldg + n + c]);
  // HF: act_fn(gate) (bf16) * up (bf16)
  out[t * ldo + c] = __float2bfloat16(rbf(g / (1.f + expf(-g))) * u);
}

int silu_mul(const void* gu, long ldg, void* out, long ldo, int T, int n, cudaStream_t s) {
  const long tot = (long)T * n;
  if (!tot) return 0;
  silu_mul_kernel<<<(tot + 255) / 256, 256, 0, s>>>((const bf16*)gu, ldg, (bf16*)out, ldo, T, n);
  return (int)cudaGetLastError();
}

__global__ void embed_kernel(const int64_t* tok, const bf16* table, bf16* out, int H, long V) {
  const long t = blockIdx.x;
  const int64_t id = tok[t];
  if (!bounds_ok(BS_EMBED_TOKEN, id, V)) return;
  const uint4* src = reinterpret_cast<const uint4*>(table + id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

int embed(const int64_t* tok, const void* table, void* out, int T, int H, long V, cudaStream_t s) {
  if (!T) return 0;
  if (H % 8) return -1;
  embed_kernel<<<T, 128, 0, s>>>(tok, (const bf16*)table, (bf16*)out, H, V);
  return (int)cudaGetLastError();
}

template <typename T>
__global__ void argmax_kernel(const T* x, long ldx, int V, float* val, int64_t* idx) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const long r = blockIdx.x;
  const T* row = x + r * ldx;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float v = to_f<T>(row[i]);
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffff, bv, o);
    int oi = __shfl_xor_sync(0xffffffff, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int j = 1; j < blockDim.x / 32; ++j)
      if (sv[j] > bv || (sv[j] == bv && si[j] < bi)) {
        bv = sv[j];
        bi = si[j];
      }
    val[r] = bv;
    idx[r] = bi;
  }
}

int argmax_rows(const void* x, long ldx, int dtype, int R, int V, float* val, int64_t* idx, cudaStream_t s) {
  if (!R) return 0;
  if (dtype == DT_BF16)
    argmax_kernel<bf16><<<R, 1024, 0, s>>>((const bf16*)x, ldx, V, val, idx);
  else
    argmax_kernel<float><<<R, 1024, 0, s>>>((const float*)x, ldx, V, val, idx);
  return (int)cudaGetLastError();
}

__global__ void sigmoid_gate_mul_kernel(const bf16* x, long ldx, const bf16* g, long ldg, bf16* out, int T, int D) {
  pdl_launch_dependents();  // the next projection (launched as a dependent) may start its prologue
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * D) return;
  const long t = i / D;
  const int c = i % D;
  const float gv = __bfloat162float(g[t * ldg + c]);
  const float sg = rbf(1.f / (1.f + expf(-gv)));
  out[t * D + c] = __float2bfloat16(__bfloat162float(x[t * ldx + c]) * sg);
}

int sigmoid_gate_mul(const void* x, long ldx, const void* g, long ldg, void* out, int T, int D, cudaStream_t s) {
  const long tot = (long)T * D;
  if (!tot) return 0;
  sigmoid_gate_mul_kernel<<<(tot + 255) / 256, 256, 0, s>>>((const bf16*)x, ldx, (const bf16*)g, ldg, (bf16*)out, T,
                                                            D);
  return (int)cudaGetLastError();
}

__global__ void shared_gate_combine_kernel(const bf16* routed, const bf16* shared, const bf16* gl, long ldgl,
                                           bf16* out, int T, int H) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * H) return;
  const long t = i / H;
  const float g = __bfloat162float(gl[t * ldgl]);
  const float sg = rbf(1.f / (1.f + expf(-g)));
  const float sh = rbf(sg * __bfloat162float(shared[i]));
  out[i] = __float2bfloat16(__bfloat162float(routed[i]) + sh);
}

int shared_gate_combine(const void* routed, const void* shared, const void* gl, long ldgl, void* out, int T, int H,
                        cudaStream_t s) {
  const long tot = (long)T * H;
  if (!tot) return 0;
  shared_gate_combine_kernel<<<(tot + 255) / 256, 256, 0, s>>>((const bf16*)routed, (const bf16*)shared,
                                                               (const bf16*)gl, ldgl, (bf16*)out, T, H);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ attention prologue
// One CTA per token. Each warp normalises one head at a time (q heads then k heads):
// RMSNorm(1+w) over head_dim -> bf16, then rotate-half RoPE on the first `rot` dims with the
// HF rounding points (cos/sin rounded to bf16, each product and the sum rounded to bf16).
// k heads and the v heads are written to the paged cache at physical row rows[t].
__global__ void qk_norm_rope_kernel(const bf16* qkv, long ldqkv, int nq, int nkv, int hd, const float* qn,
                                    const float* kn, const int* pos, const int* rows, bf16* kc, bf16* vc, bf16* qout,
                                    int rot, float theta, float eps, long kv_rows) {
  extern __shared__ float sh[];  // [warps][hd] normalised head + [rot/2] cos + [rot/2] sin
  const int t = blockIdx.x;
  const int warps = blockDim.x / 32, w = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int half = rot / 2;
  float* cs = sh + warps * hd;
  float* sn = cs + half;
  const float p = (float)pos[t];
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float inv = 1.0f / powf(theta, (float)(2 * j) / (float)rot);
    const float f = p * inv;
    cs[j] = rbf(cosf(f));
    sn[j] = rbf(sinf(f));
  }
  __syncthreads();
  const bf16* row = qkv + (long)t * ldqkv;
  const long prow = rows[t];
  const bool kv_ok = bounds_ok(BS_KV_ROW, prow, kv_rows);  // debug build: a bad row skips the KV write
  float* buf = sh + w * hd;
  for (int hh = w; hh < nq + nkv; hh += warps) {
    const bool isq = hh < nq;
    const bf16* src = isq ? row + (long)hh * 2 * hd : row + (long)nq * 2 * hd + (long)(hh - nq) * hd;
    const float* wt = isq ? qn : kn;
    float ss = 0.f;
    for (int i = lane; i < hd; i += 32) {
      float v = __bfloat162float(src[i]);
      buf[i] = v;
      ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / hd + eps);
    for (int i = lane; i < hd; i += 32) buf[i] = rbf(buf[i] * inv * wt[i]);
    __syncwarp();
    if (!isq && !kv_ok) continue;
    bf16* dst = isq ? qout + ((long)t * nq + hh) * hd : kc + (prow * nkv + (hh - nq)) * hd;
    for (int i = lane; i < hd; i += 32) {
      float o;
      if (i < rot) {
        const int j = i < half ? i : i - half;
        const float rh = i < half ? -buf[i + half] : buf[i - half];
        o = rbf(rbf(buf[i] * cs[j]) + rbf(rh * sn[j]));
      } else {
        o = buf[i];
      }
      dst[i] = __float2bfloat16(o);
    }
    __syncwarp();
  }
  // values: plain copy into the paged cache
  const bf16* vsrc = row + (long)nq * 2 * hd + (long)nkv * hd;
  bf16* vdst = vc + prow * nkv * hd;
  if (kv_ok)
    for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) vdst[i] = vsrc[i];
}

int qk_norm_rope_kv_write(const void* qkv, long ldqkv, int nq, int nkv, int hd, const float* qn, const float* kn,
                          const int* pos, const int* rows, void* kc, void* vc, void* qout, int T, int rot,
                          float theta, float eps, long kv_rows, cudaStream_t s) {
  if (!T) return 0;
  const int threads = 256, warps = threads / 32;
  const size_t smem = (size_t)(warps * hd + rot) * sizeof(float);
  qk_norm_rope_kernel<<<T, threads, smem, s>>>((const bf16*)qkv, ldqkv, nq, nkv, hd, qn, kn, pos, rows, (bf16*)kc,
                                               (bf16*)vc, (bf16*)qout, rot, theta, eps, kv_rows);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ router softmax + top-k
// One warp per token: fp32 softmax over E experts, k rounds of arg-max (ties -> lower
// expert index), renormalised weights.
// One warp per token row: fp32 softmax over the E router logits, then k rounds of a warp-wide
// argmax (ties to the lower expert id), renormalised. PER = logits per lane (E <= 32 PER) is a
// compile-time count and every loop over it and over the k <= 16 picks is unrolled, so the row
// stays in registers (a runtime-indexed array would live in local memory).
template <int PER>
__global__ void router_topk_kernel(const bf16* logits, long ld, int T, int E, int k, float* wout, int* iout) {
  const long t = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  float p[PER];
  const bf16* row = logits + t * ld;
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? __bfloat162float(row[e]) : -INFINITY;
    m = fmaxf(m, p[i]);
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    p[i] = (lane + 32 * i) < E ? expf(p[i] - m) : 0.f;
    s += p[i];
  }
  s = warp_sum(s);
  const float invs = 1.f / s;
#pragma unroll
  for (int i = 0; i < PER; ++i) p[i] = (lane + 32 * i) < E ? p[i] * invs : -1.f;
  float tw[16];
  int ti[16];
  float tot = 0.f;
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    if (r >= k) break;
    float bv = -2.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (p[i] > bv || (p[i] == bv && e < bi)) {
        bv = p[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffff, bv, o);
      int oi = __shfl_xor_sync(0xffffffff, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    // a row whose probabilities are NaN selects nothing (bi stays out of range): it gets no
    // expert (id -1, weight 0) instead of an index past the array
    const bool found = bi < E;
    tw[r] = found ? bv : 0.f;
    ti[r] = found ? bi : -1;
    tot += tw[r];
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (found && lane + 32 * i == bi) p[i] = -1.f;
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      if (r >= k) break;
      // renormalised weight, rounded through the logits dtype like the reference (.to(bf16))
      wout[t * k + r] = ti[r] >= 0 ? rbf(tw[r] / tot) : 0.f;
      iout[t * k + r] = ti[r];
    }
  }
}

int router_topk(const void* logits, long ld, int T, int E, int k, float* w, int* idx, cudaStream_t s) {
  if (!T) return 0;
  if (E > 1024 || k > 16) return -1;
  const int per = (E + 31) / 32;
  const dim3 grid((T + 7) / 8), block(256);
  if (per <= 1)
    router_topk_kernel<1><<<grid, block, 0, s>>>((const bf16*)logits, ld, T, E, k, w, idx);
  else if (per <= 2)
    router_topk_kernel<2><<<grid, block, 0, s>>>((const bf16*)logits, ld, T, E, k, w, idx);
  else if (per <= 4)
    router_topk_kernel<4><<<grid, block, 0, s>>>((const bf16*)logits, ld, T, E, k, w, idx);
  else if (per <= 8)
    router_topk_kernel<8><<<grid, block, 0, s>>>((const bf16*)logits, ld, T, E, k, w, idx);
  else if (per <= 16)
    router_topk_kernel<16><<<grid, block, 0, s>>>((const bf16*)logits, ld, T, E, k, w, idx);
  else
    router_topk_kernel<32><<<grid, block, 0, s>>>((const bf16*)logits, ld, T, E, k, w, idx);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ clock stamp
// One thread writes %globaltimer (ns) into buf[slot]: a stream-ordered timestamp that also works
// inside a captured CUDA graph, where timing events cannot be recorded (in-graph attribution).
__global__ void stamp_kernel(unsigned long long* buf, int slot) { buf[slot] = globaltimer(); }

int stamp(unsigned long long* buf, int slot, cudaStream_t s) {
  stamp_kernel<<<1, 1, 0, s>>>(buf, slot);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ debug build: canaries
__global__ void canary_check_kernel(const unsigned char* tail, int site) {
  for (int i = threadIdx.x; i < CANARY_BYTES; i += blockDim.x)
    if (tail[i] != CANARY_BYTE) {
#ifdef QB_BOUNDS
      bounds_record(ERR_CANARY, site, i, CANARY_BYTES);
#endif
      return;
    }
}

int canary_check(const void* tail, int site, cudaStream_t s) {
  canary_check_kernel<<<1, 128, 0, s>>>((const unsigned char*)tail, site);
  return (int)cudaGetLastError();
}

QB_BOUNDS_INSTALL(bounds_install_elementwise)

bool bounds_build() {
#ifdef QB_BOUNDS
  return true;
#else
  return false;
#endif
}

}  // namespace qb
