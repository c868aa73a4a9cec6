// PyTorch bindings of the sm_100a kernels. Each function checks shapes/dtypes/devices,
// allocates outputs and scratch through the PyTorch caching allocator (so calls are
// CUDA-graph capturable), and launches on the current stream. Launch failures raise.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGraphsC10Utils.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>
#include <cstring>
#include <string>
#include <vector>
#include <mutex>
#include <unordered_map>

#include "kernels.h"

namespace {

using at::Tensor;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bf16")
std::atomic<long> g_launches{0};  // kernels launched through these bindings (bench evidence)

#define LAUNCH(expr)                                                         \
  do {                                                                       \
    g_launches.fetch_add(1, std::memory_order_relaxed);                      \
    int _rc = (expr);                                                        \
    TORCH_CHECK(_rc == 0, "qwen35_b200 kernel launch failed: ", #expr, " rc=", _rc); \
  } while (0)

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Device status word shared by every kernel with bounded waits (one per device).
Tensor& status_tensor(const at::Device& dev) {
  static std::mutex mu;
  static std::unordered_map<int, Tensor> m;
  std::lock_guard<std::mutex> g(mu);
  auto it = m.find(dev.index());
  if (it == m.end()) {
    it = m.emplace(dev.index(), at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(dev))).first;
    // debug build: the bounds checks of every translation unit record into this word
    c10::cuda::CUDAGuard g(dev.index());
    int* word = it->second.data_ptr<int>();
    TORCH_CHECK(qb::bounds_install_elementwise(word) == 0 && qb::bounds_install_sequence(word) == 0,
                "bounds-check status word install failed");
  }
  return it->second;
}
int* err_ptr(const Tensor& like) { return status_tensor(like.device()).data_ptr<int>(); }

// Scratch buffers: in the debug build (-DQB_BOUNDS) each gets CANARY_BYTES of CANARY_BYTE after
// its end, compared by a check kernel after the launch that used it (bounds.cuh); in the release
// build a plain allocation.
struct Scratch {
  Tensor t;      // the buffer the kernel uses
  Tensor bytes;  // debug build: the allocation including the canary
  long nbytes = 0;
  int site = 0;
};

Scratch scratch_empty(long n, const at::TensorOptions& opt, int site) {
  Scratch sc;
  sc.site = site;
  if (!qb::bounds_build()) {
    sc.t = at::empty({n}, opt);
    return sc;
  }
  sc.nbytes = n * (long)c10::elementSize(c10::typeMetaToScalarType(opt.dtype()));
  sc.bytes = at::empty({sc.nbytes + qb::CANARY_BYTES}, opt.dtype(at::kByte));
  cudaMemsetAsync(sc.bytes.data_ptr<uint8_t>() + sc.nbytes, qb::CANARY_BYTE, qb::CANARY_BYTES, stream());
  sc.t = sc.bytes.narrow(0, 0, sc.nbytes).view(c10::typeMetaToScalarType(opt.dtype()));
  return sc;
}

void scratch_check(const Scratch& sc) {
  if (qb::bounds_build() && sc.bytes.defined()) qb::canary_check(sc.bytes.data_ptr<uint8_t>() + sc.nbytes, sc.site, stream());
}

long row_stride(const Tensor& t) { return t.dim() >= 2 ? t.stride(0) : t.size(-1); }

// ------------------------------------------------------------------ dense
// Stream-K arrival counters: one zeroed array per device, re-armed to zero by the kernel itself,
// so a GEMM (eager or replayed from a graph) needs no memset. GEMMs of one device run on one
// stream in this engine; the array is made on the first call outside a graph capture (the graph
// runner's warm-up), and a call that meets a capture first gets a zeroed array of its own.
Tensor gemm_counters(const Tensor& like, long n) {
  static std::mutex mu;
  static std::unordered_map<int, Tensor> per_dev;
  constexpr long kCounters = 1 << 15;
  const int dev = like.get_device();
  std::lock_guard<std::mutex> lock(mu);
  auto it = per_dev.find(dev);
  if (it != per_dev.end() && n <= kCounters) return it->second;
  const bool capturing = c10::cuda::currentStreamCaptureStatusMayInitCtx() != c10::cuda::CaptureStatus::None;
  if (capturing || n > kCounters) return at::zeros({n}, like.options().dtype(at::kInt));
  Tensor t = at::zeros({kCounters}, like.options().dtype(at::kInt));
  per_dev[dev] = t;
  return t;
}

Tensor linear(Tensor x, Tensor w, c10::optional<Tensor> out) {
  CHECK_CUDA(x);
  CHECK_CUDA(w);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "linear: shape mismatch");
  TORCH_CHECK(x.scalar_type() == w.scalar_type(), "linear: dtype mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "linear: inner dim must be contiguous");
  const bool bf = x.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf || x.scalar_type() == at::kHalf, "linear: bf16/f16 only");
  const int T = x.size(0), N = w.size(0), K = x.size(1);
  Tensor y = out.has_value() ? *out : at::empty({T, N}, x.options());
  TORCH_CHECK(y.stride(1) == 1, "linear: output inner dim must be contiguous");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "linear: row strides must be 16B multiples");
  // stream-K workspace when the tiles do not divide evenly over the SMs (decode projections)
  const long wsf = qb::gemm_split_ws_floats(T, N, K);
  Scratch ws;
  Tensor cnt;
  if (wsf) {
    ws = scratch_empty(wsf, x.options().dtype(at::kFloat), qb::BS_CANARY_GEMM_WS);
    cnt = gemm_counters(x, (long)((N + 127) / 128) * ((T + 15) / 16));
  }
  LAUNCH(qb::gemm_ws(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(), y.stride(0), T, N, K, bf, 0,
                     err_ptr(x), stream(), 0, wsf ? ws.t.data_ptr<float>() : nullptr,
                     wsf ? cnt.data_ptr<int>() : nullptr));
  scratch_check(ws);
  return y;
}

// ------------------------------------------------------------------ norms / glue
Tensor rmsnorm(Tensor x, Tensor w1p, double eps) {
  CHECK_BF16(x);
  const int H = x.size(-1);
  auto x2 = x.reshape({-1, H});
  TORCH_CHECK(x2.stride(1) == 1, "rmsnorm: inner dim must be contiguous");
  Tensor out = at::empty({x2.size(0), H}, x.options());
  LAUNCH(qb::rmsnorm(x2.data_ptr(), x2.stride(0), w1p.data_ptr<float>(), out.data_ptr(), H, x2.size(0), H, (float)eps,
                     stream()));
  return out.view(x.sizes());
}

void add_rmsnorm(Tensor x, Tensor res, Tensor w1p, Tensor out, double eps) {
  CHECK_BF16(x);
  CHECK_BF16(res);
  const int H = x.size(-1);
  TORCH_CHECK(res.is_contiguous() && out.is_contiguous(), "add_rmsnorm: residual/out must be contiguous");
  TORCH_CHECK(x.stride(-1) == 1, "add_rmsnorm: x inner dim contiguous");
  LAUNCH(qb::add_rmsnorm(x.data_ptr(), row_stride(x), res.data_ptr(), H, w1p.data_ptr<float>(), out.data_ptr(), H,
                         res.numel() / H, H, (float)eps, stream()));
}

Tensor gated_rmsnorm(Tensor core, Tensor z, Tensor w, double eps) {
  CHECK_BF16(core);
  TORCH_CHECK(core.is_contiguous() && core.dim() == 3, "gated_rmsnorm: core [T, heads, dv] contiguous");
  TORCH_CHECK(z.dim() == 3 && z.stride(2) == 1 && z.stride(1) == z.size(2), "gated_rmsnorm: z [T, heads, dv] view");
  Tensor out = at::empty_like(core);
  LAUNCH(qb::gated_rmsnorm(core.data_ptr(), z.data_ptr(), z.stride(0), w.data_ptr(), out.data_ptr(), core.size(0),
                           core.size(1), core.size(2), (float)eps, stream()));
  return out;
}

Tensor silu_mul(Tensor gu) {
  CHECK_BF16(gu);
  const int n = gu.size(-1) / 2;
  Tensor out = at::empty({gu.size(0), n}, gu.options());
  LAUNCH(qb::silu_mul(gu.data_ptr(), gu.stride(0), out.data_ptr(), n, gu.size(0), n, stream()));
  return out;
}

Tensor embed(Tensor tok, Tensor table) {
  TORCH_CHECK(tok.scalar_type() == at::kLong, "embed: int64 tokens");
  Tensor out = at::empty({tok.size(0), table.size(1)}, table.options());
  LAUNCH(qb::embed(tok.data_ptr<int64_t>(), table.data_ptr(), out.data_ptr(), tok.size(0), table.size(1),
                         table.size(0), stream()));
  return out;
}

std::tuple<Tensor, Tensor> argmax_rows(Tensor x) {
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "argmax_rows: [R, V] rows contiguous");
  const int dt = x.scalar_type() == at::kBFloat16 ? qb::DT_BF16 : qb::DT_F32;
  TORCH_CHECK(dt == qb::DT_F32 ? x.scalar_type() == at::kFloat : true, "argmax_rows: bf16 or fp32");
  Tensor val = at::empty({x.size(0)}, x.options().dtype(at::kFloat));
  Tensor idx = at::empty({x.size(0)}, x.options().dtype(at::kLong));
  LAUNCH(qb::argmax_rows(x.data_ptr(), x.stride(0), dt, x.size(0), x.size(1), val.data_ptr<float>(),
                         idx.data_ptr<int64_t>(), stream()));
  return {val, idx};
}

Tensor sigmoid_gate_mul(Tensor x, Tensor g) {
  CHECK_BF16(x);
  Tensor out = at::empty({x.size(0), x.size(1)}, x.options());
  LAUNCH(qb::sigmoid_gate_mul(x.data_ptr(), x.stride(0), g.data_ptr(), g.stride(0), out.data_ptr(), x.size(0),
                              x.size(1), stream()));
  return out;
}

Tensor shared_gate_combine(Tensor routed, Tensor shared, Tensor gl) {
  CHECK_BF16(routed);
  TORCH_CHECK(routed.is_contiguous() && shared.is_contiguous(), "shared_gate_combine: contiguous inputs");
  Tensor out = at::empty_like(routed);
  LAUNCH(qb::shared_gate_combine(routed.data_ptr(), shared.data_ptr(), gl.data_ptr(), gl.stride(0), out.data_ptr(),
                                 routed.size(0), routed.size(1), stream()));
  return out;
}

std::tuple<Tensor, Tensor> router_topk2(Tensor logits, int64_t k) {
  CHECK_BF16(logits);
  const int T = logits.size(0), E = logits.size(1);
  Tensor w = at::empty({T, k}, logits.options().dtype(at::kFloat));
  Tensor idx = at::empty({T, k}, logits.options().dtype(at::kInt));
  LAUNCH(qb::router_topk(logits.data_ptr(), logits.stride(0), T, E, k, w.data_ptr<float>(), idx.data_ptr<int>(),
                         stream()));
  return {w, idx};
}

// ------------------------------------------------------------------ attention
Tensor qk_norm_rope_kv_write(Tensor q, Tensor k, Tensor v, Tensor qn, Tensor kn, Tensor pos, Tensor rows, Tensor kc,
                             Tensor vc, int64_t rot, double theta, double eps) {
  CHECK_BF16(q);
  const int T = q.size(0), nq = q.size(1), hd = q.size(2), nkv = k.size(1);
  const auto* base = reinterpret_cast<const char*>(q.data_ptr());
  TORCH_CHECK(T <= 1 || (q.stride(0) == k.stride(0) && k.stride(0) == v.stride(0)),
              "qk_norm_rope: q/k/v must be views of one row");
  TORCH_CHECK(reinterpret_cast<const char*>(k.data_ptr()) == base + (long)nq * 2 * hd * 2 &&
                  reinterpret_cast<const char*>(v.data_ptr()) == base + ((long)nq * 2 * hd + (long)nkv * hd) * 2,
              "qk_norm_rope: expected the fused [q|gate]*nq, k*nkv, v*nkv row layout");
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous(), "qk_norm_rope: caches contiguous");
  Tensor qout = at::empty({T, nq, hd}, q.options());
  LAUNCH(qb::qk_norm_rope_kv_write(q.data_ptr(), q.stride(0), nq, nkv, hd, qn.data_ptr<float>(), kn.data_ptr<float>(),
                                   pos.data_ptr<int>(), rows.data_ptr<int>(), kc.data_ptr(), vc.data_ptr(),
                                   qout.data_ptr(), T, rot, (float)theta, (float)eps, kc.numel() / ((long)nkv * hd),
                                   stream()));
  return qout;
}

Tensor attention_varlen(Tensor q, Tensor kc, Tensor vc, Tensor table, Tensor seg_lane, Tensor cu, Tensor pos,
                        int64_t block_size, int64_t max_ctx) {
  CHECK_BF16(q);
  TORCH_CHECK(q.is_contiguous(), "attention: q contiguous [T, nq, hd]");
  const int T = q.size(0), nq = q.size(1), hd = q.size(2), nkv = kc.size(1);
  const int S = seg_lane.size(0);
  int dev_sms = 148;
  // splits: enough CTAs to fill the GPU twice, at least 64 keys per split
  long base_ctas = (long)T * nkv;
  int splits = (int)((2L * dev_sms + base_ctas - 1) / base_ctas);
  int max_splits = (int)((max_ctx + 63) / 64);
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  if (splits > 64) splits = 64;
  Tensor out = at::empty_like(q);
  Scratch ws;
  if (splits > 1) ws = scratch_empty((long)T * nq * splits * (hd + 2), q.options().dtype(at::kFloat), qb::BS_CANARY_ATTN_WS);
  LAUNCH(qb::attention_varlen(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), table.data_ptr<int>(), table.size(1),
                              pos.data_ptr<int>(), seg_lane.data_ptr<int>(), cu.data_ptr<int>(), S, T, nq, nkv, hd,
                              block_size, splits, splits > 1 ? ws.t.data_ptr<float>() : nullptr, out.data_ptr(),
                              stream()));
  scratch_check(ws);
  if (splits > 1) g_launches.fetch_add(1, std::memory_order_relaxed);  // the split-combine kernel
  return out;
}

Tensor attention_fa(Tensor q, Tensor kc, Tensor vc, Tensor table, Tensor seg_lane, Tensor pos, Tensor tiles,
                    int64_t block_size, int64_t splits) {
  CHECK_BF16(q);
  TORCH_CHECK(q.is_contiguous() && kc.is_contiguous() && vc.is_contiguous(), "attention_fa: contiguous");
  TORCH_CHECK(tiles.dim() == 2 && tiles.size(1) == 3 && tiles.scalar_type() == at::kInt, "attention_fa: tiles [n, 3]");
  const int T = q.size(0), nq = q.size(1), hd = q.size(2), nkv = kc.size(1);
  Tensor out = at::empty_like(q);
  Scratch ws;
  if (splits > 1) ws = scratch_empty((long)T * nq * splits * (hd + 4), q.options().dtype(at::kFloat), qb::BS_CANARY_ATTN_WS);
  LAUNCH(qb::fa_prefill(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.size(0), table.data_ptr<int>(), table.size(1),
                        pos.data_ptr<int>(), seg_lane.data_ptr<int>(), tiles.data_ptr<int>(), tiles.size(0), T, nq,
                        nkv, hd, block_size, (int)splits, splits > 1 ? ws.t.data_ptr<float>() : nullptr,
                        out.data_ptr(), err_ptr(q), stream()));
  scratch_check(ws);
  if (splits > 1) g_launches.fetch_add(1, std::memory_order_relaxed);  // the combine kernel
  return out;
}

// ------------------------------------------------------------------ deltanet
Tensor causal_conv_varlen(Tensor x, Tensor state, Tensor w, Tensor seg_lane, Tensor cu, bool commit) {
  CHECK_BF16(x);
  TORCH_CHECK(state.stride(2) == 1 && state.stride(1) == state.size(2), "conv: state [lanes, C, K-1] rows contiguous");
  const int T = x.size(0), C = x.size(1), K = w.size(1);
  Tensor out = at::empty({T, C}, x.options());
  LAUNCH(qb::causal_conv_varlen_t(x.data_ptr(), x.stride(0), state.data_ptr(), state.stride(0), w.data_ptr(),
                                  seg_lane.data_ptr<int>(), cu.data_ptr<int>(), seg_lane.size(0), T, C, K,
                                  out.data_ptr(), commit, (int)state.size(0), stream()));
  g_launches.fetch_add(1, std::memory_order_relaxed);  // output + state kernels
  return out;
}

Tensor gated_delta_varlen(Tensor qkv, Tensor ab, Tensor a_log, Tensor dt_bias, Tensor state, Tensor seg_lane,
                          Tensor cu, int64_t nk, int64_t nv, int64_t dk, int64_t dv, bool commit) {
  CHECK_BF16(qkv);
  TORCH_CHECK(state.scalar_type() == at::kFloat, "delta: fp32 state");
  TORCH_CHECK(state.stride(3) == 1 && state.stride(2) == dv && state.stride(1) == dk * dv, "delta: state layout");
  const int T = qkv.size(0);
  Tensor out = at::empty({T, nv, dv}, qkv.options());
  Scratch scratch = scratch_empty((long)T * (2 * nk * dk + 4 * nv), qkv.options().dtype(at::kFloat),
                                  qb::BS_CANARY_DN_SCRATCH);
  LAUNCH(qb::gated_delta_varlen_t(qkv.data_ptr(), qkv.stride(0), ab.data_ptr(), ab.stride(0),
                                  a_log.data_ptr<float>(), dt_bias.data_ptr<float>(), state.data_ptr<float>(),
                                  state.stride(0), seg_lane.data_ptr<int>(), cu.data_ptr<int>(), seg_lane.size(0), T,
                                  nk, nv, dk, dv, scratch.t.data_ptr<float>(), out.data_ptr(), commit, stream()));
  scratch_check(scratch);
  g_launches.fetch_add(1, std::memory_order_relaxed);  // prep + recurrence kernels
  return out;
}

Tensor deltanet_decode(Tensor proj, Tensor conv_state, Tensor conv_w, Tensor a_log, Tensor dt_bias, Tensor state,
                       Tensor norm_w, Tensor seg_lane, int64_t nk, int64_t nv, int64_t dk, int64_t dv, double eps) {
  CHECK_BF16(proj);
  TORCH_CHECK(proj.stride(1) == 1, "deltanet_decode: proj rows contiguous");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.stride(3) == 1 && state.stride(2) == dv &&
                  state.stride(1) == dk * dv, "deltanet_decode: fp32 state [lanes, nv, dk, dv]");
  TORCH_CHECK(conv_state.scalar_type() == at::kBFloat16 && conv_state.stride(2) == 1 &&
                  conv_state.stride(1) == conv_state.size(2), "deltanet_decode: conv state [lanes, C, K-1]");
  TORCH_CHECK(conv_w.is_contiguous() && norm_w.is_contiguous() && seg_lane.is_contiguous(), "deltanet_decode: contiguous");
  const int T = proj.size(0);
  TORCH_CHECK(seg_lane.size(0) == T, "deltanet_decode: one token per lane");
  Tensor out = at::empty({T, nv * dv}, proj.options());
  LAUNCH(qb::deltanet_decode(proj.data_ptr(), proj.stride(0), conv_state.data_ptr(), conv_state.stride(0),
                             conv_w.data_ptr(), a_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
                             state.data_ptr<float>(), state.stride(0), norm_w.data_ptr(), seg_lane.data_ptr<int>(), T,
                             nk, nv, dk, dv, conv_w.size(1), (float)eps, out.data_ptr(), stream(), err_ptr(proj)));
  return out;
}

Tensor gated_delta_chunked(Tensor qkv, Tensor ab, Tensor a_log, Tensor dt_bias, Tensor state, Tensor seg_lane,
                           Tensor chunks, Tensor seg_chunk0, int64_t nk, int64_t nv, int64_t dk, int64_t dv,
                           bool commit) {
  CHECK_BF16(qkv);
  TORCH_CHECK(state.scalar_type() == at::kFloat, "delta: fp32 state");
  TORCH_CHECK(state.stride(3) == 1 && state.stride(2) == dv && state.stride(1) == dk * dv, "delta: state layout");
  TORCH_CHECK(chunks.dim() == 2 && chunks.size(1) == 3, "delta: chunks [n, 3]");
  const int T = qkv.size(0), n_chunks = chunks.size(0);
  Tensor out = at::empty({T, nv, dv}, qkv.options());
  Scratch scratch = scratch_empty(qb::gated_delta_chunked_scratch(T, n_chunks, nk, nv, dk),
                                  qkv.options().dtype(at::kFloat), qb::BS_CANARY_DN_SCRATCH);
  LAUNCH(qb::gated_delta_chunked(qkv.data_ptr(), qkv.stride(0), ab.data_ptr(), ab.stride(0), a_log.data_ptr<float>(),
                                 dt_bias.data_ptr<float>(), state.data_ptr<float>(), state.stride(0),
                                 seg_lane.data_ptr<int>(), chunks.data_ptr<int>(), n_chunks,
                                 seg_chunk0.data_ptr<int>(), seg_lane.size(0), T, nk, nv, dk, dv,
                                 scratch.t.data_ptr<float>(), out.data_ptr(), commit, stream()));
  scratch_check(scratch);
  g_launches.fetch_add(2, std::memory_order_relaxed);  // prep + chunk prep + chunk state kernels
  return out;
}

// chunked gated delta rule on tcgen05 (state in TMEM): same contract as gated_delta_chunked
Tensor gated_delta_tc(Tensor qkv, Tensor ab, Tensor a_log, Tensor dt_bias, Tensor state, Tensor seg_lane, Tensor chunks,
                      Tensor seg_chunk0, int64_t nk, int64_t nv, int64_t dk, int64_t dv, bool commit) {
  CHECK_BF16(qkv);
  TORCH_CHECK(state.scalar_type() == at::kFloat, "delta_tc: fp32 state");
  TORCH_CHECK(state.stride(3) == 1 && state.stride(2) == dv && state.stride(1) == dk * dv, "delta_tc: state layout");
  TORCH_CHECK(chunks.dim() == 2 && chunks.size(1) == 3, "delta_tc: chunks [n, 3]");
  TORCH_CHECK(qkv.stride(1) == 1 && qkv.stride(0) % 8 == 0, "delta_tc: qkv rows 16-byte aligned");
  const int T = qkv.size(0), n_chunks = chunks.size(0);
  Tensor out = at::empty({T, nv, dv}, qkv.options());
  Scratch scratch = scratch_empty(qb::gated_delta_tc_scratch(T, n_chunks, nk, nv), qkv.options().dtype(at::kFloat),
                                  qb::BS_CANARY_DN_SCRATCH);
  LAUNCH(qb::gated_delta_tc(qkv.data_ptr(), qkv.stride(0), ab.data_ptr(), ab.stride(0), a_log.data_ptr<float>(),
                            dt_bias.data_ptr<float>(), state.data_ptr<float>(), state.stride(0),
                            seg_lane.data_ptr<int>(), chunks.data_ptr<int>(), n_chunks, seg_chunk0.data_ptr<int>(),
                            seg_lane.size(0), T, nk, nv, dk, dv, scratch.t.data_ptr<float>(), out.data_ptr(), commit,
                            err_ptr(qkv), stream()));
  scratch_check(scratch);
  g_launches.fetch_add(2, std::memory_order_relaxed);  // glue prep + chunk prep + state kernels
  return out;
}

// ------------------------------------------------------------------ moe
Tensor moe_routed_impl(Tensor h, Tensor topw, Tensor topi, Tensor w13, c10::optional<Tensor> s13, Tensor w2,
                       c10::optional<Tensor> s2, int64_t first, int64_t count) {
  CHECK_BF16(h);
  TORCH_CHECK(h.is_contiguous(), "moe: h contiguous");
  const int T = h.size(0), H = h.size(1), k = topi.size(1);
  const bool fp4 = s13.has_value();
  const int n13 = w13.size(1);  // 2I
  const int I = n13 / 2;
  const int cap = T * k;
  auto i32 = h.options().dtype(at::kInt);
  Tensor meta = at::empty({2 * count + 2 * cap + cap + 1}, i32);
  int* counts = meta.data_ptr<int>();
  int* offsets = counts + count;
  int* perm_tok = offsets + count;
  int* perm_slot = perm_tok + cap;
  int* inv = perm_slot + cap;
  int* n_assign = inv + cap;
  Tensor topi_c = topi.contiguous();
  Tensor out = at::empty_like(h);
  if (T == 0) return out;
  LAUNCH(qb::moe_dispatch(topi_c.data_ptr<int>(), T, k, first, count, counts, offsets, perm_tok, perm_slot, inv,
                          n_assign, stream()));
  if (fp4) {
    Tensor xh = at::empty({cap, H}, h.options().dtype(at::kHalf));
    Tensor inter = at::empty({cap, I}, h.options().dtype(at::kHalf));
    Tensor y2 = at::empty({cap, H}, h.options());
    LAUNCH(qb::moe_gather_f16(h.data_ptr(), perm_tok, n_assign, cap, H, xh.data_ptr(), stream()));
    LAUNCH(qb::moe_expert_gemm(xh.data_ptr(), H, w13.data_ptr<uint8_t>(), s13->data_ptr<uint8_t>(), n13, H, 0, 0,
                               offsets, counts, count, cap, 1, inter.data_ptr(), I, err_ptr(h), stream(), 0));
    LAUNCH(qb::moe_expert_gemm(inter.data_ptr(), I, w2.data_ptr<uint8_t>(), s2->data_ptr<uint8_t>(), H, I, 0, 0,
                               offsets, counts, count, cap, 0, y2.data_ptr(), H, err_ptr(h), stream(), 0));
    LAUNCH(qb::moe_combine(y2.data_ptr(), inv, topw.contiguous().data_ptr<float>(), T, k, H, out.data_ptr(), stream()));
  } else {
    // bf16 experts (the MTP layer of the published checkpoint): TMA-fed bf16 weight tiles
    Tensor xh = at::empty({cap, H}, h.options());
    Tensor inter = at::empty({cap, I}, h.options());
    Tensor y2 = at::empty({cap, H}, h.options());
    LAUNCH(qb::moe_gather_bf16(h.data_ptr(), perm_tok, n_assign, cap, H, xh.data_ptr(), stream()));
    LAUNCH(qb::moe_expert_gemm_bf16(xh.data_ptr(), H, w13.data_ptr(), n13, H, 0, offsets, counts, count, cap, 1,
                                    inter.data_ptr(), I, stream()));
    LAUNCH(qb::moe_expert_gemm_bf16(inter.data_ptr(), I, w2.data_ptr(), H, I, 0, offsets, counts, count, cap, 0,
                                    y2.data_ptr(), H, stream()));
    LAUNCH(qb::moe_combine(y2.data_ptr(), inv, topw.contiguous().data_ptr<float>(), T, k, H, out.data_ptr(), stream()));
  }
  return out;
}

Tensor moe_routed_bf16(Tensor h, Tensor topw, Tensor topi, Tensor w13, Tensor w2, int64_t first, int64_t count) {
  return moe_routed_impl(h, topw, topi, w13, c10::nullopt, w2, c10::nullopt, first, count);
}

// Block-scaled path: weights' e8m0 scales pre-arranged in 512-byte chunks (s13c / s2c).
// sparse_rows: many rows are routed nowhere (expert ids -1, an expert-parallel receive area):
// they are neither quantised nor written.
void moe_routed_mx_into(Tensor h, Tensor topw, Tensor topi, Tensor w13, Tensor s13c, Tensor w2, Tensor s2c,
                        int64_t first, int64_t count, bool tiled, Tensor out, bool sparse_rows = false,
                        const c10::optional<Tensor>& shared = c10::nullopt,
                        const c10::optional<Tensor>& gate = c10::nullopt) {
  CHECK_BF16(h);
  TORCH_CHECK(h.is_contiguous() && out.is_contiguous(), "moe: h and out contiguous");
  const int T = h.size(0), H = h.size(1), k = topi.size(1);
  const int n13 = w13.size(1), I = n13 / 2;
  const int cap = T * k;
  auto i32 = h.options().dtype(at::kInt);
  if (T == 0) return;
  Scratch meta = scratch_empty(2 * count + 3 * cap + 1 + count + 1, i32, qb::BS_CANARY_MOE_META);
  int* counts = meta.t.data_ptr<int>();
  int* offsets = counts + count;
  int* perm_tok = offsets + count;
  int* perm_slot = perm_tok + cap;
  int* inv = perm_slot + cap;
  int* n_assign = inv + cap;
  int* tstart = n_assign + 1;
  Tensor topi_c = topi.contiguous();
  const int BN = qb::mx_token_tile(cap, count);
  LAUNCH(qb::moe_dispatch(topi_c.data_ptr<int>(), T, k, first, count, counts, offsets, perm_tok, perm_slot, inv,
                          n_assign, stream(), BN, tstart));
  const long tiles = count + (cap + BN - 1) / BN;
  const int KM = H > I ? H : I;
  auto u8 = h.options().dtype(at::kByte);
  // hi plane then lo plane; scale chunks either hi then lo regions, or (merged) per chunk hi|lo
  const bool merged = qb::mx_merged(tiled, BN);
  const long plane = ((long)cap * KM + 127) / 128 * 128, sf_plane = tiles * (KM / 128) * 512;
  Scratch hl = scratch_empty(2 * plane, u8, qb::BS_CANARY_MOE_SCRATCH);
  Scratch sf = scratch_empty(2 * sf_plane, u8, qb::BS_CANARY_MOE_SCRATCH);
  Tensor inter = at::empty({cap, I}, h.options());
  Tensor y2 = at::empty({cap, H}, h.options());
  uint8_t *hp = hl.t.data_ptr<uint8_t>(), *lp = hp + plane;
  uint8_t *shp = sf.t.data_ptr<uint8_t>(), *slp = merged ? shp : shp + sf_plane;
  // each token quantised once, then expanded into its assignments' rows (k x fewer conversions)
  Tensor qs = at::empty({(long)T * (2 * H + H / 32)}, u8);
  LAUNCH(qb::mx_quant_expand(h.data_ptr(), T, perm_tok, n_assign, cap, H, offsets, tstart, count, BN,
                             qs.data_ptr<uint8_t>(), hp, lp, shp, slp, stream(), merged,
                             sparse_rows ? topi_c.data_ptr<int>() : nullptr, k));
  LAUNCH(qb::moe_mx_gemm(hp, lp, shp, slp, cap, w13.data_ptr<uint8_t>(), s13c.data_ptr<uint8_t>(), n13, H, offsets,
                         counts, tstart, count, BN, 1, inter.data_ptr(), I, err_ptr(h), stream(), tiled));
  LAUNCH(qb::mx_quant(inter.data_ptr(), nullptr, n_assign, cap, I, offsets, counts, tstart, count, BN, hp, lp, shp,
                      slp, stream(), merged));
  LAUNCH(qb::moe_mx_gemm(hp, lp, shp, slp, cap, w2.data_ptr<uint8_t>(), s2c.data_ptr<uint8_t>(), H, I, offsets,
                         counts, tstart, count, BN, 0, y2.data_ptr(), H, err_ptr(h), stream(), tiled));
  const bool with_shared = shared.has_value() && gate.has_value();
  if (with_shared)
    TORCH_CHECK(!sparse_rows && shared->is_contiguous() && shared->sizes() == h.sizes() && gate->dim() == 1 &&
                    gate->size(0) == T && gate->scalar_type() == at::kBFloat16,
                "moe: shared [T, H] contiguous and gate logits [T] bf16");
  LAUNCH(qb::moe_combine(y2.data_ptr(), inv, topw.contiguous().data_ptr<float>(), T, k, H, out.data_ptr(), stream(),
                         sparse_rows, with_shared ? shared->data_ptr() : nullptr,
                         with_shared ? gate->data_ptr() : nullptr, with_shared ? gate->stride(0) : 0));
  scratch_check(meta);
  scratch_check(hl);
  scratch_check(sf);
}

Tensor moe_routed_mx(Tensor h, Tensor topw, Tensor topi, Tensor w13, Tensor s13c, Tensor w2, Tensor s2c,
                     int64_t first, int64_t count, bool tiled, c10::optional<Tensor> shared,
                     c10::optional<Tensor> gate) {
  Tensor out = at::empty_like(h);
  moe_routed_mx_into(h, topw, topi, w13, s13c, w2, s2c, first, count, tiled, out, false, shared, gate);
  return out;
}

// Expert-parallel MoE (ep.cu): dispatch this rank's token rows to the ranks owning their experts,
// run this rank's experts on the rows it received (into its symmetric y area), combine the
// weighted partial outputs of this rank's tokens from every rank.
Tensor ep_moe(std::vector<int64_t> bases, int64_t rank, Tensor h, Tensor topw, Tensor topi, Tensor w13, Tensor s13c,
              Tensor w2, Tensor s2c, int64_t first, int64_t count, bool tiled, int64_t cap, int64_t experts_per_rank,
              int64_t par, Tensor state, double timeout_s) {
  CHECK_BF16(h);
  TORCH_CHECK(h.is_contiguous() && topi.is_contiguous() && topw.is_contiguous(), "ep_moe: contiguous inputs");
  TORCH_CHECK(topi.scalar_type() == at::kInt && topw.scalar_type() == at::kFloat, "ep_moe: int32 ids, fp32 weights");
  const int world = bases.size(), T = h.size(0), H = h.size(1), k = topi.size(1);
  TORCH_CHECK(T <= cap, "ep_moe: more tokens than the receive areas hold");
  std::vector<void*> b(world);
  for (int r = 0; r < world; ++r) b[r] = reinterpret_cast<void*>(bases[r]);
  const unsigned long long tns = (unsigned long long)(timeout_s * 1e9);
  Tensor slots = at::empty({T > 0 ? T : 1, world}, h.options().dtype(at::kInt));
  Tensor counts = at::empty({world}, h.options().dtype(at::kInt));
  LAUNCH(qb::ep_dispatch(b.data(), world, rank, cap, H, k, experts_per_rank, h.data_ptr(), H,
                         topi.data_ptr<int>(), topw.data_ptr<float>(), T, slots.data_ptr<int>(),
                         counts.data_ptr<int>(), state.data_ptr<int>(), tns, err_ptr(h), stream()));
  long xo, io, wo, yo;
  qb::ep_offsets(world, cap, H, k, (int)par, &xo, &io, &wo, &yo);
  char* own = reinterpret_cast<char*>(b[rank]);
  auto opt = h.options();
  const long rows = (long)world * cap;
  Tensor rx = at::from_blob(own + xo, {rows, H}, opt);
  Tensor ri = at::from_blob(own + io, {rows, k}, opt.dtype(at::kInt));
  Tensor rw = at::from_blob(own + wo, {rows, k}, opt.dtype(at::kFloat));
  Tensor ry = at::from_blob(own + yo, {rows, H}, opt);
  moe_routed_mx_into(rx, rw, ri, w13, s13c, w2, s2c, first, count, tiled, ry, true);
  Tensor out = at::empty({T, H}, opt);
  LAUNCH(qb::ep_combine(b.data(), world, rank, cap, H, k, slots.data_ptr<int>(), T, out.data_ptr(), H,
                        state.data_ptr<int>(), tns, err_ptr(h), stream()));
  return out;
}

int64_t ep_region_bytes(int64_t world, int64_t cap, int64_t H, int64_t k) {
  return qb::ep_region_bytes(world, cap, H, k);
}

Tensor moe_routed_fp4(Tensor h, Tensor topw, Tensor topi, Tensor w13, Tensor s13, Tensor w2, Tensor s2, int64_t first,
                      int64_t count) {
  return moe_routed_impl(h, topw, topi, w13, s13, w2, s2, first, count);
}

void stamp(Tensor buf, int64_t slot) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kLong, "stamp: int64 CUDA buffer");
  TORCH_CHECK(slot >= 0 && slot < buf.numel(), "stamp: slot out of range");
  LAUNCH(qb::stamp(reinterpret_cast<unsigned long long*>(buf.data_ptr<int64_t>()), (int)slot, stream()));
}

// ------------------------------------------------------------------ symmetric memory (IPC)
// One cudaMalloc'd region per rank, exported with cudaIpcGetMemHandle and mapped by every peer.
py::tuple symm_alloc(int64_t bytes) {
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, bytes) == cudaSuccess, "symm_alloc: cudaMalloc failed");
  TORCH_CHECK(cudaMemset(p, 0, bytes) == cudaSuccess, "symm_alloc: cudaMemset failed");
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, p) == cudaSuccess, "symm_alloc: cudaIpcGetMemHandle failed");
  return py::make_tuple((int64_t)reinterpret_cast<uintptr_t>(p), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t symm_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  TORCH_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess,
              "symm_open: cudaIpcOpenMemHandle failed");
  return (int64_t)reinterpret_cast<uintptr_t>(p);
}

void symm_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }
void symm_free(int64_t ptr) { cudaFree(reinterpret_cast<void*>(ptr)); }

void symm_ar_add_rmsnorm(std::vector<int64_t> bases, int64_t rank, Tensor partial, Tensor res, Tensor w1p, Tensor out,
                         double eps, int64_t slot_elems, int64_t max_blocks, Tensor epoch, double timeout_s) {
  CHECK_BF16(partial);
  CHECK_BF16(res);
  TORCH_CHECK(res.is_contiguous() && out.is_contiguous() && partial.stride(-1) == 1, "symm_ar: layouts");
  std::vector<void*> b(bases.size());
  for (size_t i = 0; i < bases.size(); ++i) b[i] = reinterpret_cast<void*>(bases[i]);
  const int H = res.size(-1);
  const int rows = res.numel() / H;
  int* ep = epoch.data_ptr<int>();
  LAUNCH(qb::symm_ar_add_rmsnorm(b.data(), (int)b.size(), (int)rank, partial.data_ptr(), partial.stride(0),
                                 res.data_ptr(), w1p.data_ptr<float>(), out.data_ptr(), rows, H, (float)eps,
                                 slot_elems, (int)max_blocks, ep, ep + 1, err_ptr(res),
                                 (unsigned long long)(timeout_s * 1e9), stream()));
}

void symm_sp_ar_add_rmsnorm(std::vector<int64_t> bases, int64_t rank, Tensor partial, Tensor res, Tensor w1p, Tensor out,
                         double eps, int64_t slot_elems, int64_t max_blocks, Tensor epoch, double timeout_s,
                         bool own, bool res_local) {
  CHECK_BF16(partial);
  CHECK_BF16(res);
  TORCH_CHECK(res.is_contiguous() && out.is_contiguous() && partial.stride(-1) == 1, "symm_sp_ar: layouts");
  std::vector<void*> b(bases.size());
  for (size_t i = 0; i < bases.size(); ++i) b[i] = reinterpret_cast<void*>(bases[i]);
  const int H = res.size(-1);
  const int rows = res.numel() / H;
  int* ep = epoch.data_ptr<int>();
  LAUNCH(qb::symm_sp_ar_add_rmsnorm(b.data(), (int)b.size(), (int)rank, partial.data_ptr(), partial.stride(0),
                                 res.data_ptr(), w1p.data_ptr<float>(), out.data_ptr(), rows, H, (float)eps,
                                 slot_elems, (int)max_blocks, ep, ep + 1, err_ptr(res),
                                 (unsigned long long)(timeout_s * 1e9), stream(), own, res_local));
}

// All-gather -> GEMM after the owner-only sequence-parallel call (own=true above): y[rows, N] =
// gathered normed rows @ w^T, each owner's rows pulled by TMA from its result area (comm.cu).
Tensor symm_gemm_ag(std::vector<int64_t> bases, int64_t rank, Tensor w, int64_t rows, int64_t hidden,
                    int64_t slot_elems, int64_t max_blocks, Tensor epoch, double timeout_s) {
  CHECK_BF16(w);
  TORCH_CHECK(w.dim() == 2 && w.size(1) == hidden && w.stride(1) == 1 && (w.stride(0) * 2) % 16 == 0,
              "symm_gemm_ag: w [N, hidden] with 16-byte rows");
  const int world = (int)bases.size();
  TORCH_CHECK(world >= 1 && world <= 8 && rank >= 0 && rank < world, "symm_gemm_ag: 1..8 ranks");
  const int per = (int)((rows + world - 1) / world);
  TORCH_CHECK((long)per * world * hidden <= slot_elems, "symm_gemm_ag: rows exceed the region");
  const long slot_stride = 3 * slot_elems;                  // elements per slot
  const long flags_base = 2 * slot_stride * 2;              // bytes
  const long ready_off = flags_base + 4L * max_blocks * 4;  // the owner-only call's ready word
  std::vector<const void*> src(world);
  qb::GemmGather g{};
  for (int o = 0; o < world; ++o) {
    char* base = reinterpret_cast<char*>(bases[o]);
    src[o] = base + (slot_elems + hidden) * 2;  // slot 0 result area, normed half of each row
    g.ready[o] = reinterpret_cast<const int*>(base + ready_off);
  }
  g.epoch = epoch.data_ptr<int>();
  g.world = world;
  g.rank = (int)rank;
  g.per = per;
  g.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  Tensor y = at::empty({rows, w.size(0)}, w.options());
  LAUNCH(qb::gemm_ag(src.data(), 2 * hidden, slot_stride, w.data_ptr(), w.stride(0), y.data_ptr(), y.stride(0),
                     (int)rows, (int)w.size(0), (int)hidden, g, err_ptr(w), stream()));
  return y;
}

// NVLS all-reduce + residual add + RMSNorm: `uc`/`mc` are this rank's unicast and multicast
// addresses of one symmetric region bound to an NVSwitch multicast object.
void nvls_ar_add_rmsnorm(int64_t uc, int64_t mc, int64_t world, int64_t rank, Tensor partial, Tensor res, Tensor w1p,
                         Tensor out, double eps, int64_t slot_elems, int64_t grid, Tensor epoch, double timeout_s) {
  CHECK_BF16(partial);
  CHECK_BF16(res);
  TORCH_CHECK(res.is_contiguous() && out.is_contiguous() && partial.stride(-1) == 1 &&
                  (partial.stride(0) * 2) % 16 == 0, "nvls_ar: layouts");
  const int H = res.size(-1);
  const int rows = res.numel() / H;
  int* ep = epoch.data_ptr<int>();
  LAUNCH(qb::nvls_ar_add_rmsnorm(reinterpret_cast<void*>(uc), reinterpret_cast<void*>(mc), (int)world, (int)rank,
                                 partial.data_ptr(), partial.stride(0), res.data_ptr(), w1p.data_ptr<float>(),
                                 out.data_ptr(), rows, H, (float)eps, slot_elems, (int)grid, ep, ep + 1, err_ptr(res),
                                 (unsigned long long)(timeout_s * 1e9), stream()));
}

int64_t nvls_region_bytes(int64_t slot_elems) { return qb::nvls_region_bytes(slot_elems); }

// GEMM -> reduce-scatter + residual add + RMSNorm + all-gather: the row-parallel projection
// x @ w^T stores its rows straight into the owner ranks' partial slots, then the pushed variant
// of the sequence-parallel kernel reduces them. Same bits as linear + symm_sp_ar_add_rmsnorm.
void symm_linear_sp_ar_add_rmsnorm(Tensor x, Tensor w, std::vector<int64_t> bases, int64_t rank, Tensor res,
                                   Tensor w1p, Tensor out, double eps, int64_t slot_elems, int64_t max_blocks,
                                   Tensor epoch, double timeout_s, bool res_local) {
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(res);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "symm_linear_sp: shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && (x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0,
              "symm_linear_sp: layouts");
  TORCH_CHECK(res.is_contiguous() && out.is_contiguous(), "symm_linear_sp: layouts");
  const int H = res.size(-1);
  const int rows = res.numel() / H;
  TORCH_CHECK(w.size(0) == H && x.size(0) == rows, "symm_linear_sp: output is [rows, hidden]");
  const int world = (int)bases.size();
  TORCH_CHECK(world >= 1 && world <= 8, "symm_linear_sp: 1..8 ranks");
  const int per = (rows + world - 1) / world;
  int* ep = epoch.data_ptr<int>();
  qb::GemmPush push{};
  for (int r = 0; r < world; ++r) push.base[r] = reinterpret_cast<void*>(bases[r]);
  push.world = world;
  push.rank = (int)rank;
  push.per = per;
  push.epoch = ep;
  push.slot_stride = 3 * slot_elems;  // a slot: partial [rows, H] then results [rows, 2H]
  TORCH_CHECK((long)per * world * H <= slot_elems, "symm_linear_sp: rows exceed the region");
  const int T = rows, N = H, K = x.size(1);
  const long wsf = qb::gemm_split_ws_floats(T, N, K);
  Tensor ws, cnt;
  if (wsf) {
    ws = at::empty({wsf}, x.options().dtype(at::kFloat));
    cnt = gemm_counters(x, (long)((N + 127) / 128) * ((T + 15) / 16));
  }
  LAUNCH(qb::gemm_ws(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), nullptr, N, T, N, K, true, 0, err_ptr(x),
                     stream(), 0, wsf ? ws.data_ptr<float>() : nullptr, wsf ? cnt.data_ptr<int>() : nullptr, &push));
  std::vector<void*> b(world);
  for (int i = 0; i < world; ++i) b[i] = reinterpret_cast<void*>(bases[i]);
  LAUNCH(qb::symm_sp_rs_add_rmsnorm(b.data(), world, (int)rank, per, res.data_ptr(), w1p.data_ptr<float>(),
                                    out.data_ptr(), rows, H, (float)eps, slot_elems, (int)max_blocks, ep, ep + 1,
                                    err_ptr(res), (unsigned long long)(timeout_s * 1e9), stream(), res_local));
}

// ------------------------------------------------------------------ status
int64_t launches() { return g_launches.load(); }
// graph replays launch the captured kernels without passing through these bindings
void add_launches(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
Tensor status(Tensor like) { return status_tensor(like.device()).clone(); }
void clear_status(Tensor like) { status_tensor(like.device()).zero_(); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("linear", &linear, "Y = X W^T on tcgen05", py::arg("x"), py::arg("w"), py::arg("out") = py::none());
  m.def("rmsnorm", &rmsnorm);
  m.def("add_rmsnorm", &add_rmsnorm);
  m.def("gated_rmsnorm", &gated_rmsnorm);
  m.def("silu_mul", &silu_mul);
  m.def("embed", &embed);
  m.def("argmax_rows", &argmax_rows);
  m.def("sigmoid_gate_mul", &sigmoid_gate_mul);
  m.def("shared_gate_combine", &shared_gate_combine);
  m.def("router_topk", &router_topk2);
  m.def("qk_norm_rope_kv_write", &qk_norm_rope_kv_write);
  m.def("attention_varlen", &attention_varlen);
  m.def("attention_fa", &attention_fa);
  m.def("moe_routed_mx", &moe_routed_mx, py::arg("h"), py::arg("topw"), py::arg("topi"), py::arg("w13"),
        py::arg("s13c"), py::arg("w2"), py::arg("s2c"), py::arg("first"), py::arg("count"), py::arg("tiled"),
        py::arg("shared") = py::none(), py::arg("gate") = py::none());
  m.def("stamp", &stamp);
  m.def("mx_probe", []() {
    Tensor t = at::zeros({8}, at::kLong);
    TORCH_CHECK(qb::mx_probe_read(reinterpret_cast<unsigned long long*>(t.data_ptr<int64_t>())) == 0, "mx_probe");
    return t;
  });
  m.def("deltanet_decode", &deltanet_decode);
  m.def("ep_moe", &ep_moe);
  m.def("ep_region_bytes", &ep_region_bytes);
  m.def("gated_delta_chunked", &gated_delta_chunked);
  m.def("gated_delta_tc", &gated_delta_tc);
  m.def("causal_conv_varlen", &causal_conv_varlen);
  m.def("gated_delta_varlen", &gated_delta_varlen);
  m.def("moe_routed_fp4", &moe_routed_fp4);
  m.def("moe_routed_bf16", &moe_routed_bf16);
  m.def("status", &status);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("symm_ar_add_rmsnorm", &symm_ar_add_rmsnorm);
  m.def("symm_sp_ar_add_rmsnorm", &symm_sp_ar_add_rmsnorm, py::arg("bases"), py::arg("rank"), py::arg("partial"),
        py::arg("res"), py::arg("w1p"), py::arg("out"), py::arg("eps"), py::arg("slot_elems"), py::arg("max_blocks"),
        py::arg("epoch"), py::arg("timeout_s"), py::arg("own") = false, py::arg("res_local") = false);
  m.def("symm_gemm_ag", &symm_gemm_ag);
  m.def("symm_linear_sp_ar_add_rmsnorm", &symm_linear_sp_ar_add_rmsnorm, py::arg("x"), py::arg("w"), py::arg("bases"),
        py::arg("rank"), py::arg("res"), py::arg("w1p"), py::arg("out"), py::arg("eps"), py::arg("slot_elems"),
        py::arg("max_blocks"), py::arg("epoch"), py::arg("timeout_s"), py::arg("res_local") = false);
  m.def("nvls_ar_add_rmsnorm", &nvls_ar_add_rmsnorm);
  m.def("nvls_region_bytes", &nvls_region_bytes);
  m.def("launches", &launches, "number of kernels launched through the bindings so far");
  m.def("add_launches", &add_launches, "account kernels launched by a CUDA-graph replay");
  m.def("clear_status", &clear_status);
}
