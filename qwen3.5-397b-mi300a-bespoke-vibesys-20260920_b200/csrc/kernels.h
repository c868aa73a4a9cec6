// Host-side launchers of every kernel in csrc/ (raw pointers, element strides, a stream).
// The torch bindings (bindings.cpp) validate tensors and call these. Each launcher returns
// 0 on success or a CUDA / driver error code.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qb {

// dtype codes used across launchers
enum DType : int { DT_BF16 = 0, DT_F16 = 1, DT_F32 = 2 };

int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, long rows, long cols, long ld_elems,
                 int box_rows, int box_cols, bool swizzle128);

// GEMM -> reduce-scatter target: every rank's symmetric sequence-parallel region (comm.cu layout)
struct GemmPush {
  void* base[8];       // region bases as mapped on this rank (own entry local)
  int world, rank;     // world == 0: no push
  int per;             // rows owned per rank (the last rank may own fewer)
  const int* epoch;    // the reduce kernel's device epoch; the slot is (epoch + 1) & 1
  long slot_stride;    // elements per slot of a region
};

// All-gather -> GEMM: the token rows are owned by the ranks in contiguous ranges (owner o holds
// rows [o per, min(T, (o+1) per))), each in its own symmetric gather area; the GEMM's producer
// loads owner o's token tiles by TMA straight from that area (a peer's memory over NVLink, no
// multicast) after owner o's ready word has reached the producing kernel's epoch.
struct GemmGather {
  const int* ready[8];  // owner o's ready word as mapped on this rank (own entry unused)
  const int* epoch;     // the producing kernel's device epoch e: slot e & 1, ready when word >= e
  int world, rank, per;
  unsigned long long timeout_ns;
};

// Y[T,N] = X[T,K] @ W[N,K]^T ; act 1 = silu(gate)*up over 64-row halves of each 128-row tile;
// with `push`, row t is stored into the owner rank's partial slot instead of Y (ldy must be N)
int gemm_ws(const void* x, long ldx, const void* w, long ldw, void* y, long ldy, int T, int N, int K, bool bf16,
            int act, int* err, cudaStream_t stream, int max_ctas = 0, float* ws = nullptr, int* cnt = nullptr,
            const GemmPush* push = nullptr);
// Y[T,N] = gathered X[T,K] @ W[N,K]^T, X row t read from owner t / per's gather area:
// src[o] = owner o's area for slot 0 as mapped here, rows `src_ld` elements apart, slot 1 at
// + slot_stride elements (bf16 only, no activation)
int gemm_ag(const void* const* src, long src_ld, long slot_stride, const void* w, long ldw, void* y, long ldy, int T,
            int N, int K, const GemmGather& g, int* err, cudaStream_t stream);
// stream-K workspace (fp32 floats; 0 = whole tiles per CTA) and CTA count; counters: one per tile
long gemm_split_ws_floats(int T, int N, int K);
int gemm_streamk_ctas(int T, int N, int K);

int rmsnorm(const void* x, long ldx, const float* w1p, void* out, long ldo, int rows, int H, float eps,
            cudaStream_t s);
int add_rmsnorm(const void* x, long ldx, void* res, long ldr, const float* w1p, void* out, long ldo, int rows, int H,
                float eps, cudaStream_t s);
int gated_rmsnorm(const void* core, const void* z, long ldz_row, const void* w, void* out, int T, int heads, int dv,
                  float eps, cudaStream_t s);
int silu_mul(const void* gu, long ldg, void* out, long ldo, int T, int n, cudaStream_t s);
int embed(const int64_t* tok, const void* table, void* out, int T, int H, long V, cudaStream_t s);
int argmax_rows(const void* x, long ldx, int dtype, int R, int V, float* val, int64_t* idx, cudaStream_t s);
int sigmoid_gate_mul(const void* x, long ldx, const void* g, long ldg, void* out, int T, int D, cudaStream_t s);
int shared_gate_combine(const void* routed, const void* shared, const void* gl, long ldgl, void* out, int T, int H,
                        cudaStream_t s);
int qk_norm_rope_kv_write(const void* qkv, long ldqkv, int nq, int nkv, int hd, const float* qn, const float* kn,
                          const int* pos, const int* rows, void* kc, void* vc, void* qout, int T, int rot,
                          float theta, float eps, long kv_rows, cudaStream_t s);
int causal_conv_varlen_t(const void* x, long ldx, void* state, long lane_stride, const void* w, const int* seg_lane,
                         const int* cu, int S, int T, int C, int K, void* out, bool commit, int lanes,
                         cudaStream_t s);
// debug build (-DQB_BOUNDS, bounds.cuh): check sites recorded in the status word, the scratch
// canary, the status-word pointer installs (one per translation unit with checks; no-ops in the
// release build) and the canary check
enum BoundsSite : int {
  BS_EMBED_TOKEN = 1,
  BS_KV_ROW = 2,
  BS_LANE = 4,
  BS_CANARY_GEMM_WS = 11,
  BS_CANARY_ATTN_WS = 12,
  BS_CANARY_DN_SCRATCH = 13,
  BS_CANARY_MOE_META = 14,
  BS_CANARY_MOE_SCRATCH = 15,
};
constexpr int CANARY_BYTES = 256;
constexpr unsigned char CANARY_BYTE = 0xA5;
bool bounds_build();
int bounds_install_elementwise(int* word);
int bounds_install_sequence(int* word);
int canary_check(const void* tail, int site, cudaStream_t s);
int gated_delta_varlen_t(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log,
                         const float* dt_bias, float* state, long lane_stride, const int* seg_lane, const int* cu,
                         int S, int T, int nk, int nv, int dk, int dv, float* scratch, void* out, bool commit,
                         cudaStream_t s);
int attention_varlen(const void* q, const void* kc, const void* vc, const int* table, int max_blocks,
                     const int* pos, const int* seg_lane, const int* cu, int S, int T, int nq, int nkv, int hd,
                     int block_size, int splits, float* ws, void* out, cudaStream_t s);
// chunked gated delta rule (deltanet.cu) and the shared DeltaNet prep kernel (sequence.cu)
int delta_prep(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log, const float* dt_bias,
               int T, int nk, int nv, int dk, float* qn, float* kn, float* gb, cudaStream_t s);
int gated_delta_chunked(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log,
                        const float* dt_bias, float* state, long lane_stride, const int* seg_lane,
                        const int* chunks, int n_chunks, const int* seg_chunk0, int S, int T, int nk, int nv, int dk,
                        int dv, float* scratch, void* out, bool commit, cudaStream_t s);
long gated_delta_chunked_scratch(int T, int n_chunks, int nk, int nv, int dk);
// chunked gated delta rule with the state in tensor memory (tcgen05), head size 128
int gated_delta_tc(const void* qkv, long ldqkv, const void* ab, long ldab, const float* a_log, const float* dt_bias,
                   float* state, long lane_stride, const int* seg_lane, const int* chunks, int n_chunks,
                   const int* seg_chunk0, int S, int T, int nk, int nv, int dk, int dv, float* scratch, void* out,
                   bool commit, int* err, cudaStream_t s);
long gated_delta_tc_scratch(int T, int n_chunks, int nk, int nv);
// DeltaNet token mixer for one token per lane (conv, l2norm, gated delta step, gated RMSNorm)
int deltanet_decode(const void* proj, long ldp, void* conv_state, long cls, const void* conv_w, const float* a_log,
                    const float* dt_bias, float* state, long sls, const void* norm_w, const int* seg_lane, int T,
                    int nk, int nv, int dk, int dv, int K, float eps, void* out, cudaStream_t s, int* err = nullptr);
// expert-parallel MoE over peer memory (ep.cu)
long ep_region_bytes(int world, int cap, int H, int k);
int ep_dispatch(void* const* bases, int world, int rank, int cap, int H, int k, int experts_per_rank, const void* x,
                long ldx, const int* topi, const float* topw, int T, int* slots, int* counts, int* state,
                unsigned long long timeout_ns, int* err, cudaStream_t s);
int ep_combine(void* const* bases, int world, int rank, int cap, int H, int k, const int* slots, int T, void* out,
               long ldo, const int* state, unsigned long long timeout_ns, int* err, cudaStream_t s);
void ep_offsets(int world, int cap, int H, int k, int par, long* x, long* i, long* w, long* y);
// in-graph clock stamp (elementwise.cu): buf[slot] = %globaltimer
int stamp(unsigned long long* buf, int slot, cudaStream_t s);
// block-scaled MoE (moe_mx.cu): token tile width, tile prefix, activation split, expert GEMM
int mx_token_tile(int cap, int count);
int mx_tile_prefix(const int* counts, int count, int BN, int* tstart, cudaStream_t s);
int mx_quant(const void* x, const int* perm, const int* n_rows, int cap, int K, const int* offsets, const int* counts,
             const int* tstart, int count, int BN, uint8_t* hi, uint8_t* lo, uint8_t* sf_hi, uint8_t* sf_lo,
             cudaStream_t s, bool merged = false);
// diagnostic wait-cycle counters of the block-scaled MoE kernel (QB_MX_PROBE=1), read and cleared
int mx_probe_read(unsigned long long* out);
// the routed MoE input quantised once per token (scratch: T x (2K + K/32) bytes), then expanded
// into the expert-sorted rows and tile scale chunks (same bytes as mx_quant with a permutation)
int mx_quant_expand(const void* x, int T, const int* perm, const int* n_rows, int cap, int K, const int* offsets,
                    const int* tstart, int count, int BN, uint8_t* qscratch, uint8_t* hi, uint8_t* lo, uint8_t* sf_hi,
                    uint8_t* sf_lo, cudaStream_t s, bool merged = false, const int* skip_ids = nullptr,
                    int k = 0);
// merged activation buffers are used (tiled codes with one TMA box per operand)
bool mx_merged(bool tiled, int BN);
int moe_mx_gemm(const uint8_t* hi, const uint8_t* lo, const uint8_t* sf_hi, const uint8_t* sf_lo, int cap,
                const uint8_t* wq, const uint8_t* sfa, int n_rows, int K, const int* offsets, const int* counts,
                const int* tstart, int count, int BN, int act, void* out, int out_cols, int* err, cudaStream_t s,
                bool tiled = false);
// tcgen05 flash attention (attention.cu); tiles = [n_tiles][segment, row0, rows]; splits > 1 splits
// every tile's key range (partials in ws, merged by a second kernel)
int fa_prefill(const void* q, const void* kc, const void* vc, long cache_rows, const int* table, int max_blocks,
               const int* pos, const int* seg_lane, const int* tiles, int n_tiles, int T, int nq, int nkv, int hd,
               int block_size, int splits, float* ws, void* out, int* err, cudaStream_t s);
int router_topk(const void* logits, long ld, int T, int E, int k, float* w, int* idx, cudaStream_t s);

// MoE: dispatch metadata + grouped MXFP4 expert GEMMs + combine
int moe_dispatch(const int* topi, int T, int k, int first, int count, int* counts, int* offsets, int* perm_tok,
                 int* perm_slot, int* inv, int* n_assign, cudaStream_t s, int tile = 0, int* tstart = nullptr);
int moe_gather_f16(const void* h, const int* perm_tok, const int* n_assign, int cap, int H, void* xh,
                   cudaStream_t s);
int moe_expert_gemm(const void* xin, int in_cols, const uint8_t* wq, const uint8_t* ws, int n_rows, int k_cols,
                    long w_expert_stride, long s_expert_stride, const int* offsets, const int* counts,
                    int count, int cap, int act, void* out, int out_cols, int* err, cudaStream_t s, int max_ctas);
int moe_gather_bf16(const void* h, const int* perm_tok, const int* n_assign, int cap, int H, void* xh,
                    cudaStream_t s);
// shared (optional, with gl / ldgl): add bf16(sigmoid(gate)) x shared to every combined row
int moe_combine(const void* y2, const int* inv, const float* topw, int T, int k, int H, void* out, cudaStream_t s,
                bool skip_empty = false, const void* shared = nullptr, const void* gl = nullptr, long ldgl = 0);
int moe_expert_gemm_bf16(const void* xin, int in_cols, const void* w, int n_rows, int k_cols, long w_expert_stride,
                         const int* offsets, const int* counts, int count, int cap, int act, void* out, int out_cols,
                         cudaStream_t s);

// one-shot all-reduce + residual add + RMSNorm over peer-mapped symmetric regions (comm.cu)
int symm_ar_add_rmsnorm(void* const* bases, int world, int rank, const void* partial, long ldp, void* res,
                        const float* w1p, void* out, int rows, int H, float eps, long slot_elems, int max_blocks,
                        int* epoch, int* done, int* err, unsigned long long timeout_ns, cudaStream_t s);
// own: the owner-only form (no all-gather; the next GEMM gathers, see comm.cu and gemm_ag)
int symm_sp_ar_add_rmsnorm(void* const* bases, int world, int rank, const void* partial, long ldp, void* res,
                        const float* w1p, void* out, int rows, int H, float eps, long slot_elems, int max_blocks,
                        int* epoch, int* done, int* err, unsigned long long timeout_ns, cudaStream_t s,
                        bool own = false, bool res_local = false);
// the same after a GEMM that pushed its rows into the owners' slots (GemmPush, per rows a rank)
// NVLS: switch-reduced all-reduce + residual add + RMSNorm over a multicast-bound region.
long nvls_region_bytes(long slot_elems);
int nvls_ar_add_rmsnorm(void* uc, void* mc, int world, int rank, const void* partial, long ldp, void* res,
                        const float* w1p, void* out, int rows, int H, float eps, long slot_elems, int grid,
                        int* epoch, int* done, int* err, unsigned long long timeout_ns, cudaStream_t s);
int symm_sp_rs_add_rmsnorm(void* const* bases, int world, int rank, int per, void* res, const float* w1p, void* out,
                           int rows, int H, float eps, long slot_elems, int max_blocks, int* epoch, int* done,
                           int* err, unsigned long long timeout_ns, cudaStream_t s, bool res_local = false);

}  // namespace qb
