// Host-callable launchers of every sm_100a kernel in this package. Kernel
// translation units include only CUDA headers; the torch-facing checks and
// tensor plumbing live in bindings.cpp.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "ar/ar_ctx.h"

namespace mbx {

// ---- allreduce (ar/allreduce.cu) -------------------------------------------
uint64_t ar_chunk_limit(const ArCtx& c, int algo);
void ar_launch(const ArCtx& c, int algo, int dtype, const void* in, void* out, uint64_t nbytes, int max_blocks,
               cudaStream_t stream);
// threads: 512 (default) or 256 per block; 256 halves a block's registers so
// it fits on an SM beside a running GEMM CTA (overlapped micro-batches).
void ar_rmsnorm_launch(const ArCtx& c, int algo, const void* in, void* residual, const void* weight, void* out, int M,
                       int H, float eps, int max_blocks, cudaStream_t stream, int threads = 512);
void ar_allgather_launch(const ArCtx& c, const void* in, void* out, uint64_t nbytes, int max_blocks,
                         cudaStream_t stream);
// Second launch of the fused GEMM->allreduce->RMSNorm (reduce own rows,
// all-gather, residual + norm). The first launch is gemm_ar_rmsnorm_launch.
void fused_rs_norm_launch(const ArCtx& c, int M, int N, int Mo, void* residual, const void* weight, void* out,
                          float eps, int max_blocks, cudaStream_t stream);
// Second launch of the push-all fused GEMM->allreduce->RMSNorm.
void fused_allsum_norm_launch(const ArCtx& c, int M, int N, void* residual, const void* weight, void* out, float eps,
                              int max_blocks, cudaStream_t stream);
void seg_submit_launch(const ArCtx& c, const void* in, uint64_t nbytes, int max_blocks, cudaStream_t stream);
void seg_wait_launch(const ArCtx& c, int dtype, const void* local, void* out, uint64_t nbytes, int max_blocks,
                     cudaStream_t stream);
// One-GPU emulation of a W-rank call (tests and single-GPU profiling): every
// rank's blocks in one cooperative launch, rank = blockIdx.y, each with its
// own context whose "peer" buffers are local allocations. `dev_scratch` is
// device memory for the world x EmuRank array (copied on `stream`).
enum EmuOp : int { kEmuAllreduce = 0, kEmuArRmsnorm = 1, kEmuFusedRsNorm = 2, kEmuAllgather = 3 };
struct EmuRank {
  ArCtx c;
  const void* in;      // allreduce / all-gather input, or the norm input
  void* out;
  void* residual;      // norm ops: residual updated in place
  const void* weight;  // norm ops: RMSNorm weight
};
void ar_emulated_launch(const EmuRank* ranks_host, int world, int op, int algo, int dtype, uint64_t nbytes, int M,
                        int N, float eps, int blocks, void* dev_scratch, cudaStream_t stream, int threads = 512);
// Raw NVLink transport kernels for bandwidth benchmarks. kMcReduce* read the
// multicast address `src` and write local `dst`; kMcStore reads local `src`
// and stores to the multicast address `dst`.
enum RawKind { kRawPush1 = 0, kRawPush4 = 1, kRawPull4 = 2, kRawMcReduce = 3, kRawMcReduceNoAcc = 4, kRawMcStore = 5 };
void raw_transport_launch(int kind, void* dst, const void* src, uint64_t nbytes, int grid, int threads,
                          cudaStream_t stream);

// ---- AWQ int4 weights (quant/awq.cu) ------------------------------------------
constexpr int kAwqGemvMaxRows = 8;
struct AwqGemvArgs {
  const void* x;          // bf16 [M, K], row stride ldx
  int64_t ldx;
  const void* qweight;    // int32 [K, N/8]
  const void* qzeros;     // int32 [K/G, N/8]
  const void* scales;     // fp16 [K/G, N], 16-byte aligned
  float* ws;              // fp32 [K/G, M, N]: per-group partial sums
  const void* residual;   // bf16 [M, N] (row stride ldo) or nullptr
  void* out;              // bf16 [M, N], row stride ldo; may alias residual
  int64_t ldo;
  int M, K, N, G;
};
// out = x @ W^T (+ residual) for M <= 8 rows, W dequantized on the fly.
void awq_gemv_launch(const AwqGemvArgs& a, cudaStream_t s);
// bf16 [N, K] (row-major, the GEMM's weight layout) from the packed tensors.
void awq_dequant_launch(const void* qweight, const void* qzeros, const void* scales, void* out, int K, int N, int G,
                        cudaStream_t s);

// ---- elementwise (ops/elementwise.cu) ----------------------------------------
void rmsnorm_launch(const void* x, void* residual, const void* w, void* out, int64_t M, int H, float eps,
                    cudaStream_t s);
// q_norm / k_norm (bf16 [128], both or neither): Qwen3's per-head RMSNorm of
// q and k, applied before the rotation in the same launch.
void rope_and_cache_launch(const void* qkv, const int* pos, const float* cos_sin, const int64_t* slots, void* q_out,
                           void* k_cache, void* v_cache, int64_t T, int nq, int nkv, int page, cudaStream_t s,
                           const void* q_norm = nullptr, const void* k_norm = nullptr, float eps = 0.f);
void silu_mul_launch(const void* x, void* out, int64_t M, int I2, cudaStream_t s);
void embedding_launch(const int* ids, const void* table, void* out, int64_t T, int H, int64_t start, int64_t rows,
                      cudaStream_t s);
void argmax_launch(const void* logits, bool bf16, int64_t ld, int64_t B, int V, int64_t offset, float* best_val,
                   int64_t* best_idx, cudaStream_t s);
void argmax_combine_launch(const float* vals, const int64_t* idxs, int W, int B, int64_t* out, cudaStream_t s);

// ---- GEMM (gemm/gemm.cu) -----------------------------------------------------
struct GemmPlan {
  int bn = 256;
  int splits = 1;
};
GemmPlan gemm_plan(int64_t M, int64_t N, int64_t K);
// C[M,N] (ldc) = A[M,K] (lda) * B[N,K]^T (ldb) (+ residual, same layout as C).
// splits > 1 needs an fp32 workspace of splits*M*N elements.
// counters: zeroed uint32 per-tile arrival counters for the in-kernel split-K
// reduction (nullptr: a separate reduce kernel folds the partials).
// ag != nullptr: A is a sequence-parallel gather buffer; the producer waits
// for the owners' all-gather flags of each m-tile before loading it.
struct GemmAgWait {
  const uint32_t* flags;       // this rank's all-gather flag words (one per owner)
  const uint32_t* epoch_word;  // device word holding the epoch to wait for
  int Mo;                      // rows per owner
};
// bf16 GEMV for 1..kGemvMaxRows rows (decode): out[M, N] = x[M, K] @ W[N, K]^T (+ residual,
// rounded like the GEMM epilogue). x and W rows 16-byte aligned, K % 8 == 0.
constexpr int kGemvMaxRows = 2;
bool gemv_bf16_supported(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M, int64_t K);
void gemv_bf16_launch(const void* x, int64_t ldx, const void* w, int64_t ldw, void* out, int64_t ldo,
                      const void* residual, int64_t M, int64_t N, int64_t K, cudaStream_t s);
// Fused decode MLP input for 1..kGemvMaxRows rows: out[M, F] = silu(x @ gate^T) *
// (x @ up^T) for a gate_up weight [2F, K] (gate rows first), rounded like
// GEMM + silu_mul.
void gemv_silu_launch(const void* x, int64_t ldx, const void* w, int64_t ldw, void* out, int64_t ldo, int64_t M,
                      int64_t N2, int64_t K, cudaStream_t s);
// Fused decode attention input for 1..kGemvMaxRows tokens: qkv = x @ W^T for a
// qkv weight [(nq + 2 nkv) * 128, K], neox RoPE of q and k at pos, q to q_out
// [M, nq, 128], k and v to the paged cache at slots (nullptr: no cache
// write); roundings of GEMM + rope_and_cache.
void gemv_rope_launch(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M, int64_t K, const int* pos,
                      const float* cos_sin, const int64_t* slots, void* q_out, void* k_cache, void* v_cache, int nq,
                      int nkv, int page, cudaStream_t s);

void gemm_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* residual,
                 int64_t M, int64_t N, int64_t K, int bn, int splits, float* workspace, uint32_t* counters,
                 uint32_t* err, cudaStream_t s, const GemmAgWait* ag = nullptr);

// Row-parallel GEMM fused with allreduce + residual add + RMSNorm: the GEMM
// epilogue stores its partial rows straight into the owner ranks' symmetric
// buffers (reduce-scatter overlapped with the remaining tiles), then one
// launch reduces, all-gathers and normalises. residual is updated in place;
// out = rmsnorm(residual) * norm_w.
// push_all: the epilogue stores every row to every rank (one exchange; best
// for small worlds) instead of to the row's owner (reduce-scatter +
// all-gather; less traffic for large worlds).
void gemm_ar_rmsnorm_launch(const ArCtx& c, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M,
                            int64_t N, int64_t K, void* residual, const void* norm_w, void* out, float eps,
                            uint32_t* err, int max_blocks, bool push_all, cudaStream_t s);

// The first launch of gemm_ar_rmsnorm_launch alone (one-GPU emulation of the
// ranks: each rank's GEMM pushes into every emulated rank's fused buffer).
void gemm_push_launch(const ArCtx& c, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N,
                      int64_t K, bool push_all, uint32_t* err, cudaStream_t s);

// ---- sequence parallel (gemm/gemm.cu, ar/allreduce.cu) ---------------------
// Rank r owns rows [r*Mo, r*Mo+Mo) of the residual stream, Mo = ceil(M/world).
// GEMM -> reduce-scatter: the epilogue pushes every output row to its owner's
// reduce-scatter slot (same buffers and flags as the fused allreduce path).
void gemm_rs_launch(const ArCtx& c, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N,
                    int64_t K, uint32_t* err, cudaStream_t s);
// Reduce-scatter of a local [M, N] tensor (e.g. the vocab-parallel embedding).
void sp_rs_push_launch(const ArCtx& c, const void* x, int M, int N, int max_blocks, cudaStream_t s);
// Reduce the owned rows (rank order, fp32, one rounding), residual shard +=
// them (bf16), normalise, and push the normed rows into every rank's gather
// buffer G ([M, N] at c.sp_off); the last block releases the all-gather flags.
void sp_rs_norm_ag_launch(const ArCtx& c, int M, int N, void* res_own, const void* w, float eps, int max_blocks,
                          cudaStream_t s);
// Wait (one tiny block) until every owner's rows of the last all-gather landed
// in G, for consumers other than the all-gather GEMM.
void sp_ag_wait_launch(const ArCtx& c, int M, cudaStream_t s);

// ---- attention (attn/attention.cu) -------------------------------------------
void prefill_attention_launch(const void* q, const void* kc, const void* vc, void* o, const int* cu_q,
                              const int* kv_len, const int* block_table, int max_blocks, const int* tiles,
                              int n_tiles, int nq, int nkv, float scale, cudaStream_t s);
// tcgen05/TMEM prefill attention (128-row query tiles, 128-key tiles).
// splits > 1 splits every query tile's keys across CTAs (partials in
// part_o [T, nq, splits, 128] / part_lse [T, nq, splits], merged in place).
void prefill_attention_tc_launch(const void* q, const void* kc, const void* vc, void* o, const int* cu_q,
                                 const int* kv_len, const int* block_table, int max_blocks, const int* tiles,
                                 int n_tiles, int T, int nq, int nkv, int num_blocks, float scale, int splits,
                                 float* part_o, float* part_lse, uint32_t* err, cudaStream_t s);
// LSE-weighted merge of split partials: rows x splits x 128 -> bf16 rows x 128.
void attn_combine_launch(const float* part_o, const float* part_lse, int64_t rows, int splits, void* out,
                         cudaStream_t s);
// counters: int32 [B * nkv], zero, for the in-kernel split-KV merge (each
// (batch, kv head)'s last CTA merges and resets its count); nullptr merges
// with a separate combine launch.
void decode_attention_launch(const void* q, const void* kc, const void* vc, void* o, const int* kv_len,
                             const int* block_table, int max_blocks, int B, int nq, int nkv, int splits,
                             float* part_o, float* part_lse, float scale, cudaStream_t s, int* counters = nullptr);

}  // namespace mbx
