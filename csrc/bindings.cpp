// Python bindings of the CUDA extension (_C): tensor checks and plumbing for
// every sm_100a kernel (launchers declared in kernels.h), the symmetric-memory
// API and the allreduce communicator core. Compiled by the host compiler only.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>

#include "kernels.h"
#include "symm/symm.h"

namespace py = pybind11;

namespace mbx {
namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }
cudaStream_t stream_of(int64_t s) { return s == 0 ? cur_stream() : reinterpret_cast<cudaStream_t>(s); }

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}
void check_bf16(const torch::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bf16");
}

// Fixed-address launch context of one communicator (all pointers are mapped
// once, so CUDA-graph replays of any launch below stay valid).
class ArComm {
 public:
  ArComm(int rank, int world, std::vector<int64_t> bufs, int64_t mc, int64_t state, int64_t status_dev,
         int64_t status_host, uint64_t half_bytes, uint64_t seg_slot_bytes, uint64_t timeout_ns,
         uint64_t fuse_half_bytes, uint64_t sp_bytes)
      : status_host_(reinterpret_cast<volatile uint32_t*>(status_host)) {
    TORCH_CHECK(world >= 1 && world <= kMaxRanks && (int)bufs.size() == world, "ArComm: bad world size");
    TORCH_CHECK(half_bytes % 4096 == 0 && fuse_half_bytes % 4096 == 0 && seg_slot_bytes % 256 == 0,
                "ArComm: buffer regions must be multiples of 4 KiB (segment slots of 256 B)");
    std::memset(&c_, 0, sizeof(c_));
    for (int i = 0; i < world; ++i) c_.bufs[i] = reinterpret_cast<char*>(bufs[i]);
    c_.mc = reinterpret_cast<char*>(mc);
    c_.state = reinterpret_cast<uint32_t*>(state);
    c_.status = reinterpret_cast<uint32_t*>(status_dev);
    c_.timeout_ns = timeout_ns;
    c_.half_bytes = half_bytes;
    c_.seg_slot_bytes = seg_slot_bytes;
    c_.fuse_off = kSigBytes + 2 * half_bytes;
    c_.fuse_half_bytes = fuse_half_bytes;
    // buffer layout: [signals][2 AR halves][2 fused halves][segment slots][G]
    c_.sp_off = sp_bytes ? kSigBytes + 2 * half_bytes + 2 * fuse_half_bytes +
                               (uint64_t)kSegSlots * kMaxRanks * seg_slot_bytes
                         : 0;
    c_.sp_bytes = sp_bytes;
    c_.trace = nullptr;
    c_.rank = rank;
    c_.world = world;
  }
  void allreduce(int64_t in, int64_t out, uint64_t nbytes, int dtype, int algo, int max_blocks, int64_t stream) {
    ar_launch(c_, algo, dtype, reinterpret_cast<const void*>(in), reinterpret_cast<void*>(out), nbytes, max_blocks,
              stream_of(stream));
  }
  void ar_rmsnorm(int64_t in, int64_t residual, int64_t weight, int64_t out, int M, int H, double eps, int algo,
                  int max_blocks, int64_t stream, int threads) {
    ar_rmsnorm_launch(c_, algo, reinterpret_cast<const void*>(in), reinterpret_cast<void*>(residual),
                      reinterpret_cast<const void*>(weight), reinterpret_cast<void*>(out), M, H, (float)eps,
                      max_blocks, stream_of(stream), threads);
  }
  void allgather(int64_t in, int64_t out, uint64_t nbytes, int max_blocks, int64_t stream) {
    ar_allgather_launch(c_, reinterpret_cast<const void*>(in), reinterpret_cast<void*>(out), nbytes, max_blocks,
                        stream_of(stream));
  }
  void seg_submit(int64_t in, uint64_t nbytes, int max_blocks, int64_t stream) {
    seg_submit_launch(c_, reinterpret_cast<const void*>(in), nbytes, max_blocks, stream_of(stream));
  }
  void seg_wait(int64_t local, int64_t out, uint64_t nbytes, int dtype, int max_blocks, int64_t stream) {
    seg_wait_launch(c_, dtype, reinterpret_cast<const void*>(local), reinterpret_cast<void*>(out), nbytes, max_blocks,
                    stream_of(stream));
  }
  void gemm_ar_rmsnorm(torch::Tensor a, torch::Tensor w, torch::Tensor residual, torch::Tensor norm_w,
                       torch::Tensor out, double eps, torch::Tensor err, int max_blocks, bool push_all) {
    check_bf16(a, "a");
    check_bf16(w, "w");
    check_bf16(residual, "residual");
    check_bf16(norm_w, "norm_w");
    check_bf16(out, "out");
    const int64_t M = a.size(0), K = a.size(1), N = w.size(0);
    TORCH_CHECK(w.size(1) == K && residual.numel() == M * N && out.numel() == M * N && norm_w.numel() == N,
                "gemm_ar_rmsnorm: shape mismatch");
    gemm_ar_rmsnorm_launch(c_, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), M, N, K, residual.data_ptr(),
                           norm_w.data_ptr(), out.data_ptr(), (float)eps,
                           reinterpret_cast<uint32_t*>(err.data_ptr<int>()), max_blocks, push_all, cur_stream());
  }
  uint64_t fused_capacity() const { return c_.fuse_half_bytes; }
  // The two launches of gemm_ar_rmsnorm one at a time (one-GPU emulation of
  // the ranks runs every rank's GEMM before any rank's reduction).
  void gemm_push(torch::Tensor a, torch::Tensor w, torch::Tensor err, bool push_all) {
    check_bf16(a, "a");
    check_bf16(w, "w");
    TORCH_CHECK(w.size(1) == a.size(1), "gemm_push: K mismatch");
    gemm_push_launch(c_, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), a.size(0), w.size(0), a.size(1),
                     push_all, reinterpret_cast<uint32_t*>(err.data_ptr<int>()), cur_stream());
  }
  void fused_allsum_norm(int M, int N, int64_t residual, int64_t weight, int64_t out, double eps, int max_blocks) {
    fused_allsum_norm_launch(c_, M, N, reinterpret_cast<void*>(residual), reinterpret_cast<const void*>(weight),
                             reinterpret_cast<void*>(out), (float)eps, max_blocks, cur_stream());
  }
  const ArCtx& ctx() const { return c_; }

  // ---- sequence parallel (rank r owns rows [r*Mo, r*Mo+Mo), Mo = ceil(M/world))
  void gemm_rs(torch::Tensor a, torch::Tensor w, torch::Tensor err) {
    check_bf16(a, "a");
    check_bf16(w, "w");
    TORCH_CHECK(w.size(1) == a.size(1), "gemm_rs: K mismatch");
    gemm_rs_launch(c_, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), a.size(0), w.size(0), a.size(1),
                   reinterpret_cast<uint32_t*>(err.data_ptr<int>()), cur_stream());
  }
  void sp_rs_push(torch::Tensor x, int max_blocks) {
    check_bf16(x, "x");
    TORCH_CHECK(x.dim() == 2, "sp_rs_push: x must be [M, N]");
    sp_rs_push_launch(c_, x.data_ptr(), (int)x.size(0), (int)x.size(1), max_blocks, cur_stream());
  }
  void sp_rs_norm_ag(int M, torch::Tensor res_own, torch::Tensor w, double eps, int max_blocks) {
    check_bf16(res_own, "res_own");
    check_bf16(w, "w");
    const int N = (int)w.numel();
    const int Mo = (M + c_.world - 1) / c_.world;
    TORCH_CHECK(res_own.numel() >= (int64_t)Mo * N, "sp_rs_norm_ag: residual shard must hold Mo rows");
    sp_rs_norm_ag_launch(c_, M, N, res_own.data_ptr(), w.data_ptr(), (float)eps, max_blocks, cur_stream());
  }
  // out[M, Nout] = G[M, K] * w[Nout, K]^T, loading each m-tile once its owners' rows landed.
  void sp_gemm_ag(int M, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> workspace,
                  torch::Tensor err) {
    check_bf16(w, "w");
    check_bf16(out, "out");
    const int64_t N = w.size(0), K = w.size(1);
    TORCH_CHECK(out.size(0) >= M && out.size(1) == N, "sp_gemm_ag: out must be [M, Nout]");
    TORCH_CHECK((uint64_t)M * K * 2 <= c_.sp_bytes, "sp_gemm_ag: rows exceed the gather buffer");
    float* ws = nullptr;
    if (workspace.has_value()) {
      const int64_t need_splits = gemm_plan(M, N, K).splits;
      TORCH_CHECK(workspace->numel() >= need_splits * M * N, "sp_gemm_ag: workspace too small");
      ws = workspace->data_ptr<float>();
    }
    GemmAgWait ag;
    ag.flags = reinterpret_cast<const uint32_t*>(c_.bufs[c_.rank] + kAgFlagOff);
    ag.epoch_word = c_.state + kStFuseEpoch;
    ag.Mo = (M + c_.world - 1) / c_.world;
    gemm_launch(c_.bufs[c_.rank] + c_.sp_off, K, w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0), nullptr, M,
                N, K, 0, 0, ws, nullptr, reinterpret_cast<uint32_t*>(err.data_ptr<int>()), cur_stream(), &ag);
  }
  void sp_ag_wait(int M) { sp_ag_wait_launch(c_, M, cur_stream()); }
  int64_t sp_gather_ptr() const { return c_.sp_off ? reinterpret_cast<int64_t>(c_.bufs[c_.rank] + c_.sp_off) : 0; }
  uint64_t sp_capacity() const { return c_.sp_bytes; }
  // Device array of >= 8 uint64 that block 0 of every later allreduce call
  // fills with %globaltimer phase marks (0 = off).
  void set_trace(int64_t ptr) { c_.trace = reinterpret_cast<uint64_t*>(ptr); }
  uint64_t chunk_limit(int algo) const { return ar_chunk_limit(c_, algo); }
  std::vector<int64_t> status() const {
    std::vector<int64_t> v(kStatusWords);
    for (int i = 0; i < kStatusWords; ++i) v[i] = status_host_[i];
    return v;
  }
  int64_t error() const { return status_host_[kStatusErr]; }
  void clear_status() {
    for (int i = 0; i < kStatusWords; ++i) status_host_[i] = 0;
  }
  bool has_multicast() const { return c_.mc != nullptr; }

 private:
  ArCtx c_;
  volatile uint32_t* status_host_;
};

// ---------------------------------------------------------------- ops
void rmsnorm(torch::Tensor x, torch::Tensor w, torch::Tensor out, double eps) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(out, "out");
  const int H = x.size(-1);
  TORCH_CHECK(w.numel() == H && out.numel() == x.numel(), "rmsnorm: shape mismatch");
  rmsnorm_launch(x.data_ptr(), nullptr, w.data_ptr(), out.data_ptr(), x.numel() / H, H, (float)eps, cur_stream());
}

void fused_add_rmsnorm(torch::Tensor x, torch::Tensor residual, torch::Tensor w, torch::Tensor out, double eps) {
  check_bf16(x, "x");
  check_bf16(residual, "residual");
  check_bf16(w, "w");
  check_bf16(out, "out");
  const int H = x.size(-1);
  TORCH_CHECK(w.numel() == H && residual.numel() == x.numel() && out.numel() == x.numel(),
              "fused_add_rmsnorm: shape mismatch");
  rmsnorm_launch(x.data_ptr(), residual.data_ptr(), w.data_ptr(), out.data_ptr(), x.numel() / H, H, (float)eps,
                 cur_stream());
}

void rope_and_cache(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                    c10::optional<torch::Tensor> slots, torch::Tensor q_out, c10::optional<torch::Tensor> k_cache,
                    c10::optional<torch::Tensor> v_cache, int64_t nq, int64_t nkv, int64_t page,
                    c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, double eps) {
  check_bf16(qkv, "qkv");
  check_bf16(q_out, "q_out");
  check_cuda(positions, "positions");
  check_cuda(cos_sin, "cos_sin");
  TORCH_CHECK(positions.scalar_type() == torch::kInt32, "positions must be int32");
  TORCH_CHECK(cos_sin.scalar_type() == torch::kFloat32 && cos_sin.dim() == 2 && cos_sin.size(1) == 128,
              "cos_sin must be fp32 [P, 128]");
  const int64_t T = qkv.size(0);
  TORCH_CHECK(qkv.size(1) == (nq + 2 * nkv) * 128, "qkv width mismatch (head_dim must be 128)");
  TORCH_CHECK(positions.numel() == T && q_out.numel() == T * nq * 128, "rope: shape mismatch");
  const int64_t* sp = nullptr;
  void *kc = nullptr, *vc = nullptr;
  if (slots.has_value()) {
    check_cuda(*slots, "slots");
    TORCH_CHECK(slots->scalar_type() == torch::kInt64 && slots->numel() == T, "slots must be int64 [T]");
    TORCH_CHECK(k_cache.has_value() && v_cache.has_value(), "caches required with slots");
    check_bf16(*k_cache, "k_cache");
    check_bf16(*v_cache, "v_cache");
    TORCH_CHECK(k_cache->dim() == 4 && k_cache->size(1) == nkv && k_cache->size(2) == page && k_cache->size(3) == 128,
                "k_cache must be [blocks, nkv, page, 128]");
    sp = slots->data_ptr<int64_t>();
    kc = k_cache->data_ptr();
    vc = v_cache->data_ptr();
  }
  const void *qn = nullptr, *kn = nullptr;
  TORCH_CHECK(q_norm.has_value() == k_norm.has_value(), "q_norm and k_norm go together");
  if (q_norm.has_value()) {
    check_bf16(*q_norm, "q_norm");
    check_bf16(*k_norm, "k_norm");
    TORCH_CHECK(q_norm->numel() == 128 && k_norm->numel() == 128 && q_norm->is_contiguous() &&
                    k_norm->is_contiguous() && qkv.is_contiguous(),
                "q_norm / k_norm must be contiguous [128] (and qkv contiguous)");
    qn = q_norm->data_ptr();
    kn = k_norm->data_ptr();
  }
  rope_and_cache_launch(qkv.data_ptr(), positions.data_ptr<int>(), cos_sin.data_ptr<float>(), sp, q_out.data_ptr(), kc,
                        vc, T, (int)nq, (int)nkv, (int)page, cur_stream(), qn, kn, (float)eps);
}

void check_awq(const torch::Tensor& qweight, const torch::Tensor& qzeros, const torch::Tensor& scales, int64_t G,
               int64_t& K, int64_t& N) {
  check_cuda(qweight, "qweight");
  check_cuda(qzeros, "qzeros");
  check_cuda(scales, "scales");
  TORCH_CHECK(qweight.scalar_type() == torch::kInt32 && qzeros.scalar_type() == torch::kInt32 &&
                  scales.scalar_type() == torch::kHalf,
              "awq: qweight / qzeros int32, scales fp16");
  TORCH_CHECK(qweight.is_contiguous() && qzeros.is_contiguous() && scales.is_contiguous(), "awq: contiguous tensors");
  K = qweight.size(0);
  N = qweight.size(1) * 8;
  TORCH_CHECK(G > 0 && K % G == 0 && qzeros.size(0) == K / G && qzeros.size(1) == N / 8 && scales.size(0) == K / G &&
                  scales.size(1) == N,
              "awq: shapes of qweight [K, N/8], qzeros [K/G, N/8], scales [K/G, N]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(scales.data_ptr()) % 16 == 0, "awq: scales must be 16-byte aligned");
}

void awq_gemv(torch::Tensor x, torch::Tensor qweight, torch::Tensor qzeros, torch::Tensor scales, int64_t G,
              torch::Tensor ws, torch::Tensor out, c10::optional<torch::Tensor> residual) {
  int64_t K, N;
  check_awq(qweight, qzeros, scales, G, K, N);
  check_bf16(x, "x");
  check_bf16(out, "out");
  TORCH_CHECK(G <= 256, "awq_gemv: group size above 256");
  TORCH_CHECK(x.dim() == 2 && x.size(1) == K && x.stride(1) == 1, "awq_gemv: x must be [M, K] with unit stride");
  const int64_t M = x.size(0);
  TORCH_CHECK(M >= 1 && M <= kAwqGemvMaxRows, "awq_gemv: 1..8 rows");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "awq_gemv: out [M, N]");
  TORCH_CHECK(ws.scalar_type() == torch::kFloat32 && ws.is_contiguous() && ws.numel() >= (K / G) * M * N,
              "awq_gemv: fp32 workspace of (K/G) * M * N");
  const void* res = nullptr;
  if (residual.has_value()) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->sizes() == out.sizes() && residual->strides() == out.strides(),
                "awq_gemv: residual laid out like out");
    res = residual->data_ptr();
  }
  AwqGemvArgs a{x.data_ptr(), x.stride(0), qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(),
                ws.data_ptr<float>(), res, out.data_ptr(), out.stride(0), (int)M, (int)K, (int)N, (int)G};
  awq_gemv_launch(a, cur_stream());
}

void awq_dequant(torch::Tensor qweight, torch::Tensor qzeros, torch::Tensor scales, int64_t G, torch::Tensor out) {
  int64_t K, N;
  check_awq(qweight, qzeros, scales, G, K, N);
  check_bf16(out, "out");
  TORCH_CHECK(out.is_contiguous() && out.numel() >= N * K, "awq_dequant: out must hold bf16 [N, K]");
  awq_dequant_launch(qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(), out.data_ptr(), (int)K, (int)N,
                     (int)G, cur_stream());
}

void silu_mul(torch::Tensor x, torch::Tensor out) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  const int I2 = x.size(-1);
  TORCH_CHECK(out.numel() * 2 == x.numel(), "silu_mul: shape mismatch");
  silu_mul_launch(x.data_ptr(), out.data_ptr(), x.numel() / I2, I2, cur_stream());
}

// out[M, F] = silu(x @ gate^T) * (x @ up^T) in one GEMV for 1-2 rows; false
// (nothing launched) when the shape or alignment does not fit it.
bool gemv_silu(torch::Tensor x, torch::Tensor w, torch::Tensor out) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(out, "out");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2 && x.size(1) == w.size(1) &&
                  out.size(0) == x.size(0) && out.size(1) * 2 == w.size(0),
              "gemv_silu: shapes must be x [M, K], w [2F, K], out [M, F]");
  TORCH_CHECK(w.stride(1) == 1 && x.stride(1) == 1 && out.stride(1) == 1, "gemv_silu: rows must be contiguous");
  if (!gemv_bf16_supported(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), x.size(0), x.size(1))) return false;
  gemv_silu_launch(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0), x.size(0),
                   w.size(0), x.size(1), cur_stream());
  return true;
}

// q_out / paged k, v = RoPE(x @ w_qkv^T) in one GEMV for 1-2 tokens (no
// q/k norm, no bias); false (nothing launched) when it does not fit.
bool gemv_rope(torch::Tensor x, torch::Tensor w, torch::Tensor positions, torch::Tensor cos_sin,
               c10::optional<torch::Tensor> slots, torch::Tensor q_out, c10::optional<torch::Tensor> k_cache,
               c10::optional<torch::Tensor> v_cache, int64_t nq, int64_t nkv, int64_t page) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(q_out, "q_out");
  check_cuda(positions, "positions");
  check_cuda(cos_sin, "cos_sin");
  const int64_t M = x.size(0);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1) && w.size(0) == (nq + 2 * nkv) * 128,
              "gemv_rope: x [M, K], w [(nq + 2 nkv) * 128, K]");
  TORCH_CHECK(positions.scalar_type() == torch::kInt32 && positions.numel() == M, "positions must be int32 [M]");
  TORCH_CHECK(cos_sin.scalar_type() == torch::kFloat32 && cos_sin.dim() == 2 && cos_sin.size(1) == 128,
              "cos_sin must be fp32 [P, 128]");
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == M * nq * 128, "q_out must be [M, nq, 128]");
  TORCH_CHECK(w.stride(1) == 1 && x.stride(1) == 1, "gemv_rope: rows must be contiguous");
  const int64_t* sp = nullptr;
  void *kc = nullptr, *vc = nullptr;
  if (slots.has_value()) {
    check_cuda(*slots, "slots");
    TORCH_CHECK(slots->scalar_type() == torch::kInt64 && slots->numel() == M, "slots must be int64 [M]");
    TORCH_CHECK(k_cache.has_value() && v_cache.has_value(), "caches required with slots");
    check_bf16(*k_cache, "k_cache");
    check_bf16(*v_cache, "v_cache");
    TORCH_CHECK(k_cache->dim() == 4 && k_cache->size(1) == nkv && k_cache->size(2) == page && k_cache->size(3) == 128,
                "k_cache must be [blocks, nkv, page, 128]");
    sp = slots->data_ptr<int64_t>();
    kc = k_cache->data_ptr();
    vc = v_cache->data_ptr();
  }
  if (!gemv_bf16_supported(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), M, x.size(1))) return false;
  gemv_rope_launch(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), M, x.size(1), positions.data_ptr<int>(),
                   cos_sin.data_ptr<float>(), sp, q_out.data_ptr(), kc, vc, (int)nq, (int)nkv, (int)page,
                   cur_stream());
  return true;
}

void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, int64_t start) {
  check_bf16(table, "table");
  check_bf16(out, "out");
  check_cuda(ids, "ids");
  TORCH_CHECK(ids.scalar_type() == torch::kInt32, "ids must be int32");
  TORCH_CHECK(out.numel() == ids.numel() * table.size(1), "embedding: shape mismatch");
  embedding_launch(ids.data_ptr<int>(), table.data_ptr(), out.data_ptr(), ids.numel(), table.size(1), start,
                   table.size(0), cur_stream());
}

void argmax(torch::Tensor logits, int64_t offset, torch::Tensor best_val, torch::Tensor best_idx) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "argmax: logits [B, V] row-major");
  TORCH_CHECK(logits.scalar_type() == torch::kBFloat16 || logits.scalar_type() == torch::kFloat32,
              "argmax: bf16 or fp32 logits");
  TORCH_CHECK(best_val.scalar_type() == torch::kFloat32 && best_idx.scalar_type() == torch::kInt64 &&
                  best_val.numel() >= logits.size(0) && best_idx.numel() >= logits.size(0),
              "argmax: outputs must be fp32/int64 [B]");
  argmax_launch(logits.data_ptr(), logits.scalar_type() == torch::kBFloat16, logits.stride(0), logits.size(0),
                logits.size(1), offset, best_val.data_ptr<float>(), best_idx.data_ptr<int64_t>(), cur_stream());
}

void argmax_combine(torch::Tensor vals, torch::Tensor idxs, torch::Tensor out) {
  check_cuda(vals, "vals");
  check_cuda(idxs, "idxs");
  TORCH_CHECK(vals.dim() == 2 && idxs.sizes() == vals.sizes() && vals.scalar_type() == torch::kFloat32 &&
                  idxs.scalar_type() == torch::kInt64,
              "argmax_combine: fp32/int64 [W, B]");
  argmax_combine_launch(vals.data_ptr<float>(), idxs.data_ptr<int64_t>(), vals.size(0), vals.size(1),
                        out.data_ptr<int64_t>(), cur_stream());
}

void gemm(torch::Tensor A, torch::Tensor B, torch::Tensor C, c10::optional<torch::Tensor> residual,
          c10::optional<torch::Tensor> workspace, torch::Tensor err, int64_t bn, int64_t splits,
          c10::optional<torch::Tensor> counters) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == torch::kBFloat16 && B.scalar_type() == torch::kBFloat16 &&
                  C.scalar_type() == torch::kBFloat16,
              "gemm: bf16 operands");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm: 2-D operands");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm: row-major operands");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && C.size(0) == M && C.size(1) == N, "gemm: shape mismatch");
  TORCH_CHECK(err.scalar_type() == torch::kInt32 && err.is_cuda(), "gemm: err must be an int32 CUDA word");
  const void* res = nullptr;
  if (residual.has_value()) {
    TORCH_CHECK(residual->scalar_type() == torch::kBFloat16 && residual->sizes() == C.sizes() &&
                    residual->strides() == C.strides(),
                "gemm: residual must match C");
    res = residual->data_ptr();
  }
  float* ws = nullptr;
  if (workspace.has_value()) {
    TORCH_CHECK(workspace->scalar_type() == torch::kFloat32 && workspace->is_cuda(), "gemm: fp32 workspace");
    const int64_t need_splits = splits > 0 ? splits : gemm_plan(M, N, K).splits;
    TORCH_CHECK(workspace->numel() >= need_splits * M * N, "gemm: workspace too small");
    ws = workspace->data_ptr<float>();
  }
  uint32_t* cnt = nullptr;
  if (counters.has_value()) {
    TORCH_CHECK(counters->scalar_type() == torch::kInt32 && counters->is_cuda() && counters->numel() >= 65536,
                "gemm: counters must be a zeroed int32 CUDA buffer of >= 65536 words");
    cnt = reinterpret_cast<uint32_t*>(counters->data_ptr<int>());
  }
  const at::cuda::CUDAGuard guard(A.device());
  gemm_launch(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), C.data_ptr(), C.stride(0), res, M, N, K, (int)bn,
              (int)splits, ws, cnt, reinterpret_cast<uint32_t*>(err.data_ptr<int>()), cur_stream());
}

std::vector<int64_t> gemm_plan_py(int64_t M, int64_t N, int64_t K) {
  GemmPlan p = gemm_plan(M, N, K);
  return {p.bn, p.splits};
}

void prefill_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor out,
                       torch::Tensor cu_q, torch::Tensor kv_len, torch::Tensor block_table, torch::Tensor tiles,
                       double scale) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  check_bf16(k_cache, "k_cache");
  check_bf16(v_cache, "v_cache");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128, "q must be [T, nq, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == 16 && k_cache.size(3) == 128,
              "k_cache must be [blocks, nkv, 16, 128]");
  for (auto* t : {&cu_q, &kv_len, &block_table, &tiles}) {
    check_cuda(*t, "index tensor");
    TORCH_CHECK(t->scalar_type() == torch::kInt32, "index tensors must be int32");
  }
  TORCH_CHECK(tiles.dim() == 2 && tiles.size(1) == 2, "tiles must be [n, 2]");
  prefill_attention_launch(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), cu_q.data_ptr<int>(),
                           kv_len.data_ptr<int>(), block_table.data_ptr<int>(), block_table.size(1),
                           tiles.data_ptr<int>(), tiles.size(0), q.size(1), k_cache.size(1), (float)scale,
                           cur_stream());
}

void prefill_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor out,
                          torch::Tensor cu_q, torch::Tensor kv_len, torch::Tensor block_table, torch::Tensor tiles,
                          double scale, torch::Tensor err, int64_t splits, c10::optional<torch::Tensor> part_o,
                          c10::optional<torch::Tensor> part_lse) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  check_bf16(k_cache, "k_cache");
  check_bf16(v_cache, "v_cache");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128, "q must be [T, nq, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == 16 && k_cache.size(3) == 128,
              "k_cache must be [blocks, nkv, 16, 128]");
  for (auto* t : {&cu_q, &kv_len, &block_table, &tiles}) {
    check_cuda(*t, "index tensor");
    TORCH_CHECK(t->scalar_type() == torch::kInt32, "index tensors must be int32");
  }
  TORCH_CHECK(tiles.dim() == 2 && tiles.size(1) == 2, "tiles must be [n, 2]");
  TORCH_CHECK(err.scalar_type() == torch::kInt32 && err.is_cuda(), "err must be an int32 CUDA word");
  float *po = nullptr, *pl = nullptr;
  if (splits > 1) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "split-KV prefill needs scratch tensors");
    TORCH_CHECK(part_o->numel() >= q.size(0) * q.size(1) * splits * 128 && part_lse->numel() >= q.size(0) * q.size(1) * splits,
                "split-KV prefill scratch too small");
    po = part_o->data_ptr<float>();
    pl = part_lse->data_ptr<float>();
  }
  prefill_attention_tc_launch(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
                              cu_q.data_ptr<int>(), kv_len.data_ptr<int>(), block_table.data_ptr<int>(),
                              block_table.size(1), tiles.data_ptr<int>(), tiles.size(0), q.size(0), q.size(1),
                              k_cache.size(1), k_cache.size(0), (float)scale, (int)splits, po, pl,
                              reinterpret_cast<uint32_t*>(err.data_ptr<int>()), cur_stream());
}

void decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor out,
                      torch::Tensor kv_len, torch::Tensor block_table, c10::optional<torch::Tensor> part_o,
                      c10::optional<torch::Tensor> part_lse, int64_t splits, double scale,
                      c10::optional<torch::Tensor> counters) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  check_bf16(k_cache, "k_cache");
  check_bf16(v_cache, "v_cache");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128, "q must be [B, nq, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == 16 && k_cache.size(3) == 128,
              "k_cache must be [blocks, nkv, 16, 128]");
  check_cuda(kv_len, "kv_len");
  check_cuda(block_table, "block_table");
  const int B = q.size(0), nq = q.size(1);
  float *po = nullptr, *pl = nullptr;
  if (splits > 1) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "decode: split-KV needs scratch tensors");
    TORCH_CHECK(part_o->numel() >= (int64_t)B * nq * splits * 128 && part_lse->numel() >= (int64_t)B * nq * splits,
                "decode: scratch too small");
    po = part_o->data_ptr<float>();
    pl = part_lse->data_ptr<float>();
  }
  int* cnt = nullptr;
  if (splits > 1 && counters.has_value()) {
    check_cuda(*counters, "counters");
    TORCH_CHECK(counters->scalar_type() == torch::kInt32 && counters->numel() >= (int64_t)B * k_cache.size(1),
                "decode: counters must be int32 with at least batch * kv_heads zeros");
    cnt = counters->data_ptr<int>();
  }
  decode_attention_launch(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), kv_len.data_ptr<int>(),
                          block_table.data_ptr<int>(), block_table.size(1), B, nq, k_cache.size(1), (int)splits, po,
                          pl, (float)scale, cur_stream(), cnt);
}

}  // namespace
}  // namespace mbx

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels: symmetric memory, allreduce, tcgen05 GEMM, attention, elementwise ops";
  using namespace mbx;
  m.attr("SIG_BYTES") = (int64_t)kSigBytes;
  m.attr("BAR_WORDS") = (int64_t)kPhases * kMaxBlocks * kMaxRanks;  // barrier flags at offset 0
  m.attr("GEMV_MAX_ROWS") = (int)kGemvMaxRows;
  m.attr("MAX_RANKS") = kMaxRanks;
  m.attr("MAX_BLOCKS") = kMaxBlocks;
  m.attr("STATE_WORDS") = (int)kStWords;
  m.attr("STATUS_WORDS") = (int)kStatusWords;
  m.attr("SEG_SLOTS") = kSegSlots;

  py::class_<SymmAlloc>(m, "SymmAlloc")
      .def_readonly("id", &SymmAlloc::id)
      .def_readonly("ptr", &SymmAlloc::ptr)
      .def_readonly("fd", &SymmAlloc::fd);
  py::class_<HostMapped>(m, "HostMapped").def_readonly("host", &HostMapped::host).def_readonly("dev", &HostMapped::dev);
  m.def("symm_granularity", &symm_granularity, py::arg("device"), py::arg("multicast"), py::arg("ndev"));
  m.def("symm_create", &symm_create, py::arg("device"), py::arg("size"));
  m.def("symm_import", &symm_import, py::arg("device"), py::arg("fd"), py::arg("size"));
  m.def("symm_free", &symm_free, py::arg("id"));
  m.def("mc_supported", &mc_supported, py::arg("device"));
  m.def("mc_create", &mc_create, py::arg("ndev"), py::arg("size"));
  m.def("mc_import", &mc_import, py::arg("fd"), py::arg("size"));
  m.def("mc_add_device", &mc_add_device, py::arg("mc_id"), py::arg("device"));
  m.def("mc_bind", &mc_bind, py::arg("mc_id"), py::arg("mem_id"), py::arg("size"));
  m.def("mc_map", &mc_map, py::arg("mc_id"), py::arg("device"), py::arg("size"));
  m.def("mc_unbind", &mc_unbind, py::arg("mc_id"), py::arg("device"), py::arg("size"));
  m.def("close_fd", &close_fd, py::arg("fd"));
  m.def("ipc_get_handle", [](int64_t p) { return py::bytes(ipc_get_handle(p)); }, py::arg("ptr"));
  m.def("ipc_open", [](py::bytes h) { return ipc_open(std::string(h)); }, py::arg("handle"));
  m.def("ipc_close", &ipc_close, py::arg("ptr"));
  m.def("host_mapped_alloc", &host_mapped_alloc, py::arg("bytes"));
  m.def("host_mapped_free", &host_mapped_free, py::arg("host"));

  py::class_<ArComm>(m, "ArComm")
      .def(py::init<int, int, std::vector<int64_t>, int64_t, int64_t, int64_t, int64_t, uint64_t, uint64_t, uint64_t,
                    uint64_t, uint64_t>(),
           py::arg("rank"), py::arg("world"), py::arg("bufs"), py::arg("mc"), py::arg("state"), py::arg("status_dev"),
           py::arg("status_host"), py::arg("half_bytes"), py::arg("seg_slot_bytes"), py::arg("timeout_ns"),
           py::arg("fuse_half_bytes") = 0, py::arg("sp_bytes") = 0)
      .def("gemm_rs", &ArComm::gemm_rs)
      .def("sp_rs_push", &ArComm::sp_rs_push)
      .def("sp_rs_norm_ag", &ArComm::sp_rs_norm_ag)
      .def("sp_gemm_ag", &ArComm::sp_gemm_ag, py::arg("M"), py::arg("w"), py::arg("out"), py::arg("workspace"),
           py::arg("err"))
      .def("sp_ag_wait", &ArComm::sp_ag_wait)
      .def("sp_gather_ptr", &ArComm::sp_gather_ptr)
      .def("sp_capacity", &ArComm::sp_capacity)
      .def("gemm_ar_rmsnorm", &ArComm::gemm_ar_rmsnorm)
      .def("gemm_push", &ArComm::gemm_push)
      .def("fused_allsum_norm", &ArComm::fused_allsum_norm)
      .def("fused_capacity", &ArComm::fused_capacity)
      .def("set_trace", &ArComm::set_trace)
      .def("allreduce", &ArComm::allreduce, py::arg("inp"), py::arg("out"), py::arg("nbytes"), py::arg("dtype"),
           py::arg("algo"), py::arg("max_blocks"), py::arg("stream"))
      .def("ar_rmsnorm", &ArComm::ar_rmsnorm, py::arg("inp"), py::arg("residual"), py::arg("weight"), py::arg("out"),
           py::arg("M"), py::arg("H"), py::arg("eps"), py::arg("algo"), py::arg("max_blocks"), py::arg("stream"),
           py::arg("threads") = 512)
      .def("allgather", &ArComm::allgather, py::arg("inp"), py::arg("out"), py::arg("nbytes"), py::arg("max_blocks"),
           py::arg("stream"))
      .def("seg_submit", &ArComm::seg_submit, py::arg("inp"), py::arg("nbytes"), py::arg("max_blocks"),
           py::arg("stream"))
      .def("seg_wait", &ArComm::seg_wait, py::arg("local"), py::arg("out"), py::arg("nbytes"), py::arg("dtype"),
           py::arg("max_blocks"), py::arg("stream"))
      .def("chunk_limit", &ArComm::chunk_limit, py::arg("algo"))
      .def("status", &ArComm::status)
      .def("error", &ArComm::error)
      .def("clear_status", &ArComm::clear_status)
      .def("has_multicast", &ArComm::has_multicast);
  m.def(
      "raw_transport",
      [](int kind, int64_t dst, int64_t src, uint64_t nbytes, int grid, int threads, int64_t stream) {
        raw_transport_launch(kind, reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), nbytes, grid,
                             threads, stream_of(stream));
      },
      py::arg("kind"), py::arg("dst"), py::arg("src"), py::arg("nbytes"), py::arg("grid"), py::arg("threads"),
      py::arg("stream"));
  m.def(
      "ce_push",
      [](int64_t dst, int64_t src, uint64_t nbytes, int64_t stream) {
        cudaError_t e = cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), nbytes,
                                        cudaMemcpyDeviceToDevice, stream_of(stream));
        TORCH_CHECK(e == cudaSuccess, "ce_push: ", cudaGetErrorString(e));
      },
      py::arg("dst"), py::arg("src"), py::arg("nbytes"), py::arg("stream"));

  m.def(
      "ar_emulated",
      [](std::vector<ArComm*> comms, int op, int algo, int dtype, std::vector<int64_t> ins, std::vector<int64_t> outs,
         std::vector<int64_t> residuals, int64_t weight, uint64_t nbytes, int M, int N, double eps, int blocks,
         int64_t scratch, int64_t scratch_bytes, int threads) {
        const int W = (int)comms.size();
        TORCH_CHECK(W >= 2 && W <= kMaxRanks && (int)ins.size() == W && (int)outs.size() == W,
                    "ar_emulated: one input and output per rank");
        TORCH_CHECK(residuals.empty() || (int)residuals.size() == W, "ar_emulated: one residual per rank");
        TORCH_CHECK((uint64_t)scratch_bytes >= sizeof(EmuRank) * W, "ar_emulated: scratch too small");
        std::vector<EmuRank> r(W);
        for (int i = 0; i < W; ++i) {
          r[i].c = comms[i]->ctx();
          TORCH_CHECK(r[i].c.rank == i && r[i].c.world == W, "ar_emulated: comms must be ranks 0..W-1 of one world");
          r[i].in = reinterpret_cast<const void*>(ins[i]);
          r[i].out = reinterpret_cast<void*>(outs[i]);
          r[i].residual = residuals.empty() ? nullptr : reinterpret_cast<void*>(residuals[i]);
          r[i].weight = reinterpret_cast<const void*>(weight);
        }
        ar_emulated_launch(r.data(), W, op, algo, dtype, nbytes, M, N, (float)eps, blocks,
                           reinterpret_cast<void*>(scratch), cur_stream(), threads);
      },
      py::arg("comms"), py::arg("op"), py::arg("algo"), py::arg("dtype"), py::arg("ins"), py::arg("outs"),
      py::arg("residuals"), py::arg("weight"), py::arg("nbytes"), py::arg("M"), py::arg("N"), py::arg("eps"),
      py::arg("blocks"), py::arg("scratch"), py::arg("scratch_bytes"), py::arg("threads") = 512);
  m.attr("EMU_ALLREDUCE") = (int)kEmuAllreduce;
  m.attr("EMU_AR_RMSNORM") = (int)kEmuArRmsnorm;
  m.attr("EMU_FUSED_RS_NORM") = (int)kEmuFusedRsNorm;
  m.attr("EMU_ALLGATHER") = (int)kEmuAllgather;
  m.attr("EMU_RANK_BYTES") = (int)sizeof(EmuRank);
  m.def("gemm", &gemm, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("residual"), py::arg("workspace"),
        py::arg("err"), py::arg("bn") = 0, py::arg("splits") = 0, py::arg("counters") = c10::nullopt);
  m.def("gemm_plan", &gemm_plan_py, py::arg("M"), py::arg("N"), py::arg("K"));
  m.def("rmsnorm", &rmsnorm);
  m.def("fused_add_rmsnorm", &fused_add_rmsnorm);
  m.def("rope_and_cache", &rope_and_cache);
  m.def("awq_gemv", &awq_gemv);
  m.def("awq_dequant", &awq_dequant);
  m.def("silu_mul", &silu_mul);
  m.def("gemv_silu", &gemv_silu, py::arg("x"), py::arg("w"), py::arg("out"));
  m.def("gemv_rope", &gemv_rope, py::arg("x"), py::arg("w"), py::arg("positions"), py::arg("cos_sin"),
        py::arg("slots"), py::arg("q_out"), py::arg("k_cache"), py::arg("v_cache"), py::arg("nq"), py::arg("nkv"),
        py::arg("page"));
  m.def("embedding", &embedding);
  m.def("argmax", &argmax);
  m.def("argmax_combine", &argmax_combine);
  m.def("prefill_attention", &prefill_attention);
  m.def("prefill_attention_tc", &prefill_attention_tc);
  m.def("decode_attention", &decode_attention, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("out"),
        py::arg("kv_len"), py::arg("block_table"), py::arg("part_o"), py::arg("part_lse"), py::arg("splits"),
        py::arg("scale"), py::arg("counters") = c10::nullopt);
}
