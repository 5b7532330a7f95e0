// PyTorch bindings of the sm_100a kernels and the C++ KV runtime.
//
// Every wrapper checks device, dtype, contiguity and shapes, then launches on
// the current CUDA stream of the tensors' device.  There is no fallback: a
// wrong argument raises, and a missing extension is reported by the Python
// loader on GPU machines.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/numpy.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "adamw.h"
#include "attention.h"
#include "ep.h"
#include "comm.h"
#include "diffusion.h"
#include "dp.h"
#include "elementwise.h"
#include "gemm.h"
#include "grpo.h"
#include "moe.h"
#include "kv_manager.h"
#include "sampling.h"

namespace {

using torch::Tensor;

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_DT(t, dt) TORCH_CHECK((t).scalar_type() == (dt), #t " has the wrong dtype")
#define CHECK_ROWS(t) TORCH_CHECK((t).dim() == 2 && (t).stride(1) == 1, #t " must be 2-D with unit inner stride")

void check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

template <typename T>
T* ptr_or_null(const c10::optional<Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

const __nv_bfloat16* bf(const Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
__nv_bfloat16* bfm(const Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

// out[N, M or M/2] = x[N, K] @ w[M, K]^T (+ bias) (+ residual)
void gemm(Tensor w, Tensor x, Tensor out, c10::optional<Tensor> bias, c10::optional<Tensor> residual, int64_t epilogue,
          bool allow_split, Tensor workspace, Tensor counters, Tensor status, bool prefetch_weights,
          int64_t split_mode) {
  CHECK_CUDA(w);
  CHECK_CUDA(x);
  CHECK_CUDA(out);
  CHECK_DT(w, torch::kBFloat16);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_ROWS(w);
  CHECK_ROWS(x);
  CHECK_ROWS(out);
  TORCH_CHECK(w.size(1) == x.size(1), "reduction dimensions differ");
  const int M = w.size(0), N = x.size(0), K = w.size(1);
  const int out_cols = epilogue == 1 ? M / 2 : M;
  TORCH_CHECK(out.size(0) == N && out.size(1) == out_cols, "output shape mismatch");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kFloat32, "bf16 or fp32 output");
  if (bias.has_value() && bias->defined()) {
    CHECK_DT(*bias, torch::kBFloat16);
    TORCH_CHECK(bias->numel() == M && bias->is_contiguous(), "bias must be [M]");
  }
  if (residual.has_value() && residual->defined()) {
    CHECK_DT(*residual, torch::kBFloat16);
    CHECK_ROWS(*residual);
    TORCH_CHECK(residual->size(0) == N && residual->size(1) == out_cols, "residual shape mismatch");
  }
  CHECK_DT(workspace, torch::kFloat32);
  CHECK_DT(counters, torch::kInt32);
  CHECK_DT(status, torch::kInt32);
  c10::cuda::CUDAGuard guard(w.device());
  osb::GemmProblem p{};
  p.w = bf(w);
  p.ldw = w.stride(0);
  p.x = bf(x);
  p.ldx = x.stride(0);
  p.M = M;
  p.N = N;
  p.K = K;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.out_f32 = out.scalar_type() == torch::kFloat32;
  p.bias = ptr_or_null<const __nv_bfloat16>(bias);
  p.residual = ptr_or_null<const __nv_bfloat16>(residual);
  p.ldr = residual.has_value() && residual->defined() ? residual->stride(0) : 0;
  p.epilogue = static_cast<int>(epilogue);
  p.allow_split = allow_split ? 1 : 0;
  TORCH_CHECK(split_mode == 0 || split_mode == 1, "split_mode: 0 cluster (DSMEM), 1 global workspace");
  p.split_mode = static_cast<int>(split_mode);
  p.workspace = workspace.data_ptr<float>();
  p.workspace_floats = workspace.numel();
  p.counters = counters.data_ptr<int>();
  p.counter_slots = counters.numel();
  p.status = status.data_ptr<int>();
  p.prefetch_weights = prefetch_weights ? 1 : 0;
  check(osb::gemm_launch(p, at::cuda::getCurrentCUDAStream()), "tcgen05 gemm");
}

// Vocabulary-head scoring without stored logits: the tcgen05 GEMM h[N, K] @ w[V, K]^T
// runs with the row-statistics epilogue into `part` ([N, ceil(V / 128), 4] fp32), then
// one warp per row folds the partials.  Outputs may be undefined tensors.
void head_stats(Tensor w, Tensor x, c10::optional<Tensor> inv_temp, c10::optional<Tensor> targets, Tensor part,
                Tensor target_logit, c10::optional<Tensor> lse1, c10::optional<Tensor> lseT,
                c10::optional<Tensor> logp, c10::optional<Tensor> logq, Tensor status) {
  CHECK_CUDA(w);
  CHECK_CUDA(x);
  CHECK_DT(w, torch::kBFloat16);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_ROWS(w);
  CHECK_ROWS(x);
  TORCH_CHECK(w.size(1) == x.size(1), "reduction dimensions differ");
  const int V = w.size(0), N = x.size(0), K = w.size(1);
  const int tiles = (V + 127) / 128;
  CHECK_DT(part, torch::kFloat32);
  TORCH_CHECK(part.is_contiguous() && part.numel() >= static_cast<long long>(N) * tiles * 4,
              "part must hold [N, ceil(V / 128), 4] floats");
  CHECK_DT(target_logit, torch::kFloat32);
  TORCH_CHECK(target_logit.numel() >= N, "target_logit needs one float per row");
  for (const c10::optional<Tensor>* o : {&lse1, &lseT, &logp, &logq})
    if (o->has_value() && (*o)->defined()) {
      CHECK_DT((**o), torch::kFloat32);
      TORCH_CHECK((*o)->numel() >= N && (*o)->is_contiguous(), "outputs need one float per row");
    }
  if (inv_temp.has_value() && inv_temp->defined()) {
    CHECK_DT((*inv_temp), torch::kFloat32);
    TORCH_CHECK(inv_temp->numel() >= N && inv_temp->is_contiguous(), "inv_temp needs one float per row");
  }
  if (targets.has_value() && targets->defined()) {
    CHECK_DT((*targets), torch::kInt32);
    TORCH_CHECK(targets->numel() >= N && targets->is_contiguous(), "targets need one int32 per row");
  }
  CHECK_DT(status, torch::kInt32);
  c10::cuda::CUDAGuard guard(w.device());
  osb::GemmProblem p{};
  p.w = bf(w);
  p.ldw = w.stride(0);
  p.x = bf(x);
  p.ldx = x.stride(0);
  p.M = V;
  p.N = N;
  p.K = K;
  p.out = part.data_ptr();     // not written in statistics mode
  p.ldo = 0;
  p.out_f32 = 1;
  p.epilogue = 2;
  p.allow_split = 0;
  p.status = status.data_ptr<int>();
  p.stat_inv_temp = ptr_or_null<const float>(inv_temp);
  p.stat_targets = ptr_or_null<const int>(targets);
  p.stat_part = part.data_ptr<float>();
  p.stat_target_logit = target_logit.data_ptr<float>();
  auto stream = at::cuda::getCurrentCUDAStream();
  check(osb::gemm_launch(p, stream), "tcgen05 head statistics gemm");
  osb::HeadStatsArgs a{};
  a.part = part.data_ptr<float>();
  a.tiles = tiles;
  a.rows = N;
  a.V = V;
  a.inv_temp = p.stat_inv_temp;
  a.targets = p.stat_targets;
  a.target_logit = target_logit.data_ptr<float>();
  a.lse1 = ptr_or_null<float>(lse1);
  a.lseT = ptr_or_null<float>(lseT);
  a.logp = ptr_or_null<float>(logp);
  a.logq = ptr_or_null<float>(logq);
  check(osb::head_stats_merge_launch(a, stream), "head statistics merge");
}

// One block-diffusion remasking step (see diffusion.h).
void remask_select(Tensor tokens, int64_t a0, int64_t bl, int64_t mask_id, Tensor drawn, c10::optional<Tensor> prio,
                   c10::optional<Tensor> logq, int64_t tc, bool subset, c10::optional<Tensor> traj,
                   c10::optional<Tensor> step_lp, Tensor out_pos, Tensor out_tok, int64_t pos_offset) {
  CHECK_CUDA(tokens);
  CHECK_DT(tokens, torch::kInt64);
  CHECK_ROWS(tokens);
  CHECK_DT(drawn, torch::kInt32);
  CHECK_DT(out_pos, torch::kInt64);
  CHECK_DT(out_tok, torch::kInt64);
  const int rows = tokens.size(0);
  TORCH_CHECK(a0 >= 0 && bl > 0 && a0 + bl <= tokens.size(1), "block outside the sequences");
  TORCH_CHECK(drawn.is_contiguous() && drawn.numel() >= rows * bl, "drawn must hold rows * bl tokens");
  TORCH_CHECK(out_pos.dim() == 2 && out_pos.size(0) == rows && out_pos.size(1) >= tc && out_pos.stride(1) == 1 &&
                  out_tok.sizes() == out_pos.sizes() && out_tok.strides() == out_pos.strides(),
              "out_pos / out_tok must be [rows, >= tc] with unit column stride");
  for (const c10::optional<Tensor>* o : {&prio, &logq})
    if (o->has_value() && (*o)->defined()) {
      CHECK_DT((**o), torch::kFloat32);
      TORCH_CHECK((*o)->is_contiguous() && (*o)->numel() >= rows * bl, "per-position inputs need rows * bl floats");
    }
  for (const c10::optional<Tensor>* o : {&traj, &step_lp})
    if (o->has_value() && (*o)->defined()) {
      CHECK_DT((**o), torch::kFloat64);
      TORCH_CHECK((*o)->is_contiguous() && (*o)->numel() >= rows, "per-row outputs need rows doubles");
    }
  c10::cuda::CUDAGuard guard(tokens.device());
  osb::RemaskArgs a{};
  a.tokens = reinterpret_cast<long long*>(tokens.data_ptr<int64_t>());
  a.ld_tokens = tokens.stride(0);
  a.a0 = static_cast<int>(a0);
  a.bl = static_cast<int>(bl);
  a.mask_id = mask_id;
  a.drawn = drawn.data_ptr<int>();
  a.prio = ptr_or_null<const float>(prio);
  a.logq = ptr_or_null<const float>(logq);
  a.tc = static_cast<int>(tc);
  a.rows = rows;
  a.subset = subset ? 1 : 0;
  a.traj = ptr_or_null<double>(traj);
  a.step_lp = ptr_or_null<double>(step_lp);
  a.out_pos = reinterpret_cast<long long*>(out_pos.data_ptr<int64_t>());
  a.out_tok = reinterpret_cast<long long*>(out_tok.data_ptr<int64_t>());
  a.out_ld = out_pos.stride(0);
  a.pos_offset = pos_offset;
  check(osb::remask_select_launch(a, at::cuda::getCurrentCUDAStream()), "remask_select");
}

void attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor table, Tensor q_start, Tensor q_len, Tensor kv_len,
               Tensor mode, Tensor tile_seq, Tensor tile_row0, int64_t tile_rows, int64_t kv_splits, Tensor out,
               double scale, Tensor status, c10::optional<Tensor> k_lo, c10::optional<Tensor> o_f32,
               c10::optional<Tensor> lse_out, c10::optional<Tensor> prior_o, c10::optional<Tensor> prior_lse) {
  CHECK_CUDA(q);
  CHECK_DT(q, torch::kBFloat16);
  CHECK_DT(k_cache, torch::kBFloat16);
  CHECK_DT(v_cache, torch::kBFloat16);
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous(), "q must be [T, Hq, D] contiguous");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes(),
              "caches must be [pages, Hkv, P, D]");
  for (const Tensor* t : {&table, &q_start, &q_len, &kv_len, &mode, &tile_seq, &tile_row0}) {
    CHECK_DT(*t, torch::kInt32);
    TORCH_CHECK(t->is_cuda() && t->is_contiguous(), "metadata must be contiguous CUDA int32");
  }
  TORCH_CHECK(out.sizes() == q.sizes() && out.is_contiguous(), "out must match q");
  c10::cuda::CUDAGuard guard(q.device());
  osb::AttentionProblem p{};
  p.q = bf(q);
  p.k_cache = bf(k_cache);
  p.v_cache = bf(v_cache);
  p.table = table.data_ptr<int>();
  p.table_stride = table.size(1);
  p.q_start = q_start.data_ptr<int>();
  p.q_len = q_len.data_ptr<int>();
  p.kv_len = kv_len.data_ptr<int>();
  p.mode = mode.data_ptr<int>();
  p.tile_seq = tile_seq.data_ptr<int>();
  p.tile_row0 = tile_row0.data_ptr<int>();
  p.num_tiles = tile_seq.numel();
  p.tile_rows = static_cast<int>(tile_rows);
  p.kv_splits = static_cast<int>(kv_splits);
  p.out = bfm(out);
  p.Hq = q.size(1);
  p.Hkv = k_cache.size(1);
  p.head_dim = q.size(2);
  p.page_size = k_cache.size(2);
  p.cache_pages = k_cache.size(0);
  p.scale = static_cast<float>(scale);
  p.status = status.data_ptr<int>();
  const long long rows = q.size(0) * q.size(1);
  if (k_lo.has_value() && k_lo->defined()) {
    CHECK_DT((*k_lo), torch::kInt32);
    TORCH_CHECK(k_lo->is_cuda() && k_lo->is_contiguous() && k_lo->numel() >= q_start.numel(), "k_lo: one per sequence");
    p.k_lo = k_lo->data_ptr<int>();
  }
  for (const c10::optional<Tensor>* o : {&o_f32, &prior_o})
    if (o->has_value() && (*o)->defined()) {
      CHECK_DT((**o), torch::kFloat32);
      TORCH_CHECK((*o)->is_cuda() && (*o)->is_contiguous() && (*o)->numel() >= rows * q.size(2),
                  "fp32 outputs / priors must hold [T, Hq, D]");
    }
  for (const c10::optional<Tensor>* o : {&lse_out, &prior_lse})
    if (o->has_value() && (*o)->defined()) {
      CHECK_DT((**o), torch::kFloat32);
      TORCH_CHECK((*o)->is_cuda() && (*o)->is_contiguous() && (*o)->numel() >= rows, "log-sum-exp rows: [T, Hq]");
    }
  p.o_f32 = ptr_or_null<float>(o_f32);
  p.lse_out = ptr_or_null<float>(lse_out);
  p.prior_o = ptr_or_null<const float>(prior_o);
  p.prior_lse = ptr_or_null<const float>(prior_lse);
  check(osb::attention_launch(p, at::cuda::getCurrentCUDAStream()), "paged attention");
}

void rmsnorm(Tensor x, Tensor w, Tensor y, double eps, c10::optional<Tensor> h, c10::optional<Tensor> delta) {
  CHECK_CUDA(x);
  CHECK_ROWS(x);
  CHECK_ROWS(y);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(w, torch::kBFloat16);
  CHECK_DT(y, torch::kBFloat16);
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(w.numel() == H && y.size(0) == T && y.size(1) == H, "rmsnorm shapes");
  const bool fused = delta.has_value() && delta->defined();
  if (fused) {
    TORCH_CHECK(h.has_value() && h->defined(), "fused add needs the residual output");
    CHECK_ROWS(*h);
    CHECK_ROWS(*delta);
  }
  c10::cuda::CUDAGuard guard(x.device());
  check(osb::rmsnorm_launch(bf(x), x.stride(0), fused ? bfm(*h) : nullptr, fused ? h->stride(0) : 0,
                            fused ? bf(*delta) : nullptr, fused ? delta->stride(0) : 0, bf(w), bfm(y), y.stride(0), T, H,
                            static_cast<float>(eps), at::cuda::getCurrentCUDAStream()),
        "rmsnorm");
}

void rope_cache(Tensor qkv, Tensor positions, c10::optional<Tensor> slots, Tensor inv_freq,
                c10::optional<Tensor> q_norm, c10::optional<Tensor> k_norm, double eps, Tensor q_out, Tensor k_cache,
                Tensor v_cache, int64_t Hq, int64_t Hkv, c10::optional<Tensor> status) {
  CHECK_CUDA(qkv);
  CHECK_ROWS(qkv);
  CHECK_DT(qkv, torch::kBFloat16);
  CHECK_DT(positions, torch::kInt32);
  CHECK_DT(inv_freq, torch::kFloat32);
  TORCH_CHECK(qkv.size(1) >= (Hq + 2 * Hkv) * 128, "qkv row too short");
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == qkv.size(0) * Hq * 128, "q_out shape");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == Hkv && k_cache.size(3) == 128, "cache layout");
  c10::cuda::CUDAGuard guard(qkv.device());
  check(osb::rope_cache_launch(bf(qkv), qkv.stride(0), positions.data_ptr<int>(), ptr_or_null<const int>(slots),
                               inv_freq.data_ptr<float>(), ptr_or_null<const __nv_bfloat16>(q_norm),
                               ptr_or_null<const __nv_bfloat16>(k_norm), static_cast<float>(eps), bfm(q_out),
                               bfm(k_cache), bfm(v_cache), qkv.size(0), Hq, Hkv, k_cache.size(2),
                               static_cast<long long>(k_cache.size(0)) * k_cache.size(2), ptr_or_null<int>(status),
                               at::cuda::getCurrentCUDAStream()),
        "rope_cache");
}

void embed(Tensor ids, Tensor table, Tensor out, c10::optional<Tensor> status) {
  CHECK_CUDA(ids);
  CHECK_DT(ids, torch::kInt32);
  CHECK_DT(table, torch::kBFloat16);
  CHECK_ROWS(out);
  TORCH_CHECK(out.size(0) == ids.numel() && out.size(1) == table.size(1), "embedding shapes");
  c10::cuda::CUDAGuard guard(ids.device());
  check(osb::embed_launch(ids.data_ptr<int>(), bf(table), table.size(0), ids.numel(), table.size(1), bfm(out),
                          out.stride(0), ptr_or_null<int>(status), at::cuda::getCurrentCUDAStream()),
        "embed");
}

void page_copy(Tensor cache, Tensor pairs) {
  // cache [layers, pages, Hkv, P, D]; pairs int32 [n, 3] (src, dst, tokens)
  CHECK_CUDA(cache);
  CHECK_DT(cache, torch::kBFloat16);
  CHECK_DT(pairs, torch::kInt32);
  TORCH_CHECK(cache.dim() == 5 && cache.is_contiguous(), "cache must be [layers, pages, Hkv, P, D]");
  c10::cuda::CUDAGuard guard(cache.device());
  check(osb::page_copy_launch(bfm(cache), cache.stride(0), cache.size(0), pairs.data_ptr<int>(), pairs.size(0),
                              cache.size(2), cache.size(3), at::cuda::getCurrentCUDAStream()),
        "page_copy");
}

// Per-row truncation arrays of the sampler / scorer (int32 top-k, float32 top-p; either optional).
static void set_truncation(const c10::optional<Tensor>& top_k, const c10::optional<Tensor>& top_p, int64_t rows,
                           const int*& k_out, const float*& p_out) {
  if (top_k.has_value() && top_k->defined()) {
    CHECK_CUDA((*top_k));
    CHECK_DT((*top_k), torch::kInt32);
    TORCH_CHECK(top_k->is_contiguous() && top_k->numel() >= rows, "top_k needs one int32 per row");
    k_out = top_k->data_ptr<int>();
  }
  if (top_p.has_value() && top_p->defined()) {
    CHECK_CUDA((*top_p));
    CHECK_DT((*top_p), torch::kFloat32);
    TORCH_CHECK(top_p->is_contiguous() && top_p->numel() >= rows, "top_p needs one float32 per row");
    p_out = top_p->data_ptr<float>();
  }
}

void sample(Tensor logits, c10::optional<Tensor> inv_temp, Tensor uniforms, Tensor tokens, c10::optional<Tensor> logq,
            c10::optional<Tensor> logp, c10::optional<Tensor> arith, c10::optional<Tensor> next_uniforms,
            c10::optional<Tensor> top_k, c10::optional<Tensor> top_p) {
  CHECK_CUDA(logits);
  CHECK_ROWS(logits);
  CHECK_DT(logits, torch::kFloat32);
  CHECK_DT(uniforms, torch::kFloat64);
  CHECK_DT(tokens, torch::kInt32);
  c10::cuda::CUDAGuard guard(logits.device());
  osb::SampleArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.V = logits.size(1);
  a.inv_temp = ptr_or_null<const float>(inv_temp);
  a.uniforms = uniforms.data_ptr<double>();
  a.uniform_stride = uniforms.dim() == 2 ? uniforms.stride(0) : 1;
  a.tokens = tokens.data_ptr<int>();
  a.logq = ptr_or_null<float>(logq);
  a.logp = ptr_or_null<float>(logp);
  a.arith = ptr_or_null<const int>(arith);
  if (next_uniforms.has_value() && next_uniforms->defined()) {
    CHECK_DT(*next_uniforms, torch::kFloat64);
    TORCH_CHECK((next_uniforms->dim() == 2 ? next_uniforms->stride(0) : 1) == a.uniform_stride,
                "next_uniforms must have the stride of uniforms");
    a.next_uniforms = next_uniforms->data_ptr<double>();
  }
  set_truncation(top_k, top_p, logits.size(0), a.top_k, a.top_p);
  check(osb::sample_launch(a, logits.size(0), at::cuda::getCurrentCUDAStream()), "sample");
}

void row_stats(Tensor logits, c10::optional<Tensor> inv_temp, c10::optional<Tensor> targets,
               c10::optional<Tensor> lse1, c10::optional<Tensor> lseT, c10::optional<Tensor> logp,
               c10::optional<Tensor> logq, c10::optional<Tensor> split_part, c10::optional<Tensor> split_count,
               c10::optional<Tensor> top_k, c10::optional<Tensor> top_p) {
  CHECK_CUDA(logits);
  CHECK_ROWS(logits);
  CHECK_DT(logits, torch::kFloat32);
  c10::cuda::CUDAGuard guard(logits.device());
  osb::RowStatsArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.V = logits.size(1);
  a.inv_temp = ptr_or_null<const float>(inv_temp);
  a.targets = ptr_or_null<const int>(targets);
  a.lse1 = ptr_or_null<float>(lse1);
  a.lseT = ptr_or_null<float>(lseT);
  a.logp = ptr_or_null<float>(logp);
  a.logq = ptr_or_null<float>(logq);
  if (split_part.has_value() && split_part->defined() && split_count.has_value() && split_count->defined()) {
    CHECK_DT(*split_part, torch::kFloat32);
    CHECK_DT(*split_count, torch::kInt32);
    TORCH_CHECK(split_part->numel() >= static_cast<long long>(osb::kRowStatsSplitRows) * osb::kRowStatsMaxSplit * 3 &&
                    split_count->numel() >= osb::kRowStatsSplitRows,
                "row-statistics split scratch too small");
    a.part = split_part->data_ptr<float>();
    a.count = split_count->data_ptr<int>();
  }
  set_truncation(top_k, top_p, logits.size(0), a.top_k, a.top_p);
  check(osb::row_stats_launch(a, logits.size(0), at::cuda::getCurrentCUDAStream()), "row_stats");
}

void gumbel_sample(Tensor logits, c10::optional<Tensor> inv_temp, Tensor seeds, c10::optional<Tensor> seed_index,
                   c10::optional<Tensor> streams, c10::optional<Tensor> row_in_seq, int64_t salt, Tensor tokens,
                   int64_t v_lo, c10::optional<Tensor> keys, c10::optional<Tensor> split_best,
                   c10::optional<Tensor> split_count) {
  CHECK_CUDA(logits);
  CHECK_ROWS(logits);
  CHECK_DT(logits, torch::kFloat32);
  CHECK_DT(seeds, torch::kInt64);
  c10::cuda::CUDAGuard guard(logits.device());
  osb::GumbelArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.V = logits.size(1);
  a.inv_temp = ptr_or_null<const float>(inv_temp);
  a.seeds = reinterpret_cast<const unsigned long long*>(seeds.data_ptr<int64_t>());
  a.seed_index = ptr_or_null<const int>(seed_index);
  a.streams = ptr_or_null<const int>(streams);
  a.row_in_seq = ptr_or_null<const int>(row_in_seq);
  a.salt = static_cast<int>(salt);
  a.tokens = tokens.data_ptr<int>();
  TORCH_CHECK(v_lo % 4 == 0, "vocabulary shards must start at a multiple of 4");
  a.v_lo = static_cast<int>(v_lo);
  if (keys.has_value() && keys->defined()) {
    CHECK_DT(*keys, torch::kInt64);
    TORCH_CHECK(keys->numel() == logits.size(0), "one key per row");
    a.keys = reinterpret_cast<unsigned long long*>(keys->data_ptr<int64_t>());
  }
  if (split_best.has_value() && split_best->defined() && split_count.has_value() && split_count->defined()) {
    CHECK_DT(*split_best, torch::kInt64);
    CHECK_DT(*split_count, torch::kInt32);
    TORCH_CHECK(split_best->numel() >= osb::kGumbelSplitRows && split_count->numel() >= osb::kGumbelSplitRows,
                "split scratch holds one word per row");
    a.row_best = reinterpret_cast<unsigned long long*>(split_best->data_ptr<int64_t>());
    a.row_count = split_count->data_ptr<int>();
  }
  check(osb::gumbel_sample_launch(a, logits.size(0), at::cuda::getCurrentCUDAStream()), "gumbel_sample");
}

void spec_verify(Tensor target, Tensor draft, Tensor candidates, int64_t n, c10::optional<Tensor> inv_temp, Tensor seeds,
                 c10::optional<Tensor> streams, int64_t salt, Tensor count, Tensor tail, Tensor valid, Tensor emitted,
                 Tensor logq, Tensor logp, c10::optional<Tensor> lseT_target, c10::optional<Tensor> lse1_target,
                 c10::optional<Tensor> lseT_draft, int64_t v_lo, int64_t V_total, c10::optional<Tensor> cand_logits,
                 c10::optional<Tensor> keys) {
  CHECK_CUDA(target);
  CHECK_ROWS(target);
  CHECK_ROWS(draft);
  CHECK_DT(target, torch::kFloat32);
  CHECK_DT(draft, torch::kFloat32);
  CHECK_DT(candidates, torch::kInt32);
  const int B = candidates.size(0);
  TORCH_CHECK(candidates.dim() == 2 && candidates.size(1) == n, "candidates must be [B, n]");
  TORCH_CHECK(target.size(0) == B * (n + 1) && draft.size(0) == B * n, "target / draft row counts");
  c10::cuda::CUDAGuard guard(target.device());
  osb::SpecArgs a{};
  a.target = target.data_ptr<float>();
  a.ld_target = target.stride(0);
  a.draft = draft.data_ptr<float>();
  a.ld_draft = draft.stride(0);
  a.candidates = candidates.data_ptr<int>();
  a.n = static_cast<int>(n);
  a.V = target.size(1);
  a.inv_temp = ptr_or_null<const float>(inv_temp);
  a.seeds = reinterpret_cast<const unsigned long long*>(seeds.data_ptr<int64_t>());
  a.streams = ptr_or_null<const int>(streams);
  a.salt = static_cast<int>(salt);
  a.count = count.data_ptr<int>();
  a.tail = tail.data_ptr<int>();
  a.valid = valid.data_ptr<int>();
  a.emitted = emitted.data_ptr<int>();
  a.logq = logq.data_ptr<float>();
  a.logp = logp.data_ptr<float>();
  a.lseT_target = ptr_or_null<const float>(lseT_target);
  a.lse1_target = ptr_or_null<const float>(lse1_target);
  a.lseT_draft = ptr_or_null<const float>(lseT_draft);
  TORCH_CHECK((a.lseT_target == nullptr) == (a.lse1_target == nullptr) &&
                  (a.lseT_target == nullptr) == (a.lseT_draft == nullptr),
              "precomputed statistics come together");
  TORCH_CHECK(v_lo % 4 == 0, "vocabulary shards must start at a multiple of 4");
  a.v_lo = static_cast<int>(v_lo);
  a.V_total = static_cast<int>(V_total);
  a.cand_logits = ptr_or_null<const float>(cand_logits);
  if (keys.has_value() && keys->defined()) {
    CHECK_DT(*keys, torch::kInt64);
    TORCH_CHECK(keys->numel() == B && a.cand_logits != nullptr, "vocabulary-parallel correction needs keys and "
                                                                 "candidate logits");
    a.keys = reinterpret_cast<unsigned long long*>(keys->data_ptr<int64_t>());
  }
  check(osb::spec_verify_launch(a, B, at::cuda::getCurrentCUDAStream()), "spec_verify");
}

// Full-vocabulary TV / forward-KL distillation: statistics, loss pieces, gradient.
void divergence_stats(Tensor s, Tensor t, Tensor out) {
  CHECK_CUDA(s);
  CHECK_ROWS(s);
  CHECK_ROWS(t);
  CHECK_DT(s, torch::kFloat32);
  CHECK_DT(t, torch::kFloat32);
  TORCH_CHECK(s.sizes() == t.sizes() && out.numel() == 4 * s.size(0), "divergence shapes");
  c10::cuda::CUDAGuard guard(s.device());
  check(osb::divergence_stats_launch(s.data_ptr<float>(), t.data_ptr<float>(), s.stride(0), t.stride(0), s.size(0),
                                     s.size(1), out.data_ptr<float>(), at::cuda::getCurrentCUDAStream()),
        "divergence_stats");
}

void divergence_loss(Tensor s, Tensor t, Tensor lse, int64_t kind, Tensor out) {
  CHECK_CUDA(s);
  CHECK_ROWS(s);
  CHECK_ROWS(t);
  TORCH_CHECK(lse.numel() == 2 * s.size(0) && out.numel() == 2 * s.size(0), "divergence loss shapes");
  c10::cuda::CUDAGuard guard(s.device());
  check(osb::divergence_loss_launch(s.data_ptr<float>(), t.data_ptr<float>(), s.stride(0), t.stride(0), s.size(0),
                                    s.size(1), lse.data_ptr<float>(), static_cast<int>(kind), out.data_ptr<float>(),
                                    at::cuda::getCurrentCUDAStream()),
        "divergence_loss");
}

void divergence_grad(Tensor s, Tensor t, Tensor lse, Tensor pieces, Tensor w, int64_t kind, Tensor grad) {
  CHECK_CUDA(s);
  CHECK_ROWS(s);
  CHECK_ROWS(t);
  CHECK_ROWS(grad);
  CHECK_DT(grad, torch::kBFloat16);
  TORCH_CHECK(grad.sizes() == s.sizes() && w.numel() == s.size(0), "divergence grad shapes");
  c10::cuda::CUDAGuard guard(s.device());
  check(osb::divergence_grad_launch(s.data_ptr<float>(), t.data_ptr<float>(), s.stride(0), t.stride(0), s.size(0),
                                    s.size(1), lse.data_ptr<float>(), pieces.data_ptr<float>(), w.data_ptr<float>(),
                                    static_cast<int>(kind), bfm(grad), grad.stride(0),
                                    at::cuda::getCurrentCUDAStream()),
        "divergence_grad");
}

// h += sum over ranks of the partials; x = rmsnorm(h) * w  (peer pointers as int64 addresses).
// pushed: parts are this rank's local receive slots, filled by the ranks' pushing GEMMs.
void allreduce_norm_impl(std::vector<int64_t> parts, std::vector<int64_t> rows, std::vector<int64_t> pads,
                         Tensor epoch, Tensor h, Tensor w, Tensor x, int64_t T, int64_t rank, double eps,
                         int64_t blocks, Tensor status, bool pushed, int64_t algorithm, int64_t wait_ns) {
  CHECK_CUDA(h);
  CHECK_ROWS(h);
  CHECK_ROWS(x);
  CHECK_DT(h, torch::kBFloat16);
  CHECK_DT(epoch, torch::kInt32);
  const int world = static_cast<int>(parts.size());
  TORCH_CHECK(world >= 1 && world <= osb::kMaxRanks && (pushed || rows.size() == parts.size()) &&
                  pads.size() == parts.size(),
              "one partial, row buffer and signal pad per rank (at most 8)");
  TORCH_CHECK(h.size(0) >= T && x.size(0) >= T && w.numel() == h.size(1), "all-reduce shapes");
  TORCH_CHECK(epoch.numel() >= 4, "the all-reduce epoch buffer holds four counters");
  c10::cuda::CUDAGuard guard(h.device());
  osb::ArArgs a{};
  for (int q = 0; q < world; ++q) {
    a.parts[q] = reinterpret_cast<const __nv_bfloat16*>(parts[q]);
    a.rows[q] = pushed ? nullptr : reinterpret_cast<__nv_bfloat16*>(rows[q]);
    a.pads[q] = reinterpret_cast<uint32_t*>(pads[q]);
  }
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>());
  a.h = bfm(h);
  a.ldh = h.stride(0);
  a.w = bf(w);
  a.x = bfm(x);
  a.ldx = x.stride(0);
  a.T = static_cast<int>(T);
  a.H = h.size(1);
  a.rank = static_cast<int>(rank);
  a.world = world;
  a.eps = static_cast<float>(eps);
  a.status = status.data_ptr<int>();
  TORCH_CHECK(algorithm >= 0 && algorithm <= 2, "all-reduce algorithm: 0 automatic, 1 one-shot, 2 two-shot");
  TORCH_CHECK(wait_ns >= 0, "wait limit must be non-negative (0 selects the default)");
  a.algorithm = static_cast<int>(algorithm);
  a.wait_ns = static_cast<unsigned long long>(wait_ns);
  if (pushed)
    check(osb::allreduce_pushed_add_rmsnorm_launch(a, static_cast<int>(blocks), at::cuda::getCurrentCUDAStream()),
          "allreduce_pushed_add_rmsnorm");
  else
    check(osb::allreduce_add_rmsnorm_launch(a, static_cast<int>(blocks), at::cuda::getCurrentCUDAStream()),
          "allreduce_add_rmsnorm");
}

void allreduce_add_rmsnorm(std::vector<int64_t> parts, std::vector<int64_t> rows, std::vector<int64_t> pads,
                           Tensor epoch, Tensor h, Tensor w, Tensor x, int64_t T, int64_t rank, double eps,
                           int64_t blocks, Tensor status, int64_t algorithm, int64_t wait_ns) {
  allreduce_norm_impl(parts, rows, pads, epoch, h, w, x, T, rank, eps, blocks, status, false, algorithm, wait_ns);
}

void allreduce_pushed_add_rmsnorm(std::vector<int64_t> parts, std::vector<int64_t> pads, Tensor epoch, Tensor h,
                                  Tensor w, Tensor x, int64_t T, int64_t rank, double eps, int64_t blocks,
                                  Tensor status, int64_t wait_ns) {
  allreduce_norm_impl(parts, {}, pads, epoch, h, w, x, T, rank, eps, blocks, status, true, 0, wait_ns);
}

osb::DpArgs dp_args(const std::vector<int64_t>& grads, const std::vector<int64_t>& params,
                    const std::vector<int64_t>& pads, Tensor counters, int64_t rank, Tensor status, int64_t wait_ns) {
  const int world = static_cast<int>(pads.size());
  TORCH_CHECK(world >= 2 && world <= osb::kMaxRanks, "data-parallel collectives need 2..8 ranks");
  TORCH_CHECK(grads.empty() || static_cast<int>(grads.size()) == world, "one gradient pointer per rank");
  TORCH_CHECK(params.empty() || static_cast<int>(params.size()) == world, "one parameter pointer per rank");
  TORCH_CHECK(rank >= 0 && rank < world, "rank out of range");
  CHECK_CUDA(counters);
  CHECK_DT(counters, torch::kInt32);
  TORCH_CHECK(counters.numel() >= 4, "counters holds 4 words");
  CHECK_DT(status, torch::kInt32);
  osb::DpArgs a{};
  for (int q = 0; q < world; ++q) {
    a.grads[q] = grads.empty() ? nullptr : reinterpret_cast<const float*>(grads[q]);
    a.params[q] = params.empty() ? nullptr : reinterpret_cast<__nv_bfloat16*>(params[q]);
    a.pads[q] = reinterpret_cast<uint32_t*>(pads[q]);
  }
  a.counters = reinterpret_cast<uint32_t*>(counters.data_ptr<int>());
  a.rank = static_cast<int>(rank);
  a.world = world;
  a.status = status.data_ptr<int>();
  a.wait_ns = static_cast<unsigned long long>(wait_ns);
  return a;
}

// shard = scale * (sum over ranks of grads[q][lo + rank * n, + n)), rank order, peer loads.
void dp_reduce_scatter(std::vector<int64_t> grads, std::vector<int64_t> pads, Tensor counters, int64_t rank,
                       int64_t lo, int64_t n, Tensor shard, double scale, Tensor status, int64_t wait_ns) {
  CHECK_CUDA(shard);
  CHECK_DT(shard, torch::kFloat32);
  TORCH_CHECK(shard.is_contiguous() && shard.numel() >= n, "shard must hold n contiguous floats");
  const c10::cuda::CUDAGuard guard(shard.device());
  const osb::DpArgs a = dp_args(grads, {}, pads, counters, rank, status, wait_ns);
  check(osb::dp_reduce_scatter_launch(a, lo, n, shard.data_ptr<float>(), static_cast<float>(scale),
                                      at::cuda::getCurrentCUDAStream()),
        "data-parallel reduce-scatter");
}

// params[q][lo + rank * n, + n) = src for every rank q (peer stores), between two barriers.
void dp_all_gather(std::vector<int64_t> params, std::vector<int64_t> pads, Tensor counters, int64_t rank, Tensor src,
                   int64_t lo, int64_t n, Tensor status, int64_t wait_ns) {
  CHECK_CUDA(src);
  CHECK_DT(src, torch::kBFloat16);
  TORCH_CHECK(src.is_contiguous() && src.numel() >= n, "src must hold n contiguous bf16 values");
  const c10::cuda::CUDAGuard guard(src.device());
  const osb::DpArgs a = dp_args({}, params, pads, counters, rank, status, wait_ns);
  check(osb::dp_all_gather_launch(a, reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), lo, n,
                                  at::cuda::getCurrentCUDAStream()),
        "data-parallel all-gather");
}

// Zeroes `bytes` at a raw device address on the current stream (signal-pad reset).
void zero_device_bytes(int64_t ptr, int64_t bytes) {
  TORCH_CHECK(ptr != 0 && bytes > 0, "zero_device_bytes needs an address and a positive size");
  check(cudaMemsetAsync(reinterpret_cast<void*>(ptr), 0, static_cast<size_t>(bytes), at::cuda::getCurrentCUDAStream()),
        "zero_device_bytes");
}

// Row-parallel GEMM whose bf16 output tile is stored into every rank's receive slot for
// this rank (dsts[q], row stride = M) and whose last CTA releases *epoch + 1 into
// flags[q]; `out` is this rank's own slot (shape / stride checks only).
void gemm_push(Tensor w, Tensor x, Tensor out, std::vector<int64_t> dsts, std::vector<int64_t> flags, Tensor epoch,
               Tensor count, bool allow_split, Tensor workspace, Tensor counters, Tensor status,
               bool prefetch_weights) {
  CHECK_CUDA(w);
  CHECK_CUDA(x);
  CHECK_CUDA(out);
  CHECK_DT(w, torch::kBFloat16);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(out, torch::kBFloat16);
  CHECK_DT(epoch, torch::kInt32);
  CHECK_DT(count, torch::kInt32);
  CHECK_ROWS(w);
  CHECK_ROWS(x);
  CHECK_ROWS(out);
  TORCH_CHECK(w.size(1) == x.size(1), "reduction dimensions differ");
  const int M = w.size(0), N = x.size(0), K = w.size(1);
  TORCH_CHECK(out.size(0) == N && out.size(1) == M, "output shape mismatch");
  const int world = static_cast<int>(dsts.size());
  TORCH_CHECK(world >= 1 && world <= 8 && flags.size() == dsts.size(), "one destination and flag per rank (at most 8)");
  c10::cuda::CUDAGuard guard(w.device());
  osb::GemmProblem p{};
  p.w = bf(w);
  p.ldw = w.stride(0);
  p.x = bf(x);
  p.ldx = x.stride(0);
  p.M = M;
  p.N = N;
  p.K = K;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.allow_split = allow_split ? 1 : 0;
  p.workspace = workspace.data_ptr<float>();
  p.workspace_floats = workspace.numel();
  p.counters = counters.data_ptr<int>();
  p.counter_slots = counters.numel();
  p.status = status.data_ptr<int>();
  p.prefetch_weights = prefetch_weights ? 1 : 0;
  p.push_world = world;
  for (int q = 0; q < world; ++q) {
    p.push_dst[q] = reinterpret_cast<__nv_bfloat16*>(dsts[q]);
    p.push_flags[q] = reinterpret_cast<uint32_t*>(flags[q]);
  }
  p.push_epoch = reinterpret_cast<const uint32_t*>(epoch.data_ptr<int>());
  p.push_count = reinterpret_cast<unsigned int*>(count.data_ptr<int>());
  check(osb::gemm_launch(p, at::cuda::getCurrentCUDAStream()), "tcgen05 gemm (push)");
}

// Expert-parallel MoE exchange: phase 0 dispatch (count exchange + peer stores), phase 1 combine (peer loads).
void ep_exchange(std::vector<int64_t> tables, std::vector<int64_t> recv_x, std::vector<int64_t> recv_y,
                 std::vector<int64_t> pads, Tensor epoch, int64_t r_max, Tensor counts, Tensor topk_idx,
                 Tensor topk_w, Tensor x, Tensor cursor, Tensor slot_of, Tensor local_offsets, Tensor h, int64_t E,
                 int64_t k, int64_t rank, int64_t blocks, int64_t phase, Tensor status, int64_t wait_ns) {
  CHECK_CUDA(x);
  CHECK_ROWS(x);
  CHECK_ROWS(h);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(h, torch::kBFloat16);
  for (const Tensor* t : {&counts, &topk_idx, &cursor, &slot_of, &local_offsets, &epoch}) {
    CHECK_DT(*t, torch::kInt32);
    TORCH_CHECK(t->is_cuda() && t->is_contiguous(), "EP metadata must be contiguous CUDA int32");
  }
  CHECK_DT(topk_w, torch::kFloat32);
  const int world = static_cast<int>(tables.size());
  TORCH_CHECK(world >= 1 && world <= osb::kEpMaxRanks && recv_x.size() == tables.size() &&
                  recv_y.size() == tables.size() && pads.size() == tables.size(),
              "one table, receive buffer, output buffer and pad per rank (at most 8)");
  const int T = x.size(0);
  TORCH_CHECK(topk_idx.numel() >= T * k && topk_w.numel() >= T * k && slot_of.numel() >= T * k, "top-k shapes");
  TORCH_CHECK(counts.numel() == E && cursor.numel() == E && local_offsets.numel() == E / world + 1, "EP shapes");
  TORCH_CHECK(h.size(0) == T && h.size(1) == x.size(1), "residual shape");
  c10::cuda::CUDAGuard guard(x.device());
  osb::EpArgs a{};
  for (int q = 0; q < world; ++q) {
    a.tables[q] = reinterpret_cast<int*>(tables[q]);
    a.recv_x[q] = reinterpret_cast<__nv_bfloat16*>(recv_x[q]);
    a.recv_y[q] = reinterpret_cast<__nv_bfloat16*>(recv_y[q]);
    a.pads[q] = reinterpret_cast<uint32_t*>(pads[q]);
  }
  a.world = world;
  a.rank = static_cast<int>(rank);
  a.E = static_cast<int>(E);
  a.E_local = static_cast<int>(E / world);
  a.k = static_cast<int>(k);
  a.T = T;
  a.H = x.size(1);
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>());
  a.r_max = r_max;
  a.counts = counts.data_ptr<int>();
  a.topk_idx = topk_idx.data_ptr<int>();
  a.topk_w = topk_w.data_ptr<float>();
  a.x = bf(x);
  a.ldx = x.stride(0);
  a.cursor = cursor.data_ptr<int>();
  a.slot_of = slot_of.data_ptr<int>();
  a.local_offsets = local_offsets.data_ptr<int>();
  a.h = bfm(h);
  a.ldh = h.stride(0);
  a.status = status.data_ptr<int>();
  TORCH_CHECK(wait_ns >= 0, "wait limit must be non-negative (0 selects the default)");
  a.wait_ns = static_cast<unsigned long long>(wait_ns);
  const int b = static_cast<int>(blocks);
  check(phase == 0 ? osb::ep_dispatch_launch(a, b, at::cuda::getCurrentCUDAStream())
                   : osb::ep_combine_launch(a, b, at::cuda::getCurrentCUDAStream()),
        "ep_exchange");
}

void logprob_grad(Tensor logits, Tensor lse, Tensor targets, Tensor w, Tensor grad) {
  CHECK_CUDA(logits);
  CHECK_ROWS(logits);
  CHECK_ROWS(grad);
  CHECK_DT(logits, torch::kFloat32);
  TORCH_CHECK(grad.scalar_type() == torch::kFloat32 || grad.scalar_type() == torch::kBFloat16,
              "fp32 or bf16 gradient");
  CHECK_DT(targets, torch::kInt32);
  TORCH_CHECK(grad.sizes() == logits.sizes() && lse.numel() == logits.size(0) && w.numel() == logits.size(0),
              "logprob_grad shapes");
  c10::cuda::CUDAGuard guard(logits.device());
  check(osb::logprob_grad_launch(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1),
                                 lse.data_ptr<float>(), targets.data_ptr<int>(), w.data_ptr<float>(), grad.data_ptr(),
                                 grad.scalar_type() == torch::kBFloat16, grad.stride(0),
                                 at::cuda::getCurrentCUDAStream()),
        "logprob_grad");
}

void grad_sq_norm(Tensor g, Tensor out) {
  CHECK_CUDA(g);
  CHECK_DT(g, torch::kFloat32);
  TORCH_CHECK(g.is_contiguous(), "flat contiguous grads");
  c10::cuda::CUDAGuard guard(g.device());
  check(osb::grad_sq_norm_launch(g.data_ptr<float>(), g.numel(), out.data_ptr<float>(),
                                 at::cuda::getCurrentCUDAStream()),
        "grad_sq_norm");
}

void grpo_loss(Tensor logp, Tensor old_logp, Tensor ref_logp, Tensor adv, Tensor mask, double beta, double eps,
               Tensor grad, Tensor row_stats, Tensor out, Tensor counter) {
  for (const Tensor* t : {&logp, &old_logp, &ref_logp, &grad}) {
    CHECK_CUDA(*t);
    CHECK_DT(*t, torch::kFloat32);
    TORCH_CHECK(t->is_contiguous() && t->sizes() == logp.sizes() && t->dim() == 2,
                "GRPO loss rows must be contiguous fp32 [B, C] tensors of one shape");
  }
  CHECK_DT(adv, torch::kFloat32);
  CHECK_DT(row_stats, torch::kFloat32);
  CHECK_DT(out, torch::kFloat32);
  CHECK_DT(counter, torch::kInt32);
  TORCH_CHECK(mask.scalar_type() == torch::kBool || mask.scalar_type() == torch::kUInt8, "mask must be bool or uint8");
  TORCH_CHECK(mask.is_contiguous() && mask.sizes() == logp.sizes(), "mask must match logp");
  const int B = static_cast<int>(logp.size(0)), C = static_cast<int>(logp.size(1));
  TORCH_CHECK(adv.is_contiguous() && adv.numel() == B, "one advantage per sequence");
  TORCH_CHECK(row_stats.is_contiguous() && row_stats.numel() >= 4LL * B, "row_stats holds 4 values per sequence");
  TORCH_CHECK(out.numel() >= 3 && counter.numel() >= 1, "out holds 3 values, counter 1");
  const c10::cuda::CUDAGuard guard(logp.device());
  osb::GrpoLossArgs a{logp.data_ptr<float>(), old_logp.data_ptr<float>(), ref_logp.data_ptr<float>(),
                      adv.data_ptr<float>(), reinterpret_cast<const unsigned char*>(mask.data_ptr()), B, C,
                      static_cast<float>(beta), static_cast<float>(eps), grad.data_ptr<float>(),
                      row_stats.data_ptr<float>(), out.data_ptr<float>(),
                      reinterpret_cast<unsigned int*>(counter.data_ptr<int>())};
  check(osb::grpo_loss_launch(a, at::cuda::getCurrentCUDAStream()), "grpo_loss");
}

void adamw(Tensor p, Tensor g, Tensor m, Tensor v, c10::optional<Tensor> publish, c10::optional<Tensor> sq_norm,
           double clip, double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step,
           c10::optional<Tensor> nonfinite, c10::optional<Tensor> step_tensor) {
  CHECK_CUDA(p);
  for (const Tensor* t : {&p, &g, &m, &v}) {
    CHECK_DT(*t, torch::kFloat32);
    TORCH_CHECK(t->is_contiguous() && t->numel() == p.numel(), "flat contiguous fp32 optimizer buffers");
  }
  if (publish.has_value() && publish->defined()) {
    CHECK_DT(*publish, torch::kBFloat16);
    TORCH_CHECK(publish->is_contiguous() && publish->numel() == p.numel(), "publish buffer shape");
  }
  c10::cuda::CUDAGuard guard(p.device());
  osb::AdamWArgs a{};
  a.params = p.data_ptr<float>();
  a.grads = g.data_ptr<float>();
  a.exp_avg = m.data_ptr<float>();
  a.exp_avg_sq = v.data_ptr<float>();
  a.publish = ptr_or_null<__nv_bfloat16>(publish);
  a.n = p.numel();
  a.sq_norm = ptr_or_null<const float>(sq_norm);
  a.clip = static_cast<float>(clip);
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.weight_decay = static_cast<float>(weight_decay);
  a.bias_correction1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  a.bias_correction2 = static_cast<float>(1.0 - std::pow(beta2, static_cast<double>(step)));
  a.nonfinite = ptr_or_null<int>(nonfinite);
  a.step_ptr = ptr_or_null<const int>(step_tensor);
  check(osb::adamw_launch(a, at::cuda::getCurrentCUDAStream()), "adamw");
}

}  // namespace

void score_stats(Tensor logits, c10::optional<Tensor> inv_temp, c10::optional<Tensor> targets, int64_t topk,
                 Tensor out) {
  CHECK_CUDA(logits);
  CHECK_ROWS(logits);
  CHECK_DT(logits, torch::kFloat32);
  CHECK_DT(out, torch::kFloat32);
  TORCH_CHECK(out.is_contiguous() && out.numel() == logits.size(0) * 4, "out must be [rows, 4]");
  c10::cuda::CUDAGuard guard(logits.device());
  check(osb::score_stats_launch(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1),
                                ptr_or_null<const float>(inv_temp), ptr_or_null<const int>(targets),
                                static_cast<int>(topk), out.data_ptr<float>(), at::cuda::getCurrentCUDAStream()),
        "score_stats");
}

// ------------------------------------------------------------------- MoE ---
void grouped_tiles(Tensor offsets, int64_t groups, int64_t tiles_m, int64_t bn, Tensor tiles, Tensor total) {
  CHECK_CUDA(offsets);
  CHECK_DT(offsets, torch::kInt32);
  CHECK_DT(tiles, torch::kInt32);
  CHECK_DT(total, torch::kInt32);
  TORCH_CHECK(offsets.numel() >= groups + 1 && tiles.numel() % 4 == 0, "grouped_tiles shapes");
  c10::cuda::CUDAGuard guard(offsets.device());
  check(osb::grouped_tiles_launch(offsets.data_ptr<int>(), groups, tiles_m, bn, tiles.data_ptr<int>(),
                                  tiles.numel() / 4, total.data_ptr<int>(), at::cuda::getCurrentCUDAStream()),
        "grouped_tiles");
}

void grouped_gemm(Tensor w, Tensor x, Tensor out, int64_t epilogue, Tensor tiles, Tensor total, int64_t groups,
                  int64_t bn, Tensor workspace, Tensor counters, Tensor status) {
  CHECK_CUDA(w);
  CHECK_CUDA(x);
  CHECK_DT(w, torch::kBFloat16);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_ROWS(w);
  CHECK_ROWS(x);
  CHECK_ROWS(out);
  TORCH_CHECK(w.size(1) == x.size(1), "reduction dimensions differ");
  TORCH_CHECK(groups > 0 && w.size(0) % groups == 0, "w must stack `groups` equal weight blocks");
  const int M = w.size(0) / groups;
  const int out_cols = epilogue == 1 ? M / 2 : M;
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == out_cols, "output shape mismatch");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kFloat32, "bf16 or fp32 output");
  CHECK_DT(tiles, torch::kInt32);
  CHECK_DT(total, torch::kInt32);
  c10::cuda::CUDAGuard guard(w.device());
  osb::GemmProblem p{};
  p.w = bf(w);
  p.ldw = w.stride(0);
  p.x = bf(x);
  p.ldx = x.stride(0);
  p.M = M;
  p.N = x.size(0);
  p.K = w.size(1);
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.out_f32 = out.scalar_type() == torch::kFloat32;
  p.epilogue = static_cast<int>(epilogue);
  p.allow_split = 0;
  p.workspace = workspace.data_ptr<float>();
  p.workspace_floats = workspace.numel();
  p.counters = counters.data_ptr<int>();
  p.counter_slots = counters.numel();
  p.status = status.data_ptr<int>();
  p.group_tiles = tiles.data_ptr<int>();
  p.group_total = total.data_ptr<int>();
  p.groups = static_cast<int>(groups);
  p.group_tile_cap = static_cast<int>(tiles.numel() / 4);
  p.group_bn = static_cast<int>(bn);
  if (x.size(0) == 0) return;
  check(osb::gemm_launch(p, at::cuda::getCurrentCUDAStream()), "grouped tcgen05 gemm");
}

void moe_route(Tensor logits, int64_t k, bool renorm, Tensor topk_idx, Tensor topk_w, Tensor counts) {
  CHECK_CUDA(logits);
  CHECK_ROWS(logits);
  CHECK_DT(logits, torch::kFloat32);
  CHECK_DT(topk_idx, torch::kInt32);
  CHECK_DT(topk_w, torch::kFloat32);
  CHECK_DT(counts, torch::kInt32);
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(topk_idx.numel() == static_cast<long long>(T) * k && topk_w.numel() == topk_idx.numel() &&
                  counts.numel() >= E,
              "moe_route shapes");
  c10::cuda::CUDAGuard guard(logits.device());
  check(osb::moe_route_launch(logits.data_ptr<float>(), logits.stride(0), T, E, k, renorm ? 1 : 0,
                              topk_idx.data_ptr<int>(), topk_w.data_ptr<float>(), counts.data_ptr<int>(),
                              at::cuda::getCurrentCUDAStream()),
        "moe_route");
}

void moe_offsets(Tensor counts, Tensor offsets, Tensor cursor) {
  CHECK_CUDA(counts);
  CHECK_DT(counts, torch::kInt32);
  CHECK_DT(offsets, torch::kInt32);
  CHECK_DT(cursor, torch::kInt32);
  const int E = counts.numel();
  TORCH_CHECK(offsets.numel() == E + 1 && cursor.numel() == E, "moe_offsets shapes");
  c10::cuda::CUDAGuard guard(counts.device());
  check(osb::moe_offsets_launch(counts.data_ptr<int>(), E, offsets.data_ptr<int>(), cursor.data_ptr<int>(),
                                at::cuda::getCurrentCUDAStream()),
        "moe_offsets");
}

void moe_dispatch(Tensor x, Tensor topk_idx, Tensor cursor, Tensor xp, Tensor slot_of) {
  CHECK_CUDA(x);
  CHECK_ROWS(x);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(xp, torch::kBFloat16);
  CHECK_DT(topk_idx, torch::kInt32);
  CHECK_DT(slot_of, torch::kInt32);
  const int T = x.size(0), H = x.size(1);
  const int k = T > 0 ? topk_idx.numel() / T : 0;
  TORCH_CHECK(xp.is_contiguous() && xp.size(1) == H && xp.size(0) >= static_cast<long long>(T) * k &&
                  slot_of.numel() == topk_idx.numel(),
              "moe_dispatch shapes");
  c10::cuda::CUDAGuard guard(x.device());
  check(osb::moe_dispatch_launch(bf(x), x.stride(0), T, k, H, topk_idx.data_ptr<int>(), cursor.data_ptr<int>(),
                                 bfm(xp), slot_of.data_ptr<int>(), at::cuda::getCurrentCUDAStream()),
        "moe_dispatch");
}

void moe_combine(Tensor y, Tensor slot_of, Tensor topk_w, Tensor h, bool accumulate) {
  CHECK_CUDA(y);
  CHECK_ROWS(y);
  CHECK_ROWS(h);
  CHECK_DT(y, torch::kBFloat16);
  CHECK_DT(h, torch::kBFloat16);
  CHECK_DT(slot_of, torch::kInt32);
  CHECK_DT(topk_w, torch::kFloat32);
  const int T = h.size(0), H = h.size(1);
  const int k = T > 0 ? slot_of.numel() / T : 0;
  TORCH_CHECK(y.size(1) == H && topk_w.numel() == slot_of.numel(), "moe_combine shapes");
  c10::cuda::CUDAGuard guard(h.device());
  check(osb::moe_combine_launch(bf(y), y.stride(0), slot_of.data_ptr<int>(), topk_w.data_ptr<float>(), T, k, H,
                                bfm(h), h.stride(0), accumulate ? 1 : 0, at::cuda::getCurrentCUDAStream()),
        "moe_combine");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels and C++ runtime of online_speculation_b200";
  m.def("gemm", &gemm);
  m.def("gemm_push", &gemm_push);
  m.def("head_stats", &head_stats);
  m.def("remask_select", &remask_select);
  m.def("allreduce_pushed_add_rmsnorm", &allreduce_pushed_add_rmsnorm);
  m.def("attention", &attention);
  m.def("rmsnorm", &rmsnorm);
  m.def("rope_cache", &rope_cache);
  m.def("embed", &embed);
  m.def("page_copy", &page_copy);
  m.def("sample", &sample);
  m.def("row_stats", &row_stats);
  m.def("gumbel_sample", &gumbel_sample);
  m.def("spec_verify", &spec_verify);
  m.def("grad_sq_norm", &grad_sq_norm);
  m.def("allreduce_add_rmsnorm", &allreduce_add_rmsnorm);
  m.def("divergence_stats", &divergence_stats);
  m.def("divergence_loss", &divergence_loss);
  m.def("divergence_grad", &divergence_grad);
  m.def("logprob_grad", &logprob_grad);
  m.def("adamw", &adamw);
  m.def("grpo_loss", &grpo_loss);
  m.def("dp_reduce_scatter", &dp_reduce_scatter);
  m.def("dp_all_gather", &dp_all_gather);
  m.def("zero_device_bytes", &zero_device_bytes);
  m.def("gemm_pick_bn", &osb::gemm_pick_bn);
  m.def("score_stats", &score_stats);
  m.def("grouped_tiles", &grouped_tiles);
  m.def("grouped_gemm", &grouped_gemm);
  m.def("moe_route", &moe_route);
  m.def("moe_offsets", &moe_offsets);
  m.def("moe_dispatch", &moe_dispatch);
  m.def("moe_combine", &moe_combine);
  m.def("ep_exchange", &ep_exchange);
  m.def("set_pdl", [](bool on) { osb::pdl_enabled() = on; });
  m.def("attention_set_trace", [](c10::optional<Tensor> buf) {
    if (buf.has_value() && buf->defined()) {
      CHECK_CUDA(*buf);
      TORCH_CHECK(buf->scalar_type() == torch::kInt64 && buf->is_contiguous() && buf->numel() >= 1024,
                  "trace buffer must be a contiguous int64 tensor of at least 1024 values");
      osb::attention_trace_buffer() = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
    } else {
      osb::attention_trace_buffer() = nullptr;
    }
  });
  m.def("gemm_set_trace", [](c10::optional<Tensor> buf) {
    if (buf.has_value() && buf->defined()) {
      CHECK_CUDA(*buf);
      TORCH_CHECK(buf->scalar_type() == torch::kInt64 && buf->is_contiguous() && buf->numel() >= 32 * 1024,
                  "trace buffer must be a contiguous int64 tensor of at least 32 x 1024 values");
      osb::gemm_trace_buffer() = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
    } else {
      osb::gemm_trace_buffer() = nullptr;
    }
  });
  m.def("allreduce_set_trace", [](c10::optional<Tensor> buf) {
    if (buf.has_value() && buf->defined()) {
      CHECK_CUDA(*buf);
      TORCH_CHECK(buf->scalar_type() == torch::kInt64 && buf->is_contiguous() && buf->numel() >= 8,
                  "trace buffer must be a contiguous int64 tensor of at least 8 values");
      osb::allreduce_trace_buffer() = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
    } else {
      osb::allreduce_trace_buffer() = nullptr;
    }
  });
  m.def("pdl_enabled", []() -> bool { return osb::pdl_enabled(); });

  pybind11::class_<osb::KVManager>(m, "KVManager")
      .def(pybind11::init<int, int>())
      .def_property_readonly("page_size", &osb::KVManager::page_size)
      .def_property_readonly("num_pages", &osb::KVManager::num_pages)
      .def_property_readonly("free_pages", &osb::KVManager::free_pages)
      .def("create", &osb::KVManager::create)
      .def("release", &osb::KVManager::release)
      .def("length", &osb::KVManager::length)
      .def("append", &osb::KVManager::append)
      .def("truncate", &osb::KVManager::truncate)
      .def("fork",
           [](osb::KVManager& self, int64_t seq, int n) {
             std::vector<int32_t> copies;
             const int64_t id = self.fork(seq, n, copies);
             return std::make_pair(id, copies);
           })
      .def("pages", &osb::KVManager::pages)
      .def("adopt", &osb::KVManager::adopt)
      .def("retain", &osb::KVManager::retain)
      .def("drop", &osb::KVManager::drop)
      .def("refcount", &osb::KVManager::refcount)
      .def("append_many",
           [](osb::KVManager& self, const std::vector<int64_t>& seqs, int n) {
             std::vector<int32_t> all;
             all.reserve(seqs.size() * n);
             for (int64_t s : seqs) {
               const auto v = self.append(s, n);
               all.insert(all.end(), v.begin(), v.end());
             }
             return all;
           })
      .def("truncate_many",
           [](osb::KVManager& self, const std::vector<int64_t>& seqs, const std::vector<int64_t>& lengths) {
             TORCH_CHECK(seqs.size() == lengths.size(), "one length per sequence");
             for (size_t i = 0; i < seqs.size(); ++i) self.truncate(seqs[i], static_cast<int>(lengths[i]));
           })
      .def("fill_table_np",
           [](const osb::KVManager& self, const std::vector<int64_t>& seqs, pybind11::array_t<int32_t> out) {
             auto buf = out.mutable_unchecked<2>();
             TORCH_CHECK(buf.shape(0) >= static_cast<ssize_t>(seqs.size()), "table rows");
             std::vector<int32_t> tmp(seqs.size() * buf.shape(1));
             self.fill_table(seqs, tmp.data(), static_cast<int>(buf.shape(1)));
             for (size_t r = 0; r < seqs.size(); ++r)
               for (ssize_t c = 0; c < buf.shape(1); ++c) buf(r, c) = tmp[r * buf.shape(1) + c];
           })
      .def("fill_table", [](const osb::KVManager& self, const std::vector<int64_t>& seqs, Tensor out) {
        TORCH_CHECK(out.device().is_cpu() && out.scalar_type() == torch::kInt32 && out.dim() == 2 &&
                        out.is_contiguous() && out.size(0) >= static_cast<int64_t>(seqs.size()),
                    "table must be a CPU int32 [rows, stride] tensor");
        self.fill_table(seqs, out.data_ptr<int32_t>(), out.size(1));
      });
}
