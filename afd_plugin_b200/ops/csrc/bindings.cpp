// torch.ops.afd_b200.* registrations for the sm_100a kernels.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGraphsC10Utils.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "launchers.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return kF32;
    case at::kBFloat16: return kBF16;
    case at::kHalf: return kF16;
    default: TORCH_CHECK(false, "afd_b200: unsupported dtype ", t.scalar_type());
  }
  return -1;
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "afd_b200: ", name, " must be a CUDA tensor");
}

void check_vec16(const at::Tensor& t, int64_t last, const char* name) {
  const int64_t align = 16 / t.element_size();
  TORCH_CHECK(last % align == 0, "afd_b200: ", name, " last dim must be a multiple of ", align);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "afd_b200: ", name, " must be 16-byte aligned");
}

// Per-device status word written by kernels whose bounded waits expire.
std::mutex g_status_mu;
std::vector<at::Tensor> g_status;

at::Tensor& status_tensor(int device) {
  std::lock_guard<std::mutex> lock(g_status_mu);
  if ((int)g_status.size() <= device) g_status.resize(device + 1);
  if (!g_status[device].defined()) {
    g_status[device] = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device));
  }
  return g_status[device];
}

int* status_ptr(const at::Tensor& like) { return status_tensor(like.get_device()).data_ptr<int>(); }

// Per-device arrival counters for merging MLA split partials inside the decode
// launch (zeroed once; every launch leaves them zero).  Decode launches on a
// device are stream-ordered in this runtime, so one array serves them all.
// Returns nullptr (the launch then runs the separate combine kernel) when the
// array is too small or does not exist yet while a graph is being captured,
// so that no allocation or memset is recorded into the graph.
constexpr int64_t kMlaArrivals = 1 << 16;

// AFD_MLA_KERNEL=mma selects the mma.sync MLA decode kernel (A/B comparisons);
// the default is the tcgen05 kernel for the shapes it takes.
bool mla_tc_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("AFD_MLA_KERNEL");
    return !(v != nullptr && std::string(v) == "mma");
  }();
  return on;
}
// AFD_MLA_BALANCED=1 runs the work-balanced MLA decode kernel (the KV tiles of
// all requests split evenly over one wave of CTAs) for the shapes the split
// kernel would take; off by default.
bool mla_balanced_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("AFD_MLA_BALANCED");
    return v != nullptr && std::string(v) == "1";
  }();
  return on;
}
std::vector<at::Tensor> g_mla_arrivals;

int* mla_arrivals(const at::Tensor& like, int64_t need) {
  if (need > kMlaArrivals) return nullptr;
  const int device = like.get_device();
  std::lock_guard<std::mutex> lock(g_status_mu);
  if ((int)g_mla_arrivals.size() <= device) g_mla_arrivals.resize(device + 1);
  if (!g_mla_arrivals[device].defined()) {
    if (c10::cuda::currentStreamCaptureStatusMayInitCtx() != c10::cuda::CaptureStatus::None) return nullptr;
    g_mla_arrivals[device] = at::zeros({kMlaArrivals}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device));
  }
  return g_mla_arrivals[device].data_ptr<int>();
}

// ------------------------------------------------------------------ norms
at::Tensor rms_norm(const at::Tensor& x, const at::Tensor& w, double eps) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous(), "rms_norm: contiguous inputs required");
  const int64_t hidden = x.size(-1);
  check_vec16(x, hidden, "x");
  auto out = at::empty_like(x);
  const int rows = (int)(x.numel() / hidden);
  c10::cuda::CUDAGuard g(x.device());
  launch_rms_norm(out.data_ptr(), x.data_ptr(), w.data_ptr(), rows, (int)hidden, (float)eps, dtype_code(x), stream());
  return out;
}

at::Tensor fused_add_rms_norm(const at::Tensor& x, at::Tensor& residual, const at::Tensor& w, double eps) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous() && residual.is_contiguous() && w.is_contiguous(), "fused_add_rms_norm: contiguous");
  TORCH_CHECK(x.sizes() == residual.sizes() && x.scalar_type() == residual.scalar_type(), "shape/dtype mismatch");
  const int64_t hidden = x.size(-1);
  check_vec16(x, hidden, "x");
  auto out = at::empty_like(x);
  c10::cuda::CUDAGuard g(x.device());
  launch_fused_add_rms_norm(out.data_ptr(), x.data_ptr(), residual.data_ptr(), w.data_ptr(),
                            (int)(x.numel() / hidden), (int)hidden, (float)eps, dtype_code(x), stream());
  return out;
}

at::Tensor silu_and_mul(const at::Tensor& x) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous(), "silu_and_mul: contiguous input required");
  const int64_t d = x.size(-1) / 2;
  check_vec16(x, d, "x");
  auto sizes = x.sizes().vec();
  sizes.back() = d;
  auto out = at::empty(sizes, x.options());
  c10::cuda::CUDAGuard g(x.device());
  launch_silu_and_mul(out.data_ptr(), x.data_ptr(), (int)(x.numel() / (2 * d)), (int)d, dtype_code(x), stream());
  return out;
}

at::Tensor argmax_rows(const at::Tensor& x) {
  check_cuda(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "argmax_rows: x [rows, n] with contiguous rows");
  auto out = at::empty({x.size(0)}, x.options().dtype(at::kInt));
  c10::cuda::CUDAGuard g(x.device());
  launch_argmax_rows(x.data_ptr(), x.stride(0), (int)x.size(0), (int)x.size(1), dtype_code(x),
                     out.data_ptr<int32_t>(), stream());
  return out;
}

// out (fp32, at least copies * span entries): out[c * span + r] = sigmoid(x[r] . w).
void gate_sigmoid_rows(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, int64_t copies, int64_t span) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.dim() == 2 &&
                  x.is_contiguous() && w.is_contiguous() && w.numel() == x.size(1),
              "gate_sigmoid_rows: x [rows, H] and w [H] bf16, contiguous");
  check_vec16(x, x.size(1), "x");
  check_vec16(w, w.numel(), "w");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && span >= x.size(0) &&
                  out.numel() >= (copies - 1) * span + x.size(0),
              "gate_sigmoid_rows: out fp32 with copies x span entries");
  c10::cuda::CUDAGuard g(x.device());
  launch_gate_sigmoid_rows(x.data_ptr(), w.data_ptr(), (int)x.size(0), (int)x.size(1), out.data_ptr<float>(),
                           (int)copies, (int)span, stream());
}

void rope_(at::Tensor& x, const at::Tensor& positions, const at::Tensor& cos_sin, bool interleaved) {
  check_cuda(x, "x");
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1, "rope_: x must be [T, H, rot] with contiguous last dim");
  TORCH_CHECK(positions.scalar_type() == at::kLong && cos_sin.scalar_type() == at::kFloat, "rope_: dtypes");
  TORCH_CHECK(cos_sin.size(1) == x.size(2), "rope_: cos_sin width must equal rot dim");
  c10::cuda::CUDAGuard g(x.device());
  launch_rope(x.data_ptr(), positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(), (int)x.size(0), (int)x.size(1),
              (int)x.size(2), x.stride(0), x.stride(1), interleaved, dtype_code(x), stream());
}

// scoring: 0 softmax, 1 sigmoid, 2 sqrt(softplus); forced [T, k] int32 (hash routing) fixes the experts.
std::tuple<at::Tensor, at::Tensor> topk_route(const at::Tensor& logits, int64_t k, int64_t scoring, bool renorm,
                                             const c10::optional<at::Tensor>& bias, int64_t n_group,
                                             int64_t topk_group, double scale,
                                             const c10::optional<at::Tensor>& forced) {
  check_cuda(logits, "logits");
  auto lf = logits.to(at::kFloat).contiguous();
  const int T = (int)lf.size(0), E = (int)lf.size(1);
  TORCH_CHECK(E <= 512 && k <= 32, "topk_route: E <= 512 and k <= 32");
  TORCH_CHECK(n_group <= 32 && (n_group <= 1 || E % n_group == 0), "topk_route: bad n_group");
  auto w = at::empty({T, k}, lf.options());
  auto ids = at::empty({T, k}, lf.options().dtype(at::kInt));
  const float* bp = nullptr;
  at::Tensor bf;
  if (bias.has_value() && bias->defined()) {
    bf = bias->to(at::kFloat).contiguous();
    bp = bf.data_ptr<float>();
  }
  const int32_t* fp = nullptr;
  if (forced.has_value() && forced->defined()) {
    TORCH_CHECK(forced->scalar_type() == at::kInt && forced->is_contiguous() && forced->size(0) == T &&
                    forced->size(1) == k, "topk_route: forced ids [T, k] int32");
    fp = forced->data_ptr<int32_t>();
  }
  TORCH_CHECK(scoring >= 0 && scoring <= 2, "topk_route: scoring 0 softmax, 1 sigmoid, 2 sqrtsoftplus");
  c10::cuda::CUDAGuard g(logits.device());
  if (T > 0)
    launch_topk_route(lf.data_ptr<float>(), bp, w.data_ptr<float>(), ids.data_ptr<int32_t>(), T, E, (int)k,
                      (int)scoring, renorm, (int)n_group, (int)topk_group, (float)scale, fp, stream());
  return {w, ids};
}

// --------------------------------------------------------------- KV cache
// With q_pe ([T, H, R], last dim contiguous), its interleaved RoPE runs in the
// same launch (in place).
void mla_cache_write(at::Tensor& cache, const at::Tensor& kv_a, const at::Tensor& w, double eps,
                     const at::Tensor& positions, const at::Tensor& cos_sin, const at::Tensor& slots, int64_t L,
                     const c10::optional<at::Tensor>& q_pe) {
  check_cuda(kv_a, "kv_a");
  const int64_t D = cache.size(-1);
  const int R = (int)(D - L);
  TORCH_CHECK(kv_a.size(1) == D && kv_a.stride(1) == 1, "mla_cache_write: kv_a [T, L+R] row-major");
  TORCH_CHECK(cache.scalar_type() == kv_a.scalar_type() && cache.is_contiguous(), "mla_cache_write: cache");
  TORCH_CHECK(kv_a.stride(0) % (16 / kv_a.element_size()) == 0, "mla_cache_write: row stride alignment");
  void* qp = nullptr;
  int qh = 0;
  int64_t qst = 0, qsh = 0;
  if (q_pe.has_value() && q_pe->defined()) {
    const at::Tensor& q = *q_pe;
    const int64_t vec = 16 / q.element_size();
    TORCH_CHECK(q.dim() == 3 && q.size(0) == kv_a.size(0) && q.size(2) == R && q.stride(2) == 1 &&
                    q.scalar_type() == kv_a.scalar_type() && q.is_cuda(),
                "mla_cache_write: q_pe [T, H, rope] with a contiguous last dim");
    TORCH_CHECK(R % vec == 0 && q.stride(0) % vec == 0 && q.stride(1) % vec == 0 &&
                    reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
                "mla_cache_write: q_pe rows must be 16-byte aligned");
    qp = q.data_ptr();
    qh = (int)q.size(1);
    qst = q.stride(0);
    qsh = q.stride(1);
  }
  c10::cuda::CUDAGuard g(kv_a.device());
  launch_mla_cache_write(cache.data_ptr(), kv_a.data_ptr(), w.data_ptr(), (float)eps, positions.data_ptr<int64_t>(),
                         cos_sin.data_ptr<float>(), slots.data_ptr<int64_t>(), (int)kv_a.size(0), (int)L, R,
                         kv_a.stride(0), dtype_code(kv_a), stream(), qp, qh, qst, qsh);
}

// qkv [T, (nq + 2 nkv) * d] (rows may be strided) -> q [T, nq, d]; k, v into
// the caches [blocks, bs, nkv, d] at slot_mapping; optional per-head norms.
at::Tensor gqa_prologue(const at::Tensor& qkv, int64_t nq, int64_t nkv, int64_t d, const c10::optional<at::Tensor>& qw,
                        const c10::optional<at::Tensor>& kw, double eps, const at::Tensor& positions,
                        const at::Tensor& cos_sin, at::Tensor& kc, at::Tensor& vc, const at::Tensor& slots) {
  check_cuda(qkv, "qkv");
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) == (nq + 2 * nkv) * d, "gqa_prologue: qkv rows");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == d, "gqa_prologue: rope over the whole head");
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous() && kc.size(-1) == d && kc.size(-2) == nkv &&
                  kc.scalar_type() == qkv.scalar_type() && vc.scalar_type() == qkv.scalar_type(),
              "gqa_prologue: caches [blocks, bs, nkv, d]");
  TORCH_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kLong, "gqa_prologue: int64 meta");
  auto check_w = [&](const c10::optional<at::Tensor>& w) -> const void* {
    if (!w.has_value() || !w->defined()) return nullptr;
    TORCH_CHECK(w->numel() == d && w->is_contiguous() && w->scalar_type() == qkv.scalar_type(), "gqa_prologue: norm w");
    return w->data_ptr();
  };
  const void* qwp = check_w(qw);
  const void* kwp = check_w(kw);
  auto q = at::empty({qkv.size(0), nq, d}, qkv.options());
  c10::cuda::CUDAGuard g(qkv.device());
  const bool ok = launch_gqa_prologue(qkv.data_ptr(), qkv.stride(0), (int)qkv.size(0), (int)nq, (int)nkv, (int)d, qwp,
                                      kwp, (float)eps, positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(),
                                      q.data_ptr(), kc.data_ptr(), vc.data_ptr(), slots.data_ptr<int64_t>(),
                                      dtype_code(qkv), stream());
  TORCH_CHECK(ok, "gqa_prologue: head size ", d, " not supported (32 / 64 / 128 / 256)");
  return q;
}

void gqa_cache_write(at::Tensor& kc, at::Tensor& vc, const at::Tensor& k, const at::Tensor& v,
                     const at::Tensor& slots) {
  check_cuda(k, "k");
  const int64_t row = k.size(1) * k.size(2);
  TORCH_CHECK(k.stride(2) == 1 && k.stride(1) == k.size(2) && v.stride(2) == 1 && v.stride(1) == v.size(2),
              "gqa_cache_write: [T, H, D] rows must be dense");
  c10::cuda::CUDAGuard g(k.device());
  launch_gqa_cache_write(kc.data_ptr(), vc.data_ptr(), k.data_ptr(), v.data_ptr(), slots.data_ptr<int64_t>(),
                         (int)k.size(0), (int)row, k.stride(0), v.stride(0), dtype_code(k), stream());
}

// -------------------------------------------------------------- attention
// q_lat [B, H, 512] and q_pe [B, H, 64] may be any strided views (last dim
// contiguous); the output is [B, H, 512], or [H, B, 512] when head_major.
at::Tensor mla_decode(const at::Tensor& q_lat, const at::Tensor& q_pe, const at::Tensor& cache,
                      const at::Tensor& block_table, const at::Tensor& seq_lens, double scale, int64_t num_splits,
                      bool head_major) {
  check_cuda(q_lat, "q_lat");
  TORCH_CHECK(q_lat.scalar_type() == at::kBFloat16 && q_pe.scalar_type() == at::kBFloat16 &&
                  cache.scalar_type() == at::kBFloat16, "mla_decode: bf16 only");
  TORCH_CHECK(q_lat.dim() == 3 && q_pe.dim() == 3 && q_lat.size(2) == 512 && q_pe.size(2) == 64 &&
                  q_lat.stride(2) == 1 && q_pe.stride(2) == 1, "mla_decode: q_lat [B,H,512], q_pe [B,H,64]");
  TORCH_CHECK(q_lat.size(0) == q_pe.size(0) && q_lat.size(1) == q_pe.size(1), "mla_decode: q halves disagree");
  TORCH_CHECK(q_lat.stride(0) % 8 == 0 && q_lat.stride(1) % 8 == 0 && q_pe.stride(0) % 8 == 0 && q_pe.stride(1) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(q_lat.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(q_pe.data_ptr()) % 16 == 0, "mla_decode: 16-byte aligned rows");
  TORCH_CHECK(cache.is_contiguous() && cache.size(-1) == 576, "mla_decode: cache [blocks, bs, 576] contiguous");
  TORCH_CHECK(q_lat.size(1) % 16 == 0, "mla_decode: heads must be a multiple of 16");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "mla_decode: int32 meta");
  TORCH_CHECK(block_table.stride(1) == 1, "mla_decode: block_table rows must be dense");
  const int B = (int)q_lat.size(0), H = (int)q_lat.size(1);
  const int bs = (int)cache.size(1), nblocks = (int)cache.size(0);
  TORCH_CHECK(bs % 32 == 0, "mla_decode: block size must be a multiple of 32");
  const int maxb = (int)block_table.size(1);
  at::Tensor out = head_major ? at::empty({H, B, 512}, q_lat.options()) : at::empty({B, H, 512}, q_lat.options());
  if (B == 0) return out;
  const int dev_sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  // The tcgen05 kernel for the head counts it is faster at (64+ heads), unless
  // AFD_MLA_KERNEL=mma asks for the mma.sync one; other shapes take mma.sync.
  const int tc_hg = mla_tc_enabled() ? mla_decode_tc_heads_per_cta(H) : 0;
  const bool use_tc = tc_hg > 0 && bs % 64 == 0;  // every tile shape divides a 64-token block
  int splits = (int)num_splits;
  if (splits <= 0) {
    splits = use_tc ? mla_decode_tc_num_splits(B, H, maxb * bs, dev_sms)
                    : mla_decode_num_splits(B * (H / 16), maxb * bs, dev_sms);
  }
  at::Tensor po, pl;
  if (splits > 1) {
    po = at::empty({B, splits, H, 512}, q_lat.options().dtype(at::kFloat));
    pl = at::empty({B, splits, H}, q_lat.options().dtype(at::kFloat));
  }
  MlaQO qo{};
  qo.q_lat = reinterpret_cast<const __nv_bfloat16*>(q_lat.data_ptr());
  qo.lat_sb = q_lat.stride(0);
  qo.lat_sh = q_lat.stride(1);
  qo.q_pe = reinterpret_cast<const __nv_bfloat16*>(q_pe.data_ptr());
  qo.pe_sb = q_pe.stride(0);
  qo.pe_sh = q_pe.stride(1);
  qo.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  qo.out_sb = head_major ? 512 : (int64_t)H * 512;
  qo.out_sh = head_major ? (int64_t)B * 512 : 512;
  c10::cuda::CUDAGuard g(q_lat.device());
  float* po_ptr = splits > 1 ? po.data_ptr<float>() : nullptr;
  float* pl_ptr = splits > 1 ? pl.data_ptr<float>() : nullptr;
  cudaError_t e = cudaErrorNotSupported;
  if (use_tc) {
    int* arr = splits > 1 ? mla_arrivals(q_lat, (int64_t)B * (H / tc_hg)) : nullptr;
    if (splits == 1 || (arr != nullptr && splits <= mla_decode_tc_max_splits(tc_hg)))
      e = launch_mla_decode_tc(qo, cache.data_ptr(), block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                               po_ptr, pl_ptr, status_ptr(q_lat), B, H, bs, nblocks, (int)block_table.stride(0), splits,
                               (float)scale, stream(), arr);
  }
  if (e == cudaErrorNotSupported && mla_balanced_enabled() && num_splits <= 0 &&
      B <= mla_decode_balanced_max_batch()) {
    int* arr = mla_arrivals(q_lat, (int64_t)B * (H / 16));
    if (arr != nullptr) {
      const int ctas = mla_decode_balanced_ctas(H, dev_sms);
      at::Tensor bpo = at::empty({2 * ctas, H, 512}, q_lat.options().dtype(at::kFloat));
      at::Tensor bpl = at::empty({2 * ctas, H}, q_lat.options().dtype(at::kFloat));
      e = launch_mla_decode_balanced(qo, cache.data_ptr(), block_table.data_ptr<int32_t>(),
                                     seq_lens.data_ptr<int32_t>(), bpo.data_ptr<float>(), bpl.data_ptr<float>(),
                                     status_ptr(q_lat), arr, B, H, bs, nblocks, (int)block_table.stride(0), ctas,
                                     (float)scale, stream());
    }
  }
  if (e == cudaErrorNotSupported) {  // nothing launched: the mma.sync kernel takes the shape
    if (use_tc && splits > 1 && num_splits <= 0) {
      // the split count was picked for the other kernel's geometry: pick again
      splits = mla_decode_num_splits(B * (H / 16), maxb * bs, dev_sms);
      if (splits > 1 && po.size(1) < splits) {
        po = at::empty({B, splits, H, 512}, q_lat.options().dtype(at::kFloat));
        pl = at::empty({B, splits, H}, q_lat.options().dtype(at::kFloat));
      }
      po_ptr = splits > 1 ? po.data_ptr<float>() : nullptr;
      pl_ptr = splits > 1 ? pl.data_ptr<float>() : nullptr;
    }
    e = launch_mla_decode(qo, cache.data_ptr(), block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), po_ptr,
                          pl_ptr, status_ptr(q_lat), B, H, 512, 64, bs, nblocks, (int)block_table.stride(0), splits,
                          (float)scale, stream(), splits > 1 ? mla_arrivals(q_lat, (int64_t)B * (H / 16)) : nullptr);
  }
  TORCH_CHECK(e == cudaSuccess, "mla_decode: launch failed: ", cudaGetErrorString(e));
  return out;
}

// DeepSeek sparse attention: q [B, H, 576] over the kept positions
// keep_pos [B, K] int32 (-1 = unused).  Output [B, H, 512].
at::Tensor mla_decode_sparse(const at::Tensor& q, const at::Tensor& cache, const at::Tensor& block_table,
                             const at::Tensor& seq_lens, const at::Tensor& keep_pos, double scale, int64_t num_splits) {
  check_cuda(q, "q");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && cache.scalar_type() == at::kBFloat16, "mla_decode_sparse: bf16 only");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 576 && q.stride(2) == 1 && q.stride(0) % 8 == 0 && q.stride(1) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0, "mla_decode_sparse: q [B, H, 576], 16-byte rows");
  TORCH_CHECK(cache.is_contiguous() && cache.dim() == 3 && cache.size(-1) == 576, "mla_decode_sparse: cache [blocks, bs, 576]");
  TORCH_CHECK(q.size(1) % 16 == 0, "mla_decode_sparse: heads must be a multiple of 16");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  keep_pos.scalar_type() == at::kInt, "mla_decode_sparse: int32 meta");
  TORCH_CHECK(block_table.stride(1) == 1, "mla_decode_sparse: block_table rows must be dense");
  TORCH_CHECK(keep_pos.dim() == 2 && keep_pos.is_contiguous() && keep_pos.size(0) == q.size(0),
              "mla_decode_sparse: keep_pos [B, K] contiguous");
  const int B = (int)q.size(0), H = (int)q.size(1), K = (int)keep_pos.size(1);
  at::Tensor out = at::empty({B, H, 512}, q.options());
  if (B == 0) return out;
  int splits = (int)num_splits;
  if (splits <= 0) {
    int dev_sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
    splits = mla_decode_num_splits(B * (H / 16), K, dev_sms);
  }
  at::Tensor po, pl;
  if (splits > 1) {
    po = at::empty({B, splits, H, 512}, q.options().dtype(at::kFloat));
    pl = at::empty({B, splits, H}, q.options().dtype(at::kFloat));
  }
  MlaQO qo{};
  qo.q_lat = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  qo.lat_sb = q.stride(0);
  qo.lat_sh = q.stride(1);
  qo.q_pe = qo.q_lat + 512;
  qo.pe_sb = q.stride(0);
  qo.pe_sh = q.stride(1);
  qo.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  qo.out_sb = (int64_t)H * 512;
  qo.out_sh = 512;
  c10::cuda::CUDAGuard g(q.device());
  launch_mla_decode_sparse(qo, cache.data_ptr(), block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                           keep_pos.data_ptr<int32_t>(), K, splits > 1 ? po.data_ptr<float>() : nullptr,
                           splits > 1 ? pl.data_ptr<float>() : nullptr, status_ptr(q), B, H, 512, (int)cache.size(1),
                           (int)block_table.stride(0), splits, (float)scale, stream(),
                           splits > 1 ? mla_arrivals(q, (int64_t)B * (H / 16)) : nullptr);
  return out;
}

at::Tensor gqa_decode(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& block_table,
                      const at::Tensor& seq_lens, double scale, int64_t num_splits) {
  check_cuda(q, "q");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && kc.scalar_type() == at::kBFloat16 && vc.scalar_type() == at::kBFloat16,
              "gqa_decode: bf16 only");
  TORCH_CHECK(q.is_contiguous() && kc.is_contiguous() && vc.is_contiguous(), "gqa_decode: contiguous tensors");
  TORCH_CHECK(q.size(2) == 128 && kc.size(3) == 128, "gqa_decode: head_dim 128 only");
  const int B = (int)q.size(0), hq = (int)q.size(1), hkv = (int)kc.size(2);
  TORCH_CHECK(hq % hkv == 0 && hq / hkv <= 16, "gqa_decode: query group of at most 16 heads");
  const int bs = (int)kc.size(1), nblocks = (int)kc.size(0), maxb = (int)block_table.size(1);
  TORCH_CHECK(bs % 32 == 0 && block_table.stride(1) == 1, "gqa_decode: block size % 32, dense table rows");
  auto out = at::empty_like(q);
  if (B == 0) return out;
  int splits = (int)num_splits;
  if (splits <= 0) {
    int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
    splits = gqa_decode_num_splits(B, hkv, maxb * bs, sms);
  }
  at::Tensor po, pl;
  if (splits > 1) {
    po = at::empty({B, splits, hq, 128}, q.options().dtype(at::kFloat));
    pl = at::empty({B, splits, hq}, q.options().dtype(at::kFloat));
  }
  c10::cuda::CUDAGuard g(q.device());
  launch_gqa_decode(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), block_table.data_ptr<int32_t>(),
                    seq_lens.data_ptr<int32_t>(), splits > 1 ? po.data_ptr<float>() : nullptr,
                    splits > 1 ? pl.data_ptr<float>() : nullptr, status_ptr(q), B, hq, hkv, 128, bs, nblocks,
                    (int)block_table.stride(0), splits, (float)scale, stream());
  return out;
}

// -------------------------------------------------------------------- MoE
std::vector<at::Tensor> moe_align(const at::Tensor& topk_ids, int64_t e_local, int64_t offset, int64_t n_shared) {
  check_cuda(topk_ids, "topk_ids");
  TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.is_contiguous(), "moe_align: int32 contiguous ids");
  TORCH_CHECK(e_local + n_shared <= 1024, "moe_align: at most 1024 local experts");
  const int T = (int)topk_ids.size(0), k = (int)topk_ids.size(1);
  const int ks = k + (int)n_shared;
  auto o = topk_ids.options();
  auto counts = at::empty({e_local + n_shared}, o), offsets = at::empty({e_local + n_shared}, o);
  auto row_token = at::empty({std::max(T * ks, 1)}, o), row_slot = at::empty({std::max(T * ks, 1)}, o);
  auto tsr = at::empty({T, ks}, o), total = at::empty({1}, o);
  c10::cuda::CUDAGuard g(topk_ids.device());
  launch_moe_align(topk_ids.data_ptr<int32_t>(), T, k, (int)n_shared, (int)e_local, (int)offset,
                   counts.data_ptr<int32_t>(),
                   offsets.data_ptr<int32_t>(), row_token.data_ptr<int32_t>(), row_slot.data_ptr<int32_t>(),
                   tsr.data_ptr<int32_t>(), total.data_ptr<int32_t>(), stream());
  return {counts, offsets, row_token, row_slot, tsr, total};
}

at::Tensor moe_gather(const at::Tensor& x, const at::Tensor& row_token, const at::Tensor& total) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous(), "moe_gather: contiguous x");
  const int64_t rows_cap = row_token.size(0), H = x.size(1);
  check_vec16(x, H, "x");
  auto xs = at::empty({rows_cap, H}, x.options());
  c10::cuda::CUDAGuard g(x.device());
  launch_moe_gather(xs.data_ptr(), x.data_ptr(), row_token.data_ptr<int32_t>(), (int)rows_cap, (int)H,
                    total.data_ptr<int32_t>(), dtype_code(x), stream());
  return xs;
}

at::Tensor grouped_gemm(const at::Tensor& a, const at::Tensor& w, const at::Tensor& offsets, const at::Tensor& counts,
                        int64_t epilogue) {
  check_cuda(a, "a");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "grouped_gemm: bf16 only");
  TORCH_CHECK(a.is_contiguous() && w.is_contiguous() && w.dim() == 3, "grouped_gemm: a [R,K], w [E,N,K] contiguous");
  const int64_t R = a.size(0), K = a.size(1), E = w.size(0), N = w.size(1);
  TORCH_CHECK(w.size(2) == K && K % 64 == 0, "grouped_gemm: K must match and be a multiple of 64");
  if (epilogue == 1) {
    TORCH_CHECK((N / 2) % 64 == 0 && N % 2 == 0, "grouped_gemm: SwiGLU needs I % 64 == 0");
  } else {
    TORCH_CHECK(N % 128 == 0, "grouped_gemm: N must be a multiple of 128");
  }
  const int64_t n_out = epilogue == 1 ? N / 2 : N;
  auto d = at::empty({R, n_out}, a.options());
  if (R == 0) return d;
  c10::cuda::CUDAGuard g(a.device());
  launch_grouped_gemm(d.data_ptr(), a.data_ptr(), w.data_ptr(), offsets.data_ptr<int32_t>(),
                      counts.data_ptr<int32_t>(), (int)E, (int)R, (int)N, (int)K, (int)epilogue, status_ptr(a),
                      stream());
  return d;
}

// An MoE layer's experts in one launch: h = SwiGLU(a x w13^T) per expert
// segment, then y = h x w2^T (epilogue 0), or with a scatter config the
// routing-weighted rows go to the Attention ranks' combine slots (epilogue 2).
// sync: int32 [>= e_local + 1], zero before the first call and left zero by
// every call ([0, e_local) per-expert tile counters, [e_local] CTA counter).
// rows_hint: the largest segment expected (picks the pass width, not the result).
// scatter (optional): meta, rw, dst_ptrs, flag_ptrs, done_ctr, counts_reset
// and cfg [J, H, total_ctas, num_dst, layer] as in grouped_gemm_scatter.
at::Tensor moe_ffn(const at::Tensor& a, const at::Tensor& w13, const at::Tensor& w2, const at::Tensor& offsets,
                   const at::Tensor& counts, at::Tensor& sync, int64_t rows_hint, int64_t w_experts,
                   const c10::optional<at::Tensor>& meta, const c10::optional<at::Tensor>& rw,
                   const c10::optional<at::Tensor>& dst_ptrs, const c10::optional<at::Tensor>& flag_ptrs,
                   const c10::optional<at::Tensor>& done_ctr, const c10::optional<at::Tensor>& counts_reset,
                   c10::optional<std::vector<int64_t>> cfg) {
  check_cuda(a, "a");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && w13.scalar_type() == at::kBFloat16 &&
                  w2.scalar_type() == at::kBFloat16, "moe_ffn: bf16 activations and weights");
  TORCH_CHECK(a.is_contiguous() && w13.is_contiguous() && w2.is_contiguous() && w13.dim() == 3 && w2.dim() == 3,
              "moe_ffn: a [R, H], w13 [E, 2I, H], w2 [E, H, I] contiguous");
  const int64_t R = a.size(0), H = a.size(1), N1 = w13.size(1), I = N1 / 2, N2 = w2.size(1);
  const int e_local = (int)counts.numel();
  TORCH_CHECK(w13.size(2) == H && H % 64 == 0 && N1 % 2 == 0 && I % 64 == 0, "moe_ffn: w13 shapes");
  TORCH_CHECK(w2.size(2) == I && N2 % 128 == 0, "moe_ffn: w2 [E, N % 128 == 0, I]");
  if (w_experts < 0) {
    TORCH_CHECK(w13.size(0) == e_local && w2.size(0) == e_local, "moe_ffn: one weight set per expert segment");
  } else {
    TORCH_CHECK(w13.size(0) == w_experts && w2.size(0) == w_experts && (w_experts == 1 || w_experts == e_local),
                "moe_ffn: w_experts must be 1 or the segment count");
  }
  TORCH_CHECK(offsets.scalar_type() == at::kInt && counts.scalar_type() == at::kInt && offsets.numel() >= e_local,
              "moe_ffn: int32 offsets / counts");
  TORCH_CHECK(sync.scalar_type() == at::kInt && sync.is_contiguous() && sync.numel() >= e_local + 1 &&
                  sync.device() == a.device(), "moe_ffn: int32 sync [>= e_local + 1] on the same device");
  const bool scatter = meta.has_value() && meta->defined();
  auto h = at::empty({R, I}, a.options());
  at::Tensor y = scatter ? at::empty({0}, a.options()) : at::empty({R, N2}, a.options());
  if (R == 0) return y;
  const int we = (int)w_experts;
  GemmSpec g0{h.data_ptr(), a.data_ptr(), w13.data_ptr(), offsets.data_ptr<int32_t>(), counts.data_ptr<int32_t>(),
              e_local, (int)R, (int)N1, (int)H, 1, we};
  GemmSpec g1{scatter ? nullptr : y.data_ptr(), h.data_ptr(), w2.data_ptr(), offsets.data_ptr<int32_t>(),
              counts.data_ptr<int32_t>(), e_local, (int)R, (int)N2, (int)I, scatter ? 2 : 0, we};
  ScatterParams sp{};
  if (scatter) {
    TORCH_CHECK(rw.has_value() && dst_ptrs.has_value() && flag_ptrs.has_value() && done_ctr.has_value() &&
                    counts_reset.has_value() && cfg.has_value() && cfg->size() == 5,
                "moe_ffn: a scatter needs meta, rw, dst_ptrs, flag_ptrs, done_ctr, counts_reset and cfg");
    const auto& c = *cfg;
    sp.meta = meta->data_ptr<int32_t>();
    sp.rw = rw->data_ptr<float>();
    sp.dst_ptrs = dst_ptrs->data_ptr<int64_t>();
    sp.J = (int)c[0];
    sp.H = (int)c[1];
    sp.total_ctas = (int)c[2];
    sp.num_dst = (int)c[3];
    sp.layer = (int)c[4];
    sp.flag_ptrs = flag_ptrs->data_ptr<int64_t>();
    sp.done_ctr = reinterpret_cast<unsigned*>(done_ctr->data_ptr());
    sp.counts_reset = counts_reset->data_ptr<int32_t>();
    sp.n_reset = (int)counts_reset->numel();
  }
  int32_t* sy = sync.data_ptr<int32_t>();
  c10::cuda::CUDAGuard guard(a.device());
  const cudaError_t e = launch_grouped_gemm_phases(g0, &g1, sy, reinterpret_cast<unsigned*>(sy + e_local),
                                                   status_ptr(a), scatter ? &sp : nullptr, stream(), (int)rows_hint);
  TORCH_CHECK(e == cudaSuccess, "moe_ffn: launch failed: ", cudaGetErrorString(e));
  return y;
}

// Dense or per-head-batched GEMM on the tcgen05 grouped kernel (no library GEMM).
//   a [T, K] (rows any stride, 16-byte aligned), w [N, K] or [1, N, K]:
//     out [T, N] (epilogue 0) or SiLU(gate) * up [T, N / 2] (epilogue 1).
//   a [E, T, K] (any strides with a contiguous last dim, e.g. a per-head view
//     of a projection), w [E, N, K]: out [T, E * N] with out[t, e * N + n] =
//     a[e, t] . w[e, n] -- a batched product written token-major.
// N % 128 == 0 (N / 2 % 64 == 0 for SwiGLU) and K % 64 == 0.  Dense epilogue 0
// only: n_valid keeps the first n_valid output columns (weights padded to a
// multiple of 128 rows), out_f32 stores fp32 (e.g. router logits).  With ws
// (fp32, zero) and ctr (int32, zero) a GEMM with few output tiles splits K
// over the SMs; both are left zero.
at::Tensor tc_gemm(const at::Tensor& a, const at::Tensor& w, int64_t epilogue, int64_t n_valid, bool out_f32,
                   const c10::optional<at::Tensor>& ws, const c10::optional<at::Tensor>& ctr) {
  check_cuda(a, "a");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && w.is_contiguous(),
              "tc_gemm: bf16, contiguous weights");
  TORCH_CHECK(a.stride(-1) == 1 && reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0, "tc_gemm: 16-byte aligned a");
  const bool batched = a.dim() == 3;
  TORCH_CHECK(a.dim() == 2 || batched, "tc_gemm: a [T, K] or [E, T, K]");
  const int64_t E = batched ? a.size(0) : 1, T = a.size(-2), K = a.size(-1);
  const at::Tensor w3 = w.dim() == 2 ? w.unsqueeze(0) : w;
  TORCH_CHECK(w3.dim() == 3 && w3.size(0) == E && w3.size(2) == K, "tc_gemm: w [E, N, K] matching a");
  const int64_t N = w3.size(1);
  TORCH_CHECK(K % 64 == 0, "tc_gemm: K must be a multiple of 64");
  for (int d = 0; d + 1 < a.dim(); ++d)
    TORCH_CHECK(a.stride(d) % 8 == 0, "tc_gemm: activation strides must be multiples of 16 bytes");
  if (epilogue == 1) {
    TORCH_CHECK(!batched && N % 128 == 0, "tc_gemm: SwiGLU for a dense [T, K] input with N % 128 == 0");
  } else {
    TORCH_CHECK(epilogue == 0 && N % 128 == 0, "tc_gemm: epilogue 0 or 1, N % 128 == 0");
  }
  const bool narrow = n_valid > 0 && n_valid < N;
  TORCH_CHECK(!(narrow || out_f32) || (!batched && epilogue == 0), "tc_gemm: n_valid / out_f32 need a dense epilogue 0");
  TORCH_CHECK(n_valid >= 0 && n_valid <= N, "tc_gemm: 0 <= n_valid <= N");
  const int64_t n_out = epilogue == 1 ? N / 2 : (narrow ? n_valid : N * E);
  auto d = at::empty({T, n_out}, a.options().dtype(out_f32 ? at::kFloat : at::kBFloat16));
  if (T == 0) return d;
  GemmSpec g{d.data_ptr(), a.data_ptr(), w3.data_ptr(), nullptr, nullptr, (int)E, (int)T, (int)N, (int)K,
             batched ? 3 : (int)epilogue, -1};
  g.fixed_count = (int)T;
  g.out_f32 = out_f32 ? 1 : 0;
  g.n_valid = narrow ? (int)n_valid : 0;
  // Split K when the output tiles alone would leave SMs idle (few weight rows):
  // one wave of items over the SMs, fp32 partials reduced in the workspace.
  const int64_t tiles = E * (epilogue == 1 ? (N / 2) / 64 : N / 128);
  const int sms = (int)grouped_gemm_grid(1 << 30);
  if (epilogue == 0 && ws.has_value() && ctr.has_value() && tiles * 2 <= sms) {
    TORCH_CHECK(ws->scalar_type() == at::kFloat && ctr->scalar_type() == at::kInt && ws->device() == a.device() &&
                    ctr->device() == a.device(), "tc_gemm: fp32 workspace and int32 tile counters on a's device");
    const int64_t cols = narrow ? n_valid : N * E;
    if (T * cols <= ws->numel() && tiles <= ctr->numel()) {
      g.k_splits = (int)std::min<int64_t>(K / 64, sms / tiles);
      g.acc_ws = ws->data_ptr<float>();
      g.tile_ctr = ctr->data_ptr<int32_t>();
    }
  }
  g.a_ld = a.stride(-2);
  g.a_plane = batched ? a.stride(0) : 0;
  c10::cuda::CUDAGuard guard(a.device());
  const cudaError_t e =
      launch_grouped_gemm_phases(g, nullptr, nullptr, nullptr, status_ptr(a), nullptr, stream(), (int)T);
  TORCH_CHECK(e == cudaSuccess, "tc_gemm: launch failed: ", cudaGetErrorString(e));
  return d;
}

// Dense SwiGLU MLP in one launch: h = SiLU(x w_gate^T) * (x w_up^T), y = h w2^T,
// as the two phases of the tcgen05 kernel over one segment of T rows.
// x [T, H] (rows any 16-byte multiple apart), w13 [2I, H], w2 [H, I]; sync as in moe_ffn.
at::Tensor dense_ffn(const at::Tensor& x, const at::Tensor& w13, const at::Tensor& w2, at::Tensor& sync) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w13.scalar_type() == at::kBFloat16 &&
                  w2.scalar_type() == at::kBFloat16 && w13.is_contiguous() && w2.is_contiguous(),
              "dense_ffn: bf16, contiguous weights");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "dense_ffn: x [T, H], 16-byte aligned rows");
  const int64_t T = x.size(0), H = x.size(1);
  const at::Tensor a13 = w13.dim() == 3 ? w13[0] : w13, a2 = w2.dim() == 3 ? w2[0] : w2;
  const int64_t N1 = a13.size(0), I = N1 / 2, N2 = a2.size(0);
  TORCH_CHECK(a13.size(1) == H && H % 64 == 0 && N1 % 128 == 0 && I % 64 == 0, "dense_ffn: w13 [2I, H]");
  TORCH_CHECK(a2.size(1) == I && N2 % 128 == 0, "dense_ffn: w2 [N % 128 == 0, I]");
  TORCH_CHECK(sync.scalar_type() == at::kInt && sync.numel() >= 2 && sync.device() == x.device(),
              "dense_ffn: int32 sync [>= 2]");
  auto h = at::empty({T, I}, x.options());
  auto y = at::empty({T, N2}, x.options());
  if (T == 0) return y;
  GemmSpec g0{h.data_ptr(), x.data_ptr(), a13.data_ptr(), nullptr, nullptr, 1, (int)T, (int)N1, (int)H, 1, 1};
  g0.fixed_count = (int)T;
  g0.a_ld = x.stride(0);
  GemmSpec g1{y.data_ptr(), h.data_ptr(), a2.data_ptr(), nullptr, nullptr, 1, (int)T, (int)N2, (int)I, 0, 1};
  g1.fixed_count = (int)T;
  int32_t* sy = sync.data_ptr<int32_t>();
  c10::cuda::CUDAGuard guard(x.device());
  const cudaError_t e = launch_grouped_gemm_phases(g0, &g1, sy, reinterpret_cast<unsigned*>(sy + 1), status_ptr(x),
                                                   nullptr, stream(), (int)T);
  TORCH_CHECK(e == cudaSuccess, "dense_ffn: launch failed: ", cudaGetErrorString(e));
  return y;
}

// CTAs of one moe_ffn launch (both phases share the persistent grid).
int64_t moe_ffn_grid(int64_t e_local, int64_t n1, int64_t n2) {
  return grouped_gemm_grid((int)(e_local * ((n1 / 2) / 64 + n2 / 128)));
}

at::Tensor moe_combine(const at::Tensor& ys, const at::Tensor& topk_w, const at::Tensor& tsr,
                       const c10::optional<at::Tensor>& shared) {
  const int k_routed = (int)topk_w.size(1);
  check_cuda(ys, "ys");
  const int T = (int)tsr.size(0), k = (int)tsr.size(1);
  const int64_t H = ys.size(1);
  check_vec16(ys, H, "ys");
  TORCH_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.is_contiguous(), "moe_combine: fp32 weights");
  auto out = at::empty({T, H}, ys.options());
  if (T == 0) return out;
  const void* sp = nullptr;
  if (shared.has_value() && shared->defined()) {
    TORCH_CHECK(shared->is_contiguous() && shared->scalar_type() == ys.scalar_type(), "moe_combine: shared");
    sp = shared->data_ptr();
  }
  c10::cuda::CUDAGuard g(ys.device());
  launch_moe_combine(out.data_ptr(), ys.data_ptr(), topk_w.data_ptr<float>(), tsr.data_ptr<int32_t>(), T, k, k_routed,
                     (int)H, sp, dtype_code(ys), stream());
  return out;
}

void decode_advance(at::Tensor& input_ids, at::Tensor& positions, at::Tensor& slots, at::Tensor& seq_lens,
                    const at::Tensor& next_tokens, const at::Tensor& block_table, int64_t block_size,
                    int64_t wrap_at, int64_t wrap_to) {
  check_cuda(input_ids, "input_ids");
  TORCH_CHECK(input_ids.scalar_type() == at::kInt && positions.scalar_type() == at::kLong &&
                  slots.scalar_type() == at::kLong && seq_lens.scalar_type() == at::kInt &&
                  next_tokens.scalar_type() == at::kInt && block_table.scalar_type() == at::kInt,
              "decode_advance: dtypes");
  const int batch = (int)input_ids.size(0);
  if (batch == 0) return;
  c10::cuda::CUDAGuard g(input_ids.device());
  launch_decode_advance(input_ids.data_ptr<int32_t>(), positions.data_ptr<int64_t>(), slots.data_ptr<int64_t>(),
                        seq_lens.data_ptr<int32_t>(), next_tokens.data_ptr<int32_t>(), block_table.data_ptr<int32_t>(),
                        batch, (int)block_table.stride(0), (int)block_size, wrap_at, wrap_to, stream());
}

// ------------------------------------------------------- fused AFD transfer
int64_t iptr(const at::Tensor& t) { return reinterpret_cast<int64_t>(t.data_ptr()); }

void afd_epoch(at::Tensor& epoch) {
  c10::cuda::CUDAGuard g(epoch.device());
  launch_afd_epoch(reinterpret_cast<uint64_t*>(epoch.data_ptr()), stream());
}

void afd_stamp(at::Tensor& buf, int64_t idx) {
  TORCH_CHECK(buf.scalar_type() == at::kLong && buf.is_contiguous() && idx >= 0 && idx < buf.numel(),
              "afd_stamp: int64 buffer and an index inside it");
  c10::cuda::CUDAGuard g(buf.device());
  launch_afd_stamp(reinterpret_cast<uint64_t*>(buf.data_ptr()), (int)idx, stream());
}

void afd_wait(const at::Tensor& flag, int64_t index, const at::Tensor& epoch, int64_t arrivals, int64_t timeout_ns) {
  c10::cuda::CUDAGuard g(flag.device());
  launch_afd_wait(reinterpret_cast<const uint64_t*>(flag.data_ptr()) + index,
                  reinterpret_cast<const uint64_t*>(epoch.data_ptr()), (uint64_t)arrivals, timeout_ns,
                  status_ptr(flag), stream());
}

// cfg (int64): [E, k, scoring, renorm, n_group, topk_group, moe, has_shared, num_ffn, e_local, t_cap,
//               attn_rank, home_f, layer]; ptrs [5, F]: tok, rid, rwt, tcount, arrive flags on each FFN rank
//               ([6, F] adds the e4m3 rows' scale buffers: rows then travel as e4m3 with 1 x 128 scales).
// done_ctr: int32 [>= 1 + ceil(T / 16)], zero before the first use and left zero by every call
// ([0] send-kernel completion, [1:] router token tiles).
// cfg[14] (optional) = prenorm: attn_out is already the FFN input; residual and norm_w are then unused.
// hash_table [vocab, k] int32 + input_ids [T] int32: hash-routed layer (experts from the table).
void afd_dispatch(const at::Tensor& attn_out, at::Tensor& residual, const at::Tensor& norm_w, double eps,
                  const at::Tensor& gate_w, const c10::optional<at::Tensor>& gate_bias, double scale,
                  const at::Tensor& ptrs, at::Tensor& fmask, at::Tensor& done_ctr, std::vector<int64_t> cfg,
                  const c10::optional<at::Tensor>& hash_table, const c10::optional<at::Tensor>& input_ids) {
  check_cuda(attn_out, "attn_out");
  TORCH_CHECK(attn_out.scalar_type() == at::kBFloat16 && residual.scalar_type() == at::kBFloat16,
              "afd_dispatch: bf16 activations");
  TORCH_CHECK(attn_out.is_contiguous() && residual.is_contiguous() && gate_w.is_contiguous(), "afd_dispatch: layout");
  TORCH_CHECK(cfg.size() == 14 || cfg.size() == 15, "afd_dispatch: cfg has 14 or 15 entries");
  TORCH_CHECK(ptrs.scalar_type() == at::kLong && ptrs.dim() == 2 && (ptrs.size(0) == 5 || ptrs.size(0) == 6),
              "afd_dispatch: ptrs [5, F] (bf16 rows) or [6, F] (e4m3 rows + scales)");
  DispatchParams p{};
  p.attn_out = attn_out.data_ptr();
  p.residual = residual.data_ptr();
  p.norm_w = norm_w.data_ptr();
  p.eps = (float)eps;
  p.gate_w = gate_w.data_ptr();
  at::Tensor gb;
  if (gate_bias.has_value() && gate_bias->defined()) {
    gb = gate_bias->to(at::kFloat).contiguous();
    p.gate_bias = gb.data_ptr<float>();
  }
  p.E = (int)cfg[0];
  p.k = (int)cfg[1];
  p.scoring = (int)cfg[2];
  p.renorm = cfg[3] != 0;
  p.n_group = (int)cfg[4];
  p.topk_group = (int)cfg[5];
  p.scale = (float)scale;
  p.T = (int)attn_out.size(0);
  p.H = (int)attn_out.size(1);
  p.moe = (int)cfg[6];
  p.has_shared = (int)cfg[7];
  p.num_ffn = (int)cfg[8];
  p.e_local = (int)cfg[9];
  p.t_cap = (int)cfg[10];
  p.attn_rank = (int)cfg[11];
  p.home_f = (int)cfg[12];
  p.layer = (int)cfg[13];
  p.prenorm = cfg.size() == 15 ? (int)cfg[14] : 0;
  if (hash_table.has_value() && hash_table->defined()) {
    TORCH_CHECK(input_ids.has_value() && input_ids->defined() && input_ids->scalar_type() == at::kInt &&
                    input_ids->is_contiguous() && input_ids->numel() == attn_out.size(0),
                "afd_dispatch: hash routing needs int32 input_ids [T]");
    TORCH_CHECK(hash_table->scalar_type() == at::kInt && hash_table->is_contiguous() &&
                    hash_table->size(1) == (int64_t)cfg[1], "afd_dispatch: hash table [vocab, k] int32");
    p.hash_table = hash_table->data_ptr<int32_t>();
    p.input_ids = input_ids->data_ptr<int32_t>();
  }
  TORCH_CHECK(p.k <= 16 && p.H % 16 == 0 && p.H <= 8192 && p.T <= p.t_cap && p.num_ffn <= 32 && p.E <= 512,
              "afd_dispatch: k <= 16, H % 16 == 0, H <= 8192, T <= t_cap, at most 32 FFN ranks, E <= 512");
  const int64_t tiles = (p.T + 15) / 16;
  TORCH_CHECK(done_ctr.scalar_type() == at::kInt && done_ctr.is_contiguous() && done_ctr.numel() >= 1 + tiles,
              "afd_dispatch: done counters need 1 + ceil(T / 16) int32 entries");
  at::Tensor h_scratch = at::empty({std::max<int64_t>(p.T, 1), p.H}, attn_out.options());
  at::Tensor logits = at::empty({std::max<int64_t>(p.T, 1), std::max(p.E, 1)}, attn_out.options().dtype(at::kFloat));
  p.h = h_scratch.data_ptr();
  p.logits = logits.data_ptr<float>();
  const int64_t* pt = ptrs.data_ptr<int64_t>();
  const int64_t F = ptrs.size(1);
  p.tok_ptrs = pt;
  p.rid_ptrs = pt + F;
  p.rwt_ptrs = pt + 2 * F;
  p.tcount_ptrs = pt + 3 * F;
  p.flag_ptrs = pt + 4 * F;
  if (ptrs.size(0) == 6) {
    TORCH_CHECK(p.H % 128 == 0, "afd_dispatch: e4m3 rows need H % 128 == 0");
    p.scale_ptrs = pt + 5 * F;
  }
  p.fmask = fmask.data_ptr<int32_t>();
  p.done_ctr = reinterpret_cast<unsigned*>(done_ctr.data_ptr());
  p.route_ctr = p.done_ctr + 1;
  p.status = status_ptr(attn_out);
  c10::cuda::CUDAGuard g(attn_out.device());
  launch_afd_dispatch(p, stream());
}

// cfg: [A, t_cap, k, e_local, e_offset, cap, ratio, home_a0, moe(, n_chunks, shared_base, shared_stride)]
// With `flag`, every CTA first waits (bounded) until flag[flag_index] >= epoch * arrivals.
void afd_expand(const at::Tensor& tok, const at::Tensor& rid, const at::Tensor& rwt, const at::Tensor& tcount,
                at::Tensor& x, at::Tensor& meta, at::Tensor& rw, at::Tensor& counts, std::vector<int64_t> cfg,
                const c10::optional<at::Tensor>& flag, int64_t flag_index, const c10::optional<at::Tensor>& epoch,
                int64_t arrivals, int64_t timeout_ns, const c10::optional<at::Tensor>& tok_scale,
                const c10::optional<at::Tensor>& home_x) {
  check_cuda(tok, "tok");
  TORCH_CHECK(cfg.size() == 9 || cfg.size() == 12, "afd_expand: cfg has 9 or 12 entries");
  ExpandParams p{};
  p.tok = tok.data_ptr();
  p.rid = rid.data_ptr<int32_t>();
  p.rwt = rwt.data_ptr<float>();
  p.tcount = tcount.data_ptr<int32_t>();
  p.x = x.data_ptr();
  p.meta = meta.data_ptr<int32_t>();
  p.rw = rw.data_ptr<float>();
  p.counts = counts.data_ptr<int32_t>();
  p.A = (int)cfg[0];
  p.t_cap = (int)cfg[1];
  p.k = (int)cfg[2];
  p.H = (int)tok.size(-1);
  p.e_local = (int)cfg[3];
  p.e_offset = (int)cfg[4];
  p.cap = (int)cfg[5];
  p.ratio = (int)cfg[6];
  p.home_a0 = (int)cfg[7];
  p.moe = (int)cfg[8];
  if (cfg.size() == 12) {
    p.n_chunks = (int)cfg[9];
    p.shared_base = (int)cfg[10];
    p.shared_stride = (int)cfg[11];
  }
  TORCH_CHECK(p.A <= 64 && p.k <= 16 && p.k + p.n_chunks <= 32 && p.H % 8 == 0,
              "afd_expand: at most 64 sources, k <= 16, k + shared chunks <= 32");
  // a row's meta word packs source (8 bits), token (16 bits) and slot (8 bits)
  TORCH_CHECK(p.t_cap >= 1 && p.t_cap <= 65535, "afd_expand: t_cap must be in [1, 65535] (16-bit token index)");
  if (flag.has_value() && flag->defined()) {
    TORCH_CHECK(epoch.has_value() && epoch->defined(), "afd_expand: a wait needs the epoch tensor");
    p.flag = reinterpret_cast<const uint64_t*>(flag->data_ptr()) + flag_index;
    p.epoch = reinterpret_cast<const uint64_t*>(epoch->data_ptr());
    p.arrivals = (uint64_t)arrivals;
    p.timeout_ns = timeout_ns;
  }
  if (tok_scale.has_value() && tok_scale->defined()) {
    TORCH_CHECK(tok.scalar_type() == at::kByte && tok_scale->scalar_type() == at::kFloat && p.H % 128 == 0,
                "afd_expand: e4m3 rows are uint8 [A, t_cap, H] with fp32 scales [A, t_cap, H / 128]");
    p.tok_scale = tok_scale->data_ptr<float>();
    if (home_x.has_value() && home_x->defined()) {
      TORCH_CHECK(home_x->scalar_type() == at::kBFloat16 && home_x->numel() >= (int64_t)p.ratio * p.t_cap * p.H,
                  "afd_expand: home_x [ratio * t_cap, H] bf16");
      p.home_x = home_x->data_ptr();
    }
  }
  p.status = status_ptr(tok);
  c10::cuda::CUDAGuard g(tok.device());
  launch_afd_expand(p, stream());
}

// cfg: [A, t_cap, k, J, e_local, e_offset, ratio, home_a0, moe, has_shared, f_rank, num_ffn, layer, echo
//       (, home_slots = J - k)]
void afd_combine_send(const at::Tensor& staging, const at::Tensor& rid, const at::Tensor& rwt,
                      const at::Tensor& tcount, const at::Tensor& dst_ptrs, const at::Tensor& flag_ptrs,
                      at::Tensor& done_ctr, int64_t H, std::vector<int64_t> cfg,
                      const c10::optional<at::Tensor>& tok_scale) {
  check_cuda(staging, "staging");
  TORCH_CHECK(cfg.size() == 14 || cfg.size() == 15, "afd_combine_send: cfg has 14 or 15 entries");
  CombineSendParams p{};
  p.staging = staging.data_ptr();
  p.rid = rid.data_ptr<int32_t>();
  p.rwt = rwt.data_ptr<float>();
  p.tcount = tcount.data_ptr<int32_t>();
  p.A = (int)cfg[0];
  p.t_cap = (int)cfg[1];
  p.k = (int)cfg[2];
  p.J = (int)cfg[3];
  p.H = (int)H;
  p.e_local = (int)cfg[4];
  p.e_offset = (int)cfg[5];
  p.ratio = (int)cfg[6];
  p.home_a0 = (int)cfg[7];
  p.moe = (int)cfg[8];
  p.has_shared = (int)cfg[9];
  p.f_rank = (int)cfg[10];
  p.num_ffn = (int)cfg[11];
  p.layer = (int)cfg[12];
  p.echo = (int)cfg[13];
  p.home_slots = cfg.size() == 15 ? (int)cfg[14] : p.J - p.k;
  if (tok_scale.has_value() && tok_scale->defined()) {
    TORCH_CHECK(p.echo && staging.scalar_type() == at::kByte && H % 128 == 0,
                "afd_combine_send: e4m3 staging rows are an echo-mode stand-in only");
    p.tok_scale = tok_scale->data_ptr<float>();
  }
  TORCH_CHECK(p.home_slots >= 0 && p.k + p.home_slots <= p.J, "afd_combine_send: home slots exceed J");
  TORCH_CHECK(p.A <= 64 && p.k <= 16 && p.J <= 32 && p.J >= p.k, "afd_combine_send: at most 64 sources, k <= J <= 32");
  TORCH_CHECK(p.t_cap >= 1 && p.t_cap <= 65535, "afd_combine_send: t_cap must be in [1, 65535] (16-bit token index)");
  p.dst_ptrs = dst_ptrs.data_ptr<int64_t>();
  p.flag_ptrs = flag_ptrs.data_ptr<int64_t>();
  p.done_ctr = reinterpret_cast<unsigned*>(done_ctr.data_ptr());
  c10::cuda::CUDAGuard g(staging.device());
  launch_afd_combine_send(p, stream());
}

at::Tensor afd_combine(const at::Tensor& comb, const at::Tensor& fmask, int64_t T, const at::Tensor& flags,
                       int64_t layer, const at::Tensor& epoch, int64_t arrivals, int64_t timeout_ns) {
  check_cuda(comb, "comb");
  TORCH_CHECK(comb.dim() == 3 && comb.is_contiguous() && comb.scalar_type() == at::kBFloat16, "afd_combine: comb");
  auto out = at::empty({T, comb.size(2)}, comb.options());
  CombineParams p{};
  p.out = out.data_ptr();
  p.comb = comb.data_ptr();
  p.fmask = fmask.data_ptr<int32_t>();
  p.T = (int)T;
  p.H = (int)comb.size(2);
  p.F = (int)comb.size(1);
  p.flag = reinterpret_cast<const uint64_t*>(flags.data_ptr());
  p.layer = (int)layer;
  p.epoch = reinterpret_cast<const uint64_t*>(epoch.data_ptr());
  p.arrivals = (uint64_t)arrivals;
  p.timeout_ns = timeout_ns;
  p.status = status_ptr(comb);
  c10::cuda::CUDAGuard g(comb.device());
  launch_afd_combine(p, stream());
  return out;
}

// Grouped GEMM whose epilogue scatters rows into peer combine buffers.
// sp_ptrs (int64 [4]): meta, rw, dst_ptr_table, flag_ptr_table; sp_cfg: [J, H, total_ctas, num_dst, layer, n_reset]
void check_w8(const at::Tensor& w, const at::Tensor& scale, int64_t N, int64_t K, const char* who);

void grouped_gemm_scatter(const at::Tensor& a, const at::Tensor& w, const at::Tensor& offsets, const at::Tensor& counts,
                          int64_t w_experts, const at::Tensor& meta, const at::Tensor& rw, const at::Tensor& dst_ptrs,
                          const at::Tensor& flag_ptrs, at::Tensor& done_ctr, at::Tensor& counts_reset,
                          std::vector<int64_t> cfg, const c10::optional<at::Tensor>& w_scale) {
  check_cuda(a, "a");
  TORCH_CHECK(cfg.size() == 5, "grouped_gemm_scatter: cfg [J, H, total_ctas, num_dst, layer]");
  const int64_t R = a.size(0), K = a.size(1), N = w.size(1);
  TORCH_CHECK(N % 128 == 0 && K % 64 == 0 && w.size(2) == K, "grouped_gemm_scatter: shapes");
  const bool w8 = w_scale.has_value() && w_scale->defined();
  if (w8) check_w8(w, *w_scale, N, K, "grouped_gemm_scatter");
  ScatterParams sp{};
  sp.meta = meta.data_ptr<int32_t>();
  sp.rw = rw.data_ptr<float>();
  sp.dst_ptrs = dst_ptrs.data_ptr<int64_t>();
  sp.J = (int)cfg[0];
  sp.H = (int)cfg[1];
  sp.total_ctas = (int)cfg[2];
  sp.num_dst = (int)cfg[3];
  sp.layer = (int)cfg[4];
  sp.flag_ptrs = flag_ptrs.data_ptr<int64_t>();
  sp.done_ctr = reinterpret_cast<unsigned*>(done_ctr.data_ptr());
  sp.counts_reset = counts_reset.data_ptr<int32_t>();
  sp.n_reset = (int)counts_reset.numel();
  c10::cuda::CUDAGuard g(a.device());
  if (w8) {
    launch_grouped_gemm_w8(nullptr, a.data_ptr(), w.data_ptr(), w_scale->data_ptr<float>(), offsets.data_ptr<int32_t>(),
                           counts.data_ptr<int32_t>(), (int)counts.numel(), (int)R, (int)N, (int)K, 2, status_ptr(a),
                           stream(), (int)w_experts, &sp);
    return;
  }
  launch_grouped_gemm(nullptr, a.data_ptr(), w.data_ptr(), offsets.data_ptr<int32_t>(), counts.data_ptr<int32_t>(),
                      (int)counts.numel(), (int)R, (int)N, (int)K, 2, status_ptr(a), stream(), (int)w_experts, &sp);
}

// fp8 weights w [E, N, K] (float8_e4m3fn), block scales [E, ceil(N / 128), K / 128] fp32.
void check_w8(const at::Tensor& w, const at::Tensor& scale, int64_t N, int64_t K, const char* who) {
  TORCH_CHECK(w.scalar_type() == at::kFloat8_e4m3fn && w.is_contiguous(), who, ": fp8 e4m3 weights, contiguous");
  TORCH_CHECK(K % 128 == 0, who, ": K must be a multiple of 128 for fp8 weights");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.is_contiguous() && scale.dim() == 3 &&
                  scale.size(0) == w.size(0) && scale.size(1) == (N + 127) / 128 && scale.size(2) == K / 128,
              who, ": block scales [E, ceil(N/128), K/128] fp32");
}

// D = A x W^T per expert segment with fp8 block-scaled weights; epilogue 0 plain, 1 SwiGLU.
at::Tensor grouped_gemm_w8(const at::Tensor& a, const at::Tensor& w, const at::Tensor& w_scale,
                           const at::Tensor& offsets, const at::Tensor& counts, int64_t epilogue, int64_t w_experts) {
  check_cuda(a, "a");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && a.is_contiguous(), "grouped_gemm_w8: bf16 activations, contiguous");
  const int64_t R = a.size(0), K = a.size(1), N = w.size(-2);
  TORCH_CHECK(w.dim() == 3 && w.size(-1) == K, "grouped_gemm_w8: w [E, N, K]");
  check_w8(w, w_scale, N, K, "grouped_gemm_w8");
  if (epilogue == 1) {
    TORCH_CHECK(N % 2 == 0 && (N / 2) % 128 == 0, "grouped_gemm_w8: SwiGLU needs I % 128 == 0 (scale blocks)");
  } else {
    TORCH_CHECK(N % 128 == 0, "grouped_gemm_w8: N must be a multiple of 128");
  }
  const int64_t n_out = epilogue == 1 ? N / 2 : N;
  auto d = at::empty({R, n_out}, a.options());
  c10::cuda::CUDAGuard g(a.device());
  launch_grouped_gemm_w8(d.data_ptr(), a.data_ptr(), w.data_ptr(), w_scale.data_ptr<float>(), offsets.data_ptr<int32_t>(),
                         counts.data_ptr<int32_t>(), (int)counts.numel(), (int)R, (int)N, (int)K, (int)epilogue,
                         status_ptr(a), stream(), (int)w_experts, nullptr);
  return d;
}

// Tensor-parallel all-reduce of x [rows, H] bf16 in place over the symmetric
// heap (see tp_allreduce.cu); `max_ctas` is the flag table's CTA capacity.
void tp_allreduce_(at::Tensor& x, const at::Tensor& slot_ptrs, const at::Tensor& flag_ptrs,
                   const at::Tensor& local_slots, const at::Tensor& local_flags, at::Tensor& epoch, at::Tensor& done,
                   int64_t rank, int64_t world, int64_t slot_elems, int64_t max_ctas, int64_t timeout_ns) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "tp_allreduce: x [rows, H] bf16");
  TORCH_CHECK(x.size(1) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "tp_allreduce: 16-byte rows");
  TORCH_CHECK(x.numel() <= slot_elems, "tp_allreduce: ", x.numel(), " elements exceed the slot size ", slot_elems);
  TORCH_CHECK(slot_ptrs.numel() == world && flag_ptrs.numel() == world && world >= 1 && world <= 16 && rank < world,
              "tp_allreduce: pointer tables");
  TORCH_CHECK(epoch.scalar_type() == at::kLong && done.scalar_type() == at::kInt, "tp_allreduce: epoch int64, done int32");
  TPAllReduceParams p{};
  p.x = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  p.rows = (int)x.size(0);
  p.H = (int)x.size(1);
  p.rows_per_cta = tp_allreduce_rows_per_cta(p.rows, (int)max_ctas);
  p.world = (int)world;
  p.rank = (int)rank;
  p.slot_elems = slot_elems;
  p.slot_ptrs = slot_ptrs.data_ptr<int64_t>();
  p.flag_ptrs = flag_ptrs.data_ptr<int64_t>();
  p.local_slots = reinterpret_cast<const __nv_bfloat16*>(local_slots.data_ptr());
  p.local_flags = reinterpret_cast<const uint64_t*>(local_flags.data_ptr());
  p.epoch = reinterpret_cast<uint64_t*>(epoch.data_ptr());
  p.done_ctr = reinterpret_cast<unsigned*>(done.data_ptr());
  p.status = status_ptr(x);
  p.timeout_ns = timeout_ns;
  c10::cuda::CUDAGuard g(x.device());
  const cudaError_t e = launch_tp_allreduce(p, stream());
  TORCH_CHECK(e == cudaSuccess, "tp_allreduce: launch failed: ", cudaGetErrorString(e));
}

at::Tensor grouped_gemm_ex(const at::Tensor& a, const at::Tensor& w, const at::Tensor& offsets,
                           const at::Tensor& counts, int64_t epilogue, int64_t w_experts) {
  check_cuda(a, "a");
  const int64_t R = a.size(0), K = a.size(1), N = w.size(-2);
  const int64_t n_out = epilogue == 1 ? N / 2 : N;
  TORCH_CHECK(K % 64 == 0 && w.size(-1) == K, "grouped_gemm_ex: K");
  auto d = at::empty({R, n_out}, a.options());
  c10::cuda::CUDAGuard g(a.device());
  launch_grouped_gemm(d.data_ptr(), a.data_ptr(), w.data_ptr(), offsets.data_ptr<int32_t>(),
                      counts.data_ptr<int32_t>(), (int)counts.numel(), (int)R, (int)N, (int)K, (int)epilogue,
                      status_ptr(a), stream(), (int)w_experts, nullptr);
  return d;
}

// ------------------------------------------------------------------ gated delta net
// x [T, >= C] (last dim contiguous, rows may be strided); weight [C, K]; state [slots, C, K - 1].
at::Tensor gdn_conv(const at::Tensor& x, const at::Tensor& weight, at::Tensor& state, const at::Tensor& cu_seqlens,
                    const at::Tensor& slots, const c10::optional<at::Tensor>& reset) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && weight.scalar_type() == at::kBFloat16 &&
                  state.scalar_type() == at::kBFloat16, "gdn_conv: bf16 tensors");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && weight.is_contiguous() && state.is_contiguous(), "gdn_conv: layout");
  const int C = (int)weight.size(0), K = (int)weight.size(1);
  TORCH_CHECK(K >= 2 && K <= 8 && x.size(1) >= C && state.size(1) == C && state.size(2) == K - 1,
              "gdn_conv: 2 <= K <= 8, state [slots, C, K - 1]");
  TORCH_CHECK(cu_seqlens.scalar_type() == at::kInt && slots.scalar_type() == at::kInt, "gdn_conv: int32 metadata");
  auto y = at::empty({x.size(0), C}, x.options());
  GdnConvParams p{};
  p.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  p.ldx = x.stride(0);
  p.weight = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  p.state = reinterpret_cast<__nv_bfloat16*>(state.data_ptr());
  p.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  p.cu_seqlens = cu_seqlens.data_ptr<int32_t>();
  p.slots = slots.data_ptr<int32_t>();
  p.reset = (reset.has_value() && reset->defined()) ? reset->data_ptr<int32_t>() : nullptr;
  p.num_seqs = (int)slots.size(0);
  p.C = C;
  p.K = K;
  if (p.num_seqs == 0 || x.size(0) == 0) return y;
  c10::cuda::CUDAGuard g(x.device());
  launch_gdn_conv(p, stream());
  return y;
}

// qkv [T, 2 nk dk + nv dv] (q | k | v); z [T, nv dv]; a, b [T, nv]; state [slots, nv, dk, dv] fp32.
at::Tensor gdn_recurrent(const at::Tensor& qkv, const at::Tensor& z, const at::Tensor& a, const at::Tensor& b,
                         const at::Tensor& A_log, const at::Tensor& dt_bias, const at::Tensor& norm_w, double eps,
                         at::Tensor& state, const at::Tensor& cu_seqlens, const at::Tensor& slots,
                         const c10::optional<at::Tensor>& reset, int64_t nk) {
  check_cuda(qkv, "qkv");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && z.scalar_type() == at::kBFloat16 &&
                  a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gdn_recurrent: bf16 inputs");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.dim() == 4,
              "gdn_recurrent: fp32 state [slots, nv, dk, dv]");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat, "gdn_recurrent: fp32 A_log / dt_bias");
  TORCH_CHECK(qkv.stride(1) == 1 && z.stride(1) == 1 && a.stride(1) == 1 && b.stride(1) == 1 && a.stride(0) == b.stride(0),
              "gdn_recurrent: last dims contiguous, a / b with one row stride");
  const int nv = (int)state.size(1), dk = (int)state.size(2), dv = (int)state.size(3);
  TORCH_CHECK(nk > 0 && nv % nk == 0 && dv >= dk && dv % 32 == 0 && dv <= 256 && norm_w.numel() == dv,
              "gdn_recurrent: nv % nk == 0, dk <= dv <= 256, dv % 32 == 0");
  TORCH_CHECK(qkv.size(1) >= 2 * nk * dk + nv * dv && z.size(1) >= nv * dv && a.size(1) >= nv, "gdn_recurrent: widths");
  auto out = at::empty({qkv.size(0), (int64_t)nv * dv}, qkv.options());
  GdnRecurrentParams p{};
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  p.ld_qkv = qkv.stride(0);
  p.z = reinterpret_cast<const __nv_bfloat16*>(z.data_ptr());
  p.ld_z = z.stride(0);
  p.a = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
  p.b = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
  p.ld_ab = a.stride(0);
  p.A_log = A_log.data_ptr<float>();
  p.dt_bias = dt_bias.data_ptr<float>();
  p.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr());
  p.eps = (float)eps;
  p.state = state.data_ptr<float>();
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.cu_seqlens = cu_seqlens.data_ptr<int32_t>();
  p.slots = slots.data_ptr<int32_t>();
  p.reset = (reset.has_value() && reset->defined()) ? reset->data_ptr<int32_t>() : nullptr;
  p.num_seqs = (int)slots.size(0);
  p.nk = (int)nk;
  p.nv = nv;
  p.dk = dk;
  p.dv = dv;
  if (p.num_seqs == 0 || qkv.size(0) == 0) return out;
  c10::cuda::CUDAGuard g(qkv.device());
  TORCH_CHECK(launch_gdn_recurrent(p, stream()), "gdn_recurrent: key head dim must be 32, 64 or 128");
  return out;
}

// ------------------------------------------------------------------ status
int64_t gg_grid(int64_t n_items) { return grouped_gemm_grid((int)n_items); }

int64_t read_status(int64_t device) { return status_tensor((int)device).item<int>(); }
void reset_status(int64_t device) { status_tensor((int)device).zero_(); }
at::Tensor status_word(int64_t device) { return status_tensor((int)device); }

}  // namespace

TORCH_LIBRARY(afd_b200, m) {
  m.def("rms_norm(Tensor x, Tensor w, float eps) -> Tensor");
  m.def("fused_add_rms_norm(Tensor x, Tensor(a!) residual, Tensor w, float eps) -> Tensor");
  m.def("silu_and_mul(Tensor x) -> Tensor");
  m.def("argmax_rows(Tensor x) -> Tensor");
  m.def("rope_(Tensor(a!) x, Tensor positions, Tensor cos_sin, bool interleaved) -> ()");
  m.def("topk_route(Tensor logits, int k, int scoring, bool renorm, Tensor? bias, int n_group, int topk_group, "
        "float scale, Tensor? forced=None) -> (Tensor, Tensor)");
  m.def("mla_cache_write(Tensor(a!) cache, Tensor kv_a, Tensor w, float eps, Tensor positions, Tensor cos_sin, "
        "Tensor slots, int L, Tensor(b!)? q_pe=None) -> ()");
  m.def("gqa_cache_write(Tensor(a!) kc, Tensor(b!) vc, Tensor k, Tensor v, Tensor slots) -> ()");
  m.def("gqa_prologue(Tensor qkv, int nq, int nkv, int d, Tensor? qw, Tensor? kw, float eps, Tensor positions, "
        "Tensor cos_sin, Tensor(a!) kc, Tensor(b!) vc, Tensor slots) -> Tensor");
  m.def("mla_decode(Tensor q_lat, Tensor q_pe, Tensor cache, Tensor block_table, Tensor seq_lens, float scale, "
        "int num_splits, bool head_major) -> Tensor");
  m.def("mla_decode_sparse(Tensor q, Tensor cache, Tensor block_table, Tensor seq_lens, Tensor keep_pos, float scale, "
        "int num_splits) -> Tensor");
  m.def("gqa_decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_table, Tensor seq_lens, float scale, "
        "int num_splits) -> Tensor");
  m.def("moe_align(Tensor topk_ids, int e_local, int offset, int n_shared) -> Tensor[]");
  m.def("moe_gather(Tensor x, Tensor row_token, Tensor total) -> Tensor");
  m.def("grouped_gemm(Tensor a, Tensor w, Tensor offsets, Tensor counts, int epilogue) -> Tensor");
  m.def("moe_combine(Tensor ys, Tensor topk_w, Tensor token_slot_row, Tensor? shared) -> Tensor");
  m.def("decode_advance(Tensor(a!) input_ids, Tensor(b!) positions, Tensor(c!) slots, Tensor(d!) seq_lens, "
        "Tensor next_tokens, Tensor block_table, int block_size, int wrap_at, int wrap_to) -> ()");
  m.def("gdn_conv(Tensor x, Tensor weight, Tensor(a!) state, Tensor cu_seqlens, Tensor slots, Tensor? reset) -> Tensor");
  m.def("gdn_recurrent(Tensor qkv, Tensor z, Tensor a, Tensor b, Tensor A_log, Tensor dt_bias, Tensor norm_w, "
        "float eps, Tensor(a!) state, Tensor cu_seqlens, Tensor slots, Tensor? reset, int nk) -> Tensor");
  m.def("afd_epoch(Tensor(a!) epoch) -> ()");
  m.def("afd_stamp(Tensor(a!) buf, int idx) -> ()");
  m.def("afd_wait(Tensor flag, int index, Tensor epoch, int arrivals, int timeout_ns) -> ()");
  m.def("afd_dispatch(Tensor attn_out, Tensor(a!) residual, Tensor norm_w, float eps, Tensor gate_w, Tensor? gate_bias, "
        "float scale, Tensor ptrs, Tensor(b!) fmask, Tensor(c!) done_ctr, int[] cfg, Tensor? hash_table=None, "
        "Tensor? input_ids=None) -> ()");
  m.def("afd_expand(Tensor tok, Tensor rid, Tensor rwt, Tensor tcount, Tensor(a!) x, Tensor(b!) meta, Tensor(c!) rw, "
        "Tensor(d!) counts, int[] cfg, Tensor? flag=None, int flag_index=0, Tensor? epoch=None, int arrivals=0, "
        "int timeout_ns=0, Tensor? tok_scale=None, Tensor? home_x=None) -> ()");
  m.def("afd_combine_send(Tensor staging, Tensor rid, Tensor rwt, Tensor tcount, Tensor dst_ptrs, Tensor flag_ptrs, "
        "Tensor(a!) done_ctr, int H, int[] cfg, Tensor? tok_scale=None) -> ()");
  m.def("afd_combine(Tensor comb, Tensor fmask, int T, Tensor flags, int layer, Tensor epoch, int arrivals, "
        "int timeout_ns) -> Tensor");
  m.def("grouped_gemm_scatter(Tensor a, Tensor w, Tensor offsets, Tensor counts, int w_experts, Tensor meta, Tensor rw, "
        "Tensor dst_ptrs, Tensor flag_ptrs, Tensor(a!) done_ctr, Tensor(b!) counts_reset, int[] cfg, "
        "Tensor? w_scale=None) -> ()");
  m.def("grouped_gemm_w8(Tensor a, Tensor w, Tensor w_scale, Tensor offsets, Tensor counts, int epilogue, "
        "int w_experts) -> Tensor");
  m.def("grouped_gemm_ex(Tensor a, Tensor w, Tensor offsets, Tensor counts, int epilogue, int w_experts) -> Tensor");
  m.def("gate_sigmoid_rows(Tensor x, Tensor w, Tensor(a!) out, int copies, int span) -> ()");
  m.def("tp_allreduce_(Tensor(a!) x, Tensor slot_ptrs, Tensor flag_ptrs, Tensor local_slots, Tensor local_flags, "
        "Tensor(b!) epoch, Tensor(c!) done, int rank, int world, int slot_elems, int max_ctas, int timeout_ns) -> ()");
  m.def("grouped_gemm_grid(int n_items) -> int");
  m.def("moe_ffn(Tensor a, Tensor w13, Tensor w2, Tensor offsets, Tensor counts, Tensor(a!) sync, int rows_hint, "
        "int w_experts=-1, Tensor? meta=None, Tensor? rw=None, Tensor? dst_ptrs=None, Tensor? flag_ptrs=None, "
        "Tensor(b!)? done_ctr=None, Tensor(c!)? counts_reset=None, int[]? cfg=None) -> Tensor");
  m.def("moe_ffn_grid(int e_local, int n1, int n2) -> int");
  m.def("tc_gemm(Tensor a, Tensor w, int epilogue=0, int n_valid=0, bool out_f32=False, Tensor(a!)? ws=None, "
        "Tensor(b!)? ctr=None) -> Tensor");
  m.def("dense_ffn(Tensor x, Tensor w13, Tensor w2, Tensor(a!) sync) -> Tensor");
  m.def("read_status(int device) -> int");
  m.def("reset_status(int device) -> ()");
  m.def("status_word(int device) -> Tensor");
}

TORCH_LIBRARY_IMPL(afd_b200, CUDA, m) {
  m.impl("rms_norm", &rms_norm);
  m.impl("fused_add_rms_norm", &fused_add_rms_norm);
  m.impl("silu_and_mul", &silu_and_mul);
  m.impl("argmax_rows", &argmax_rows);
  m.impl("gate_sigmoid_rows", &gate_sigmoid_rows);
  m.impl("tp_allreduce_", &tp_allreduce_);
  m.impl("gqa_prologue", &gqa_prologue);
  m.impl("rope_", &rope_);
  m.impl("topk_route", &topk_route);
  m.impl("mla_cache_write", &mla_cache_write);
  m.impl("gqa_cache_write", &gqa_cache_write);
  m.impl("mla_decode", &mla_decode);
  m.impl("mla_decode_sparse", &mla_decode_sparse);
  m.impl("gqa_decode", &gqa_decode);
  m.impl("moe_align", &moe_align);
  m.impl("moe_gather", &moe_gather);
  m.impl("grouped_gemm", &grouped_gemm);
  m.impl("moe_combine", &moe_combine);
  m.impl("decode_advance", &decode_advance);
  m.impl("afd_epoch", &afd_epoch);
  m.impl("afd_stamp", &afd_stamp);
  m.impl("gdn_conv", &gdn_conv);
  m.impl("gdn_recurrent", &gdn_recurrent);
  m.impl("afd_wait", &afd_wait);
  m.impl("afd_dispatch", &afd_dispatch);
  m.impl("afd_combine", &afd_combine);
  m.impl("grouped_gemm_scatter", &grouped_gemm_scatter);
  m.impl("grouped_gemm_ex", &grouped_gemm_ex);
  m.impl("moe_ffn", &moe_ffn);
  m.impl("tc_gemm", &tc_gemm);
  m.impl("dense_ffn", &dense_ffn);
  m.impl("grouped_gemm_w8", &grouped_gemm_w8);
  m.impl("afd_expand", &afd_expand);
  m.impl("afd_combine_send", &afd_combine_send);
}

TORCH_LIBRARY_IMPL(afd_b200, CompositeExplicitAutograd, m) {
  m.impl("read_status", &read_status);
  m.impl("reset_status", &reset_status);
  m.impl("status_word", &status_word);
  m.impl("grouped_gemm_grid", &gg_grid);
  m.impl("moe_ffn_grid", &moe_ffn_grid);
}
