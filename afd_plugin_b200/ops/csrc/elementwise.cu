// Memory-bound kernels: RMSNorm (+fused residual add), SiLU-and-mul, RoPE,
// routing top-k, KV-cache writes (the MLA one with the query's RoPE, the GQA
// attention prologue with QK-norm and RoPE).  Every kernel computes in fp32.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "device_state.h"
#include "launchers.h"
#include "routing.cuh"

namespace afd {

// ============================================================ RMSNorm
// One group of TPR threads per row; each thread owns H/(8*TPR) 16-byte vectors.
template <typename T, int TPR, bool kAddResidual>
__global__ void rms_norm_kernel(T* __restrict__ out, const T* __restrict__ x, T* __restrict__ residual,
                                const T* __restrict__ w, int rows, int hidden, float eps) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  constexpr int VN = Vec16<T>::N;
  constexpr int kRowsPerBlock = (TPR >= 256) ? 1 : 256 / TPR;
  const int sub = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  const int row = blockIdx.x * kRowsPerBlock + sub;
  __shared__ float red[kRowsPerBlock][(TPR + 31) / 32];
  const bool active = row < rows;
  const int nvec = hidden / VN;
  float ss = 0.f;
  // Cache up to 4 vectors per thread in registers (H <= 4*8*TPR), else re-read.
  constexpr int kCache = 4;
  Vec16<T> cache[kCache];
  if (active) {
    const T* xr = x + (size_t)row * hidden;
    T* rr = kAddResidual ? residual + (size_t)row * hidden : nullptr;
    int c = 0;
    for (int v = lane; v < nvec; v += TPR, ++c) {
      Vec16<T> a = load16(xr + v * VN);
      if constexpr (kAddResidual) {
        Vec16<T> r = load16(rr + v * VN);
#pragma unroll
        for (int i = 0; i < VN; ++i) a.v[i] = from_f32<T>(to_f32(a.v[i]) + to_f32(r.v[i]));
        store16(rr + v * VN, a);
      }
#pragma unroll
      for (int i = 0; i < VN; ++i) {
        float f = to_f32(a.v[i]);
        ss += f * f;
      }
      if (c < kCache) cache[c] = a;
    }
  }
  if constexpr (TPR <= 32) {
    ss = warp_sum(ss, TPR);
  } else {
    ss = warp_sum(ss, 32);
    if ((threadIdx.x & 31) == 0) red[sub][lane / 32] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int i = 0; i < TPR / 32; ++i) ss += red[sub][i];
  }
  if (!active) return;
  const float inv = rsqrtf(ss / (float)hidden + eps);
  const T* src = kAddResidual ? residual + (size_t)row * hidden : x + (size_t)row * hidden;
  T* orow = out + (size_t)row * hidden;
  int c = 0;
  for (int v = lane; v < nvec; v += TPR, ++c) {
    Vec16<T> a = (c < kCache) ? cache[c] : load16(src + v * VN);
    Vec16<T> ww = load16(w + v * VN);
    Vec16<T> o;
#pragma unroll
    for (int i = 0; i < VN; ++i) o.v[i] = from_f32<T>(to_f32(a.v[i]) * inv * to_f32(ww.v[i]));
    store16(orow + v * VN, o);
  }
}

template <typename T, bool kAdd>
static void rms_norm_dispatch(void* out, const void* x, void* res, const void* w, int rows, int hidden, float eps,
                              cudaStream_t s) {
  constexpr int VN = Vec16<T>::N;
  const int nvec = hidden / VN;
  auto go = [&](auto tpr_tag) {
    constexpr int TPR = decltype(tpr_tag)::value;
    constexpr int RPB = (TPR >= 256) ? 1 : 256 / TPR;
    dim3 grid((rows + RPB - 1) / RPB);
    launch_pdl(rms_norm_kernel<T, TPR, kAdd>, dim3(grid), dim3(RPB * TPR), 0, s, (T*)out, (const T*)x, (T*)res, (const T*)w,
               rows, hidden, eps);
  };
  if (nvec <= 8) go(std::integral_constant<int, 8>{});
  else if (nvec <= 16) go(std::integral_constant<int, 16>{});
  else if (nvec <= 32) go(std::integral_constant<int, 32>{});
  else if (nvec <= 64) go(std::integral_constant<int, 64>{});
  else if (nvec <= 128) go(std::integral_constant<int, 128>{});
  else go(std::integral_constant<int, 256>{});
}

// ============================================================ SiLU * up
template <typename T>
__global__ void silu_and_mul_kernel(T* __restrict__ out, const T* __restrict__ in, int rows, int d) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  constexpr int VN = Vec16<T>::N;
  const int nvec = d / VN;
  const size_t total = (size_t)rows * nvec;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / nvec;
    const int v = (int)(i % nvec);
    const T* row = in + r * 2 * d;
    Vec16<T> g = load16(row + v * VN);
    Vec16<T> u = load16(row + d + v * VN);
    Vec16<T> o;
#pragma unroll
    for (int k = 0; k < VN; ++k) {
      float gf = to_f32(g.v[k]);
      o.v[k] = from_f32<T>(gf / (1.f + __expf(-gf)) * to_f32(u.v[k]));
    }
    store16(out + r * d + v * VN, o);
  }
}

// ============================================================ RoPE (in place)
// x: [T, H, rot] with strides (st, sh, 1); cos_sin: [P, rot] fp32 = [cos | sin].
template <typename T>
__global__ void rope_kernel(T* __restrict__ x, const int64_t* __restrict__ pos, const float* __restrict__ cos_sin,
                            int tokens, int heads, int rot, int64_t st, int64_t sh, bool interleaved) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  const int half = rot / 2;
  const size_t total = (size_t)tokens * heads * half;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int p = (int)(i % half);
    const size_t th = i / half;
    const int h = (int)(th % heads);
    const int t = (int)(th / heads);
    const float* cs = cos_sin + pos[t] * rot;
    const float c = cs[p], s = cs[half + p];
    T* base = x + t * st + h * sh;
    const int i0 = interleaved ? 2 * p : p;
    const int i1 = interleaved ? 2 * p + 1 : p + half;
    const float a = to_f32(base[i0]), b = to_f32(base[i1]);
    base[i0] = from_f32<T>(a * c - b * s);
    base[i1] = from_f32<T>(b * c + a * s);
  }
}

// ============================================================ routing top-k
// One warp per token (see routing.cuh for the selection rules).
__global__ void topk_route_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                  float* __restrict__ out_w, int32_t* __restrict__ out_id, int tokens, int E, int k,
                                  int scoring, bool renorm, int n_group, int topk_group, float scale,
                                  const int32_t* __restrict__ forced) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (warp >= tokens) return;
  float w;
  int id;
  warp_route(logits + (size_t)warp * E, bias, E, k, scoring, renorm, n_group, topk_group, scale, w, id,
             forced ? forced + (size_t)warp * k : nullptr);
  if (lane < k) {
    out_w[(size_t)warp * k + lane] = w;
    out_id[(size_t)warp * k + lane] = id;
  }
}

// ============================================================ MLA cache write
// kv_a [T, L + R]: latent (RMSNorm) || k_pe (interleaved RoPE) -> cache[slot].
// With q_pe, the token's query rope part is rotated in place by the same
// launch (q_pe [T, q_heads, R] strided; same position, same interleaved
// pairing), so decode needs no separate query-rope launch.  One CTA per
// token: warp 0 writes the cache row, the other warps (kQWarps) rotate the
// query in 16-byte vectors whose loads are all in flight together.
constexpr int kQWarps = 3;

template <typename T>
__global__ void mla_cache_write_kernel(T* __restrict__ cache, const T* __restrict__ kv_a, const T* __restrict__ w,
                                       float eps, const int64_t* __restrict__ pos, const float* __restrict__ cos_sin,
                                       const int64_t* __restrict__ slots, int tokens, int L, int R,
                                       int64_t kv_stride, T* __restrict__ q_pe, int q_heads, int64_t q_st,
                                       int64_t q_sh) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  constexpr int VN = Vec16<T>::N;
  const float* cs = cos_sin + pos[t] * R;
  if (warp > 0) {
    T* qt = q_pe + (size_t)t * q_st;
    const int per_head = R / VN;
    for (int i = threadIdx.x - 32; i < q_heads * per_head; i += kQWarps * 32) {
      const int h = i / per_head, c0 = (i % per_head) * VN;
      T* x = qt + (size_t)h * q_sh + c0;
      Vec16<T> v = load16(x);
#pragma unroll
      for (int j = 0; j < VN / 2; ++j) {
        const int p = c0 / 2 + j;
        const float c = cs[p], s = cs[R / 2 + p];
        const float a = to_f32(v.v[2 * j]), b = to_f32(v.v[2 * j + 1]);
        v.v[2 * j] = from_f32<T>(a * c - b * s);
        v.v[2 * j + 1] = from_f32<T>(b * c + a * s);
      }
      store16(x, v);
    }
    return;
  }
  const T* src = kv_a + (size_t)t * kv_stride;
  T* dst = cache + slots[t] * (int64_t)(L + R);
  float ss = 0.f;
  for (int v = lane; v < L / VN; v += 32) {
    Vec16<T> a = load16(src + v * VN);
#pragma unroll
    for (int i = 0; i < VN; ++i) ss += to_f32(a.v[i]) * to_f32(a.v[i]);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)L + eps);
  for (int v = lane; v < L / VN; v += 32) {
    Vec16<T> a = load16(src + v * VN);
    Vec16<T> ww = load16(w + v * VN);
#pragma unroll
    for (int i = 0; i < VN; ++i) a.v[i] = from_f32<T>(to_f32(a.v[i]) * inv * to_f32(ww.v[i]));
    store16(dst + v * VN, a);
  }
  for (int p = lane; p < R / 2; p += 32) {
    const float c = cs[p], s = cs[R / 2 + p];
    const float a = to_f32(src[L + 2 * p]), b = to_f32(src[L + 2 * p + 1]);
    dst[L + 2 * p] = from_f32<T>(a * c - b * s);
    dst[L + 2 * p + 1] = from_f32<T>(b * c + a * s);
  }
}

// GQA cache write: k, v [T, Hkv, D] -> caches [slots, Hkv, D].
template <typename T>
__global__ void gqa_cache_write_kernel(T* __restrict__ kc, T* __restrict__ vc, const T* __restrict__ k,
                                       const T* __restrict__ v, const int64_t* __restrict__ slots, int tokens,
                                       int row_elems, int64_t k_stride, int64_t v_stride) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  constexpr int VN = Vec16<T>::N;
  const int nv = row_elems / VN;
  const size_t total = (size_t)tokens * nv;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / nv);
    const int c = (int)(i % nv);
    const int64_t s = slots[t];
    store16(kc + s * row_elems + c * VN, load16(k + t * k_stride + c * VN));
    store16(vc + s * row_elems + c * VN, load16(v + t * v_stride + c * VN));
  }
}

// GQA attention prologue, one CTA per token, one warp per head of the qkv
// projection row [q heads | k heads | v heads] x D: optional per-head RMSNorm
// of q and k (Qwen3 QK-norm; rounded to the storage type as the separate
// norm kernel does), NeoX RoPE on the whole head (pairs c, c + D/2, i.e.
// lanes l and l ^ 16 with D/32 elements per lane), q into q_out [T, nq, D],
// k and v into the paged caches at the token's slot.
template <typename T, int E>
__global__ void gqa_prologue_kernel(const T* __restrict__ qkv, int64_t qkv_stride, int nq, int nkv,
                                    const T* __restrict__ qw, const T* __restrict__ kw, float eps,
                                    const int64_t* __restrict__ pos, const float* __restrict__ cos_sin,
                                    T* __restrict__ q_out, T* __restrict__ kc, T* __restrict__ vc,
                                    const int64_t* __restrict__ slots) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  constexpr int D = 32 * E, half = D / 2;
  const int t = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x / 32;
  const T* row = qkv + (size_t)t * qkv_stride;
  const float* cs = cos_sin + pos[t] * D;
  const int64_t slot = slots[t];
  for (int h = warp; h < nq + 2 * nkv; h += nwarps) {
    const T* src = row + (size_t)h * D + lane * E;
    float x[E];
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = to_f32(src[i]);
    if (h >= nq + nkv) {  // v head: straight into the cache
      T* dst = vc + ((size_t)slot * nkv + (h - nq - nkv)) * D + lane * E;
#pragma unroll
      for (int i = 0; i < E; ++i) dst[i] = from_f32<T>(x[i]);
      continue;
    }
    const bool is_q = h < nq;
    const T* nw = is_q ? qw : kw;
    if (nw != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < E; ++i) ss += x[i] * x[i];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
      for (int i = 0; i < E; ++i) x[i] = to_f32(from_f32<T>(x[i] * inv * to_f32(nw[lane * E + i])));
    }
    T* dst = is_q ? q_out + ((size_t)t * nq + h) * D + lane * E : kc + ((size_t)slot * nkv + (h - nq)) * D + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, x[i], 16);
      const int c = lane * E + i;
      const int p = c < half ? c : c - half;
      const float cv = cs[p], sv = cs[half + p];
      dst[i] = from_f32<T>(c < half ? x[i] * cv - other * sv : x[i] * cv + other * sv);
    }
  }
}

static int grid_for(size_t work, int block) {
  size_t g = (work + block - 1) / block;
  const size_t cap = (size_t)device_sm_count() * 32;
  return (int)(g > cap ? cap : (g ? g : 1));
}

}  // namespace afd

using namespace afd;

#define AFD_DTYPE_SWITCH(dt, T, ...)                        \
  switch (dt) {                                             \
    case kF32: { using T = float; __VA_ARGS__; break; }     \
    case kBF16: { using T = __nv_bfloat16; __VA_ARGS__; break; } \
    case kF16: { using T = __half; __VA_ARGS__; break; }    \
  }

void launch_rms_norm(void* out, const void* x, const void* w, int rows, int hidden, float eps, int dtype,
                     cudaStream_t s) {
  AFD_DTYPE_SWITCH(dtype, T, (rms_norm_dispatch<T, false>(out, x, nullptr, w, rows, hidden, eps, s)));
}

void launch_fused_add_rms_norm(void* out, const void* x, void* residual, const void* w, int rows, int hidden,
                               float eps, int dtype, cudaStream_t s) {
  AFD_DTYPE_SWITCH(dtype, T, (rms_norm_dispatch<T, true>(out, x, residual, w, rows, hidden, eps, s)));
}

void launch_silu_and_mul(void* out, const void* in, int rows, int d, int dtype, cudaStream_t s) {
  AFD_DTYPE_SWITCH(dtype, T, {
    const size_t work = (size_t)rows * d / Vec16<T>::N;
    launch_pdl(silu_and_mul_kernel<T>, dim3(grid_for(work, 256)), dim3(256), 0, s, (T*)out, (const T*)in, rows, d);
  });
}

void launch_rope(void* x, const int64_t* pos, const float* cos_sin, int tokens, int heads, int rot, int64_t st,
                 int64_t sh, bool interleaved, int dtype, cudaStream_t s) {
  AFD_DTYPE_SWITCH(dtype, T, {
    const size_t work = (size_t)tokens * heads * rot / 2;
    launch_pdl(rope_kernel<T>, dim3(grid_for(work, 256)), dim3(256), 0, s, (T*)x, pos, cos_sin, tokens, heads, rot, st, sh,
               interleaved);
  });
}

void launch_topk_route(const float* logits, const float* bias, float* w, int32_t* ids, int tokens, int E, int k,
                       int scoring, bool renorm, int n_group, int topk_group, float scale, const int32_t* forced,
                       cudaStream_t s) {
  const int warps_per_block = 4;
  dim3 grid((tokens + warps_per_block - 1) / warps_per_block);
  launch_pdl(topk_route_kernel, dim3(grid), dim3(32 * warps_per_block), 0, s, logits, bias, w, ids, tokens, E, k, scoring,
             renorm, n_group, topk_group, scale, forced);
}

void launch_mla_cache_write(void* cache, const void* kv_a, const void* w, float eps, const int64_t* pos,
                            const float* cos_sin, const int64_t* slots, int tokens, int L, int R, int64_t kv_stride,
                            int dtype, cudaStream_t s, void* q_pe, int q_heads, int64_t q_st, int64_t q_sh) {
  if (tokens == 0) return;
  AFD_DTYPE_SWITCH(dtype, T, {
    const int threads = q_pe != nullptr ? 32 * (1 + kQWarps) : 32;
    launch_pdl(mla_cache_write_kernel<T>, dim3(tokens), dim3(threads), 0, s, (T*)cache, (const T*)kv_a, (const T*)w, eps, pos,
               cos_sin, slots, tokens, L, R, kv_stride, (T*)q_pe, q_heads, q_st, q_sh);
  });
}

template <typename T>
static void gqa_prologue_typed(const void* qkv, int64_t qkv_stride, int tokens, int nq, int nkv, int e,
                               const void* qw, const void* kw, float eps, const int64_t* pos, const float* cos_sin,
                               void* q_out, void* kc, void* vc, const int64_t* slots, cudaStream_t s) {
  const int threads = 32 * std::min(8, nq + 2 * nkv);
  auto go = [&](auto ec) {
    constexpr int E = decltype(ec)::value;
    launch_pdl(gqa_prologue_kernel<T, E>, dim3(tokens), dim3(threads), 0, s, (const T*)qkv, qkv_stride, nq, nkv, (const T*)qw,
               (const T*)kw, eps, pos, cos_sin, (T*)q_out, (T*)kc, (T*)vc, slots);
  };
  switch (e) {
    case 1: go(std::integral_constant<int, 1>{}); break;
    case 2: go(std::integral_constant<int, 2>{}); break;
    case 4: go(std::integral_constant<int, 4>{}); break;
    default: go(std::integral_constant<int, 8>{}); break;
  }
}

bool launch_gqa_prologue(const void* qkv, int64_t qkv_stride, int tokens, int nq, int nkv, int d, const void* qw,
                         const void* kw, float eps, const int64_t* pos, const float* cos_sin, void* q_out, void* kc,
                         void* vc, const int64_t* slots, int dtype, cudaStream_t s) {
  const int e = d / 32;
  if (d % 32 != 0 || d > 256 || (e & (e - 1))) return false;
  if (tokens <= 0) return true;
  AFD_DTYPE_SWITCH(dtype, T, {
    gqa_prologue_typed<T>(qkv, qkv_stride, tokens, nq, nkv, e, qw, kw, eps, pos, cos_sin, q_out, kc, vc, slots, s);
  });
  return true;
}

void launch_gqa_cache_write(void* kc, void* vc, const void* k, const void* v, const int64_t* slots, int tokens,
                            int row_elems, int64_t k_stride, int64_t v_stride, int dtype, cudaStream_t s) {
  AFD_DTYPE_SWITCH(dtype, T, {
    const size_t work = (size_t)tokens * row_elems / Vec16<T>::N;
    launch_pdl(gqa_cache_write_kernel<T>, dim3(grid_for(work, 256)), dim3(256), 0, s, (T*)kc, (T*)vc, (const T*)k, (const T*)v,
               slots, tokens, row_elems, k_stride, v_stride);
  });
}

// ============================================================ decode advance
// Device-resident decode loop: the sampled token becomes the next input and
// every sequence moves one position (slot from its block table).
__global__ void decode_advance_kernel(int32_t* __restrict__ input_ids, int64_t* __restrict__ positions,
                                      int64_t* __restrict__ slots, int32_t* __restrict__ seq_lens,
                                      const int32_t* __restrict__ next_tokens, const int32_t* __restrict__ table,
                                      int batch, int table_stride, int block_size, int64_t wrap_at,
                                      int64_t wrap_to) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  int64_t p = positions[b] + 1;
  // Optional wrap keeps a long benchmark loop inside the allocated context window.
  if (wrap_at > 0 && p >= wrap_at) p = wrap_to;
  input_ids[b] = next_tokens[b];
  positions[b] = p;
  seq_lens[b] = (int32_t)(p + 1);
  slots[b] = (int64_t)table[(size_t)b * table_stride + p / block_size] * block_size + p % block_size;
}

// ============================================================ row argmax
// One CTA per row, 16-byte loads; ties go to the lowest index (torch.argmax).
template <typename T, bool kVec>
__global__ void __launch_bounds__(512) argmax_rows_kernel(const T* __restrict__ x, int64_t ld, int n,
                                                         int32_t* __restrict__ out) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  __shared__ float s_v[16];
  __shared__ int s_i[16];
  const T* row = x + (size_t)blockIdx.x * ld;
  constexpr int V = 16 / sizeof(T);
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int nv = kVec ? n / V : 0;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const Vec16<T> c = load16(row + (size_t)v * V);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float f = to_f32(c.v[j]);
      if (f > best) {
        best = f;
        bi = v * V + j;
      }
    }
  }
  for (int i = nv * V + threadIdx.x; i < n; i += blockDim.x) {
    const float f = to_f32(row[i]);
    if (f > best || (f == best && i < bi)) {
      best = f;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_v[warp] = best;
    s_i[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)blockDim.x / 32; ++w)
      if (s_v[w] > best || (s_v[w] == best && s_i[w] < bi)) {
        best = s_v[w];
        bi = s_i[w];
      }
    out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

void launch_decode_advance(int32_t* input_ids, int64_t* positions, int64_t* slots, int32_t* seq_lens,
                           const int32_t* next_tokens, const int32_t* table, int batch, int table_stride,
                           int block_size, int64_t wrap_at, int64_t wrap_to, cudaStream_t s) {
  decode_advance_kernel<<<(batch + 127) / 128, 128, 0, s>>>(input_ids, positions, slots, seq_lens, next_tokens,
                                                            table, batch, table_stride, block_size, wrap_at, wrap_to);
}

template <typename T>
static void argmax_rows_go(const void* x, int64_t ld, int rows, int n, int32_t* out, cudaStream_t s) {
  const T* p = static_cast<const T*>(x);
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((ld * (int64_t)sizeof(T)) % 16 == 0);
  if (vec)
    launch_pdl(argmax_rows_kernel<T, true>, dim3(rows), dim3(512), 0, s, p, ld, n, out);
  else
    launch_pdl(argmax_rows_kernel<T, false>, dim3(rows), dim3(512), 0, s, p, ld, n, out);
}

// ============================================================ gated shared expert
// out[c * span + r] = sigmoid(x[r] . w) for every copy c < copies: one warp
// per row, 16-byte loads, fp32 dot product (Qwen3.5's shared-expert gate,
// written into the routing weights of each shared-expert chunk's rows).
__global__ void gate_sigmoid_rows_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                        int rows, int H, float* __restrict__ out, int copies, int span) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int VN = Vec16<__nv_bfloat16>::N;
  const __nv_bfloat16* xr = x + (size_t)row * H;
  float acc = 0.f;
  for (int v = lane; v < H / VN; v += 32) {
    const Vec16<__nv_bfloat16> a = load16(xr + v * VN), b = load16(w + v * VN);
#pragma unroll
    for (int i = 0; i < VN; ++i) acc += to_f32(a.v[i]) * to_f32(b.v[i]);
  }
  acc = warp_sum(acc);
  const float g = 1.f / (1.f + expf(-acc));
  for (int c = lane; c < copies; c += 32) out[(size_t)c * span + row] = g;
}

void launch_gate_sigmoid_rows(const void* x, const void* w, int rows, int H, float* out, int copies, int span,
                              cudaStream_t s) {
  if (rows <= 0) return;
  const int warps = 4;
  launch_pdl(gate_sigmoid_rows_kernel, dim3((rows + warps - 1) / warps), dim3(32 * warps), 0, s, (const __nv_bfloat16*)x,
             (const __nv_bfloat16*)w, rows, H, out, copies, span);
}

void launch_argmax_rows(const void* x, int64_t ld, int rows, int n, int dtype, int32_t* out, cudaStream_t s) {
  if (rows <= 0) return;
  if (dtype == kBF16)
    argmax_rows_go<__nv_bfloat16>(x, ld, rows, n, out, s);
  else if (dtype == kF16)
    argmax_rows_go<__half>(x, ld, rows, n, out, s);
  else
    argmax_rows_go<float>(x, ld, rows, n, out, s);
}
