// Fused Attention<->FFN transfer kernels over NVLink peer memory.
//
// Per-rank protocol: a token row crosses NVLink once per FFN rank that owns
// one of its experts (or is its home rank for the shared expert / dense MLP)
// and comes back as one pre-reduced row per such rank.
//
// afd_dispatch      (Attention side, per layer and ubatch), two kernels:
//   norm    residual += attn_out; h = RMSNorm(residual) * w (one CTA per
//           token); h goes straight to every FFN rank's token buffer (the home
//           rank only for a dense layer), so the rows travel while routing runs
//   router  logits = h . gate^T on the tensor cores, split over (token tile,
//           expert tile) CTAs; the last CTA of a token tile runs the top-k and
//           sends the token's routing (k ids + weights) to every FFN rank; the
//           last tile publishes the token count and bumps every FFN rank's
//           arrival counter (release, system scope).
// afd_expand        (FFN side) waits for every Attention rank, then copies
//   each received row into the contiguous segment of every local expert it
//   routes to (local HBM), and home rows into the shared-expert chunks'
//   segments, building the grouped GEMM's row -> (source, token, slot) map.
// afd_combine_send  (FFN side, after the expert GEMMs) sums a token's local
//   expert outputs (+ shared expert) and stores one row into the source
//   Attention rank's combine slot; the last CTA bumps every Attention rank's
//   counter.
// afd_combine       (Attention side) waits for every FFN rank and sums the
//   token's FFN slots.
// afd_wait / afd_epoch: bounded arrival wait and per-stage epoch bump.
//
// Counters only grow: the n-th use of a stage expects epoch[stage] * arrivals,
// so captured graphs replay without resets.  No wait is unbounded: on expiry
// a kernel records kStatusWaitTimeout and returns.
#include <cuda_fp8.h>

#include <cstdlib>

#include "common.cuh"
#include "device_state.h"
#include "launchers.h"
#include "routing.cuh"

namespace afd {
namespace fused {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRouterThreads = 512;
constexpr int kRouterWarps = kRouterThreads / 32;
constexpr int kMaxSlots = 32;     // routed slots + shared-expert chunks
constexpr int kMaxA = 64;         // Attention ranks
constexpr int kNormMaxVec = 4;    // H <= 8 * kThreads * kNormMaxVec = 8192
constexpr int kRouteTile = 16;    // tokens per router CTA (one m16 MMA tile, one warp each for top-k)
constexpr int kMaxRouteE = 512;   // experts (matches the warp top-k)

using bf16 = __nv_bfloat16;

AFD_DEVICE uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
AFD_DEVICE void red_release_sys_add(uint64_t* p, uint64_t v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
AFD_DEVICE void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
AFD_DEVICE void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// 16-byte load that bypasses L1 (rows written by a peer GPU).
AFD_DEVICE Vec16<bf16> load16_cg(const bf16* p) {
  Vec16<bf16> out;
  *reinterpret_cast<int4*>(out.v) = __ldcg(reinterpret_cast<const int4*>(p));
  return out;
}
AFD_DEVICE uint32_t ld32(const bf16* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Bounded spin until *flag >= target; returns false on timeout.
AFD_DEVICE bool wait_flag(const uint64_t* flag, uint64_t target, int64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(flag) < target) {
    if ((int64_t)(globaltimer_ns() - t0) > timeout_ns) return false;
    __nanosleep(64);
  }
  return true;
}

// CTA-level completion count.  Thread 0 makes the CTA's stores (peer stores
// included) visible at system scope -- bar.sync puts the other threads'
// stores under that fence -- and counts the CTA in; the last of `expected`
// CTAs resets the counter and runs `publish`, whose flag updates are
// releases.  One system fence per CTA, all in parallel: the last CTA adds no
// fence of its own besides the release, so a chain of fences never forms.
template <typename Publish>
AFD_DEVICE void finish_grid(unsigned* ctr, unsigned expected, Publish publish) {
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    if (atomicAdd(ctr, 1u) == expected - 1) {
      *ctr = 0u;
      publish();
    }
  }
}

// Exclusive prefix of the per-source token counts in shared memory; returns
// the total.  Called by one thread after the arrival acquire.
AFD_DEVICE int source_prefix(const int32_t* tcount, int A, int* pre) {
  int run = 0;
  for (int a = 0; a < A; ++a) {
    pre[a] = run;
    run += __ldcg(tcount + a);
  }
  pre[A] = run;
  return run;
}
AFD_DEVICE int source_of(const int* pre, int A, int q) {
  int a = 0;
  while (a + 1 < A && pre[a + 1] <= q) ++a;
  return a;
}

// out[v] = sum over the rows selected by `mask` of src + bit * stride, for this
// lane's 16-byte vectors; four vectors per row are loaded before any is used.
template <bool kBypassL1>
AFD_DEVICE void warp_sum_rows(bf16* out, const bf16* src, size_t stride, unsigned mask, int H, int lane,
                              float scale = 1.f) {
  const int nv = H / 8;
  for (int v0 = lane; v0 < nv; v0 += 128) {
    float acc[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[u][q] = 0.f;
    for (unsigned m = mask; m; m &= m - 1) {
      const bf16* row = src + (size_t)(__ffs(m) - 1) * stride;
      Vec16<bf16> x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + u * 32;
        if (v < nv) x[u] = kBypassL1 ? load16_cg(row + v * 8) : load16(row + v * 8);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v0 + u * 32 < nv)
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[u][q] += __bfloat162float(x[u].v[q]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = v0 + u * 32;
      if (v < nv) {
        Vec16<bf16> o;
#pragma unroll
        for (int q = 0; q < 8; ++q) o.v[q] = __float2bfloat16_rn(acc[u][q] * scale);
        store16(out + v * 8, o);
      }
    }
  }
}

// Column chunk `cc` (256 columns: one 16-byte vector per lane) of the sum of
// the rows selected by `mask`; the rows' loads go out four at a time, so a
// token's slots cost one or two memory round trips instead of one per slot.
constexpr int kChunkCols = 256;
template <bool kBypassL1>
AFD_DEVICE void warp_sum_chunk(bf16* out, const bf16* src, size_t stride, unsigned mask, int H, int cc, int lane) {
  const int col = cc * kChunkCols + lane * 8;
  if (col >= H) return;
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0.f;
  while (mask) {
    int r[4];
    int n = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      r[u] = mask ? __ffs(mask) - 1 : -1;
      if (mask) {
        mask &= mask - 1;
        ++n;
      }
    }
    Vec16<bf16> x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (u < n) {
        const bf16* row = src + (size_t)r[u] * stride + col;
        x[u] = kBypassL1 ? load16_cg(row) : load16(row);
      }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (u < n)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(x[u].v[q]);
  }
  Vec16<bf16> o;
#pragma unroll
  for (int q = 0; q < 8; ++q) o.v[q] = __float2bfloat16_rn(acc[q]);
  store16(out + col, o);
}

// e4m3 <-> bf16 helpers for rows that travel as fp8 with one scale per 128 columns.
AFD_DEVICE uint2 pack_e4m3x8(const Vec16<bf16>& y, float inv) {
  uint32_t w[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
        make_float2(__bfloat162float(y.v[4 * i]) * inv, __bfloat162float(y.v[4 * i + 1]) * inv), __NV_SATFINITE,
        __NV_E4M3);
    const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
        make_float2(__bfloat162float(y.v[4 * i + 2]) * inv, __bfloat162float(y.v[4 * i + 3]) * inv), __NV_SATFINITE,
        __NV_E4M3);
    w[i] = (uint32_t)lo | ((uint32_t)hi << 16);
  }
  return make_uint2(w[0], w[1]);
}
// 16 e4m3 values -> 16 bf16 times `scale` (two 16-byte vectors).
AFD_DEVICE void unpack_e4m3x16(uint4 raw, float scale, Vec16<bf16>& a, Vec16<bf16>& b) {
  const uint32_t in[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)((in[i] >> (16 * h)) & 0xFFFFu), __NV_E4M3);
      __half2 h2;
      *reinterpret_cast<__half2_raw*>(&h2) = hr;
      const float2 f = __half22float2(h2);
      Vec16<bf16>& dst = i < 2 ? a : b;
      const int j = (i & 1) * 4 + h * 2;
      dst.v[j] = __float2bfloat16_rn(f.x * scale);
      dst.v[j + 1] = __float2bfloat16_rn(f.y * scale);
    }
  }
}

__global__ void epoch_kernel(uint64_t* epoch) { *epoch += 1; }

// Phase timing: the device clock when the stream reaches this point.
__global__ void stamp_kernel(uint64_t* buf, int idx) { buf[idx] = globaltimer_ns(); }

__global__ void wait_kernel(const uint64_t* flag, const uint64_t* epoch, uint64_t arrivals, int64_t timeout_ns,
                            int* status) {
  if (threadIdx.x != 0) return;
  if (!wait_flag(flag, (*epoch) * arrivals, timeout_ns)) atomicExch(status, kStatusWaitTimeout);
}

// The token count was stored by the norm kernel (an earlier kernel, so it is
// complete); the arrival is a release on every FFN rank's counter.
AFD_DEVICE void publish_dispatch(const DispatchParams& p) {
  for (int f = 0; f < p.num_ffn; ++f) red_release_sys_add(reinterpret_cast<uint64_t*>(p.flag_ptrs[f]) + p.layer, 1ull);
}

// ---- dispatch, step 1 (one CTA per token): residual += attn_out;
// h = RMSNorm(residual) * w (or h = attn_out when the model normalised it
// already, prenorm), kept locally for the router and stored straight
// into the FFN ranks' token buffers: every FFN rank for an MoE layer (the
// routing, which follows, tells each rank which rows it answers), the home
// rank only for a dense layer.  A dense layer has no router step, so this
// kernel also publishes the arrival.
__global__ void __launch_bounds__(kThreads) dispatch_norm_kernel(DispatchParams p) {
  __shared__ float s_red[kWarps];
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  const int nv = p.H / 8;
  const bf16* a = static_cast<const bf16*>(p.attn_out) + (size_t)t * p.H;
  bf16* r = static_cast<bf16*>(p.residual) + (size_t)t * p.H;
  Vec16<bf16> x[kNormMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < kNormMaxVec; ++u) {
    const int v = threadIdx.x + u * kThreads;
    if (v < nv) {
      const Vec16<bf16> xa = load16(a + v * 8);
      if (p.prenorm) {
        x[u] = xa;
        continue;
      }
      const Vec16<bf16> xr = load16(r + v * 8);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        x[u].v[j] = __float2bfloat16_rn(__bfloat162float(xa.v[j]) + __bfloat162float(xr.v[j]));
        const float f = __bfloat162float(x[u].v[j]);
        ss += f * f;
      }
      store16(r + v * 8, x[u]);
    }
  }
  float inv = 1.f;
  if (!p.prenorm) {
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot += s_red[w];
    inv = rsqrtf(tot / (float)p.H + p.eps);
  }
  const bf16* nw = static_cast<const bf16*>(p.norm_w);
  bf16* h = static_cast<bf16*>(p.h) + (size_t)t * p.H;
  const size_t row_off = ((size_t)p.attn_rank * p.t_cap + t) * p.H;
  const int f_lo = p.moe ? 0 : p.home_f;
  const int f_hi = p.moe ? p.num_ffn : (p.has_shared ? p.home_f + 1 : p.home_f);
  const size_t row = (size_t)p.attn_rank * p.t_cap + t;
#pragma unroll
  for (int u = 0; u < kNormMaxVec; ++u) {
    const int v = threadIdx.x + u * kThreads;
    const bool valid = v < nv;
    Vec16<bf16> y = x[u];
    if (valid && !p.prenorm) {
      const Vec16<bf16> w = load16(nw + v * 8);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        y.v[j] = __float2bfloat16_rn(__bfloat162float(x[u].v[j]) * inv * __bfloat162float(w.v[j]));
    }
    if (valid && p.moe) store16(h + v * 8, y);
    if (p.scale_ptrs != nullptr) {
      // e4m3 with one scale per 128 columns: the 16 vectors of a group sit in one half-warp
      float amax = 0.f;
      if (valid) {
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(__bfloat162float(y.v[j])));
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float sc = fmaxf(amax, 1e-12f) / 448.f;
      if (valid) {
        const uint2 q = pack_e4m3x8(y, 1.f / sc);
        for (int f = f_lo; f < f_hi; ++f) {
          *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(p.tok_ptrs[f]) + row * p.H + v * 8) = q;
          if ((threadIdx.x & 15) == 0) reinterpret_cast<float*>(p.scale_ptrs[f])[row * (p.H / 128) + v / 16] = sc;
        }
      }
    } else if (valid) {
      for (int f = f_lo; f < f_hi; ++f) store16(reinterpret_cast<bf16*>(p.tok_ptrs[f]) + row_off + v * 8, y);
    }
  }
  if (t == 0 && threadIdx.x < p.num_ffn)  // token count for every FFN rank (plain store)
    reinterpret_cast<volatile int*>(p.tcount_ptrs[threadIdx.x])[p.attn_rank] = p.T;
  if (!p.moe) {
    if (threadIdx.x == 0) p.fmask[t] = p.has_shared ? (int32_t)(1u << p.home_f) : 0;
    finish_grid(p.done_ctr, gridDim.x, [&] { publish_dispatch(p); });
  }
  // MoE layers: the router kernel publishes; this kernel's stores are complete
  // when it finishes, which precedes the router's release.
}

// ---- dispatch, step 2 (MoE layers): router logits on the tensor cores, top-k,
// routing metadata, arrival.
// Grid (token tiles of 16, expert tiles of 8 * NT).  Each of the 16 warps takes
// every 16th 16-wide K step (split K); the CTA sums the partial tiles.  The
// last CTA to finish a token tile (per-tile counter) routes its tokens, one
// warp per token, sends the ids / weights to every FFN rank and records which
// FFN ranks answer each token; the last token tile publishes the arrival.
template <int NT>
__global__ void __launch_bounds__(kRouterThreads, 1) dispatch_router_kernel(DispatchParams p) {
  constexpr int EB = 8 * NT;
  __shared__ __align__(16) float sbuf[kRouteTile * kMaxRouteE];
  __shared__ int s_last;
  static_assert(kRouterWarps * kRouteTile * EB <= kRouteTile * kMaxRouteE, "split-K buffer");
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRouteTile;
  const int nt = min(kRouteTile, p.T - t0);
  const int e0 = blockIdx.y * EB;
  const bf16* h = static_cast<const bf16*>(p.h);
  const bf16* gate = static_cast<const bf16*>(p.gate_w);
  const int g = lane >> 2, c = (lane & 3) * 2;  // MMA fragment row group / column pair
  const bool ok0 = g < nt, ok1 = g + 8 < nt;
  const bf16* h0 = h + (size_t)(t0 + (ok0 ? g : 0)) * p.H + c;
  const bf16* h1 = h + (size_t)(t0 + (ok1 ? g + 8 : 0)) * p.H + c;
  const bf16* gp[NT];
  bool okE[NT];
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int e = e0 + n * 8 + g;
    okE[n] = e < p.E;
    gp[n] = gate + (size_t)(okE[n] ? e : 0) * p.H + c;
  }
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  if (p.H % 64 == 0) {
    // 64-column chunks, split over the warps.  K is permuted inside a chunk
    // (the same way for both operands, so the dot products are unchanged):
    // lane q = lane % 4 owns columns [16q, 16q + 16) and reads them with two
    // 16-byte loads per row; MMA step j takes its pairs 16q + 4j + {0,1} and
    // + {2,3}.  A quad of lanes reads 128 contiguous bytes of each row.
    const int q = lane & 3;
    const bf16* hr0 = h + (size_t)(t0 + (ok0 ? g : 0)) * p.H + 16 * q;
    const bf16* hr1 = h + (size_t)(t0 + (ok1 ? g + 8 : 0)) * p.H + 16 * q;
    const bf16* gr[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) gr[n] = gate + (size_t)(okE[n] ? e0 + n * 8 + g : 0) * p.H + 16 * q;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    const int kchunks = p.H / 64;
#pragma unroll(NT >= 4 ? 1 : 2)
    for (int kc = warp; kc < kchunks; kc += kRouterWarps) {
      const int k = kc * 64;
      uint4 a0[2], a1[2], bv[NT][2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        a0[hh] = ok0 ? __ldg(reinterpret_cast<const uint4*>(hr0 + k + 8 * hh)) : z;
        a1[hh] = ok1 ? __ldg(reinterpret_cast<const uint4*>(hr1 + k + 8 * hh)) : z;
#pragma unroll
        for (int n = 0; n < NT; ++n) bv[n][hh] = okE[n] ? __ldg(reinterpret_cast<const uint4*>(gr[n] + k + 8 * hh)) : z;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int hh = j >> 1;
        const bool hi = j & 1;  // words 0,1 or 2,3 of the 16-byte vector
        uint32_t a[4];
        a[0] = hi ? a0[hh].z : a0[hh].x;
        a[1] = hi ? a1[hh].z : a1[hh].x;
        a[2] = hi ? a0[hh].w : a0[hh].y;
        a[3] = hi ? a1[hh].w : a1[hh].y;
#pragma unroll
        for (int n = 0; n < NT; ++n)
          mma_bf16_16816(acc[n], a, hi ? bv[n][hh].z : bv[n][hh].x, hi ? bv[n][hh].w : bv[n][hh].y);
      }
    }
  }
  const int ksteps = p.H % 64 == 0 ? 0 : p.H / 16;
#pragma unroll 4
  for (int ks = warp; ks < ksteps; ks += kRouterWarps) {
    const int k = ks * 16;
    uint32_t a[4];
    a[0] = ok0 ? ld32(h0 + k) : 0u;
    a[1] = ok1 ? ld32(h1 + k) : 0u;
    a[2] = ok0 ? ld32(h0 + k + 8) : 0u;
    a[3] = ok1 ? ld32(h1 + k + 8) : 0u;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const uint32_t b0 = okE[n] ? ld32(gp[n] + k) : 0u;
      const uint32_t b1 = okE[n] ? ld32(gp[n] + k + 8) : 0u;
      mma_bf16_16816(acc[n], a, b0, b1);
    }
  }
  // split-K reduction: red[warp][16][EB]
  float* red = sbuf;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    red[(warp * kRouteTile + g) * EB + n * 8 + c] = acc[n][0];
    red[(warp * kRouteTile + g) * EB + n * 8 + c + 1] = acc[n][1];
    red[(warp * kRouteTile + g + 8) * EB + n * 8 + c] = acc[n][2];
    red[(warp * kRouteTile + g + 8) * EB + n * 8 + c + 1] = acc[n][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kRouteTile * EB; i += kRouterThreads) {
    const int r = i / EB, col = i % EB;
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kRouterWarps; ++w) sum += red[(w * kRouteTile + r) * EB + col];
    if (r < nt && e0 + col < p.E) p.logits[(size_t)(t0 + r) * p.E + e0 + col] = sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_gpu();
    s_last = (atomicAdd(&p.route_ctr[blockIdx.x], 1u) == gridDim.y - 1);
    if (s_last) fence_acq_rel_gpu();
  }
  __syncthreads();
  if (!s_last) return;
  float* lg = sbuf;  // [16][E]
  for (int i = threadIdx.x; i < nt * p.E; i += kRouterThreads) lg[i] = __ldcg(p.logits + (size_t)t0 * p.E + i);
  __syncthreads();
  if (warp < nt) {
    const int t = t0 + warp;
    float w;
    int id;
    const int32_t* forced = p.hash_table ? p.hash_table + (size_t)p.input_ids[t] * p.k : nullptr;
    warp_route(lg + warp * p.E, p.gate_bias, p.E, p.k, p.scoring, p.renorm, p.n_group, p.topk_group, p.scale, w,
               id, forced);
    const unsigned bit = lane < p.k ? (1u << (id / p.e_local)) : 0u;
    const unsigned mask = __reduce_or_sync(0xffffffffu, bit) | (p.has_shared ? (1u << p.home_f) : 0u);
    const size_t off = ((size_t)p.attn_rank * p.t_cap + t) * p.k;
    if (lane < p.k) {
      for (int f = 0; f < p.num_ffn; ++f) {
        reinterpret_cast<int32_t*>(p.rid_ptrs[f])[off + lane] = id;
        reinterpret_cast<float*>(p.rwt_ptrs[f])[off + lane] = w;
      }
    }
    if (lane == 0) p.fmask[t] = (int32_t)mask;
  }
  if (threadIdx.x == 0) p.route_ctr[blockIdx.x] = 0u;
  finish_grid(p.done_ctr, gridDim.x, [&] { publish_dispatch(p); });
}

// ---- FFN side: wait for every Attention rank, then one warp per received
// (source, token) row: copy it into the segment of every local expert it
// routes to, and (home sources) into every shared-expert chunk's segment.
// Expert counters start at zero (cleared after the previous use).
__global__ void __launch_bounds__(kThreads) expand_kernel(ExpandParams p) {
  __shared__ int s_pre[kMaxA + 1];
  __shared__ int s_row[kWarps][kMaxSlots];
  __shared__ int s_ok;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  pdl_wait();  // before reading the epoch: the first layer's predecessor bumps it
  pdl_launch_dependents();
  bool ok = true;
  if (threadIdx.x == 0 && p.flag) ok = wait_flag(p.flag, (*p.epoch) * p.arrivals, p.timeout_ns);
  if (threadIdx.x == 0) {
    if (!ok) atomicExch(p.status, kStatusWaitTimeout);
    s_ok = ok;
    if (ok) {
      source_prefix(p.tcount, p.A, s_pre);
      if (blockIdx.x == 0) {
        if (p.n_chunks > 0) {
          const int home_total = s_pre[p.home_a0 + p.ratio] - s_pre[p.home_a0];
          for (int ch = 0; ch < p.n_chunks; ++ch) p.counts[p.e_local + ch] = home_total;
        } else {
          for (int i = 0; i < p.ratio; ++i) p.counts[p.e_local + i] = s_pre[p.home_a0 + i + 1] - s_pre[p.home_a0 + i];
        }
      }
    }
  }
  __syncthreads();
  const bool fp8 = p.tok_scale != nullptr;
  if (!s_ok || (!p.moe && !fp8)) return;
  const bf16* tok = static_cast<const bf16*>(p.tok);
  bf16* x = static_cast<bf16*>(p.x);
  bf16* home_x = static_cast<bf16*>(p.home_x);
  const int nv = p.H / 8;
  const int total = s_pre[p.A];
  const int slots = p.k + p.n_chunks;
  for (int q = blockIdx.x * kWarps + warp; q < total; q += gridDim.x * kWarps) {
    const int a = source_of(s_pre, p.A, q);
    const int t = q - s_pre[a];
    const int pair = a * p.t_cap + t;
    const size_t base = (size_t)pair * p.k;
    const bool home = a >= p.home_a0 && a < p.home_a0 + p.ratio;
    if (fp8) {
      // e4m3 rows: dequantise once into every target (expert segments, shared
      // chunks, and the bf16 copy of home rows used by the dense / shared GEMMs).
      int row = -1;
      if (p.moe && lane < p.k) {
        const int le = __ldcg(p.rid + base + lane) - p.e_offset;
        if (le >= 0 && le < p.e_local) {
          const int slot = atomicAdd(&p.counts[le], 1);
          if (slot < p.cap) {
            row = le * p.cap + slot;
            p.meta[row] = (a << 24) | (t << 8) | lane;
            p.rw[row] = __ldcg(p.rwt + base + lane);
          } else {
            atomicExch(p.status, kStatusBadIndex);
          }
        }
      } else if (p.moe && lane >= p.k && lane < slots && home) {
        row = p.shared_base + (lane - p.k) * p.shared_stride + (s_pre[a] - s_pre[p.home_a0]) + t;
        p.meta[row] = (a << 24) | (t << 8) | lane;
        p.rw[row] = 1.f;
      }
      if (lane < slots) s_row[warp][lane] = row;
      const unsigned used = __ballot_sync(0xffffffffu, row >= 0);
      __syncwarp();
      bf16* hx = home && home_x ? home_x + ((size_t)(a - p.home_a0) * p.t_cap + t) * p.H : nullptr;
      if (used || hx) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.tok) + (size_t)pair * p.H;
        const float* sc = p.tok_scale + (size_t)pair * (p.H / 128);
        for (int c = lane; c < p.H / 16; c += 32) {
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(src + c * 16));
          Vec16<bf16> lo, hi;
          unpack_e4m3x16(raw, __ldcg(sc + c / 8), lo, hi);
          for (unsigned m = used; m; m &= m - 1) {
            bf16* dst = x + (size_t)s_row[warp][__ffs(m) - 1] * p.H + c * 16;
            store16(dst, lo);
            store16(dst + 8, hi);
          }
          if (hx) {
            store16(hx + c * 16, lo);
            store16(hx + c * 16 + 8, hi);
          }
        }
      }
      __syncwarp();
      continue;
    }
    int row = -1;
    if (lane < p.k) {
      const int le = __ldcg(p.rid + base + lane) - p.e_offset;
      if (le >= 0 && le < p.e_local) {
        const int slot = atomicAdd(&p.counts[le], 1);
        if (slot < p.cap) {
          row = le * p.cap + slot;
          p.meta[row] = (a << 24) | (t << 8) | lane;
          p.rw[row] = __ldcg(p.rwt + base + lane);
        } else {
          atomicExch(p.status, kStatusBadIndex);
        }
      }
    } else if (lane < slots && a >= p.home_a0 && a < p.home_a0 + p.ratio) {
      row = p.shared_base + (lane - p.k) * p.shared_stride + (s_pre[a] - s_pre[p.home_a0]) + t;
      p.meta[row] = (a << 24) | (t << 8) | lane;
      p.rw[row] = 1.f;
    }
    if (lane < slots) s_row[warp][lane] = row;
    const unsigned used = __ballot_sync(0xffffffffu, row >= 0);
    __syncwarp();
    if (used) {
      const bf16* src = tok + (size_t)pair * p.H;
      for (int v0 = lane; v0 < nv; v0 += 128) {
        Vec16<bf16> xv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (v0 + u * 32 < nv) xv[u] = load16_cg(src + (v0 + u * 32) * 8);
        for (unsigned m = used; m; m &= m - 1) {
          bf16* dst = x + (size_t)s_row[warp][__ffs(m) - 1] * p.H;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (v0 + u * 32 < nv) store16(dst + (v0 + u * 32) * 8, xv[u]);
        }
      }
    }
    __syncwarp();
  }
}

// One warp per received (source, token): sum this rank's slots for the token
// (routed experts it owns; the shared-expert slots for home sources) and
// store the row into the source's combine slot [t][f_rank].
__global__ void __launch_bounds__(kThreads) combine_send_kernel(CombineSendParams p) {
  __shared__ int s_pre[kMaxA + 1];
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) source_prefix(p.tcount, p.A, s_pre);
  __syncthreads();
  const int total = s_pre[p.A];
  // Expert-output sums go one (token, 256-column chunk) per warp; the
  // transport-only echo mode keeps one warp per token.
  const int nch = p.echo ? 1 : (p.H + kChunkCols - 1) / kChunkCols;
  for (int item = blockIdx.x * kWarps + warp; item < total * nch; item += gridDim.x * kWarps) {
    const int q = item / nch, cc = item - q * nch;
    const int a = source_of(s_pre, p.A, q);
    const int t = q - s_pre[a];
    const int pair = a * p.t_cap + t;
    const bool home = p.has_shared && a >= p.home_a0 && a < p.home_a0 + p.ratio;
    bool hit = false;
    float w = 0.f;  // echo mode: the slot's routing weight (1 for a shared slot)
    if (lane < p.k) {
      if (p.moe) {
        const int le = p.rid[(size_t)pair * p.k + lane] - p.e_offset;
        if (le >= 0 && le < p.e_local) {
          hit = true;
          w = p.echo ? p.rwt[(size_t)pair * p.k + lane] : 1.f;
        }
      }
    } else if (lane < p.k + p.home_slots) {
      hit = home;
      w = home ? 1.f : 0.f;
    }
    const unsigned used = __ballot_sync(0xffffffffu, hit);
    if (!used) continue;
    bf16* dst = reinterpret_cast<bf16*>(p.dst_ptrs[a]) + ((size_t)t * p.num_ffn + p.f_rank) * p.H;
    if (p.echo && p.tok_scale != nullptr) {
      // transport-only stand-in with e4m3 rows: dequantise and scale
      const float wsum = warp_sum(w);
      const uint8_t* src = static_cast<const uint8_t*>(p.staging) + (size_t)pair * p.H;
      const float* sc = p.tok_scale + (size_t)pair * (p.H / 128);
      for (int c = lane; c < p.H / 16; c += 32) {
        Vec16<bf16> lo, hi;
        unpack_e4m3x16(__ldcg(reinterpret_cast<const uint4*>(src + c * 16)), __ldcg(sc + c / 8) * wsum, lo, hi);
        store16(dst + c * 16, lo);
        store16(dst + c * 16 + 8, hi);
      }
    } else if (p.echo) {
      const float wsum = warp_sum(w);
      warp_sum_rows<true>(dst, static_cast<const bf16*>(p.staging) + (size_t)pair * p.H, 0, 1u, p.H, lane, wsum);
    } else {
      warp_sum_chunk<false>(dst, static_cast<const bf16*>(p.staging) + (size_t)pair * p.J * p.H, (size_t)p.H, used,
                            p.H, cc, lane);
    }
  }
  finish_grid(p.done_ctr, gridDim.x, [&] {
    for (int a = 0; a < p.A; ++a) red_release_sys_add(reinterpret_cast<uint64_t*>(p.flag_ptrs[a]) + p.layer, 1ull);
  });
}

// One warp per token: out[t] = sum of the FFN slots that answer token t.
__global__ void __launch_bounds__(kThreads) combine_kernel(CombineParams p) {
  __shared__ bool ok;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) ok = wait_flag(p.flag + p.layer, (*p.epoch) * p.arrivals, p.timeout_ns);
  __syncthreads();
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(p.status, kStatusWaitTimeout);
    return;
  }
  const int nch = (p.H + kChunkCols - 1) / kChunkCols;
  for (int item = blockIdx.x * kWarps + warp; item < p.T * nch; item += gridDim.x * kWarps) {
    const int t = item / nch, cc = item - t * nch;
    const unsigned mask = (unsigned)p.fmask[t];
    warp_sum_chunk<true>(static_cast<bf16*>(p.out) + (size_t)t * p.H,
                         static_cast<const bf16*>(p.comb) + (size_t)t * p.F * p.H, (size_t)p.H, mask, p.H, cc, lane);
  }
}

}  // namespace fused

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("AFD_DISABLE_PDL");
    return !(v && v[0] == '1');
  }();
  return on;
}

}  // namespace afd

using namespace afd;

void launch_afd_epoch(uint64_t* epoch, cudaStream_t s) { fused::epoch_kernel<<<1, 1, 0, s>>>(epoch); }

void launch_afd_stamp(uint64_t* buf, int idx, cudaStream_t s) { fused::stamp_kernel<<<1, 1, 0, s>>>(buf, idx); }

void launch_afd_wait(const uint64_t* flag, const uint64_t* epoch, uint64_t arrivals, int64_t timeout_ns, int* status,
                     cudaStream_t s) {
  fused::wait_kernel<<<1, 32, 0, s>>>(flag, epoch, arrivals, timeout_ns, status);
}

// Two launches: norm + row stores (one CTA per token), then the router for
// MoE layers.  The router's expert tile widens with the token count so the
// grid stays near two CTAs per SM.
void launch_afd_dispatch(const DispatchParams& p, cudaStream_t s) {
  using namespace fused;
  if (p.T <= 0) return;
  launch_pdl(dispatch_norm_kernel, dim3(p.T), dim3(kThreads), 0, s, p);
  if (!p.moe) return;
  const int mt = (p.T + kRouteTile - 1) / kRouteTile;
  const int target = device_sm_count() * 2;
  if (mt * ((p.E + 7) / 8) <= target)
    launch_pdl(dispatch_router_kernel<1>, dim3(mt, (p.E + 7) / 8), dim3(kRouterThreads), 0, s, p);
  else if (mt * ((p.E + 15) / 16) <= target)
    launch_pdl(dispatch_router_kernel<2>, dim3(mt, (p.E + 15) / 16), dim3(kRouterThreads), 0, s, p);
  else
    launch_pdl(dispatch_router_kernel<4>, dim3(mt, (p.E + 31) / 32), dim3(kRouterThreads), 0, s, p);
}

static int warp_grid(int items, int max_ctas) {
  return std::max(1, std::min((items + fused::kWarps - 1) / fused::kWarps, max_ctas));
}

void launch_afd_expand(const ExpandParams& p, cudaStream_t s) {
  launch_pdl(fused::expand_kernel, dim3(warp_grid(p.A * p.t_cap, device_sm_count())), dim3(fused::kThreads), 0, s, p);
}

void launch_afd_combine_send(const CombineSendParams& p, cudaStream_t s) {
  const int nch = p.echo ? 1 : (p.H + fused::kChunkCols - 1) / fused::kChunkCols;
  launch_pdl(fused::combine_send_kernel, dim3(warp_grid(p.A * p.t_cap * nch, 2 * device_sm_count())),
             dim3(fused::kThreads), 0, s, p);
}

void launch_afd_combine(const CombineParams& p, cudaStream_t s) {
  const int nch = (p.H + fused::kChunkCols - 1) / fused::kChunkCols;
  launch_pdl(fused::combine_kernel, dim3(warp_grid(p.T * nch, 2 * device_sm_count())), dim3(fused::kThreads), 0, s,
             p);
}
