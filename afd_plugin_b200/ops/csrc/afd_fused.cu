// Fused Attention<->FFN transfer kernels over NVLink peer memory.
//
// Per-rank protocol: a token row crosses NVLink once per FFN rank that owns
// one of its experts (or is its home rank for the shared expert / dense MLP)
// and comes back as one pre-reduced row per such rank.
//
// afd_dispatch      (Attention side, per layer and ubatch), three kernels:
//   norm    residual += attn_out; h = RMSNorm(residual) * w (one CTA per token)
//   router  logits = h . gate^T on the tensor cores, split over (token tile,
//           expert tile) CTAs; the last CTA of a token tile runs the top-k and
//           sends the token's routing (k ids + weights) to every FFN rank
//   send    one warp per (token, destination FFN rank) stores h into that
//           rank's token buffer; the last CTA publishes the token count and
//           bumps every FFN rank's arrival counter (release, system scope).
// afd_expand        (FFN side) copies each received row into the contiguous
//   segment of every local expert it routes to (local HBM), building the
//   grouped GEMM's row -> (source, token, slot) map.
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
#include "common.cuh"
#include "launchers.h"
#include "routing.cuh"

namespace afd {
namespace fused {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxK = 16;
constexpr int kNormMaxVec = 4;    // H <= 8 * kThreads * kNormMaxVec = 8192
constexpr int kRouteTile = 16;    // tokens per router CTA (one m16 MMA tile)
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

// Warp-wide row copy of H bf16 elements (H % 8 == 0), four 16-byte loads in flight per lane.
AFD_DEVICE void warp_copy_row(bf16* dst, const bf16* src, int H, int lane) {
  const int nv = H / 8;
  int v = lane;
  for (; v + 96 < nv; v += 128) {
    Vec16<bf16> x0 = load16(src + v * 8), x1 = load16(src + (v + 32) * 8);
    Vec16<bf16> x2 = load16(src + (v + 64) * 8), x3 = load16(src + (v + 96) * 8);
    store16(dst + v * 8, x0);
    store16(dst + (v + 32) * 8, x1);
    store16(dst + (v + 64) * 8, x2);
    store16(dst + (v + 96) * 8, x3);
  }
  for (; v < nv; v += 32) store16(dst + v * 8, load16(src + v * 8));
}

// Last-CTA completion: every CTA makes its peer stores visible system-wide and
// counts itself; the last one resets the counter and runs `publish`.
template <typename Publish>
AFD_DEVICE void finish_grid(unsigned* done_ctr, Publish publish) {
  __shared__ int s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(done_ctr, 1u) == gridDim.x - 1);
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *done_ctr = 0u;
    __threadfence_system();
    publish();
  }
}

__global__ void epoch_kernel(uint64_t* epoch) { *epoch += 1; }

__global__ void wait_kernel(const uint64_t* flag, const uint64_t* epoch, uint64_t arrivals, int64_t timeout_ns,
                            int* status) {
  if (threadIdx.x != 0) return;
  if (!wait_flag(flag, (*epoch) * arrivals, timeout_ns)) atomicExch(status, kStatusWaitTimeout);
}

// ---- dispatch, step 1 (one CTA per token): residual += attn_out; h = RMSNorm(residual) * w.
// h goes to local scratch; with a shared expert / dense MLP the home FFN rank
// gets the row right here (its destination does not depend on routing).
__global__ void __launch_bounds__(kThreads) dispatch_norm_kernel(DispatchParams p) {
  __shared__ float s_red[kWarps];
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
      const Vec16<bf16> xa = load16(a + v * 8), xr = load16(r + v * 8);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        x[u].v[j] = __float2bfloat16_rn(__bfloat162float(xa.v[j]) + __bfloat162float(xr.v[j]));
        const float f = __bfloat162float(x[u].v[j]);
        ss += f * f;
      }
      store16(r + v * 8, x[u]);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) s_red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) tot += s_red[w];
  const float inv = rsqrtf(tot / (float)p.H + p.eps);
  const bf16* nw = static_cast<const bf16*>(p.norm_w);
  bf16* h = static_cast<bf16*>(p.h) + (size_t)t * p.H;
  bf16* home = p.has_shared ? reinterpret_cast<bf16*>(p.tok_ptrs[p.home_f]) +
                                  ((size_t)p.attn_rank * p.t_cap + t) * p.H
                            : nullptr;
#pragma unroll
  for (int u = 0; u < kNormMaxVec; ++u) {
    const int v = threadIdx.x + u * kThreads;
    if (v < nv) {
      const Vec16<bf16> w = load16(nw + v * 8);
      Vec16<bf16> y;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        y.v[j] = __float2bfloat16_rn(__bfloat162float(x[u].v[j]) * inv * __bfloat162float(w.v[j]));
      store16(h + v * 8, y);
      if (home) store16(home + v * 8, y);
    }
  }
  if (!p.moe && threadIdx.x == 0) p.fmask[t] = p.has_shared ? (int32_t)(1u << p.home_f) : 0;
  if (home) __threadfence_system();
}

// ---- dispatch, step 2 (MoE layers): router logits on the tensor cores, then top-k.
// Grid (token tiles of 16, expert tiles of 8 * NT).  Each warp takes every 8th
// 16-wide K step (split K), the CTA sums the eight partial tiles.  The last
// CTA to finish a token tile (per-tile counter) routes its 16 tokens: writes
// the ids / weights to every FFN rank and the destination mask locally.
template <int NT>
__global__ void __launch_bounds__(kThreads) dispatch_router_kernel(DispatchParams p) {
  constexpr int EB = 8 * NT;
  __shared__ __align__(16) float sbuf[kRouteTile * kMaxRouteE];
  __shared__ int s_last;
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
  const int ksteps = p.H / 16;
#pragma unroll 4
  for (int ks = warp; ks < ksteps; ks += kWarps) {
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
  for (int i = threadIdx.x; i < kRouteTile * EB; i += kThreads) {
    const int r = i / EB, col = i % EB;
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) sum += red[(w * kRouteTile + r) * EB + col];
    if (r < nt && e0 + col < p.E) p.logits[(size_t)(t0 + r) * p.E + e0 + col] = sum;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&p.route_ctr[blockIdx.x], 1u) == gridDim.y - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* lg = sbuf;  // [16][E]
  for (int i = threadIdx.x; i < nt * p.E; i += kThreads) lg[i] = __ldcg(p.logits + (size_t)t0 * p.E + i);
  __syncthreads();
  for (int i = warp; i < nt; i += kWarps) {
    const int t = t0 + i;
    float w;
    int id;
    warp_route(lg + i * p.E, p.gate_bias, p.E, p.k, p.scoring, p.renorm, p.n_group, p.topk_group, p.scale, w, id);
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
  __threadfence_system();
}

// ---- dispatch, step 3: one warp per (token, FFN rank) row store; the last CTA
// publishes the token count and bumps every FFN rank's arrival counter.
__global__ void __launch_bounds__(kThreads) dispatch_send_kernel(DispatchParams p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kWarps + warp;
  const int t = gw / p.num_ffn, f = gw % p.num_ffn;
  if (t < p.T) {
    const unsigned mask = (unsigned)p.fmask[t];
    if (((mask >> f) & 1u) && !(p.has_shared && f == p.home_f)) {
      bf16* dst = reinterpret_cast<bf16*>(p.tok_ptrs[f]) + ((size_t)p.attn_rank * p.t_cap + t) * p.H;
      warp_copy_row(dst, static_cast<const bf16*>(p.h) + (size_t)t * p.H, p.H, lane);
    }
  }
  finish_grid(p.done_ctr, [&] {
    for (int ff = 0; ff < p.num_ffn; ++ff)
      atomicExch_system(reinterpret_cast<int*>(p.tcount_ptrs[ff]) + p.attn_rank, p.T);
    __threadfence_system();
    for (int ff = 0; ff < p.num_ffn; ++ff)
      red_release_sys_add(reinterpret_cast<uint64_t*>(p.flag_ptrs[ff]) + p.layer, 1ull);
  });
}

// One warp per (source, token): copy the row into every local expert segment it
// routes to.  Counters start at zero (cleared after the previous use).
__global__ void __launch_bounds__(kThreads) expand_kernel(ExpandParams p) {
  __shared__ int s_row[kWarps][kMaxK];
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (blockIdx.x == 0 && threadIdx.x < p.ratio) p.counts[p.e_local + threadIdx.x] = p.tcount[p.home_a0 + threadIdx.x];
  if (!p.moe) return;
  const bf16* tok = static_cast<const bf16*>(p.tok);
  bf16* x = static_cast<bf16*>(p.x);
  const int nv = p.H / 8;
  for (int pair = blockIdx.x * kWarps + warp; pair < p.A * p.t_cap; pair += gridDim.x * kWarps) {
    const int a = pair / p.t_cap, t = pair % p.t_cap;
    if (t >= p.tcount[a]) continue;
    const size_t base = (size_t)pair * p.k;
    int row = -1;
    if (lane < p.k) {
      const int le = p.rid[base + lane] - p.e_offset;
      if (le >= 0 && le < p.e_local) {
        const int slot = atomicAdd(&p.counts[le], 1);
        if (slot < p.cap) {
          row = le * p.cap + slot;
          p.meta[row] = (a << 24) | (t << 8) | lane;
          p.rw[row] = p.rwt[base + lane];
        } else {
          atomicExch(p.status, kStatusBadIndex);
        }
      }
      s_row[warp][lane] = row;
    }
    const unsigned used = __ballot_sync(0xffffffffu, row >= 0);
    __syncwarp();
    if (used) {
      const bf16* src = tok + (size_t)pair * p.H;
      for (int v = lane; v < nv; v += 32) {
        const Vec16<bf16> xv = load16_cg(src + v * 8);
        for (unsigned m = used; m; m &= m - 1) store16(x + (size_t)s_row[warp][__ffs(m) - 1] * p.H + v * 8, xv);
      }
    }
    __syncwarp();
  }
}

// One warp per (source, token): sum this rank's slots for the token and store
// the row into the source's combine slot [t][f_rank].
__global__ void __launch_bounds__(kThreads) combine_send_kernel(CombineSendParams p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int nv = p.H / 8;
  for (int pair = blockIdx.x * kWarps + warp; pair < p.A * p.t_cap; pair += gridDim.x * kWarps) {
    const int a = pair / p.t_cap, t = pair % p.t_cap;
    if (t >= p.tcount[a]) continue;
    const bool home = p.has_shared && a >= p.home_a0 && a < p.home_a0 + p.ratio;
    bool hit = false;
    float w = 0.f;  // echo mode: the slot's routing weight (1 for the shared slot)
    if (lane < p.k) {
      if (p.moe) {
        const int le = p.rid[(size_t)pair * p.k + lane] - p.e_offset;
        if (le >= 0 && le < p.e_local) {
          hit = true;
          w = p.echo ? p.rwt[(size_t)pair * p.k + lane] : 1.f;
        }
      }
    } else if (lane == p.k) {
      hit = home;
      w = home ? 1.f : 0.f;
    }
    const unsigned used = __ballot_sync(0xffffffffu, hit);
    if (!used) continue;
    bf16* dst = reinterpret_cast<bf16*>(p.dst_ptrs[a]) + ((size_t)t * p.num_ffn + p.f_rank) * p.H;
    if (p.echo) {
      const float wsum = warp_sum(w);
      const bf16* row = static_cast<const bf16*>(p.staging) + (size_t)pair * p.H;
      for (int v = lane; v < nv; v += 32) {
        Vec16<bf16> xv = load16_cg(row + v * 8);
#pragma unroll
        for (int q = 0; q < 8; ++q) xv.v[q] = __float2bfloat16_rn(__bfloat162float(xv.v[q]) * wsum);
        store16(dst + v * 8, xv);
      }
    } else {
      const bf16* st = static_cast<const bf16*>(p.staging) + (size_t)pair * p.J * p.H;
      for (int v = lane; v < nv; v += 32) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (unsigned m = used; m; m &= m - 1) {
          const Vec16<bf16> xv = load16(st + (size_t)(__ffs(m) - 1) * p.H + v * 8);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(xv.v[q]);
        }
        Vec16<bf16> o;
#pragma unroll
        for (int q = 0; q < 8; ++q) o.v[q] = __float2bfloat16_rn(acc[q]);
        store16(dst + v * 8, o);
      }
    }
  }
  finish_grid(p.done_ctr, [&] {
    for (int a = 0; a < p.A; ++a) red_release_sys_add(reinterpret_cast<uint64_t*>(p.flag_ptrs[a]) + p.layer, 1ull);
  });
}

// One warp per token: out[t] = sum of the FFN slots that answer token t.
__global__ void __launch_bounds__(kThreads) combine_kernel(CombineParams p) {
  __shared__ bool ok;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) ok = wait_flag(p.flag + p.layer, (*p.epoch) * p.arrivals, p.timeout_ns);
  __syncthreads();
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(p.status, kStatusWaitTimeout);
    return;
  }
  const int nv = p.H / 8;
  for (int t = blockIdx.x * kWarps + warp; t < p.T; t += gridDim.x * kWarps) {
    const unsigned mask = (unsigned)p.fmask[t];
    const bf16* base = static_cast<const bf16*>(p.comb) + (size_t)t * p.F * p.H;
    bf16* out = static_cast<bf16*>(p.out) + (size_t)t * p.H;
    for (int v = lane; v < nv; v += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (unsigned m = mask; m; m &= m - 1) {
        const Vec16<bf16> xv = load16_cg(base + (size_t)(__ffs(m) - 1) * p.H + v * 8);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(xv.v[q]);
      }
      Vec16<bf16> o;
#pragma unroll
      for (int q = 0; q < 8; ++q) o.v[q] = __float2bfloat16_rn(acc[q]);
      store16(out + v * 8, o);
    }
  }
}

}  // namespace fused
}  // namespace afd

using namespace afd;

void launch_afd_epoch(uint64_t* epoch, cudaStream_t s) { fused::epoch_kernel<<<1, 1, 0, s>>>(epoch); }

void launch_afd_wait(const uint64_t* flag, const uint64_t* epoch, uint64_t arrivals, int64_t timeout_ns, int* status,
                     cudaStream_t s) {
  fused::wait_kernel<<<1, 32, 0, s>>>(flag, epoch, arrivals, timeout_ns, status);
}

// Three launches: norm (one CTA per token), router (MoE layers only), send.
// The router's expert tile widens with the token count so the grid stays
// near two CTAs per SM.
void launch_afd_dispatch(const DispatchParams& p, cudaStream_t s) {
  using namespace fused;
  const int T = std::max(1, p.T);
  if (p.T > 0) dispatch_norm_kernel<<<p.T, kThreads, 0, s>>>(p);
  if (p.moe && p.T > 0) {
    const int mt = (T + kRouteTile - 1) / kRouteTile;
    const int target = 148 * 2;
    if (mt * ((p.E + 7) / 8) <= target)
      dispatch_router_kernel<1><<<dim3(mt, (p.E + 7) / 8), kThreads, 0, s>>>(p);
    else if (mt * ((p.E + 15) / 16) <= target)
      dispatch_router_kernel<2><<<dim3(mt, (p.E + 15) / 16), kThreads, 0, s>>>(p);
    else
      dispatch_router_kernel<4><<<dim3(mt, (p.E + 31) / 32), kThreads, 0, s>>>(p);
  }
  const int warps = T * p.num_ffn;
  dispatch_send_kernel<<<(warps + kWarps - 1) / kWarps, kThreads, 0, s>>>(p);
}

static int warp_grid(int items, int max_ctas) {
  return std::max(1, std::min((items + fused::kWarps - 1) / fused::kWarps, max_ctas));
}

void launch_afd_expand(const ExpandParams& p, cudaStream_t s) {
  fused::expand_kernel<<<warp_grid(p.A * p.t_cap, 148 * 4), fused::kThreads, 0, s>>>(p);
}

void launch_afd_combine_send(const CombineSendParams& p, cudaStream_t s) {
  fused::combine_send_kernel<<<warp_grid(p.A * p.t_cap, 148 * 4), fused::kThreads, 0, s>>>(p);
}

void launch_afd_combine(const CombineParams& p, cudaStream_t s) {
  fused::combine_kernel<<<warp_grid(p.T, 148 * 2), fused::kThreads, 0, s>>>(p);
}
