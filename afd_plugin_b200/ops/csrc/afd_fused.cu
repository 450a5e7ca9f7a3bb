// Fused Attention<->FFN transfer kernels over NVLink peer memory.
//
// Per-rank protocol: a token row crosses NVLink once per FFN rank that owns
// one of its experts (or is its home rank for the shared expert / dense MLP)
// and comes back as one pre-reduced row per such rank.
//
// afd_dispatch      (Attention side, per layer and ubatch)
//   residual += attn_out; h = RMSNorm(residual) * w           (post-attn norm)
//   logits = h . gate^T; (weight, expert) = top-k routing      (router)
//   h is stored (16-byte stores) into each destination FFN rank's token
//   buffer; the token's routing (k ids + weights) goes to every FFN rank.  The
//   last CTA publishes the token count and bumps every FFN rank's arrival
//   counter (release, system scope).
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

constexpr int kTPC = 4;         // tokens per dispatch CTA
constexpr int kThreads = 256;
constexpr int kMaxK = 16;

AFD_DEVICE uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
AFD_DEVICE void red_release_sys_add(uint64_t* p, uint64_t v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded spin until *flag >= target; returns false on timeout.
AFD_DEVICE bool wait_flag(const uint64_t* flag, uint64_t target, int64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(flag) < target) {
    if ((int64_t)(globaltimer_ns() - t0) > timeout_ns) return false;
    __nanosleep(64);
  }
  return true;
}

// CTA-wide 16-byte row copy of H bf16 elements.
AFD_DEVICE void copy_row(__nv_bfloat16* dst, const __nv_bfloat16* src, int H) {
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) store16(dst + v * 8, load16(src + v * 8));
}

__global__ void epoch_kernel(uint64_t* epoch) { *epoch += 1; }

__global__ void wait_kernel(const uint64_t* flag, const uint64_t* epoch, uint64_t arrivals, int64_t timeout_ns,
                            int* status) {
  if (threadIdx.x != 0) return;
  if (!wait_flag(flag, (*epoch) * arrivals, timeout_ns)) atomicExch(status, kStatusWaitTimeout);
}

__global__ void __launch_bounds__(kThreads) dispatch_kernel(DispatchParams p) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __nv_bfloat16* hbuf = reinterpret_cast<__nv_bfloat16*>(dsm);                      // [kTPC][H]
  float* logits = reinterpret_cast<float*>(dsm + (size_t)kTPC * p.H * 2);            // [kTPC][E]
  __shared__ int s_id[kTPC][kMaxK];
  __shared__ float s_w[kTPC][kMaxK];
  __shared__ unsigned s_mask[kTPC];
  __shared__ float s_red[kThreads / 32];
  __shared__ int s_last;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const __nv_bfloat16* attn_out = static_cast<const __nv_bfloat16*>(p.attn_out);
  __nv_bfloat16* residual = static_cast<__nv_bfloat16*>(p.residual);
  const __nv_bfloat16* norm_w = static_cast<const __nv_bfloat16*>(p.norm_w);
  const __nv_bfloat16* gate_w = static_cast<const __nv_bfloat16*>(p.gate_w);
  const int t0 = blockIdx.x * kTPC;
  const int nt = max(0, min(kTPC, p.T - t0));
  const int VN = 8;
  const int nv = p.H / VN;

  // ---- residual add + RMSNorm (one token at a time, whole CTA)
  for (int i = 0; i < nt; ++i) {
    const int t = t0 + i;
    const __nv_bfloat16* a = attn_out + (size_t)t * p.H;
    __nv_bfloat16* r = residual + (size_t)t * p.H;
    float ss = 0.f;
    for (int v = threadIdx.x; v < nv; v += kThreads) {
      Vec16<__nv_bfloat16> x = load16(a + v * VN), y = load16(r + v * VN);
#pragma unroll
      for (int j = 0; j < VN; ++j) {
        x.v[j] = __float2bfloat16_rn(__bfloat162float(x.v[j]) + __bfloat162float(y.v[j]));
        const float f = __bfloat162float(x.v[j]);
        ss += f * f;
      }
      store16(r + v * VN, x);
      store16(hbuf + (size_t)i * p.H + v * VN, x);
    }
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) tot += s_red[w];
    const float inv = rsqrtf(tot / (float)p.H + p.eps);
    for (int v = threadIdx.x; v < nv; v += kThreads) {
      Vec16<__nv_bfloat16> x = load16(hbuf + (size_t)i * p.H + v * VN), w = load16(norm_w + v * VN);
#pragma unroll
      for (int j = 0; j < VN; ++j)
        x.v[j] = __float2bfloat16_rn(__bfloat162float(x.v[j]) * inv * __bfloat162float(w.v[j]));
      store16(hbuf + (size_t)i * p.H + v * VN, x);
    }
    __syncthreads();
  }

  // ---- router logits (gate rows read once per CTA for all its tokens)
  if (threadIdx.x < kTPC) s_mask[threadIdx.x] = p.has_shared ? (1u << p.home_f) : 0u;
  __syncthreads();
  if (p.moe && nt > 0) {
    for (int e = warp; e < p.E; e += kThreads / 32) {
      float acc[kTPC] = {0.f, 0.f, 0.f, 0.f};
      const __nv_bfloat16* g = gate_w + (size_t)e * p.H;
      for (int v = lane; v < nv; v += 32) {
        Vec16<__nv_bfloat16> gw = load16(g + v * VN);
#pragma unroll
        for (int i = 0; i < kTPC; ++i) {
          if (i < nt) {
            Vec16<__nv_bfloat16> x = load16(hbuf + (size_t)i * p.H + v * VN);
#pragma unroll
            for (int j = 0; j < VN; ++j) acc[i] += __bfloat162float(x.v[j]) * __bfloat162float(gw.v[j]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kTPC; ++i) {
        const float s = warp_sum(acc[i]);
        if (lane == 0 && i < nt) logits[i * p.E + e] = s;
      }
    }
    __syncthreads();
    if (warp < nt) {  // top-k, one warp per token
      float w;
      int id;
      warp_route(logits + warp * p.E, p.gate_bias, p.E, p.k, p.scoring, p.renorm, p.n_group, p.topk_group, p.scale,
                 w, id);
      if (lane < p.k) {
        s_id[warp][lane] = id;
        s_w[warp][lane] = w;
        atomicOr(&s_mask[warp], 1u << (id / p.e_local));
      }
    }
    __syncthreads();
  }

  // ---- stores into the FFN ranks (peer memory)
  for (int i = 0; i < nt; ++i) {
    const int t = t0 + i;
    const unsigned mask = s_mask[i];
    const size_t tok_off = (size_t)p.attn_rank * p.t_cap + t;
    for (int f = 0; f < p.num_ffn; ++f) {
      if (mask & (1u << f))
        copy_row(reinterpret_cast<__nv_bfloat16*>(p.tok_ptrs[f]) + tok_off * p.H, hbuf + (size_t)i * p.H, p.H);
      if (p.moe && threadIdx.x < p.k) {
        reinterpret_cast<int32_t*>(p.rid_ptrs[f])[tok_off * p.k + threadIdx.x] = s_id[i][threadIdx.x];
        reinterpret_cast<float*>(p.rwt_ptrs[f])[tok_off * p.k + threadIdx.x] = s_w[i][threadIdx.x];
      }
    }
    if (threadIdx.x == 0) p.fmask[t] = (int32_t)mask;
  }

  // ---- completion: the last CTA publishes counts and arrives at every FFN rank
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(p.done_ctr, 1u) == gridDim.x - 1);
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    for (int f = 0; f < p.num_ffn; ++f) atomicExch_system(reinterpret_cast<int*>(p.tcount_ptrs[f]) + p.attn_rank, p.T);
    *p.done_ctr = 0u;
    __threadfence_system();
    for (int f = 0; f < p.num_ffn; ++f)
      red_release_sys_add(reinterpret_cast<uint64_t*>(p.flag_ptrs[f]) + p.layer, 1ull);
  }
}

// One CTA per (source, token): copy the row into every local expert segment it
// routes to.  Counters start at zero (cleared after the previous use).
__global__ void __launch_bounds__(kThreads) expand_kernel(ExpandParams p) {
  __shared__ int s_row[kMaxK];
  if (blockIdx.x == 0 && threadIdx.x < p.ratio) p.counts[p.e_local + threadIdx.x] = p.tcount[p.home_a0 + threadIdx.x];
  if (!p.moe) return;
  const __nv_bfloat16* tok = static_cast<const __nv_bfloat16*>(p.tok);
  __nv_bfloat16* x = static_cast<__nv_bfloat16*>(p.x);
  for (int pair = blockIdx.x; pair < p.A * p.t_cap; pair += gridDim.x) {
    const int a = pair / p.t_cap, t = pair % p.t_cap;
    if (t >= p.tcount[a]) continue;
    const size_t base = (size_t)pair * p.k;
    if (threadIdx.x < p.k) {
      const int le = p.rid[base + threadIdx.x] - p.e_offset;
      int row = -1;
      if (le >= 0 && le < p.e_local) {
        const int slot = atomicAdd(&p.counts[le], 1);
        if (slot < p.cap) {
          row = le * p.cap + slot;
          p.meta[row] = (a << 24) | (t << 8) | threadIdx.x;
          p.rw[row] = p.rwt[base + threadIdx.x];
        } else {
          atomicExch(p.status, kStatusBadIndex);
        }
      }
      s_row[threadIdx.x] = row;
    }
    __syncthreads();
    for (int j = 0; j < p.k; ++j)
      if (s_row[j] >= 0) copy_row(x + (size_t)s_row[j] * p.H, tok + (size_t)pair * p.H, p.H);
    __syncthreads();
  }
}

// One CTA per (source, token): sum this rank's slots for the token and store
// the row into the source's combine slot [t][f_rank].
__global__ void __launch_bounds__(kThreads) combine_send_kernel(CombineSendParams p) {
  __shared__ float s_w[kMaxK + 1];
  __shared__ int s_any;
  __shared__ int s_last;
  const int VN = 8;
  const int nv = p.H / VN;
  for (int pair = blockIdx.x; pair < p.A * p.t_cap; pair += gridDim.x) {
    const int a = pair / p.t_cap, t = pair % p.t_cap;
    if (t >= p.tcount[a]) continue;
    const bool home = p.has_shared && a >= p.home_a0 && a < p.home_a0 + p.ratio;
    if (threadIdx.x == 0) s_any = home ? 1 : 0;
    __syncthreads();
    if (threadIdx.x <= p.k) {
      float w = 0.f;  // weight of a slot this rank filled (1, or the routing weight in echo mode)
      if (threadIdx.x < p.k) {
        if (p.moe) {
          const int le = p.rid[(size_t)pair * p.k + threadIdx.x] - p.e_offset;
          if (le >= 0 && le < p.e_local) {
            w = p.echo ? p.rwt[(size_t)pair * p.k + threadIdx.x] : 1.f;
            atomicOr(&s_any, 1);
          }
        }
      } else {
        w = home ? 1.f : 0.f;
      }
      s_w[threadIdx.x] = w;
    }
    __syncthreads();
    if (s_any) {
      __nv_bfloat16* dst =
          reinterpret_cast<__nv_bfloat16*>(p.dst_ptrs[a]) + ((size_t)t * p.num_ffn + p.f_rank) * p.H;
      if (p.echo) {
        float wsum = 0.f;
        for (int j = 0; j <= p.k; ++j) wsum += s_w[j];
        const __nv_bfloat16* row = static_cast<const __nv_bfloat16*>(p.staging) + (size_t)pair * p.H;
        for (int v = threadIdx.x; v < nv; v += kThreads) {
          Vec16<__nv_bfloat16> x = load16(row + v * VN);
#pragma unroll
          for (int q = 0; q < VN; ++q) x.v[q] = __float2bfloat16_rn(__bfloat162float(x.v[q]) * wsum);
          store16(dst + v * VN, x);
        }
      } else {
        const __nv_bfloat16* st = static_cast<const __nv_bfloat16*>(p.staging) + (size_t)pair * p.J * p.H;
        for (int v = threadIdx.x; v < nv; v += kThreads) {
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int j = 0; j < p.J; ++j) {
            if (s_w[j] == 0.f) continue;
            Vec16<__nv_bfloat16> x = load16(st + (size_t)j * p.H + v * VN);
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(x.v[q]);
          }
          Vec16<__nv_bfloat16> o;
#pragma unroll
          for (int q = 0; q < 8; ++q) o.v[q] = __float2bfloat16_rn(acc[q]);
          store16(dst + v * VN, o);
        }
      }
    }
    __syncthreads();
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(p.done_ctr, 1u) == gridDim.x - 1);
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *p.done_ctr = 0u;
    __threadfence_system();
    for (int a = 0; a < p.A; ++a) red_release_sys_add(reinterpret_cast<uint64_t*>(p.flag_ptrs[a]) + p.layer, 1ull);
  }
}

// out[t] = sum of the FFN slots that answer token t.
__global__ void __launch_bounds__(kThreads) combine_kernel(CombineParams p) {
  __shared__ bool ok;
  if (threadIdx.x == 0) ok = wait_flag(p.flag + p.layer, (*p.epoch) * p.arrivals, p.timeout_ns);
  __syncthreads();
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(p.status, kStatusWaitTimeout);
    return;
  }
  const int VN = 8;
  const int nv = p.H / VN;
  for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
    const unsigned mask = (unsigned)p.fmask[t];
    const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(p.comb) + (size_t)t * p.F * p.H;
    for (int v = threadIdx.x; v < nv; v += kThreads) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int f = 0; f < p.F; ++f) {
        if (!(mask & (1u << f))) continue;
        Vec16<__nv_bfloat16> x = load16(base + (size_t)f * p.H + v * VN);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(x.v[q]);
      }
      Vec16<__nv_bfloat16> o;
#pragma unroll
      for (int q = 0; q < 8; ++q) o.v[q] = __float2bfloat16_rn(acc[q]);
      store16(static_cast<__nv_bfloat16*>(p.out) + (size_t)t * p.H + v * VN, o);
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

void launch_afd_dispatch(const DispatchParams& p, cudaStream_t s) {
  const int grid = std::max(1, (p.T + fused::kTPC - 1) / fused::kTPC);
  const size_t smem = (size_t)fused::kTPC * p.H * 2 + (size_t)fused::kTPC * p.E * 4;
  static size_t attr = 0;
  if (smem > 48 * 1024 && smem > attr) {
    cudaFuncSetAttribute(fused::dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = smem;
  }
  fused::dispatch_kernel<<<grid, fused::kThreads, smem, s>>>(p);
}

static int pair_grid(int pairs) { return std::max(1, std::min(pairs, 148 * 8)); }

void launch_afd_expand(const ExpandParams& p, cudaStream_t s) {
  fused::expand_kernel<<<pair_grid(p.A * p.t_cap), fused::kThreads, 0, s>>>(p);
}

void launch_afd_combine_send(const CombineSendParams& p, cudaStream_t s) {
  fused::combine_send_kernel<<<pair_grid(p.A * p.t_cap), fused::kThreads, 0, s>>>(p);
}

void launch_afd_combine(const CombineParams& p, cudaStream_t s) {
  const int grid = std::max(1, std::min(p.T, 148 * 4));
  fused::combine_kernel<<<grid, fused::kThreads, 0, s>>>(p);
}
