// Fused Attention<->FFN transfer kernels over NVLink peer memory.
//
// afd_dispatch  (Attention side, one kernel per layer and ubatch)
//   residual += attn_out; h = RMSNorm(residual) * w           (post-attn norm)
//   logits = h . gate^T; (weight, expert) = top-k routing      (router)
//   for every routed (token, k): claim a row of the owning FFN rank's
//   per-expert receive segment with a system-scope atomic on that rank's
//   counter, then store h (bf16, 16-byte stores) plus (source, token, slot)
//   metadata and the routing weight straight into the peer's memory.  The
//   token is also stored once into its home FFN rank's shared-expert /
//   dense-MLP segment.  The last CTA publishes the shared-segment count and
//   bumps every FFN rank's arrival counter (release, system scope).
// afd_wait      one thread spins (bounded by globaltimer) until a counter
//               reaches epoch * arrivals (acquire, system scope).
// afd_combine   (Attention side) waits for every FFN rank's arrival and sums
//               the k routed slots + the shared slot of each token.
// afd_epoch     bumps the per-step epoch that all counters are compared to.
//
// Counters only grow: the n-th step expects epoch n times the number of
// arriving ranks, so graphs replay without resetting them.  No wait is
// unbounded: on expiry the kernel records kStatusWaitTimeout and returns.
#include "common.cuh"
#include "launchers.h"
#include "routing.cuh"

namespace afd {
namespace fused {

constexpr int kTPC = 4;         // tokens per dispatch CTA
constexpr int kThreads = 256;
constexpr int kMaxSlots = 17;   // top-k (<= 16) + one shared/dense slot

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
  __shared__ int s_row[kTPC][kMaxSlots];
  __shared__ int s_dst[kTPC][kMaxSlots];
  __shared__ float s_w[kTPC][kMaxSlots];
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
    // ---- top-k per token, one warp each
    if (warp < nt) {
      float w;
      int id;
      warp_route(logits + warp * p.E, p.gate_bias, p.E, p.k, p.scoring, p.renorm, p.n_group, p.topk_group, p.scale,
                 w, id);
      if (lane < p.k) {
        const int f = id / p.e_local, le = id % p.e_local;
        // claim a row in the owner's segment for expert `le`
        int* cnt = reinterpret_cast<int*>(p.cnt_ptrs[f]);
        const int slot = atomicAdd_system(cnt + le, 1);
        s_row[warp][lane] = (slot < p.cap) ? le * p.cap + slot : -1;
        s_dst[warp][lane] = f;
        s_w[warp][lane] = w;
        if (slot >= p.cap) atomicExch(p.status, kStatusBadIndex);
      }
    }
  }
  const int n_route = p.moe ? p.k : 0;
  const int n_slots = n_route + (p.has_shared ? 1 : 0);
  if (threadIdx.x < nt && p.has_shared) {
    const int i = threadIdx.x;
    s_row[i][n_route] = p.e_local * p.cap + p.src_local * p.t_cap + (t0 + i);
    s_dst[i][n_route] = p.home_f;
    s_w[i][n_route] = 1.f;
  }
  __syncthreads();

  // ---- stores into the FFN ranks' receive segments (peer memory)
  for (int i = 0; i < nt; ++i) {
    for (int j = 0; j < n_slots; ++j) {
      const int row = s_row[i][j];
      if (row < 0) continue;
      const int f = s_dst[i][j];
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.x_ptrs[f]) + (size_t)row * p.H;
      for (int v = threadIdx.x; v < nv; v += kThreads) store16(dst + v * VN, load16(hbuf + (size_t)i * p.H + v * VN));
      if (threadIdx.x == 0) {
        const int slot_id = (j == n_route) ? p.k : j;  // shared/dense output lands in slot k
        reinterpret_cast<int32_t*>(p.meta_ptrs[f])[row] =
            ((p.attn_rank & 0xFF) << 24) | (((t0 + i) & 0xFFFF) << 8) | (slot_id & 0xFF);
        reinterpret_cast<float*>(p.w_ptrs[f])[row] = s_w[i][j];
      }
    }
  }

  // ---- completion: the last CTA publishes counts and arrives at every FFN rank
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(p.done_ctr, 1u) == gridDim.x - 1);
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    if (p.has_shared) {
      int* cnt = reinterpret_cast<int*>(p.cnt_ptrs[p.home_f]);
      atomicExch_system(cnt + p.e_local + p.src_local, p.T);
    }
    *p.done_ctr = 0u;
    __threadfence_system();
    for (int f = 0; f < p.num_ffn; ++f)
      red_release_sys_add(reinterpret_cast<uint64_t*>(p.flag_ptrs[f]) + p.layer, 1ull);
  }
}

// out[t] = sum of the token's routed slots and its shared slot.
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
    const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(p.comb) + (size_t)t * p.J * p.H;
    for (int v = threadIdx.x; v < nv; v += kThreads) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < p.n_routed; ++j) {
        Vec16<__nv_bfloat16> x = load16(base + (size_t)j * p.H + v * VN);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(x.v[q]);
      }
      if (p.shared_slot >= 0) {
        Vec16<__nv_bfloat16> x = load16(base + (size_t)p.shared_slot * p.H + v * VN);
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

// Transport-only FFN stand-in for connector benchmarks: every received row is
// weighted and stored back into its source rank's combine slot, exactly like
// the scatter epilogue of the expert GEMM but without the math.
__global__ void __launch_bounds__(kThreads) echo_kernel(EchoParams p) {
  __shared__ int s_last;
  const int VN = 8;
  const int nv = p.H / VN;
  const int n_seg = p.e_local + p.ratio;
  for (int seg = blockIdx.y; seg < n_seg; seg += gridDim.y) {
    const int cnt = p.counts[seg];
    const int row0 = seg < p.e_local ? seg * p.cap : p.e_local * p.cap + (seg - p.e_local) * p.t_cap;
    for (int i = blockIdx.x; i < cnt; i += gridDim.x) {
      const int r = row0 + i;
      const int m = p.meta[r];
      const int src = (m >> 24) & 0xFF, tok = (m >> 8) & 0xFFFF, slot = m & 0xFF;
      const float w = p.rw[r];
      const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.x) + (size_t)r * p.H;
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.dst_ptrs[src]) + ((size_t)tok * p.J + slot) * p.H;
      for (int v = threadIdx.x; v < nv; v += kThreads) {
        Vec16<__nv_bfloat16> a = load16(x + v * VN);
#pragma unroll
        for (int j = 0; j < VN; ++j) a.v[j] = __float2bfloat16_rn(__bfloat162float(a.v[j]) * w);
        store16(dst + v * VN, a);
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(p.done_ctr, 1u) == gridDim.x * gridDim.y - 1);
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    for (int i = 0; i < n_seg; ++i) p.counts[i] = 0;
    *p.done_ctr = 0u;
    __threadfence_system();
    for (int a = 0; a < p.num_dst; ++a)
      red_release_sys_add(reinterpret_cast<uint64_t*>(p.flag_ptrs[a]) + p.layer, 1ull);
  }
}

}  // namespace fused
}  // namespace afd

using namespace afd;

void launch_afd_echo(const EchoParams& p, cudaStream_t s) {
  fused::echo_kernel<<<dim3(16, 148), fused::kThreads, 0, s>>>(p);
}

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

void launch_afd_combine(const CombineParams& p, cudaStream_t s) {
  const int grid = std::max(1, std::min(p.T, 148 * 4));
  fused::combine_kernel<<<grid, fused::kThreads, 0, s>>>(p);
}
