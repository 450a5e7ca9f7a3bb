// One-shot all-reduce over NVLink peer memory for tensor-parallel attention
// (the row-parallel o_proj's partial outputs), in place on a [rows, H] bf16
// tensor.
//
// Every rank owns, in its symmetric heap, W slots per parity (one per source
// rank) and a flag per (CTA, source).  CTA c of rank r takes rows
// [c * rows_per_cta, ...):
//   1. push: stores its rows into slot r of every rank's heap (plain 16-byte
//      stores; its own slot is local), for the call's parity (epoch & 1);
//   2. release: one system-scope fence, then flag[c][r] = epoch on every rank;
//   3. wait: flag[c][p] >= epoch for every source p (bounded by the device
//      clock; on expiry the status word records a timeout and the rows are
//      left as the local partial);
//   4. sum: out = sum over p of slot p, accumulated in fp32, rounded once.
// The last CTA to finish advances the epoch (a device counter, so the
// launch replays from a CUDA graph).  Slots alternate by parity: a rank can
// only write slot set e+1 of a peer after that peer's call e flag, i.e. after
// the peer has finished reading slot set e-1.
//
// Peer pointers are dereferenced only by plain ld/st/red instructions.
#include <algorithm>

#include "common.cuh"
#include "device_state.h"
#include "launchers.h"

namespace afd {
namespace tpar {

constexpr int kThreads = 256;
using bf16 = __nv_bfloat16;

AFD_DEVICE uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
AFD_DEVICE void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
AFD_DEVICE void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads) tp_allreduce_kernel(TPAllReduceParams p) {
  __shared__ int s_ok;
  const uint64_t epoch = *p.epoch;
  const int par = (int)(epoch & 1);
  const int row0 = blockIdx.x * p.rows_per_cta;
  const int row1 = min(p.rows, row0 + p.rows_per_cta);
  const int nv = p.H / 8;  // 16-byte vectors per row
  bf16* x = p.x;
  // 1. push this CTA's rows into slot [par][rank] of every rank
  for (int i = threadIdx.x; i < (row1 - row0) * nv; i += kThreads) {
    const int r = row0 + i / nv, v = i % nv;
    const uint4 val = *reinterpret_cast<const uint4*>(x + (size_t)r * p.H + v * 8);
    for (int q = 0; q < p.world; ++q) {
      bf16* slot = reinterpret_cast<bf16*>(p.slot_ptrs[q]) + ((size_t)par * p.world + p.rank) * p.slot_elems;
      *reinterpret_cast<uint4*>(slot + (size_t)r * p.H + v * 8) = val;
    }
  }
  __syncthreads();
  // 2. release: the stores above (bar.sync puts them under this thread's fence)
  if (threadIdx.x == 0) {
    fence_sys();
    for (int q = 0; q < p.world; ++q)
      st_release_sys(reinterpret_cast<uint64_t*>(p.flag_ptrs[q]) + (size_t)blockIdx.x * p.world + p.rank, epoch);
    // 3. every source's rows for this CTA
    bool ok = true;
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < p.world && ok; ++q) {
      const uint64_t* f = p.local_flags + (size_t)blockIdx.x * p.world + q;
      while (ld_acquire_sys(f) < epoch) {
        if ((int64_t)(globaltimer_ns() - t0) > p.timeout_ns) {
          ok = false;
          break;
        }
        __nanosleep(32);
      }
    }
    if (!ok) atomicExch(p.status, kStatusWaitTimeout);
    s_ok = ok;
  }
  __syncthreads();
  // 4. sum the slots (local memory) in fp32
  if (s_ok) {
    const bf16* base = p.local_slots + (size_t)par * p.world * p.slot_elems;
    for (int i = threadIdx.x; i < (row1 - row0) * nv; i += kThreads) {
      const int r = row0 + i / nv, v = i % nv;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int q = 0; q < p.world; ++q) {
        const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(base + (size_t)q * p.slot_elems + (size_t)r * p.H + v * 8));
        const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(e[j]);
      }
      uint4 out;
      uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        o[j] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      *reinterpret_cast<uint4*>(x + (size_t)r * p.H + v * 8) = out;
    }
  }
  // the last CTA advances the epoch for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.done_ctr, 1u) == gridDim.x - 1) {
      *p.done_ctr = 0u;
      *p.epoch = epoch + 1;
    }
  }
}

}  // namespace tpar
}  // namespace afd

using namespace afd;

int tp_allreduce_rows_per_cta(int rows, int max_ctas) {
  // one row per CTA while the flag table has a row of flags for each
  return std::max(1, (rows + max_ctas - 1) / max_ctas);
}

cudaError_t launch_tp_allreduce(const TPAllReduceParams& p, cudaStream_t s) {
  if (p.rows <= 0) return cudaSuccess;
  const int grid = (p.rows + p.rows_per_cta - 1) / p.rows_per_cta;
  tpar::tp_allreduce_kernel<<<grid, tpar::kThreads, 0, s>>>(p);
  return cudaGetLastError();
}
