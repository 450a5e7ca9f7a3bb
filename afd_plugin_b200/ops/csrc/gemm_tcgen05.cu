// Grouped expert GEMM on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// For every local expert e with a row segment [off_e, off_e + cnt_e) of the
// activation matrix A [rows, K]:   D[r, n] = sum_k A[r, k] * W[e, n, k].
// Decode batches give a handful of tokens per expert, so the product is
// computed transposed ("swap AB"): the 128-row weight tile is the MMA's M
// operand and the expert's tokens (<= 256 per pass) are its N operand, so each
// weight byte is streamed from HBM exactly once per pass.
//
// CTA = (128 weight rows, expert).  Warp roles:
//   warp 0  TMA producer: W tile (128 x 64) + up to four 64-token A tiles per
//           stage into 128B-swizzled shared memory, mbarrier transaction counts;
//   warp 1  TMEM allocator and single-thread MMA issuer (tcgen05.mma kind::f16,
//           fp32 accumulators in TMEM, tcgen05.commit frees each stage);
//   warps 2-5  epilogue: tcgen05.ld TMEM -> registers -> global.
// Epilogue 1 fuses SwiGLU: the weight tile holds 64 gate rows and the matching
// 64 up rows, and the output is silu(gate) * up.
//
// Every wait is bounded; on expiry the CTA records kStatusWaitTimeout and
// winds down (TMEM is always released).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <type_traits>

#include <cuda_fp8.h>

#include "common.cuh"
#include "device_state.h"
#include "launchers.h"

namespace afd {
PFN_cuTensorMapEncodeTiled_v12000 get_tensor_map_encoder();

namespace gg {

constexpr int kBK = 64;            // K per stage (128 B of bf16)
constexpr int kBM = 128;           // weight rows per CTA (MMA M)
constexpr int kSub = 64;           // tokens per A sub-tile
constexpr int kThreads = 6 * 32;
constexpr int kWBytes = kBM * kBK * 2;          // 16 KB
constexpr int kSubBytes = kSub * kBK * 2;       // 8 KB

// Pipeline: a ring of STAGES stages, each one weight tile (128 rows x 64 K,
// 16 KB) plus SUB activation sub-tiles (64 tokens x 64 K, 8 KB each, adjacent
// so one MMA of N = 64 * n_sub covers them).  A pass covers SUB * 64 tokens
// of an expert; wider segments take several passes over its weights.  The
// shapes instantiated trade pass width for weight bytes in flight per SM:
// (4 stages, 256 tokens), (6, 128) and (8, 64).
constexpr uint32_t kAccCols = 256;              // one accumulator: 128 lanes x up to 256 fp32 columns
constexpr uint32_t kTmemCols = 2 * kAccCols;    // two accumulators

template <int STAGES, int SUB>
struct Smem {
  alignas(1024) uint8_t w[STAGES][kWBytes];
  alignas(1024) uint8_t a[STAGES][SUB * kSubBytes];
  float xchg[32 * 64];  // SwiGLU exchange: [col][row] for the 64 up rows
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int last_split;
};

// K-major, 128B-swizzled operand descriptor (8-row groups 1024 B apart).
AFD_DEVICE uint64_t make_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;              // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;    // stride byte offset
  d |= (uint64_t)1 << 46;              // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;              // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both K-major.
AFD_DEVICE uint32_t make_idesc(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

AFD_DEVICE void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
AFD_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
AFD_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
AFD_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

AFD_DEVICE void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

AFD_DEVICE uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Scatter epilogue bookkeeping: every CTA of the layer arrives once; the last
// one clears the local expert counters and signals every Attention rank.
// Local destinations (num_dst == 0) need device-scope ordering only.
AFD_DEVICE void scatter_arrive(const ScatterParams& sp) {
  if (sp.num_dst > 0) __threadfence_system(); else __threadfence();
  if (atomicAdd(sp.done_ctr, 1u) == (unsigned)sp.total_ctas - 1) {
    for (int i = 0; i < sp.n_reset; ++i) sp.counts_reset[i] = 0;
    *sp.done_ctr = 0u;
    if (sp.num_dst > 0) __threadfence_system(); else __threadfence();
    for (int a = 0; a < sp.num_dst; ++a)
      asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(reinterpret_cast<uint64_t*>(sp.flag_ptrs[a]) +
                                                                     sp.layer),
                   "l"(1ull)
                   : "memory");
  }
}

// Work item = (expert e, weight tile nt); items are ordered expert-major so the
// CTAs working on one expert at the same time share its activation tiles in L2.
struct Item {
  int e, nt, cnt, seg;
};

AFD_DEVICE bool next_item(int& idx, int n_items, int n_tiles, const int32_t* counts, const int32_t* offsets,
                          Item& it) {
  for (; idx < n_items; idx += gridDim.x) {
    const int e = idx / n_tiles;
    const int c = counts[e];
    if (c > 0) {
      it.e = e;
      it.nt = idx % n_tiles;
      it.cnt = c;
      it.seg = offsets[e];
      idx += gridDim.x;
      return true;
    }
  }
  return false;
}

// AND of `pred` over the 128 epilogue threads (named barrier 1).
AFD_DEVICE bool bar_red_and_epilogue(bool pred) {
  uint32_t out;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(out)
      : "r"((uint32_t)pred)
      : "memory");
  return out != 0;
}

// Acquire load of a device-scope counter written by other CTAs of this grid.
AFD_DEVICE int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Later async-proxy (TMA) reads of global memory see generic-proxy writes made
// visible to this thread before the fence.
AFD_DEVICE void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Work item of a (possibly two-phase) launch: phase, expert, weight tile.
// Items are numbered phase-major, then expert-major, so the CTAs working on
// one expert at the same time share its activation tiles in L2, and every
// phase-1 item comes after all phase-0 items.
struct PItem {
  int ph, e, nt, cnt, seg, kb0, kb1;  // K blocks [kb0, kb1) of the weight rows
};

AFD_DEVICE bool next_phase_item(int& idx, const GGArgs& g, int n0, int n_all, PItem& it) {
  for (; idx < n_all; idx += gridDim.x) {
    const int ph = idx < n0 ? 0 : 1;
    const GGPhase& P = g.ph[ph];
    const int j = ph ? idx - n0 : idx;
    const int per_e = P.n_tiles * P.k_splits;
    const int e = j / per_e;
    const int c = P.counts ? P.counts[e] : P.fixed_count;
    if (c > 0) {
      const int rem = j - e * per_e;
      const int ks = rem % P.k_splits;
      const int kb_total = P.k_dim / kBK;
      it.ph = ph;
      it.e = e;
      it.nt = rem / P.k_splits;
      it.cnt = c;
      it.seg = P.offsets ? P.offsets[e] : 0;
      it.kb0 = ks * P.kb_per;
      it.kb1 = min(kb_total, it.kb0 + P.kb_per);
      idx += gridDim.x;
      return true;
    }
  }
  return false;
}

// Persistent grouped GEMM: one CTA per SM walks its work items; the TMA
// producer runs ahead across item boundaries, the accumulator is double
// buffered in TMEM so the epilogue of one item overlaps the MMAs of the next.
//
// Two-phase launches (an MoE layer's gate_up -> SwiGLU -> down in one kernel):
// phase 1 reads phase 0's output.  Every phase-0 item adds one to its
// expert's counter once its rows are stored; a phase-1 item of expert e waits
// (bounded) until all of e's phase-0 tiles are counted, then reads them with
// TMA.  Items are handed out phase-major in a fixed order, so a waiting CTA
// only waits for items that come earlier and never wait themselves: the wait
// always ends.  One launch keeps the SMs busy across the phase boundary (no
// kernel boundary, no tail of the first GEMM), and the intermediate rows stay
// in L2.  The last CTA to finish clears the counters for the next launch.
template <int STAGES, int SUB>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(
    const __grid_constant__ CUtensorMap w_map0, const __grid_constant__ CUtensorMap a_map0,
    const __grid_constant__ CUtensorMap w_map1, const __grid_constant__ CUtensorMap a_map1,
    const __grid_constant__ GGArgs g, const ScatterParams sp) {
  constexpr int kPassRows = SUB * kSub;
  extern __shared__ uint8_t smem_raw[];
  using SmemT = Smem<STAGES, SUB>;
  SmemT& sm = *reinterpret_cast<SmemT*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int n0 = g.ph[0].n_tiles * g.ph[0].k_splits * g.ph[0].n_experts;
  const int n_all = n0 + (g.n_phases > 1 ? g.ph[1].n_tiles * g.ph[1].k_splits * g.ph[1].n_experts : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // Set-up above overlaps the previous kernel; everything below reads its results.
  pdl_wait();
  pdl_launch_dependents();

  // Rows of the 128-row weight tile: [r0, r0 + 64) and [r1, r1 + 64).  SwiGLU
  // tiles pair 64 gate rows with the matching 64 up rows.
  auto w_rows = [&](const PItem& it, int& r0, int& r1) {
    const GGPhase& P = g.ph[it.ph];
    if (P.epi == 1) {
      r0 = it.e * P.w_stride_rows + it.nt * 64;
      r1 = it.e * P.w_stride_rows + P.n_w / 2 + it.nt * 64;
    } else {
      r0 = it.e * P.w_stride_rows + it.nt * kBM;
      r1 = r0 + 64;
    }
  };

  if (warp == 0) {
    // ----------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&w_map0);
      prefetch_tensormap(&a_map0);
      if (g.n_phases > 1) {
        prefetch_tensormap(&w_map1);
        prefetch_tensormap(&a_map1);
      }
      int it_count = 0, idx = blockIdx.x;
      PItem it;
      bool ok = true;
      const uint64_t pol_keep = l2_policy_evict_last(), pol_stream = l2_policy_evict_first();
      while (ok && next_phase_item(idx, g, n0, n_all, it)) {
        const GGPhase& P = g.ph[it.ph];
        const CUtensorMap* wm = it.ph ? &w_map1 : &w_map0;
        const CUtensorMap* am = it.ph ? &a_map1 : &a_map0;
        if (it.ph == 1 && g.ph[0].done != nullptr) {
          // this expert's phase-0 rows: wait until every tile of them is stored
          const int need = g.ph[0].n_tiles;
          const uint64_t t0 = globaltimer_ns();
          while (ld_acquire_gpu(g.ph[0].done + it.e) < need) {
            if ((int64_t)(globaltimer_ns() - t0) > g.dep_timeout_ns) {
              atomicExch(g.status, kStatusWaitTimeout);
              ok = false;
              break;
            }
            __nanosleep(128);
          }
          if (!ok) break;
          fence_proxy_async_global();
        }
        int r0, r1;
        w_rows(it, r0, r1);
        const int n_pass = (it.cnt + kPassRows - 1) / kPassRows;
        for (int p = 0; p < n_pass && ok; ++p) {
          const int n_sub = min(SUB, (it.cnt - p * kPassRows + kSub - 1) / kSub);
          for (int kb = it.kb0; kb < it.kb1; ++kb, ++it_count) {
            const int st = it_count % STAGES;
            if (!mbar_wait_bounded(&sm.empty[st], ((it_count / STAGES) & 1) ^ 1)) {
              atomicExch(g.status, kStatusWaitTimeout);
              ok = false;
              break;
            }
            mbar_expect_tx(&sm.full[st], kWBytes + n_sub * kSubBytes);
            // A weight tile read by several passes (a segment wider than a pass,
            // e.g. a shared-expert chunk that sees every token) stays in L2 for
            // the next pass; one read once is the first to leave.
            if (g.l2_hints) {
              const uint64_t pol = n_pass > 1 ? pol_keep : pol_stream;
              tma_load_2d_hint(sm.w[st], wm, &sm.full[st], kb * kBK, r0, pol);
              tma_load_2d_hint(sm.w[st] + kWBytes / 2, wm, &sm.full[st], kb * kBK, r1, pol);
            } else {
              tma_load_2d(sm.w[st], wm, &sm.full[st], kb * kBK, r0);
              tma_load_2d(sm.w[st] + kWBytes / 2, wm, &sm.full[st], kb * kBK, r1);
            }
            for (int s2 = 0; s2 < n_sub; ++s2) {
              const int arow = it.seg + p * kPassRows + s2 * kSub;
              if (P.a3d)
                tma_load_3d(sm.a[st] + s2 * kSubBytes, am, &sm.full[st], kb * kBK, arow, it.e);
              else
                tma_load_2d(sm.a[st] + s2 * kSubBytes, am, &sm.full[st], kb * kBK, arow);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it_count = 0, acc_count = 0, idx = blockIdx.x;
      int fail_ab = 0, fail_par = 0;  // the accumulator barrier whose phase a timeout leaves open
      PItem it;
      bool ok = true;
      while (ok && next_phase_item(idx, g, n0, n_all, it)) {
        const int n_pass = (it.cnt + kPassRows - 1) / kPassRows;
        for (int p = 0; p < n_pass && ok; ++p, ++acc_count) {
          const int n_sub = min(SUB, (it.cnt - p * kPassRows + kSub - 1) / kSub);
          const uint32_t idesc = make_idesc(kBM, n_sub * kSub);
          const int ab = acc_count & 1;
          fail_ab = ab;
          fail_par = (acc_count >> 1) & 1;
          if (!mbar_wait_bounded(&sm.acc_empty[ab], ((acc_count >> 1) & 1) ^ 1)) {
            atomicExch(g.status, kStatusWaitTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tacc = tmem + ab * kAccCols;
          for (int kb = it.kb0; kb < it.kb1; ++kb, ++it_count) {
            const int st = it_count % STAGES;
            if (!mbar_wait_bounded(&sm.full[st], (it_count / STAGES) & 1)) {
              atomicExch(g.status, kStatusWaitTimeout);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t wa = smem_u32(sm.w[st]);
            const uint32_t aa = smem_u32(sm.a[st]);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma(tacc, make_desc(wa + kk * 32), make_desc(aa + kk * 32), idesc, ((kb - it.kb0) | kk) != 0);
            umma_commit(&sm.empty[st]);
          }
          if (ok) umma_commit(&sm.acc_full[ab]);
        }
      }
      if (!ok) {
        // a commit's arrival marks every MMA issued before it complete: wait (bounded)
        // for it so that no MMA still writes TMEM when the CTA deallocates it
        umma_commit(&sm.acc_full[fail_ab]);
        mbar_wait_bounded(&sm.acc_full[fail_ab], fail_par);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;           // TMEM lanes 32*quarter .. +31
    const int row = quarter * 32 + lane;    // weight row within the tile
    int acc_count = 0, idx = blockIdx.x;
    PItem it;
    bool ok = true;
    while (ok && next_phase_item(idx, g, n0, n_all, it)) {
      const GGPhase& P = g.ph[it.ph];
      const int epi = P.epi;
      __nv_bfloat16* __restrict__ d = P.d;
      const int ld_d = P.ld_d;
      const int n_pass = (it.cnt + kPassRows - 1) / kPassRows;
      for (int p = 0; p < n_pass; ++p, ++acc_count) {
        const int ab = acc_count & 1;
        // The four epilogue warps agree on the outcome of the bounded wait, so
        // the named barriers below are reached by all of them or by none.
        ok = bar_red_and_epilogue(mbar_wait_bounded(&sm.acc_full[ab], (acc_count >> 1) & 1));
        if (!ok) {
          if (lane == 0) atomicExch(g.status, kStatusWaitTimeout);
          break;
        }
        tc_fence_after();
        const int n_cols = min(kPassRows, it.cnt - p * kPassRows);
        const int r_base = it.seg + p * kPassRows;
        const uint32_t tacc = tmem + ab * kAccCols + ((uint32_t)(quarter * 32) << 16);
        for (int c0 = 0; c0 < n_cols; c0 += 32) {
          float v[32];
          tmem_ld32(tacc + c0, v);
          if (P.k_splits > 1) {
            // partial sum of this K slice: fp32 atomics into the tile's workspace rows
            const int col = it.nt * kBM + row + (epi == 3 ? it.e * P.n_w : 0);
            const int rb = epi == 3 ? r_base - it.seg : r_base;
            if (epi == 3 || col < P.n_valid) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (c0 + j < n_cols) atomicAdd(P.acc_ws + (size_t)(rb + c0 + j) * ld_d + col, v[j]);
            }
          } else if (epi == 0 && P.out_f32) {
            const int col = it.nt * kBM + row;
            float* df = reinterpret_cast<float*>(d);
            if (col < P.n_valid) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (c0 + j < n_cols) df[(size_t)(r_base + c0 + j) * ld_d + col] = v[j];
            }
          } else if (epi == 0 || epi == 3) {
            // epilogue 3: rows relative to the segment, columns in the expert's block
            const int col = it.nt * kBM + row + (epi == 3 ? it.e * P.n_w : 0);
            const int rb = epi == 3 ? r_base - it.seg : r_base;
            if (epi == 3 || col < P.n_valid) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (c0 + j < n_cols) d[(size_t)(rb + c0 + j) * ld_d + col] = __float2bfloat16_rn(v[j]);
            }
          } else if (epi == 2) {
            // routing weight applied, row stored into the source rank's slot
            const int col = it.nt * kBM + row;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (c0 + j < n_cols) {
                const int r = r_base + c0 + j;
                const int m = sp.meta[r];
                const int src = (m >> 24) & 0xFF, tok = (m >> 8) & 0xFFFF, slot = m & 0xFF;
                __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(sp.dst_ptrs[src]);
                dst[((size_t)tok * sp.J + slot) * sp.H + col] = __float2bfloat16_rn(sp.rw[r] * v[j]);
              }
            }
          } else {
            if (quarter >= 2) {
#pragma unroll
              for (int j = 0; j < 32; ++j) sm.xchg[j * 64 + (row - 64)] = v[j];
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (quarter < 2) {
              const int col = it.nt * 64 + row;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (c0 + j < n_cols) {
                  const float gt = v[j];
                  const float u = sm.xchg[j * 64 + row];
                  d[(size_t)(r_base + c0 + j) * ld_d + col] = __float2bfloat16_rn(gt / (1.f + __expf(-gt)) * u);
                }
              }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
          }
        }
        tc_fence_before();
        if (lane == 0) mbar_arrive(&sm.acc_empty[ab]);
      }
      if (ok && P.k_splits > 1) {
        // the last K slice of a tile to finish turns the fp32 sums into the output
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (warp == 2 && lane == 0) {
          int* ctr = P.tile_ctr + it.e * P.n_tiles + it.nt;
          const int last = atomicAdd(ctr, 1) == P.k_splits - 1;
          if (last) *ctr = 0;
          sm.last_split = last;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (sm.last_split) {
          __threadfence();
          const int col = it.nt * kBM + row + (epi == 3 ? it.e * P.n_w : 0);
          const int rb = epi == 3 ? 0 : it.seg;
          if (epi == 3 || col < P.n_valid) {
            for (int r = 0; r < it.cnt; ++r) {
              float* src = P.acc_ws + (size_t)(rb + r) * ld_d + col;
              const float x = __ldcg(src);
              __stcg(src, 0.f);
              if (P.out_f32)
                reinterpret_cast<float*>(d)[(size_t)(rb + r) * ld_d + col] = x;
              else
                d[(size_t)(rb + r) * ld_d + col] = __float2bfloat16_rn(x);
            }
          }
        }
      }
      if (ok && P.done != nullptr) {
        // this tile's rows are stored: count it for the expert's phase-1 items
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (warp == 2 && lane == 0) atomicAdd(P.done + it.e, 1);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
  if (threadIdx.x == 0) {
    // Every role of this CTA is done reading counts and storing rows.
    if (g.ph[0].done != nullptr) {
      __threadfence();
      if (atomicAdd(g.finish_ctr, 1u) == gridDim.x - 1) {
        for (int e = 0; e < g.ph[0].n_experts; ++e) g.ph[0].done[e] = 0;
        *g.finish_ctr = 0u;
        __threadfence();
      }
    }
    if (g.ph[0].epi == 2 || (g.n_phases > 1 && g.ph[1].epi == 2)) scatter_arrive(sp);
  }
}

// ===================================================================== fp8 weights
// Block-scaled fp8 (e4m3) weights with bf16 activations ("W8A16"): TMA streams
// 128-row x 128-K fp8 weight tiles (half the HBM bytes of bf16), twelve
// converter warps dequantise each tile with its 128 x 128 block scale into two
// 128B-swizzled bf16 tiles in shared memory, and the tcgen05 MMA reads those.
// Warp roles: 0 TMA producer, 1 TMEM + MMA issuer, 2-5 epilogue, 6-17 converter.
// Decode gives a few tokens per expert, so a pass takes 64 tokens and the
// shared memory goes to pipeline depth (4 TMA stages) and to the converted ring.
namespace gg8 {

constexpr int kBK = 128;                       // K per stage (one fp8 row = 128 B)
constexpr int kBM = 128;
constexpr int kSub = 64;
constexpr int kMaxSub = 1;                     // tokens per pass <= 64
constexpr int kStages = 4;
constexpr int kCvt = 2;
constexpr int kCvtWarps = 12;
constexpr int kCvtThreads = kCvtWarps * 32;
constexpr int kThreads = (6 + kCvtWarps) * 32;
constexpr int kWBytes = kBM * kBK;             // 16 KB fp8
constexpr int kWcHalf = kBM * 64 * 2;          // 16 KB: 128 rows x 64 K bf16
constexpr int kSubBytes = kSub * 64 * 2;       // 8 KB: 64 tokens x 64 K bf16
constexpr int kAHalf = kMaxSub * kSubBytes;    // 16 KB: one K half of the A stage
constexpr uint32_t kAccCols = 128;
constexpr uint32_t kTmemCols = 256;

struct Smem {
  alignas(1024) uint8_t w[kStages][kWBytes];
  alignas(1024) uint8_t a[kStages][2 * kAHalf];
  alignas(1024) uint8_t wc[kCvt][2 * kWcHalf];
  float xchg[32 * 64];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t cfull[kCvt];
  uint64_t cempty[kCvt];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
};

// Two fp32 products in one packed multiply (sm_100 mul.f32x2).
AFD_DEVICE float2 mul_f32x2(float2 a, float s) {
  uint64_t x = ((uint64_t)__float_as_uint(a.y) << 32) | __float_as_uint(a.x);
  const uint64_t ss = ((uint64_t)__float_as_uint(s) << 32) | __float_as_uint(s);
  uint64_t y;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(y) : "l"(x), "l"(ss));
  return make_float2(__uint_as_float((uint32_t)y), __uint_as_float((uint32_t)(y >> 32)));
}

AFD_DEVICE uint4 cvt16(uint4 raw, float scale, uint4& hi) {
  // 16 e4m3 values -> 16 bf16 (scaled); returns the first 8, `hi` the last 8.
  // Per pair: e4m3x2 -> f16x2 (exact), f16 -> f32 (exact), one packed fp32
  // multiply by the block scale, one rounding to bf16x2.
  const uint32_t in[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t pair = (__nv_fp8x2_storage_t)(h ? (in[i] >> 16) : (in[i] & 0xFFFFu));
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
      __half2 h2;
      *reinterpret_cast<__half2_raw*>(&h2) = hr;
      const float2 f = mul_f32x2(__half22float2(h2), scale);
      out[i * 2 + h] = pack_bf16(f.x, f.y);
    }
  }
  hi = make_uint4(out[4], out[5], out[6], out[7]);
  return make_uint4(out[0], out[1], out[2], out[3]);
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_w8_kernel(
    const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap a_map,
    const float* __restrict__ w_scale, __nv_bfloat16* __restrict__ d, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ counts, int n_w, int w_stride_rows, int k_dim, int ld_d, int n_tiles, int n_experts,
    int w_experts, int* __restrict__ status, const ScatterParams sp, int l2_hints) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int kb_total = k_dim / kBK;
  const int n_items = n_tiles * n_experts;
  constexpr int kPassRows = kMaxSub * kSub;
  const int nblk_n = (n_w + 127) / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int c = 0; c < kCvt; ++c) {
      mbar_init(&sm.cfull[c], kCvtThreads);
      mbar_init(&sm.cempty[c], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  gg::tc_fence_before();
  __syncthreads();
  gg::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_wait();
  pdl_launch_dependents();

  // rows of the 128-row weight tile: [r0, r0 + 64) and [r1, r1 + 64)
  auto w_rows = [&](const gg::Item& it, int& r0, int& r1) {
    if (EPI == 1) {
      r0 = it.nt * 64;
      r1 = n_w / 2 + it.nt * 64;
    } else {
      r0 = it.nt * kBM;
      r1 = r0 + 64;
    }
  };

  if (warp == 0) {
    // ----------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&w_map);
      prefetch_tensormap(&a_map);
      int it_count = 0, idx = blockIdx.x;
      gg::Item it;
      bool ok = true;
      const uint64_t pol_keep = l2_policy_evict_last(), pol_stream = l2_policy_evict_first();
      while (ok && gg::next_item(idx, n_items, n_tiles, counts, offsets, it)) {
        int r0, r1;
        w_rows(it, r0, r1);
        const int wb = it.e * w_stride_rows;
        const int n_pass = (it.cnt + kPassRows - 1) / kPassRows;
        for (int p = 0; p < n_pass && ok; ++p) {
          const int n_sub = min(kMaxSub, (it.cnt - p * kPassRows + kSub - 1) / kSub);
          for (int kb = 0; kb < kb_total; ++kb, ++it_count) {
            const int st = it_count % kStages;
            if (!mbar_wait_bounded(&sm.empty[st], ((it_count / kStages) & 1) ^ 1)) {
              atomicExch(status, kStatusWaitTimeout);
              ok = false;
              break;
            }
            mbar_expect_tx(&sm.full[st], kWBytes + 2 * n_sub * kSubBytes);
            // as in the bf16 kernel: weight tiles of a single pass leave L2 first
            if (l2_hints) {
              const uint64_t pol = n_pass > 1 ? pol_keep : pol_stream;
              tma_load_2d_hint(sm.w[st], &w_map, &sm.full[st], kb * kBK, wb + r0, pol);
              tma_load_2d_hint(sm.w[st] + kWBytes / 2, &w_map, &sm.full[st], kb * kBK, wb + r1, pol);
            } else {
              tma_load_2d(sm.w[st], &w_map, &sm.full[st], kb * kBK, wb + r0);
              tma_load_2d(sm.w[st] + kWBytes / 2, &w_map, &sm.full[st], kb * kBK, wb + r1);
            }
            for (int h = 0; h < 2; ++h)
              for (int s2 = 0; s2 < n_sub; ++s2)
                tma_load_2d(sm.a[st] + h * kAHalf + s2 * kSubBytes, &a_map, &sm.full[st], kb * kBK + h * 64,
                            it.seg + p * kPassRows + s2 * kSub);
          }
        }
      }
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------- converter
    const int ct = threadIdx.x - 6 * 32;  // 0 .. kCvtThreads - 1
    int it_count = 0, idx = blockIdx.x;
    gg::Item it;
    bool ok = true;
    while (ok && gg::next_item(idx, n_items, n_tiles, counts, offsets, it)) {
      int r0, r1;
      w_rows(it, r0, r1);
      const int ew = w_experts == 1 ? 0 : it.e;
      const float* sc_lo = w_scale + ((size_t)ew * nblk_n + r0 / 128) * kb_total;
      const float* sc_hi = w_scale + ((size_t)ew * nblk_n + r1 / 128) * kb_total;
      const int n_pass = (it.cnt + kPassRows - 1) / kPassRows;
      for (int p = 0; p < n_pass && ok; ++p) {
        // the block scales of the next K block load while this one converts
        float s_lo = sc_lo[0], s_hi = sc_hi[0];
        for (int kb = 0; kb < kb_total; ++kb, ++it_count) {
          const int st = it_count % kStages;
          const int cs = it_count % kCvt;
          const int kn = kb + 1 < kb_total ? kb + 1 : kb;
          const float s_lo_next = sc_lo[kn], s_hi_next = sc_hi[kn];
          if (!mbar_wait_bounded(&sm.full[st], (it_count / kStages) & 1) ||
              !mbar_wait_bounded(&sm.cempty[cs], ((it_count / kCvt) & 1) ^ 1)) {
            atomicExch(status, kStatusWaitTimeout);
            ok = false;
            break;
          }
          const uint8_t* src = sm.w[st];
          uint8_t* dst = sm.wc[cs];
#pragma unroll
          for (int q = ct; q < kBM * 8; q += kCvtThreads) {
            const int r = q >> 3, c = q & 7;
            const uint4 raw = *reinterpret_cast<const uint4*>(src + r * 128 + ((c ^ (r & 7)) << 4));
            uint4 hi;
            const uint4 lo = cvt16(raw, r < 64 ? s_lo : s_hi, hi);
            uint8_t* tile = dst + (c >> 2) * kWcHalf + r * 128;
            // Chunks 0-3 of a source row go to the first K half, 4-7 to the
            // second (16 KB apart, the same banks): the second half stores its
            // odd chunk first, so each store instruction writes eight distinct
            // 16-byte bank groups per row.
            const int d0 = (c & 3) * 2;
            const bool h1 = c >= 4;
            *reinterpret_cast<uint4*>(tile + (((h1 ? d0 + 1 : d0) ^ (r & 7)) << 4)) = h1 ? hi : lo;
            *reinterpret_cast<uint4*>(tile + (((h1 ? d0 : d0 + 1) ^ (r & 7)) << 4)) = h1 ? lo : hi;
          }
          s_lo = s_lo_next;
          s_hi = s_hi_next;
          fence_proxy_async();
          mbar_arrive(&sm.cfull[cs]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it_count = 0, acc_count = 0, idx = blockIdx.x;
      int fail_ab = 0, fail_par = 0;  // the accumulator barrier whose phase a timeout leaves open
      gg::Item it;
      bool ok = true;
      while (ok && gg::next_item(idx, n_items, n_tiles, counts, offsets, it)) {
        const int n_pass = (it.cnt + kPassRows - 1) / kPassRows;
        for (int p = 0; p < n_pass && ok; ++p, ++acc_count) {
          // N = this pass's tokens rounded up to 16 (the MMA reads the first
          // N rows of the 64-row activation tile)
          const int n_tok = min(kPassRows, it.cnt - p * kPassRows);
          const uint32_t idesc = gg::make_idesc(kBM, (n_tok + 15) / 16 * 16);
          const int ab = acc_count & 1;
          fail_ab = ab;
          fail_par = (acc_count >> 1) & 1;
          if (!mbar_wait_bounded(&sm.acc_empty[ab], ((acc_count >> 1) & 1) ^ 1)) {
            atomicExch(status, kStatusWaitTimeout);
            ok = false;
            break;
          }
          gg::tc_fence_after();
          const uint32_t tacc = tmem + ab * kAccCols;
          for (int kb = 0; kb < kb_total; ++kb, ++it_count) {
            const int st = it_count % kStages;
            const int cs = it_count % kCvt;
            if (!mbar_wait_bounded(&sm.full[st], (it_count / kStages) & 1) ||
                !mbar_wait_bounded(&sm.cfull[cs], (it_count / kCvt) & 1)) {
              atomicExch(status, kStatusWaitTimeout);
              ok = false;
              break;
            }
            gg::tc_fence_after();
            const uint32_t wa = smem_u32(sm.wc[cs]);
            const uint32_t aa = smem_u32(sm.a[st]);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const int h = kk >> 2;
              gg::umma(tacc, gg::make_desc(wa + h * kWcHalf + (kk & 3) * 32),
                       gg::make_desc(aa + h * kAHalf + (kk & 3) * 32), idesc, (kb | kk) != 0);
            }
            gg::umma_commit(&sm.empty[st]);
            gg::umma_commit(&sm.cempty[cs]);
          }
          if (ok) gg::umma_commit(&sm.acc_full[ab]);
        }
      }
      if (!ok) {
        // drain the issued MMAs before the CTA deallocates TMEM (see the bf16 kernel)
        gg::umma_commit(&sm.acc_full[fail_ab]);
        mbar_wait_bounded(&sm.acc_full[fail_ab], fail_par);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int acc_count = 0, idx = blockIdx.x;
    gg::Item it;
    bool ok = true;
    while (ok && gg::next_item(idx, n_items, n_tiles, counts, offsets, it)) {
      const int n_pass = (it.cnt + kPassRows - 1) / kPassRows;
      for (int p = 0; p < n_pass; ++p, ++acc_count) {
        const int ab = acc_count & 1;
        if (!mbar_wait_bounded(&sm.acc_full[ab], (acc_count >> 1) & 1)) {
          atomicExch(status, kStatusWaitTimeout);
          ok = false;
          break;
        }
        gg::tc_fence_after();
        const int n_cols = min(kPassRows, it.cnt - p * kPassRows);
        const int r_base = it.seg + p * kPassRows;
        const uint32_t tacc = tmem + ab * kAccCols + ((uint32_t)(quarter * 32) << 16);
        for (int c0 = 0; c0 < n_cols; c0 += 32) {
          float v[32];
          gg::tmem_ld32(tacc + c0, v);
          if (EPI == 0) {
            const int col = it.nt * kBM + row;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (c0 + j < n_cols) d[(size_t)(r_base + c0 + j) * ld_d + col] = __float2bfloat16_rn(v[j]);
          } else if (EPI == 2) {
            const int col = it.nt * kBM + row;
#pragma unroll 4
            for (int j = 0; j < 32; ++j) {
              if (c0 + j < n_cols) {
                const int r = r_base + c0 + j;
                const int m = sp.meta[r];
                const int src = (m >> 24) & 0xFF, tok = (m >> 8) & 0xFFFF, slot = m & 0xFF;
                __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(sp.dst_ptrs[src]);
                dst[((size_t)tok * sp.J + slot) * sp.H + col] = __float2bfloat16_rn(sp.rw[r] * v[j]);
              }
            }
          } else {
            if (quarter >= 2) {
#pragma unroll
              for (int j = 0; j < 32; ++j) sm.xchg[j * 64 + (row - 64)] = v[j];
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (quarter < 2) {
              const int col = it.nt * 64 + row;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (c0 + j < n_cols) {
                  const float g = v[j];
                  const float u = sm.xchg[j * 64 + row];
                  d[(size_t)(r_base + c0 + j) * ld_d + col] = __float2bfloat16_rn(g / (1.f + __expf(-g)) * u);
                }
              }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
          }
        }
        gg::tc_fence_before();
        if (lane == 0) mbar_arrive(&sm.acc_empty[ab]);
      }
    }
    if (EPI == 2) {
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (warp == 2 && lane == 0) gg::scatter_arrive(sp);
    }
  }
  gg::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    gg::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

}  // namespace gg8

static void encode_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {kBK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  get_tensor_map_encoder()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace gg
}  // namespace afd

using namespace afd;

int grouped_gemm_grid(int n_items) {
  const int sms = device_sm_count();
  return n_items < sms ? (n_items > 0 ? n_items : 1) : sms;
}

namespace {

// Activation map: rows of K elements a_ld apart, or (a_plane > 0) one plane
// of rows_cap rows per expert, a_plane elements apart.
void encode_activations(CUtensorMap* map, const GemmSpec& g) {
  const uint64_t ld = g.a_ld > 0 ? (uint64_t)g.a_ld : (uint64_t)g.k;
  if (g.a_plane <= 0 && ld == (uint64_t)g.k) {
    gg::encode_2d(map, g.a, g.rows_cap, g.k, gg::kSub);
    return;
  }
  const int rank = g.a_plane > 0 ? 3 : 2;
  const cuuint64_t dims[3] = {(cuuint64_t)g.k, (cuuint64_t)g.rows_cap, (cuuint64_t)g.e_local};
  const cuuint64_t strides[2] = {ld * 2, (cuuint64_t)(g.a_plane > 0 ? g.a_plane : 0) * 2};
  const cuuint32_t box[3] = {gg::kBK, gg::kSub, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  get_tensor_map_encoder()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(g.a), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

GGPhase make_phase(const GemmSpec& g, CUtensorMap* wmap, CUtensorMap* amap) {
  const int w_experts = g.w_experts < 0 ? g.e_local : g.w_experts;
  gg::encode_2d(wmap, g.w, (uint64_t)w_experts * g.n, g.k, 64);
  encode_activations(amap, g);
  GGPhase P{};
  P.a3d = g.a_plane > 0 ? 1 : 0;
  P.fixed_count = g.fixed_count;
  P.out_f32 = g.out_f32;
  P.n_valid = g.n_valid > 0 ? g.n_valid : g.n;
  const int kb_total = g.k / gg::kBK;
  P.k_splits = (g.k_splits > 1 && g.acc_ws && g.tile_ctr) ? min(g.k_splits, kb_total) : 1;
  P.kb_per = (kb_total + P.k_splits - 1) / P.k_splits;
  P.k_splits = (kb_total + P.kb_per - 1) / P.kb_per;  // no empty slices
  P.acc_ws = g.acc_ws;
  P.tile_ctr = g.tile_ctr;
  P.d = static_cast<__nv_bfloat16*>(g.d);
  P.offsets = g.offsets;
  P.counts = g.counts;
  P.done = nullptr;
  P.n_w = g.n;
  P.w_stride_rows = (w_experts == 1) ? 0 : g.n;
  P.k_dim = g.k;
  P.n_experts = g.e_local;
  P.epi = g.epilogue;
  if (g.epilogue == 1) {
    P.n_tiles = (g.n / 2) / 64;
    P.ld_d = g.n / 2;
  } else {
    P.n_tiles = g.n / gg::kBM;
    P.ld_d = g.epilogue == 3 ? g.n * g.e_local : (g.n_valid > 0 ? g.n_valid : g.n);
  }
  return P;
}

template <int STAGES, int SUB>
cudaError_t launch_kernel(const CUtensorMap& w0, const CUtensorMap& a0, const CUtensorMap& w1, const CUtensorMap& a1,
                          const GGArgs& args, const ScatterParams& sp, int n_items, cudaStream_t s) {
  const int smem = (int)sizeof(gg::Smem<STAGES, SUB>) + 1024;
  static PerDeviceOnce attr;
  cudaError_t e = attr.run([&] {
    return cudaFuncSetAttribute(gg::grouped_gemm_kernel<STAGES, SUB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem);
  });
  if (e != cudaSuccess) return e;
  const int grid = grouped_gemm_grid(n_items);
  return launch_pdl(gg::grouped_gemm_kernel<STAGES, SUB>, dim3(grid), dim3(gg::kThreads), (size_t)smem, s, w0, a0,
                    w1, a1, args, sp);
}

// Tokens per pass for a launch whose segments are expected to need rows_hint
// rows per pass.  Measured on B200 at decode shapes: 64-token passes (8
// stages) stream routed experts fastest (0.92-0.99 of HBM); with a few
// whole-batch segments among them (shared-expert chunks) 128-token passes (6
// stages) win even though those segments take two passes (callers pass 128
// then); 256-token passes (4 stages) suit dense GEMMs over a 256-row batch.
// AFD_GG_PIPE=64|128|256 forces one shape for experiments.
int pipe_rows(int rows_hint) {
  static const int forced = [] {
    const char* v = std::getenv("AFD_GG_PIPE");
    const int r = v ? std::atoi(v) : 0;
    return (r == 64 || r == 128 || r == 256) ? r : 0;
  }();
  if (forced) return forced;
  if (rows_hint <= 64) return 64;
  return rows_hint <= 128 ? 128 : 256;
}

}  // namespace

int grouped_gemm_launch_grid(int n_items) { return grouped_gemm_grid(n_items); }

cudaError_t launch_grouped_gemm_phases(const GemmSpec& g0, const GemmSpec* g1, int* done, unsigned* finish_ctr,
                                       int* status, const ScatterParams* sp, cudaStream_t s, int rows_hint) {
  CUtensorMap w0, a0, w1, a1;
  GGArgs args{};
  args.ph[0] = make_phase(g0, &w0, &a0);
  args.n_phases = 1;
  if (g1 != nullptr) {
    args.ph[1] = make_phase(*g1, &w1, &a1);
    args.n_phases = 2;
    args.ph[0].done = done;
  } else {
    w1 = w0;
    a1 = a0;
  }
  args.status = status;
  args.finish_ctr = finish_ctr;
  args.dep_timeout_ns = 2000000000ll;  // 2 s: phase-0 tiles of an expert are minutes' worth of margin away
  args.l2_hints = (l2_hint_mask() & kL2HintGemm) ? 1 : 0;
  ScatterParams none{};
  const ScatterParams& spv = sp ? *sp : none;
  int n_items = args.ph[0].n_tiles * args.ph[0].k_splits * args.ph[0].n_experts;
  if (g1 != nullptr) n_items += args.ph[1].n_tiles * args.ph[1].k_splits * args.ph[1].n_experts;
  switch (pipe_rows(rows_hint)) {
    case 64:
      return launch_kernel<8, 1>(w0, a0, w1, a1, args, spv, n_items, s);
    case 128:
      return launch_kernel<6, 2>(w0, a0, w1, a1, args, spv, n_items, s);
    default:
      return launch_kernel<4, 4>(w0, a0, w1, a1, args, spv, n_items, s);
  }
}

void launch_grouped_gemm(void* d, const void* a, const void* w, const int32_t* expert_offsets,
                         const int32_t* expert_counts, int e_local, int rows_cap, int n, int k, int epilogue,
                         int* status, cudaStream_t s, int w_experts, const ScatterParams* sp) {
  GemmSpec g{d, a, w, expert_offsets, expert_counts, e_local, rows_cap, n, k, epilogue, w_experts};
  launch_grouped_gemm_phases(g, nullptr, nullptr, nullptr, status, sp, s);
}


void launch_grouped_gemm_w8(void* d, const void* a, const void* w, const float* w_scale, const int32_t* expert_offsets,
                            const int32_t* expert_counts, int e_local, int rows_cap, int n, int k, int epilogue,
                            int* status, cudaStream_t s, int w_experts, const ScatterParams* sp) {
  if (w_experts < 0) w_experts = e_local;
  CUtensorMap wmap, amap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)w_experts * n};
    const cuuint64_t strides[1] = {(cuuint64_t)k};
    const cuuint32_t box[2] = {gg::gg8::kBK, 64};
    const cuuint32_t estr[2] = {1, 1};
    get_tensor_map_encoder()(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  gg::encode_2d(&amap, a, rows_cap, k, gg::gg8::kSub);
  const int smem = (int)sizeof(gg::gg8::Smem) + 1024;
  const int w_stride = (w_experts == 1) ? 0 : n;
  ScatterParams none{};
  const ScatterParams& spv = sp ? *sp : none;
  auto go = [&](auto epi_tag, int n_tiles, int ld) {
    constexpr int EPI = decltype(epi_tag)::value;
    static PerDeviceOnce attr;
    attr.run([&] {
      return cudaFuncSetAttribute(gg::gg8::grouped_gemm_w8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  smem);
    });
    const int grid = grouped_gemm_grid(n_tiles * e_local);
    launch_pdl(gg::gg8::grouped_gemm_w8_kernel<EPI>, dim3(grid), dim3(gg::gg8::kThreads), (size_t)smem, s, wmap, amap, w_scale,
               (__nv_bfloat16*)d, expert_offsets, expert_counts, n, w_stride, k, ld, n_tiles, e_local, w_experts,
               status, spv, (l2_hint_mask() & kL2HintGemm) ? 1 : 0);
  };
  if (epilogue == 1) {
    go(std::integral_constant<int, 1>{}, (n / 2) / 64, n / 2);
  } else if (epilogue == 2) {
    go(std::integral_constant<int, 2>{}, n / gg::gg8::kBM, n);
  } else {
    go(std::integral_constant<int, 0>{}, n / gg::gg8::kBM, n);
  }
}
