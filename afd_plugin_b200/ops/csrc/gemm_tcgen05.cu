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

#include <type_traits>

#include "common.cuh"
#include "launchers.h"

namespace afd {
PFN_cuTensorMapEncodeTiled_v12000 get_tensor_map_encoder();

namespace gg {

constexpr int kBK = 64;            // K per stage (128 B of bf16)
constexpr int kBM = 128;           // weight rows per CTA (MMA M)
constexpr int kSub = 64;           // tokens per A sub-tile
constexpr int kMaxSub = 4;         // tokens per pass <= 256 (MMA N)
constexpr int kStages = 4;
constexpr int kThreads = 6 * 32;
constexpr int kWBytes = kBM * kBK * 2;          // 16 KB
constexpr int kSubBytes = kSub * kBK * 2;       // 8 KB
constexpr int kABytes = kMaxSub * kSubBytes;    // 32 KB
constexpr uint32_t kTmemCols = 256;

struct Smem {
  alignas(1024) uint8_t w[kStages][kWBytes];
  alignas(1024) uint8_t a[kStages][kABytes];
  float xchg[32 * 64];  // SwiGLU exchange: [col][row] for the 64 up rows
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint64_t acc_empty;
  uint32_t tmem_base;
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
AFD_DEVICE void scatter_arrive(const ScatterParams& sp) {
  __threadfence_system();
  if (atomicAdd(sp.done_ctr, 1u) == (unsigned)sp.total_ctas - 1) {
    for (int i = 0; i < sp.n_reset; ++i) sp.counts_reset[i] = 0;
    *sp.done_ctr = 0u;
    __threadfence_system();
    for (int a = 0; a < sp.num_dst; ++a)
      asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(reinterpret_cast<uint64_t*>(sp.flag_ptrs[a]) +
                                                                     sp.layer),
                   "l"(1ull)
                   : "memory");
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(
    const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap a_map,
    __nv_bfloat16* __restrict__ d, const int32_t* __restrict__ offsets, const int32_t* __restrict__ counts, int n_w,
    int w_stride_rows, int k_dim, int ld_d, int* __restrict__ status, const ScatterParams sp) {
  const int e = blockIdx.y;
  const int cnt = counts[e];
  if (cnt == 0) {
    if (EPI == 2 && threadIdx.x == 0) scatter_arrive(sp);
    return;
  }
  const int seg = offsets[e];
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int nt = blockIdx.x;
  const int kb_total = k_dim / kBK;
  const int n_pass = (cnt + kMaxSub * kSub - 1) / (kMaxSub * kSub);
  // Weight rows of this tile (two 64-row halves).
  int w_row0, w_row1;
  if (EPI == 1) {
    const int inter = n_w / 2;
    w_row0 = e * w_stride_rows + nt * 64;
    w_row1 = e * w_stride_rows + inter + nt * 64;
  } else {
    w_row0 = e * w_stride_rows + nt * kBM;
    w_row1 = w_row0 + 64;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
    mbar_init(&sm.acc_empty, 4);
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
  bool ok = true;

  if (warp == 0) {
    // ----------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&w_map);
      prefetch_tensormap(&a_map);
      int it = 0;
      for (int p = 0; p < n_pass && ok; ++p) {
        const int rows_left = cnt - p * kMaxSub * kSub;
        const int n_sub = min(kMaxSub, (rows_left + kSub - 1) / kSub);
        for (int kb = 0; kb < kb_total; ++kb, ++it) {
          const int st = it % kStages;
          if (it >= kStages && !mbar_wait_bounded(&sm.empty[st], ((it / kStages) - 1) & 1)) {
            atomicExch(status, kStatusWaitTimeout);
            ok = false;
            break;
          }
          mbar_expect_tx(&sm.full[st], kWBytes + n_sub * kSubBytes);
          tma_load_2d(sm.w[st], &w_map, &sm.full[st], kb * kBK, w_row0);
          tma_load_2d(sm.w[st] + kWBytes / 2, &w_map, &sm.full[st], kb * kBK, w_row1);
          for (int s = 0; s < n_sub; ++s)
            tma_load_2d(sm.a[st] + s * kSubBytes, &a_map, &sm.full[st], kb * kBK,
                        seg + p * kMaxSub * kSub + s * kSub);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0;
      for (int p = 0; p < n_pass && ok; ++p) {
        const int rows_left = cnt - p * kMaxSub * kSub;
        const int n_sub = min(kMaxSub, (rows_left + kSub - 1) / kSub);
        const uint32_t idesc = make_idesc(kBM, n_sub * kSub);
        if (p > 0 && !mbar_wait_bounded(&sm.acc_empty, (p - 1) & 1)) {
          atomicExch(status, kStatusWaitTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < kb_total; ++kb, ++it) {
          const int st = it % kStages;
          if (!mbar_wait_bounded(&sm.full[st], (it / kStages) & 1)) {
            atomicExch(status, kStatusWaitTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t wa = smem_u32(sm.w[st]);
          const uint32_t aa = smem_u32(sm.a[st]);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma(tmem, make_desc(wa + kk * 32), make_desc(aa + kk * 32), idesc, (kb | kk) != 0);
          umma_commit(&sm.empty[st]);
        }
        if (ok) umma_commit(&sm.acc_full);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;           // TMEM lanes 32*quarter .. +31
    const int row = quarter * 32 + lane;    // weight row within the tile
    for (int p = 0; p < n_pass; ++p) {
      if (!mbar_wait_bounded(&sm.acc_full, p & 1)) {
        atomicExch(status, kStatusWaitTimeout);
        break;
      }
      tc_fence_after();
      const int rows_left = cnt - p * kMaxSub * kSub;
      const int n_cols = min(kMaxSub * kSub, rows_left);
      const int r_base = seg + p * kMaxSub * kSub;
      for (int c0 = 0; c0 < n_cols; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + c0, v);
        if (EPI == 0) {
          const int col = nt * kBM + row;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < n_cols) d[(size_t)(r_base + c0 + j) * ld_d + col] = __float2bfloat16_rn(v[j]);
        } else if (EPI == 2) {
          // routing weight applied, row stored into the source rank's slot (peer memory)
          const int col = nt * kBM + row;
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
            const int col = nt * 64 + row;
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
      tc_fence_before();
      if (lane == 0) mbar_arrive(&sm.acc_empty);
    }
    if (EPI == 2) {
      __threadfence_system();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (warp == 2 && lane == 0) scatter_arrive(sp);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

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

void launch_grouped_gemm(void* d, const void* a, const void* w, const int32_t* expert_offsets,
                         const int32_t* expert_counts, int e_local, int rows_cap, int n, int k, int epilogue,
                         int* status, cudaStream_t s, int w_experts, const ScatterParams* sp) {
  if (w_experts < 0) w_experts = e_local;
  CUtensorMap wmap, amap;
  gg::encode_2d(&wmap, w, (uint64_t)w_experts * n, k, 64);
  gg::encode_2d(&amap, a, rows_cap, k, gg::kSub);
  const int smem = (int)sizeof(gg::Smem) + 1024;
  const int w_stride = (w_experts == 1) ? 0 : n;
  ScatterParams none{};
  const ScatterParams& spv = sp ? *sp : none;
  auto go = [&](auto epi_tag, dim3 grid, int ld) {
    constexpr int EPI = decltype(epi_tag)::value;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(gg::grouped_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      set = true;
    }
    gg::grouped_gemm_kernel<EPI><<<grid, gg::kThreads, smem, s>>>(wmap, amap, (__nv_bfloat16*)d, expert_offsets,
                                                                    expert_counts, n, w_stride, k, ld, status, spv);
  };
  if (epilogue == 1) {
    go(std::integral_constant<int, 1>{}, dim3((n / 2) / 64, e_local), n / 2);
  } else if (epilogue == 2) {
    go(std::integral_constant<int, 2>{}, dim3(n / gg::kBM, e_local), n);
  } else {
    go(std::integral_constant<int, 0>{}, dim3(n / gg::kBM, e_local), n);
  }
}
