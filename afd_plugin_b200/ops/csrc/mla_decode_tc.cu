// Absorbed-MLA paged decode on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA = (request b, group of HG heads, KV split); 64-token KV tiles
// (576 bf16 per token: 512 latent + 64 rope) stream into a two-stage ring by
// TMA (128B swizzle; one cache block of 64 tokens per tile).  Per tile:
//
//   S  = Q K^T      tcgen05.mma M=64 (the HG heads, padded), N=64 tokens,
//                   K=576: A = the query in shared memory, B = the tile
//                   (K-major).  S lands in TMEM with head h in lane
//                   32*(h/16) + h%16, one fp32 column per token.
//   softmax         one thread per head reads its 64 scores (tcgen05.ld),
//                   keeps the running max / sum in registers and writes
//                   P^T (heads x 64 tokens, bf16) into shared memory in the
//                   swizzled K-major layout the next MMA reads.
//   O^T += V^T P^T  tcgen05.mma M=128 latent rows (four blocks of 512),
//                   N=HG, K=64 tokens: A = the same KV tile read MN-major
//                   (latent contiguous), B = P^T.  O^T stays in TMEM for the
//                   whole split.
//
// The running max is raised lazily: O^T is rescaled (tcgen05.ld / st by the
// four softmax warps) only when a head's maximum grows by more than 2^8, so
// un-rescaled probabilities stay below 256 and fp32 accumulation is exact
// enough; the final normalisation uses the same (possibly stale) maximum.
//
// Warp roles: 0-3 softmax / O correction / epilogue (TMEM lanes 32w..32w+31),
// 4 TMA producer, 5 TMEM allocator and single-thread MMA issuer.  The MMA
// thread polls for whichever of S(t+1) (tile landed) and PV(t) (P written)
// is ready, so the softmax of one tile overlaps the next tile's QK^T on the
// tensor core and a stage is released as soon as its PV is done.  A split writes a
// normalised fp32 partial and its log-sum-exp; the last CTA of a (request,
// head group) merges them (per-group arrival counter, reset by that CTA).
//
// Every wait is bounded; on expiry the CTA records kStatusWaitTimeout, stops
// issuing work and still releases its TMEM.
//
// The decode op uses this kernel for layers with 64 or more heads (32 heads
// per CTA, where it measured faster than the mma.sync kernel of
// mla_decode.cu); with 16 heads per CTA the per-tile hand-offs between the
// MMA thread and the one softmax warp cost more than the mma.sync kernel's
// math, so 16-head groups stay there (see pick_shape).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "device_state.h"
#include "launchers.h"

namespace afd {
PFN_cuTensorMapEncodeTiled_v12000 get_tensor_map_encoder();

namespace mtc {

constexpr int kD = 576, kL = 512;
constexpr int kBoxes = kD / 64;                        // 9 column boxes of 128 B
constexpr int kThreads = 6 * 32;
constexpr int kSoftmaxThreads = 128;
constexpr float kRescaleLog2 = 8.f;                    // raise the max only past 2^8
// S = Q K^T can accumulate its 36 K-steps into kNA independent TMEM
// accumulators (boxes j, j + kNA, ...) that the softmax sums; three measured
// no faster than one on B200, so one is used.
constexpr int kNA = 1;

// Shapes: HG heads per CTA, TILE tokens per stage (32 or 64; a cache block
// holds whole tiles), STAGES stages in the ring.
template <int HG, int TILE, int STAGES>
struct Cfg {
  static constexpr int kBoxBytes = TILE * 128;                // one 64-column box of the tile
  static constexpr int kStageBytes = kBoxes * kBoxBytes;
  // TMEM columns: S buffers [2][kNA][TILE], then O^T [4 latent blocks][HG].
  static constexpr uint32_t kSStride = kNA * TILE;
  static constexpr uint32_t kOCol = 2 * kSStride;
  static constexpr uint32_t kUsed = kOCol + 4 * HG;
  static constexpr uint32_t kTmemCols = kUsed <= 32 ? 32 : kUsed <= 64 ? 64 : kUsed <= 128 ? 128 : kUsed <= 256 ? 256 : 512;
};

template <int HG, int TILE, int STAGES>
struct Smem {
  // The query is the M=64 operand: rows HG..63 of each box read past it (into
  // the following boxes or the KV stages) and only feed unused TMEM lanes.
  alignas(1024) uint8_t q[kBoxes * HG * 128];
  alignas(1024) uint8_t kv[STAGES][Cfg<HG, TILE, STAGES>::kStageBytes];
  alignas(1024) uint8_t p[2][HG * 128];  // P^T rows of 128 B (TILE tokens used)
  float alpha[HG];
  float inv_l[HG];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t o_done;  // one completion per PV issue
  uint64_t o_last;  // the last PV of the split
  uint64_t q_ready;
  uint32_t tmem_base;
  int rescale;
  int last;
};

AFD_DEVICE bool mbar_test_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// mbarrier wait bounded by the device clock (1 s): a protocol fault ends the
// CTA with an error status instead of spinning.
constexpr uint64_t kWaitNs = 1000000000ull;
AFD_DEVICE bool wait(uint64_t* bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, phase)) return true;
    if (globaltimer_ns() - t0 > kWaitNs) return false;
  }
}

// 128B-swizzled operand descriptor.  K-major: rows of 128 B, 8-row groups
// `sbo` apart (lbo unused).  MN-major: 64 contiguous MN elements per 128 B
// row, MN blocks of 64 `lbo` apart, 8-row K groups `sbo` apart.
AFD_DEVICE uint64_t desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32; a_mn: A is MN-major.
AFD_DEVICE uint32_t idesc_bf16(int m, int n, bool a_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

AFD_DEVICE void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
AFD_DEVICE void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
AFD_DEVICE void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
AFD_DEVICE void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 16 / 32 / 64 consecutive fp32 columns (one lane per thread).
template <int N>
AFD_DEVICE void tmem_ld(uint32_t taddr, float (&v)[N]);
template <>
AFD_DEVICE void tmem_ld<16>(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
AFD_DEVICE void tmem_ld<32>(uint32_t taddr, float (&v)[32]) {
  float a[16], b[16];
  tmem_ld<16>(taddr, a);
  tmem_ld<16>(taddr + 16, b);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = a[i];
    v[16 + i] = b[i];
  }
}
template <>
AFD_DEVICE void tmem_ld<64>(uint32_t taddr, float (&v)[64]) {
  uint32_t r[32];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr + 32 * h));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[32 * h + i] = __uint_as_float(r[i]);
  }
}
template <int N>
AFD_DEVICE void tmem_st(uint32_t taddr, const float (&v)[N]);
template <>
AFD_DEVICE void tmem_st<16>(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}

// The four softmax warps agree on a predicate (bar.red.and over 128 threads),
// so every named barrier after it is reached by all of them or by none.
AFD_DEVICE bool all128(bool pred) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.b32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.b32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((int)pred));
  return r != 0;
}
AFD_DEVICE bool any128(bool pred) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.b32 p, %1, 0;\n bar.red.or.pred q, 1, 128, p;\n selp.b32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((int)pred));
  return r != 0;
}
AFD_DEVICE void sync128() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Byte offset of (row, col) in a 128B-swizzled K-major tile of 128 B rows:
// 16-byte chunk index XOR (row % 8), 8-row groups 1024 B apart.
AFD_DEVICE uint32_t swz_row(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

// out[b, h, :] = sum_s w_s o_s with w_s = 2^(lse_s - max) / sum, for the HG
// heads of group hg (the last CTA to arrive; partials read through L2).
template <int HG>
AFD_DEVICE void merge_group(const MlaQO& qo, const float* part_o, const float* part_lse, int b, int hg, int heads,
                            int num_splits, int tid, float* wsm) {
  const float* pl = part_lse + (size_t)b * num_splits * heads + hg * HG;
  for (int i = tid; i < num_splits * HG; i += kSoftmaxThreads) wsm[i] = __ldcg(pl + (size_t)(i / HG) * heads + i % HG);
  sync128();
  if (tid < HG) {
    float mx = -INFINITY;
    for (int sp = 0; sp < num_splits; ++sp) mx = fmaxf(mx, wsm[sp * HG + tid]);
    float wsum = 0.f;
    for (int sp = 0; sp < num_splits; ++sp) {
      const float v = wsm[sp * HG + tid];
      const float w = (v == -INFINITY) ? 0.f : exp2f(v - mx);
      wsm[sp * HG + tid] = w;
      wsum += w;
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    for (int sp = 0; sp < num_splits; ++sp) wsm[sp * HG + tid] *= inv;
  }
  sync128();
  const int c = tid * 4;  // four latent columns per thread
  const float* base = part_o + ((size_t)b * num_splits * heads + (size_t)hg * HG) * kL + c;
#pragma unroll 1
  for (int h0 = 0; h0 < HG; h0 += 8) {
    float4 acc[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < num_splits; ++sp) {
      const float* ps = base + ((size_t)sp * heads + h0) * kL;
      float4 x[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) x[h] = __ldcg(reinterpret_cast<const float4*>(ps + (size_t)h * kL));
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        const float w = wsm[sp * HG + h0 + h];
        acc[h].x += w * x[h].x;
        acc[h].y += w * x[h].y;
        acc[h].z += w * x[h].z;
        acc[h].w += w * x[h].w;
      }
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      __nv_bfloat16* ob = qo.out + (size_t)b * qo.out_sb + (size_t)(hg * HG + h0 + h) * qo.out_sh + c;
      *reinterpret_cast<__nv_bfloat162*>(ob) = __floats2bfloat162_rn(acc[h].x, acc[h].y);
      *reinterpret_cast<__nv_bfloat162*>(ob + 2) = __floats2bfloat162_rn(acc[h].z, acc[h].w);
    }
  }
}

template <int HG, int TILE, int STAGES, int MIN_CTAS>
__global__ void __launch_bounds__(kThreads, MIN_CTAS) mla_decode_tc_kernel(
    const __grid_constant__ CUtensorMap kv_map, const MlaQO qo, const int32_t* __restrict__ block_table,
    const int32_t* __restrict__ seq_lens, float* __restrict__ part_o, float* __restrict__ part_lse,
    int* __restrict__ status, int heads, int block_size, int max_blocks, int num_splits, float scale_log2,
    int* __restrict__ arrivals) {
  static_assert(HG == 16 || HG == 32, "heads per CTA");
  static_assert(TILE == 32 || TILE == 64, "tokens per stage");
  constexpr uint32_t kQBox = HG * 128;
  constexpr int kTile = TILE, kStages = STAGES;
  constexpr int kBoxBytes = Cfg<HG, TILE, STAGES>::kBoxBytes;
  constexpr int kStageBytes = Cfg<HG, TILE, STAGES>::kStageBytes;
  constexpr uint32_t kSStride = Cfg<HG, TILE, STAGES>::kSStride;
  constexpr uint32_t kOCol = Cfg<HG, TILE, STAGES>::kOCol;
  constexpr uint32_t kTmemCols = Cfg<HG, TILE, STAGES>::kTmemCols;
  static_assert(Cfg<HG, TILE, STAGES>::kUsed <= 512, "TMEM columns");
  extern __shared__ uint8_t smem_raw[];
  using SmemT = Smem<HG, TILE, STAGES>;
  SmemT& sm = *reinterpret_cast<SmemT*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int b = blockIdx.x, hg = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int seq_len = seq_lens[b];
  const int n_tiles_total = (seq_len + kTile - 1) / kTile;
  const int tiles_per_split = (n_tiles_total + num_splits - 1) / num_splits;
  const int tile_begin = split * tiles_per_split;
  const int n_tiles = max(0, min(n_tiles_total, tile_begin + tiles_per_split) - tile_begin);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], 4);
      mbar_init(&sm.p_full[s], 1);
    }
    mbar_init(&sm.o_done, 1);
    mbar_init(&sm.o_last, 1);
    mbar_init(&sm.q_ready, 4);
    fence_barrier_init();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) prefetch_tensormap(&kv_map);
    int my_row = 0, issued = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int st = i % kStages;
      if ((i & 31) == 0) {  // cache rows of the next 32 tiles, one block-table load per lane
        const int ti = i + lane;
        if (ti < n_tiles) {
          const int t0 = (tile_begin + ti) * kTile;
          my_row = block_table[(size_t)b * max_blocks + t0 / block_size] * block_size + (t0 % block_size);
        }
      }
      const int row = __shfl_sync(0xffffffffu, my_row, i & 31);
      int ok = 1;
      if (lane == 0) ok = wait(&sm.empty[st], ((i / kStages) & 1) ^ 1);
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        if (lane == 0) atomicExch(status, kStatusWaitTimeout);
        break;
      }
      if (lane == 0) {
        mbar_expect_tx(&sm.full[st], kStageBytes);
#pragma unroll
        for (int bx = 0; bx < kBoxes; ++bx) tma_load_2d(sm.kv[st] + bx * kBoxBytes, &kv_map, &sm.full[st], bx * 64, row);
      }
      ++issued;
    }
    // No copy may still be landing in shared memory when the CTA exits (the
    // loads of a split that stopped early): wait, bounded, for the last ones.
    if (lane == 0)
      for (int i = max(0, issued - kStages); i < issued; ++i) wait(&sm.full[i % kStages], (i / kStages) & 1);
  } else if (warp == 5) {
    // ------------------------------------------------------- MMA issuer
    // Two kinds of work, issued as soon as each is ready (non-blocking polls):
    // S(t) = Q K^T once tile t has landed, and O^T += V^T P^T for tile u once
    // its P is written.  S(t) also waits until PV(t-2) is issued, so the
    // commit that announces S(t) covers PV(t-2): the softmax warps then know
    // at most PV(t-1) is outstanding when they wait to rescale O.
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16(64, kTile, false);
      const uint32_t idesc_o = idesc_bf16(128, HG, true);
      const uint32_t q_base = smem_u32(sm.q);
      bool ok = wait(&sm.q_ready, 0);
      int qk = 0, pv = 0;
      uint64_t idle_since = 0;
      while (ok && pv < n_tiles) {
        bool did = false;
        if (qk < n_tiles && qk <= pv + 1) {
          const int st = qk % kStages, sb = qk & 1;
          if (mbar_test_wait(&sm.full[st], (qk / kStages) & 1) &&
              mbar_test_wait(&sm.s_free[sb], ((qk >> 1) & 1) ^ 1)) {
            fence_after();
            const uint32_t kv = smem_u32(sm.kv[st]);
#pragma unroll 1
            for (int j = 0; j < kBoxes; ++j)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma(tmem + sb * kSStride + (j % kNA) * kTile, desc_sw128(q_base + j * kQBox + kk * 32, 16, 1024),
                    desc_sw128(kv + j * kBoxBytes + kk * 32, 16, 1024), idesc_s, (j >= kNA || kk != 0) ? 1u : 0u);
            commit(&sm.s_full[sb]);
            ++qk;
            did = true;
          }
        }
        if (pv < qk && mbar_test_wait(&sm.p_full[pv & 1], (pv >> 1) & 1)) {
          const int st = pv % kStages;
          fence_after();
          const uint32_t kv = smem_u32(sm.kv[st]);
          const uint32_t pb = smem_u32(sm.p[pv & 1]);
#pragma unroll
          for (int mb = 0; mb < 4; ++mb)
#pragma unroll
            for (int kk = 0; kk < kTile / 16; ++kk)
              mma(tmem + kOCol + mb * HG, desc_sw128(kv + 2 * mb * kBoxBytes + kk * 2048, kBoxBytes, 1024),
                  desc_sw128(pb + kk * 32, 16, 1024), idesc_o, (pv > 0 || kk > 0) ? 1u : 0u);
          commit(&sm.empty[st]);
          commit(&sm.o_done);
          ++pv;
          did = true;
        }
        if (did) {
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = globaltimer_ns();
        } else if (globaltimer_ns() - idle_since > kWaitNs) {
          ok = false;
        }
      }
      // The commit's arrival also marks every MMA issued so far complete: after
      // a timeout this thread waits (bounded) for it, so no MMA still writes
      // TMEM when the CTA deallocates it.
      commit(&sm.o_last);
      if (!ok) {
        atomicExch(status, kStatusWaitTimeout);
        wait(&sm.o_last, 0);
      }
    }
  } else {
    // ----------------------------------------- softmax / correction / epilogue
    const int tid = threadIdx.x;                 // 0..127 = TMEM lane
    const int h = (warp * 16) + lane;            // head of this thread's S lane (lane < 16)
    const bool owns_head = lane < 16 && h < HG;
    // Q (HG heads x 576) -> swizzled K-major boxes; the producer is already streaming.
    for (int c = tid; c < HG * (kD / 8); c += kSoftmaxThreads) {
      const int r = c / (kD / 8), col = (c % (kD / 8)) * 8;
      const int hh = hg * HG + r;
      const __nv_bfloat16* src = (col < kL) ? qo.q_lat + (size_t)b * qo.lat_sb + (size_t)hh * qo.lat_sh + col
                                            : qo.q_pe + (size_t)b * qo.pe_sb + (size_t)hh * qo.pe_sh + (col - kL);
      *reinterpret_cast<uint4*>(sm.q + (col >> 6) * kQBox + swz_row(r, (col & 63) >> 3)) =
          *reinterpret_cast<const uint4*>(src);
    }
    fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.q_ready);

    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
      const int sb = t & 1;
      ok = all128(wait(&sm.s_full[sb], (t >> 1) & 1));
      if (!ok) break;
      fence_after();
      float s[kTile];
      if (warp * 16 < HG) {
        const uint32_t ta = tmem + sb * kSStride + ((uint32_t)(warp * 32) << 16);
        tmem_ld<kTile>(ta, s);
#pragma unroll
        for (int a = 1; a < kNA; ++a) {
          float s2[kTile];
          tmem_ld<kTile>(ta + a * kTile, s2);
#pragma unroll
          for (int j = 0; j < kTile; ++j) s[j] += s2[j];
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free[sb]);
      float alpha = 1.f;
      bool rescale = false;
      if (owns_head) {
        const int tok0 = (tile_begin + t) * kTile;
        float mx[8];  // eight independent chains
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
#pragma unroll
        for (int j = 0; j < kTile; ++j) {
          s[j] = (tok0 + j < seq_len) ? s[j] * scale_log2 : -INFINITY;
          mx[j & 7] = fmaxf(mx[j & 7], s[j]);
        }
        const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        if (mt > m_run + kRescaleLog2 || m_run == -INFINITY) {
          const float m_new = fmaxf(mt, m_run);
          alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - m_new);
          rescale = t > 0;
          m_run = m_new;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        float ls[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) ls[c] = 0.f;
        uint8_t* prow = sm.p[sb] + (h >> 3) * 1024;
#pragma unroll
        for (int c = 0; c < kTile / 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float p0 = exp2f(s[8 * c + 2 * k] - m_use);
            const float p1 = exp2f(s[8 * c + 2 * k + 1] - m_use);
            ls[c] += p0 + p1;
            w[k] = pack_bf16(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + swz_row(h & 7, c)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l_run = l_run * alpha + (((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7])));
        sm.alpha[h] = alpha;
      }
      fence_proxy_async();  // P^T stores -> visible to the tensor core
      if (any128(rescale)) {
        // O^T (through tile t-1) times alpha per head column, once its last MMA is done.
        ok = all128(wait(&sm.o_done, (t - 1) & 1));
        if (!ok) break;
        fence_after();
#pragma unroll 1
        for (int mb = 0; mb < 4; ++mb) {
#pragma unroll
          for (int c0 = 0; c0 < HG; c0 += 16) {
            const uint32_t ta = tmem + kOCol + mb * HG + c0 + ((uint32_t)(warp * 32) << 16);
            float o[16];
            tmem_ld<16>(ta, o);
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] *= sm.alpha[c0 + j];
            tmem_st<16>(ta, o);
          }
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      }
      fence_before();
      sync128();
      if (tid == 0) mbar_arrive(&sm.p_full[sb]);
    }

    // ---- epilogue: O^T / l -> bf16 output, or a normalised fp32 partial
    if (owns_head) {
      sm.inv_l[h] = l_run > 0.f ? 1.f / l_run : 0.f;
      if (num_splits > 1)
        part_lse[((size_t)b * num_splits + split) * heads + hg * HG + h] =
            l_run > 0.f ? m_run + log2f(l_run) : -INFINITY;
    }
    ok = all128(ok && (n_tiles == 0 || wait(&sm.o_last, 0)));
    if (ok && n_tiles > 0) {
      fence_after();
      for (int mb = 0; mb < 4; ++mb) {
        const int col = mb * 128 + tid;  // latent index of this thread's TMEM lane
#pragma unroll
        for (int c0 = 0; c0 < HG; c0 += 16) {
          float o[16];
          tmem_ld<16>(tmem + kOCol + mb * HG + c0 + ((uint32_t)(warp * 32) << 16), o);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int hh = hg * HG + c0 + j;
            const float v = o[j] * sm.inv_l[c0 + j];
            if (num_splits == 1)
              qo.out[(size_t)b * qo.out_sb + (size_t)hh * qo.out_sh + col] = __float2bfloat16_rn(v);
            else
              part_o[(((size_t)b * num_splits + split) * heads + hh) * kL + col] = v;
          }
        }
      }
    } else if (ok) {  // an empty split: a zero partial with lse = -inf
      if (num_splits == 1) {
        for (int i = tid; i < HG * kL; i += kSoftmaxThreads)
          qo.out[(size_t)b * qo.out_sb + (size_t)(hg * HG + i / kL) * qo.out_sh + i % kL] = __float2bfloat16_rn(0.f);
      } else {
        for (int i = tid; i < HG * kL; i += kSoftmaxThreads)
          part_o[(((size_t)b * num_splits + split) * heads + hg * HG + i / kL) * kL + i % kL] = 0.f;
      }
    }
    if (!ok && tid == 0) atomicExch(status, kStatusWaitTimeout);
    if (num_splits > 1 && arrivals != nullptr) {
      __threadfence();
      sync128();
      if (tid == 0) {
        int* ctr = arrivals + (size_t)b * gridDim.y + hg;
        const int prev = atomicAdd(ctr, 1);
        sm.last = prev == num_splits - 1;
        if (sm.last) *ctr = 0;
      }
      sync128();
      if (sm.last) {
        __threadfence();
        merge_group<HG>(qo, part_o, part_lse, b, hg, heads, num_splits, tid, reinterpret_cast<float*>(sm.p[0]));
      }
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 5) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

}  // namespace mtc
}  // namespace afd

using namespace afd;

namespace {

// A kernel shape: heads per CTA, tokens per stage, stages, resident CTAs per SM.
struct TcShape {
  int hg, tile, stages, ctas;
};

// Measured on B200 (MLA decode, ~1 K context): with 32 heads per CTA
// (64 or more heads) 64-token tiles in two stages beat the mma.sync kernel
// (DeepSeek-V3 128 heads, 64 requests x 2100 tokens: 222 vs 244 us); with 16
// heads per CTA no shape does (256 requests: 100 us at best vs 72), so those
// layers keep the mma.sync kernel (hg = 0 here).  AFD_MLA_TC_SHAPE=tile,stages
// selects a shape for any head count that is a multiple of 16 (comparisons).
TcShape pick_shape(int heads) {
  static const int forced = [] {
    const char* v = std::getenv("AFD_MLA_TC_SHAPE");
    if (v == nullptr) return 0;
    int t = 0, st = 0;
    if (std::sscanf(v, "%d,%d", &t, &st) != 2) return 0;
    return t * 16 + st;
  }();
  const int hg = (heads % 32 == 0 && heads >= 64) ? 32 : (heads % 16 == 0 ? 16 : 0);
  if (hg == 0) return {0, 64, 2, 1};
  if (forced) {
    const int tile = forced / 16, stages = forced % 16;
    return {hg, tile, stages, (hg == 16 && tile == 32 && stages == 2) ? 2 : 1};
  }
  if (hg == 32) return {32, 64, 2, 1};
  return {0, 64, 2, 1};
}

template <int HG, int TILE, int STAGES, int CTAS>
cudaError_t launch_shape(const CUtensorMap& map, const MlaQO& qo, const int32_t* block_table, const int32_t* seq_lens,
                         float* po, float* pl, int* status, int batch, int heads, int block_size, int max_blocks,
                         int num_splits, float scale_log2, int* arrivals, cudaStream_t s) {
  static PerDeviceOnce once;
  const int smem = (int)sizeof(mtc::Smem<HG, TILE, STAGES>) + 1024;
  cudaError_t e = once.run([smem] {
    return cudaFuncSetAttribute(mtc::mla_decode_tc_kernel<HG, TILE, STAGES, CTAS>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  if (e != cudaSuccess) return e;
  dim3 grid(batch, heads / HG, num_splits);
  mtc::mla_decode_tc_kernel<HG, TILE, STAGES, CTAS><<<grid, mtc::kThreads, smem, s>>>(
      map, qo, block_table, seq_lens, po, pl, status, heads, block_size, max_blocks, num_splits, scale_log2, arrivals);
  return cudaGetLastError();
}

}  // namespace

int mla_decode_tc_heads_per_cta(int heads) { return pick_shape(heads).hg; }

int mla_decode_tc_num_splits(int batch, int heads, int max_seq_len, int num_sms) {
  // cost = waves x (tiles per split + the CTA's fixed start-up / drain, about
  // two tiles), in tiles; the smallest split count of the cheapest cost wins
  // (splits also cost a partial round trip through L2 and a merge).
  const TcShape sh = pick_shape(heads);
  if (sh.hg == 0) return 1;
  const long groups = (long)batch * (heads / sh.hg);
  const long slots = (long)num_sms * sh.ctas;
  const int tiles = (max_seq_len + sh.tile - 1) / sh.tile;
  const int max_s = std::max(1, std::min(16, tiles / 2));
  int best = 1;
  long best_cost = -1;
  for (int sp = 1; sp <= max_s; ++sp) {
    const long waves = (groups * sp + slots - 1) / slots;
    const long cost = waves * ((tiles + sp - 1) / sp + 2);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

// The merge of split partials stages one weight per (split, head) in P's buffer.
int mla_decode_tc_max_splits(int heads_per_cta) { return (int)(2 * heads_per_cta * 128 / sizeof(float)) / heads_per_cta; }

cudaError_t launch_mla_decode_tc(const MlaQO& qo, const void* cache, const int32_t* block_table,
                                 const int32_t* seq_lens, float* partial_o, float* partial_lse, int* status, int batch,
                                 int heads, int block_size, int num_blocks, int max_blocks_per_seq, int num_splits,
                                 float scale, cudaStream_t s, int* arrivals) {
  const TcShape sh = pick_shape(heads);
  if (sh.hg == 0 || block_size % sh.tile != 0) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(cache) & 15u) != 0) return cudaErrorMisalignedAddress;
  if (num_splits > 1 && (arrivals == nullptr || num_splits > mla_decode_tc_max_splits(sh.hg))) return cudaErrorInvalidValue;
  auto encode = get_tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)mtc::kD, (cuuint64_t)num_blocks * block_size};
  const cuuint64_t strides[1] = {(cuuint64_t)mtc::kD * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)sh.tile};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(cache), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const float sl2 = scale * 1.4426950408889634f;
#define AFD_MTC_LAUNCH(HG, T, ST, C)                                                                                  \
  if (sh.hg == HG && sh.tile == T && sh.stages == ST)                                                                 \
    return launch_shape<HG, T, ST, C>(map, qo, block_table, seq_lens, partial_o, partial_lse, status, batch, heads,   \
                                      block_size, max_blocks_per_seq, num_splits, sl2, arrivals, s);
  AFD_MTC_LAUNCH(16, 32, 2, 2)
  AFD_MTC_LAUNCH(16, 32, 4, 1)
  AFD_MTC_LAUNCH(16, 64, 2, 1)
  AFD_MTC_LAUNCH(32, 32, 4, 1)
  AFD_MTC_LAUNCH(32, 64, 2, 1)
#undef AFD_MTC_LAUNCH
  return cudaErrorNotSupported;
}
