// Absorbed-MLA paged decode for sm_100a.
//
// One CTA = (request b, group of 16 heads, KV split).  A producer warp streams
// 32-token KV tiles (576 bf16 per token) from the paged cache into shared
// memory with TMA (cp.async.bulk.tensor, 128B swizzle; the 64-token cache
// blocks are contiguous rows of a 2-D tensor map), completing on mbarriers;
// four math warps compute S = Q K^T (tokens split over warps), an online
// softmax (exp2 domain) and O += P V (latent dims split over warps) with
// tensor-core MMAs reading the swizzled tiles through ldmatrix.  With several
// splits each CTA writes a normalised partial O plus its log-sum-exp; the last
// CTA of a (request, head group) to finish merges them (a per-group arrival
// counter that it resets), or, without counters, a combine kernel does.  The
// producer warp starts streaming KV tiles while the math warps load the query.
//
// Memory-bound by design: per token per layer it reads 1152 B of cache and
// does ~37 kFLOP for 16 heads, well under the tensor-core ceiling; the
// pipeline's job is to keep enough tile bytes in flight to saturate HBM.
//
// Sparse variant (DeepSeek sparse attention, kSparse = true): the CTA walks a
// per-request list of kept positions instead of the whole sequence.  The
// rows are scattered over the paged cache, so the producer warp gathers them
// with per-thread cp.async (one token row of 1152 B per lane, 16 B per copy,
// written at the same swizzled offsets the TMA path produces) and each lane
// signals the stage's mbarrier with cp.async.mbarrier.arrive.noinc; unused
// or out-of-range entries are zero-filled (src-size 0) and masked out of the
// softmax.  The math warps are shared with the dense path.
//
// Every mbarrier wait is bounded; on expiry the CTA records
// kStatusWaitTimeout in `status` and leaves its loop.
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "device_state.h"
#include "launchers.h"

namespace afd {
namespace mla {

constexpr int kHeads = 16;        // heads per CTA (MMA M)
constexpr int kTile = 32;         // tokens per pipeline stage
constexpr int kStages = 2;
constexpr int kMathWarps = 4;
constexpr int kThreads = (kMathWarps + 1) * 32;
constexpr int kBoxCols = 64;      // 128 B of bf16 per swizzle row
constexpr int kD = 576, kL = 512; // DeepSeek MLA latent + rope
constexpr int kBoxes = kD / kBoxCols;                 // 9
constexpr int kTileBytes = kTile * kD * 2;            // 36864
constexpr int kBoxBytes = kTile * kBoxCols * 2;       // 4096
constexpr int kQBoxBytes = kHeads * kBoxCols * 2;     // 2048
constexpr int kSStride = 36;                          // padded fp32 row of S

struct Smem {
  alignas(1024) uint8_t kv[kStages][kTileBytes];
  alignas(1024) uint8_t q[kBoxes * kQBoxBytes];
  float s[2][kHeads * kSStride];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int last;  // this CTA merges its group's split partials
};

// Byte offset of element (row, col) inside a 128B-swizzled tile made of
// `kBoxes` column boxes of `rows` x 64 bf16.
AFD_DEVICE uint32_t swz(int row, int col, int box_bytes) {
  const int box = col >> 6;
  const int chunk = (col & 63) >> 3;
  return box * box_bytes + row * 128 + ((chunk ^ (row & 7)) << 4) + ((col & 7) << 1);
}

// 16-byte global -> shared copy; `src_bytes` 0 writes zeros without reading.
AFD_DEVICE void cp_async_16_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// The mbarrier receives one arrival once this thread's earlier cp.async copies land.
AFD_DEVICE void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
AFD_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Entry `tok` of request b's kept-position list is a real token.
AFD_DEVICE bool sparse_entry_valid(const int32_t* __restrict__ keep_pos, int b, int tok, int num_keep, int seq_len) {
  if (tok >= num_keep) return false;
  const int p = keep_pos[(size_t)b * num_keep + tok];
  return p >= 0 && p < seq_len;
}

// out[b, h, :] = sum_s w_s o_s / sum_s w_s with w_s = 2^(lse_s - max_s lse),
// for the 16 heads of group hg, by the 128 math threads of the CTA that
// arrived last.  Partials are read through L2 (other CTAs of this launch wrote
// them).  The split log-sum-exps are staged in shared memory with independent
// loads, turned into normalised weights per head, and then every thread owns
// four latent columns of all 16 heads, so each split's rows arrive as eight
// independent 16-byte loads per thread instead of a chain of dependent ones.
constexpr int kMergeMaxSplits = (2 * kHeads * kSStride) / kHeads;  // the weights live in Smem::s

AFD_DEVICE void merge_group(const MlaQO& qo, const float* part_o, const float* part_lse, int b, int hg, int heads,
                            int num_splits, int tid, float* wsm) {
  const float* pl = part_lse + (size_t)b * num_splits * heads + hg * kHeads;
  for (int i = tid; i < num_splits * kHeads; i += kMathWarps * 32)
    wsm[i] = __ldcg(pl + (size_t)(i / kHeads) * heads + (i % kHeads));
  asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
  if (tid < kHeads) {
    float mx = -INFINITY;
    for (int sp = 0; sp < num_splits; ++sp) mx = fmaxf(mx, wsm[sp * kHeads + tid]);
    float wsum = 0.f;
    for (int sp = 0; sp < num_splits; ++sp) {
      const float v = wsm[sp * kHeads + tid];
      const float w = (v == -INFINITY) ? 0.f : exp2f(v - mx);
      wsm[sp * kHeads + tid] = w;
      wsum += w;
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    for (int sp = 0; sp < num_splits; ++sp) wsm[sp * kHeads + tid] *= inv;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
  static_assert(kL / 4 == kMathWarps * 32, "one float4 column per math thread");
  const int c = tid * 4;
  const float* base = part_o + ((size_t)b * num_splits * heads + (size_t)hg * kHeads) * kL + c;
#pragma unroll 1
  for (int h0 = 0; h0 < kHeads; h0 += 8) {
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
        const float w = wsm[sp * kHeads + h0 + h];
        acc[h].x += w * x[h].x;
        acc[h].y += w * x[h].y;
        acc[h].z += w * x[h].z;
        acc[h].w += w * x[h].w;
      }
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      __nv_bfloat16* ob = qo.out + (size_t)b * qo.out_sb + (size_t)(hg * kHeads + h0 + h) * qo.out_sh + c;
      *reinterpret_cast<__nv_bfloat162*>(ob) = __floats2bfloat162_rn(acc[h].x, acc[h].y);
      *reinterpret_cast<__nv_bfloat162*>(ob + 2) = __floats2bfloat162_rn(acc[h].z, acc[h].w);
    }
  }
}

template <bool kSparse>
__global__ void __launch_bounds__(kThreads, 2) mla_decode_kernel(
    const __grid_constant__ CUtensorMap kv_map, const MlaQO qo, const int32_t* __restrict__ block_table, const int32_t* __restrict__ seq_lens, float* __restrict__ part_o,
    float* __restrict__ part_lse, int* __restrict__ status, int heads, int block_size, int max_blocks,
    int num_splits, float scale_log2, const __nv_bfloat16* __restrict__ cache, const int32_t* __restrict__ keep_pos,
    int num_keep, int* __restrict__ arrivals, int l2_stream) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int b = blockIdx.x;
  const int hg = blockIdx.y;
  const int split = blockIdx.z;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int seq_len = seq_lens[b];
  const int seq = kSparse ? num_keep : seq_len;  // entries this CTA's splits walk
  const int n_tiles_total = (seq + kTile - 1) / kTile;
  const int tiles_per_split = (n_tiles_total + num_splits - 1) / num_splits;
  const int tile_begin = split * tiles_per_split;
  const int tile_end = min(n_tiles_total, tile_begin + tiles_per_split);
  const int n_tiles = max(0, tile_end - tile_begin);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], kSparse ? kTile : 1);
      mbar_init(&sm.empty[s], kMathWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp < kMathWarps) {
    // Q tile (16 heads x 576) -> swizzled smem by the math warps while the
    // producer's first tiles are in flight.  The latent part and the rope
    // part come from separate (strided) tensors.
    for (int c = threadIdx.x; c < kHeads * (kD / 8); c += kMathWarps * 32) {
      const int r = c / (kD / 8);
      const int col = (c % (kD / 8)) * 8;
      const int h = hg * kHeads + r;
      const __nv_bfloat16* src =
          (col < kL) ? qo.q_lat + (size_t)b * qo.lat_sb + (size_t)h * qo.lat_sh + col
                     : qo.q_pe + (size_t)b * qo.pe_sb + (size_t)h * qo.pe_sh + (col - kL);
      *reinterpret_cast<uint4*>(sm.q + swz(r, col, kQBoxBytes)) = *reinterpret_cast<const uint4*>(src);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
  }

  if (warp == kMathWarps) {
    // ------------------------------------------------------------ producer
    if constexpr (kSparse) {
      // one kept token per lane (kTile == 32), its 72 16-byte chunks gathered
      const uint32_t kv_smem = smem_u32(sm.kv[0]);
      for (int i = 0; i < n_tiles; ++i) {
        const int st = i % kStages;
        if (i >= kStages &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(&sm.empty[st], ((i / kStages) - 1) & 1))) {
          if (lane == 0) atomicExch(status, kStatusWaitTimeout);
          break;
        }
        const int tok = (tile_begin + i) * kTile + lane;
        const bool valid = sparse_entry_valid(keep_pos, b, tok, num_keep, seq_len);
        const __nv_bfloat16* src = cache;
        if (valid) {
          const int p = keep_pos[(size_t)b * num_keep + tok];
          const int blk = block_table[(size_t)b * max_blocks + p / block_size];
          src = cache + ((size_t)blk * block_size + p % block_size) * kD;
        }
        const uint32_t dst = kv_smem + st * kTileBytes;
        const uint32_t nbytes = valid ? 16u : 0u;
#pragma unroll 8
        for (int c = 0; c < kD / 8; ++c) cp_async_16_zfill(dst + swz(lane, c * 8, kBoxBytes), src + (valid ? c * 8 : 0), nbytes);
        cp_async_mbar_arrive_noinc(&sm.full[st]);
      }
      cp_async_wait_all();
    } else {
      // The cache rows of 32 tiles at a time are looked up by the warp's
      // lanes together (one block-table load each), so no global load sits
      // between a stage's release and its next TMA.
      if (lane == 0) prefetch_tensormap(&kv_map);
      // With one head group the KV rows are read once per step: they are the
      // first to leave L2 (weights and activations of the next kernels stay).
      const bool stream_kv = l2_stream && gridDim.y == 1;
      const uint64_t pol = l2_policy_evict_first();
      int my_row = 0;
      for (int i = 0; i < n_tiles; ++i) {
        const int st = i % kStages;
        if ((i & 31) == 0) {
          const int ti = i + lane;
          if (ti < n_tiles) {
            const int t0 = (tile_begin + ti) * kTile;
            my_row = block_table[(size_t)b * max_blocks + t0 / block_size] * block_size + (t0 % block_size);
          }
        }
        const int row = __shfl_sync(0xffffffffu, my_row, i & 31);
        int ok = 1;
        if (lane == 0 && i >= kStages) ok = mbar_wait_bounded(&sm.empty[st], ((i / kStages) - 1) & 1);
        if (!__shfl_sync(0xffffffffu, ok, 0)) {  // the whole warp leaves together
          if (lane == 0) atomicExch(status, kStatusWaitTimeout);
          break;
        }
        if (lane == 0) {
          mbar_expect_tx(&sm.full[st], kTileBytes);
#pragma unroll
          for (int bx = 0; bx < kBoxes; ++bx) {
            if (stream_kv)
              tma_load_2d_hint(sm.kv[st] + bx * kBoxBytes, &kv_map, &sm.full[st], bx * kBoxCols, row, pol);
            else
              tma_load_2d(sm.kv[st] + bx * kBoxBytes, &kv_map, &sm.full[st], bx * kBoxCols, row);
          }
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- math warps
  const int r0 = lane >> 2;  // fragment rows r0, r0 + 8 (heads)
  const int qd = lane & 3;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const uint32_t q_base = smem_u32(sm.q);
  bool ok = true;

  for (int i = 0; i < n_tiles && ok; ++i) {
    const int st = i % kStages;
    if (!mbar_wait_bounded(&sm.full[st], (i / kStages) & 1)) {
      atomicExch(status, kStatusWaitTimeout);
      ok = false;
      break;
    }
    const uint32_t kv_base = smem_u32(sm.kv[st]);
    const int tok0 = (tile_begin + i) * kTile;

    // ---- S[16 x 8] for tokens 8*warp .. 8*warp+7; four independent
    // accumulators keep four MMA chains in flight instead of one.
    float sacc4[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a) sacc4[a][0] = sacc4[a][1] = sacc4[a][2] = sacc4[a][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kD / 16; kk += 2) {
      uint32_t a0[4], a1[4];
      {
        const int r = lane & 15;
        const int c = kk * 16 + (lane >> 4) * 8;
        ldmatrix_x4(a0[0], a0[1], a0[2], a0[3], q_base + swz(r, c, kQBoxBytes));
        ldmatrix_x4(a1[0], a1[1], a1[2], a1[3], q_base + swz(r, c + 16, kQBoxBytes));
      }
      uint32_t b0, b1, b2, b3;
      {
        const int mi = lane >> 3;
        const int row = warp * 8 + (lane & 7);
        const int c = kk * 16 + mi * 8;
        ldmatrix_x4(b0, b1, b2, b3, kv_base + swz(row, c, kBoxBytes));
      }
      mma_bf16_16816(sacc4[(kk >> 1) & 3], a0, b0, b1);
      mma_bf16_16816(sacc4[((kk >> 1) + 2) & 3], a1, b2, b3);
    }
    float sacc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sacc[j] = (sacc4[0][j] + sacc4[1][j]) + (sacc4[2][j] + sacc4[3][j]);
    // scale + mask, publish to smem
    float* sS = sm.s[i & 1];
    {
      const int tcol = warp * 8 + qd * 2;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tok = tok0 + tcol + (j & 1);
        const bool keep = kSparse ? sparse_entry_valid(keep_pos, b, tok, num_keep, seq_len) : (tok < seq);
        sacc[j] = keep ? sacc[j] * scale_log2 : -INFINITY;
      }
      *reinterpret_cast<float2*>(&sS[r0 * kSStride + tcol]) = make_float2(sacc[0], sacc[1]);
      *reinterpret_cast<float2*>(&sS[(r0 + 8) * kSStride + tcol]) = make_float2(sacc[2], sacc[3]);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));

    // ---- online softmax on rows r0 and r0+8 (quad covers all 32 tokens)
    float sv[2][8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float* srow = &sS[(r0 + 8 * h) * kSStride];
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const float2 lo = *reinterpret_cast<const float2*>(&srow[ks * 16 + qd * 2]);
        const float2 hi = *reinterpret_cast<const float2*>(&srow[ks * 16 + 8 + qd * 2]);
        sv[h][ks * 4 + 0] = lo.x;
        sv[h][ks * 4 + 1] = lo.y;
        sv[h][ks * 4 + 2] = hi.x;
        sv[h][ks * 4 + 3] = hi.y;
      }
    }
    float alpha[2];
    uint32_t pa[2][4];  // A fragments of P for k-steps 0 and 1
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mt = sv[h][0];
#pragma unroll
      for (int j = 1; j < 8; ++j) mt = fmaxf(mt, sv[h][j]);
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      const float m_new = fmaxf(m_run[h], mt);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      alpha[h] = exp2f(m_run[h] - m_use);
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sv[h][j] = exp2f(sv[h][j] - m_use);
        ls += sv[h][j];
      }
      ls += __shfl_xor_sync(0xffffffffu, ls, 1);
      ls += __shfl_xor_sync(0xffffffffu, ls, 2);
      l_run[h] = l_run[h] * alpha[h] + ls;
      m_run[h] = m_new;
    }
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      pa[ks][0] = pack_bf16(sv[0][ks * 4 + 0], sv[0][ks * 4 + 1]);
      pa[ks][1] = pack_bf16(sv[1][ks * 4 + 0], sv[1][ks * 4 + 1]);
      pa[ks][2] = pack_bf16(sv[0][ks * 4 + 2], sv[0][ks * 4 + 3]);
      pa[ks][3] = pack_bf16(sv[1][ks * 4 + 2], sv[1][ks * 4 + 3]);
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }

    // ---- O[16 x 128 (this warp's latent slice)] += P V
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        const int n0 = warp * 128 + np * 16;
        const int mi = lane >> 3;
        const int row = ks * 16 + (mi & 1) * 8 + (lane & 7);
        const int c = n0 + (mi >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3, kv_base + swz(row, c, kBoxBytes));
        mma_bf16_16816(o[np * 2], pa[ks], b0, b1);
        mma_bf16_16816(o[np * 2 + 1], pa[ks], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[st]);
  }

  // ---- epilogue
  const int h_lo = hg * kHeads + r0;
  const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
  const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
  if (num_splits == 1) {
    __nv_bfloat16* o0 = qo.out + (size_t)b * qo.out_sb + (size_t)h_lo * qo.out_sh;
    __nv_bfloat16* o1 = qo.out + (size_t)b * qo.out_sb + (size_t)(h_lo + 8) * qo.out_sh;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int col = warp * 128 + n * 8 + qd * 2;
      *reinterpret_cast<__nv_bfloat162*>(&o0[col]) = __floats2bfloat162_rn(o[n][0] * inv0, o[n][1] * inv0);
      *reinterpret_cast<__nv_bfloat162*>(&o1[col]) = __floats2bfloat162_rn(o[n][2] * inv1, o[n][3] * inv1);
    }
  } else {
    float* po = part_o + (((size_t)b * num_splits + split) * heads) * kL;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int col = warp * 128 + n * 8 + qd * 2;
      *reinterpret_cast<float2*>(&po[(size_t)h_lo * kL + col]) = make_float2(o[n][0] * inv0, o[n][1] * inv0);
      *reinterpret_cast<float2*>(&po[(size_t)(h_lo + 8) * kL + col]) = make_float2(o[n][2] * inv1, o[n][3] * inv1);
    }
    if (warp == 0 && qd == 0) {
      float* pl = part_lse + ((size_t)b * num_splits + split) * heads;
      pl[h_lo] = l_run[0] > 0.f ? m_run[0] + log2f(l_run[0]) : -INFINITY;
      pl[h_lo + 8] = l_run[1] > 0.f ? m_run[1] + log2f(l_run[1]) : -INFINITY;
    }
    if (arrivals != nullptr) {
      // Release this CTA's partials, count it in; the last arrival merges.
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
      if (threadIdx.x == 0) {
        int* ctr = arrivals + (size_t)b * gridDim.y + hg;
        const int prev = atomicAdd(ctr, 1);
        sm.last = prev == num_splits - 1;
        if (sm.last) *ctr = 0;  // ready for the next launch (stream-ordered)
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
      if (!sm.last) return;
      __threadfence();
      merge_group(qo, part_o, part_lse, b, hg, heads, num_splits, threadIdx.x, &sm.s[0][0]);
    }
  }
}

// Merge split partials: out[b,h,:] = sum_s w_s o_s / sum_s w_s, w_s = 2^(lse_s - max).
__global__ void mla_combine_kernel(const MlaQO qo, const float* __restrict__ part_o,
                                   const float* __restrict__ part_lse, int heads, int num_splits, int L) {
  const int b = blockIdx.x, h = blockIdx.y;
  const float* pl = part_lse + (size_t)b * num_splits * heads + h;
  float mx = -INFINITY;
  for (int s = 0; s < num_splits; ++s) mx = fmaxf(mx, pl[(size_t)s * heads]);
  float wsum = 0.f;
  for (int s = 0; s < num_splits; ++s) {
    const float v = pl[(size_t)s * heads];
    wsum += (v == -INFINITY) ? 0.f : exp2f(v - mx);
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  for (int c = threadIdx.x * 4; c < L; c += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < num_splits; ++s) {
      const float v = pl[(size_t)s * heads];
      if (v == -INFINITY) continue;
      const float w = exp2f(v - mx);
      const float4 x = *reinterpret_cast<const float4*>(part_o + (((size_t)b * num_splits + s) * heads + h) * L + c);
      acc.x += w * x.x;
      acc.y += w * x.y;
      acc.z += w * x.z;
      acc.w += w * x.w;
    }
    __nv_bfloat16* ob = qo.out + (size_t)b * qo.out_sb + (size_t)h * qo.out_sh + c;
    *reinterpret_cast<__nv_bfloat162*>(ob) = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    *reinterpret_cast<__nv_bfloat162*>(ob + 2) = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
  }
}

// ---------------------------------------------------------------------------
// Work-balanced variant (stream-K over the KV tiles of all requests).
//
// The split kernel gives every request the same number of CTAs, so with one
// split per request a 256-request batch fills 256 of 296 CTA slots and the
// wave lasts a whole request.  Here the requests' tile ranges are laid end to
// end -- request b owns global tiles [P_b, P_{b+1}), P the exclusive prefix of
// max(1, ceil(seq_len / 32)) -- and CTA c of a head group takes global tiles
// [c W, (c + 1) W) with W = ceil(P_B / C): every CTA streams the same number
// of tiles.  A CTA's range crosses request boundaries; each piece (segment)
// runs the split kernel's producer / math pipeline (the stage ring continues
// across segments).  A request inside one CTA is written out directly;
// otherwise each covering CTA leaves a normalised partial in slot 2 c
// (the request is the CTA's first segment) or 2 c + 1 (its last), and the
// last of them to arrive merges.  Every CTA derives P from seq_lens itself,
// so a captured graph replays with new lengths.
constexpr int kBalMaxBatch = 1024;

struct BalSmem {
  Smem core;  // stages, query, S, barriers: the split kernel's layout
  int prefix[kBalMaxBatch + 1];
  int wsum[kThreads / 32];
  int carry;
  float mx[kHeads], inv[kHeads];  // merge: per-head max log-sum-exp and 1 / weight sum
};

// out[b, h, :] for the heads of group hg from the n_chunks partials of
// request b (chunk j lives in CTA first_cta + j; slot 2 c + 1 for the first
// chunk when the request starts inside that CTA's range, else 2 c).
AFD_DEVICE void merge_balanced(const MlaQO& qo, const float* part_o, const float* part_lse, int b, int hg, int heads,
                               int first_cta, int n_chunks, bool first_in_second_slot, int tid, float* mx_s,
                               float* inv_s) {
  auto slot = [&](int j) { return (first_cta + j) * 2 + ((j == 0 && first_in_second_slot) ? 1 : 0); };
  if (tid < kHeads) {
    const int h = hg * kHeads + tid;
    float mx = -INFINITY;
    for (int j = 0; j < n_chunks; ++j) mx = fmaxf(mx, __ldcg(part_lse + (size_t)slot(j) * heads + h));
    float wsum = 0.f;
    for (int j = 0; j < n_chunks; ++j) {
      const float v = __ldcg(part_lse + (size_t)slot(j) * heads + h);
      wsum += (v == -INFINITY) ? 0.f : exp2f(v - mx);
    }
    mx_s[tid] = mx;
    inv_s[tid] = wsum > 0.f ? 1.f / wsum : 0.f;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
  const int c = tid * 4;
#pragma unroll 1
  for (int h0 = 0; h0 < kHeads; h0 += 8) {
    float4 acc[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < n_chunks; ++j) {
      const int sl = slot(j);
      const float* ps = part_o + ((size_t)sl * heads + (size_t)hg * kHeads + h0) * kL + c;
      const float* pl = part_lse + (size_t)sl * heads + hg * kHeads + h0;
      float4 x[8];
      float w[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        x[h] = __ldcg(reinterpret_cast<const float4*>(ps + (size_t)h * kL));
        const float v = __ldcg(pl + h);
        w[h] = (v == -INFINITY) ? 0.f : exp2f(v - mx_s[h0 + h]) * inv_s[h0 + h];
      }
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        acc[h].x += w[h] * x[h].x;
        acc[h].y += w[h] * x[h].y;
        acc[h].z += w[h] * x[h].z;
        acc[h].w += w[h] * x[h].w;
      }
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      __nv_bfloat16* ob = qo.out + (size_t)b * qo.out_sb + (size_t)(hg * kHeads + h0 + h) * qo.out_sh + c;
      *reinterpret_cast<__nv_bfloat162*>(ob) = __floats2bfloat162_rn(acc[h].x, acc[h].y);
      *reinterpret_cast<__nv_bfloat162*>(ob + 2) = __floats2bfloat162_rn(acc[h].z, acc[h].w);
    }
  }
}

// Exclusive prefix of the per-request tile counts into bs.prefix[0..batch]
// (all threads of the CTA; batch <= kBalMaxBatch).
AFD_DEVICE void tile_prefix(BalSmem& bs, const int32_t* __restrict__ seq_lens, int batch) {
  const int tid = threadIdx.x, warp = tid / 32, lane = tid & 31;
  if (tid == 0) bs.carry = 0;
  __syncthreads();
  for (int base = 0; base < batch; base += kThreads) {
    const int i = base + tid;
    const int v = i < batch ? max(1, (seq_lens[i] + kTile - 1) / kTile) : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) bs.wsum[warp] = x;
    __syncthreads();
    int before = bs.carry;
    for (int w = 0; w < warp; ++w) before += bs.wsum[w];
    if (i < batch) bs.prefix[i] = before + x - v;
    __syncthreads();
    if (tid == kThreads - 1) bs.carry = before + x;  // the chunk's last inclusive sum
    __syncthreads();
  }
  if (tid == 0) bs.prefix[batch] = bs.carry;
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 2) mla_decode_bal_kernel(
    const __grid_constant__ CUtensorMap kv_map, const MlaQO qo, const int32_t* __restrict__ block_table,
    const int32_t* __restrict__ seq_lens, float* __restrict__ part_o, float* __restrict__ part_lse,
    int* __restrict__ status, int* __restrict__ arrivals, int batch, int heads, int block_size, int max_blocks,
    float scale_log2, int l2_stream) {
  extern __shared__ uint8_t smem_raw[];
  BalSmem& bs = *reinterpret_cast<BalSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Smem& sm = bs.core;
  const int c = blockIdx.x, C = gridDim.x;
  const int hg = blockIdx.y, G = gridDim.y;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;

  tile_prefix(bs, seq_lens, batch);
  const int T = bs.prefix[batch];
  const int W = (T + C - 1) / C;
  const int g0 = c * W;
  const int g1 = min(T, g0 + W);
  if (g0 >= g1) return;  // more CTAs than tiles: this one has none (uniform over the CTA)
  // first request of this CTA's range: the last b with prefix[b] <= g0
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (bs.prefix[mid] <= g0) lo = mid; else hi = mid - 1;
  }
  const int b0 = lo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kMathWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kMathWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) prefetch_tensormap(&kv_map);
    const bool stream_kv = l2_stream && G == 1;
    const uint64_t pol = l2_policy_evict_first();
    int it = 0;
    bool ok = true;
    for (int b = b0; ok && b < batch && bs.prefix[b] < g1; ++b) {
      const int p0 = bs.prefix[b];
      const int t_lo = max(g0, p0) - p0;
      const int t_hi = min(g1, bs.prefix[b + 1]) - p0;
      const int seq_b = seq_lens[b];
      int my_row = 0;
      for (int i = t_lo; i < t_hi; ++i, ++it) {
        const int st = it % kStages;
        if (((i - t_lo) & 31) == 0) {  // rows of the segment's next 32 tiles, one lookup per lane
          const int ti = i + lane;
          my_row = 0;  // a tile past the sequence (an empty request's masked tile) reads row 0
          if (ti < t_hi && ti * kTile < seq_b) {
            const int t0 = ti * kTile;
            my_row = block_table[(size_t)b * max_blocks + t0 / block_size] * block_size + (t0 % block_size);
          }
        }
        const int row = __shfl_sync(0xffffffffu, my_row, (i - t_lo) & 31);
        int okl = 1;
        if (lane == 0 && it >= kStages) okl = mbar_wait_bounded(&sm.empty[st], ((it / kStages) - 1) & 1);
        if (!__shfl_sync(0xffffffffu, okl, 0)) {  // the whole warp leaves together
          if (lane == 0) atomicExch(status, kStatusWaitTimeout);
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_expect_tx(&sm.full[st], kTileBytes);
#pragma unroll
          for (int bx = 0; bx < kBoxes; ++bx) {
            if (stream_kv)
              tma_load_2d_hint(sm.kv[st] + bx * kBoxBytes, &kv_map, &sm.full[st], bx * kBoxCols, row, pol);
            else
              tma_load_2d(sm.kv[st] + bx * kBoxBytes, &kv_map, &sm.full[st], bx * kBoxCols, row);
          }
        }
      }
    }
    // no copy may still land in shared memory when the CTA exits: wait (bounded) for the last ones
    if (lane == 0)
      for (int i = max(0, it - kStages); i < it; ++i) mbar_wait_bounded(&sm.full[i % kStages], (i / kStages) & 1);
    return;
  }

  // -------------------------------------------------------------- math warps
  const int r0 = lane >> 2;  // fragment rows r0, r0 + 8 (heads)
  const int qd = lane & 3;
  const int tid = threadIdx.x;
  const uint32_t q_base = smem_u32(sm.q);
  int it = 0;
  int seg = 0;
  bool ok = true;
  for (int b = b0; ok && b < batch && bs.prefix[b] < g1; ++b, ++seg) {
    const int p0 = bs.prefix[b], p1 = bs.prefix[b + 1];
    const int t_lo = max(g0, p0) - p0;
    const int t_hi = min(g1, p1) - p0;
    const int seq = seq_lens[b];
    // request b's query; the previous segment's readers of sm.q are done
    asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
    for (int q = tid; q < kHeads * (kD / 8); q += kMathWarps * 32) {
      const int r = q / (kD / 8);
      const int col = (q % (kD / 8)) * 8;
      const int h = hg * kHeads + r;
      const __nv_bfloat16* src =
          (col < kL) ? qo.q_lat + (size_t)b * qo.lat_sb + (size_t)h * qo.lat_sh + col
                     : qo.q_pe + (size_t)b * qo.pe_sb + (size_t)h * qo.pe_sh + (col - kL);
      *reinterpret_cast<uint4*>(sm.q + swz(r, col, kQBoxBytes)) = *reinterpret_cast<const uint4*>(src);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));

    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.f, 0.f};

    for (int i = t_lo; i < t_hi; ++i, ++it) {
      const int st = it % kStages;
      if (!mbar_wait_bounded(&sm.full[st], (it / kStages) & 1)) {
        atomicExch(status, kStatusWaitTimeout);
        ok = false;
        break;
      }
      const uint32_t kv_base = smem_u32(sm.kv[st]);
      const int tok0 = i * kTile;
      // S[16 x 8] for tokens 8*warp .. 8*warp+7 (four accumulators in flight)
      float sacc4[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a) sacc4[a][0] = sacc4[a][1] = sacc4[a][2] = sacc4[a][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kD / 16; kk += 2) {
        uint32_t a0[4], a1[4];
        {
          const int r = lane & 15;
          const int cc = kk * 16 + (lane >> 4) * 8;
          ldmatrix_x4(a0[0], a0[1], a0[2], a0[3], q_base + swz(r, cc, kQBoxBytes));
          ldmatrix_x4(a1[0], a1[1], a1[2], a1[3], q_base + swz(r, cc + 16, kQBoxBytes));
        }
        uint32_t b0r, b1r, b2r, b3r;
        {
          const int mi = lane >> 3;
          const int row = warp * 8 + (lane & 7);
          const int cc = kk * 16 + mi * 8;
          ldmatrix_x4(b0r, b1r, b2r, b3r, kv_base + swz(row, cc, kBoxBytes));
        }
        mma_bf16_16816(sacc4[(kk >> 1) & 3], a0, b0r, b1r);
        mma_bf16_16816(sacc4[((kk >> 1) + 2) & 3], a1, b2r, b3r);
      }
      float sacc[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) sacc[j] = (sacc4[0][j] + sacc4[1][j]) + (sacc4[2][j] + sacc4[3][j]);
      float* sS = sm.s[it & 1];
      {
        const int tcol = warp * 8 + qd * 2;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int tok = tok0 + tcol + (j & 1);
          sacc[j] = tok < seq ? sacc[j] * scale_log2 : -INFINITY;
        }
        *reinterpret_cast<float2*>(&sS[r0 * kSStride + tcol]) = make_float2(sacc[0], sacc[1]);
        *reinterpret_cast<float2*>(&sS[(r0 + 8) * kSStride + tcol]) = make_float2(sacc[2], sacc[3]);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));

      // online softmax on rows r0 and r0 + 8 (the quad covers all 32 tokens)
      float sv[2][8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float* srow = &sS[(r0 + 8 * h) * kSStride];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const float2 lo2 = *reinterpret_cast<const float2*>(&srow[ks * 16 + qd * 2]);
          const float2 hi2 = *reinterpret_cast<const float2*>(&srow[ks * 16 + 8 + qd * 2]);
          sv[h][ks * 4 + 0] = lo2.x;
          sv[h][ks * 4 + 1] = lo2.y;
          sv[h][ks * 4 + 2] = hi2.x;
          sv[h][ks * 4 + 3] = hi2.y;
        }
      }
      float alpha[2];
      uint32_t pa[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float mt = sv[h][0];
#pragma unroll
        for (int j = 1; j < 8; ++j) mt = fmaxf(mt, sv[h][j]);
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
        const float m_new = fmaxf(m_run[h], mt);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        alpha[h] = exp2f(m_run[h] - m_use);
        float ls = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          sv[h][j] = exp2f(sv[h][j] - m_use);
          ls += sv[h][j];
        }
        ls += __shfl_xor_sync(0xffffffffu, ls, 1);
        ls += __shfl_xor_sync(0xffffffffu, ls, 2);
        l_run[h] = l_run[h] * alpha[h] + ls;
        m_run[h] = m_new;
      }
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        pa[ks][0] = pack_bf16(sv[0][ks * 4 + 0], sv[0][ks * 4 + 1]);
        pa[ks][1] = pack_bf16(sv[1][ks * 4 + 0], sv[1][ks * 4 + 1]);
        pa[ks][2] = pack_bf16(sv[0][ks * 4 + 2], sv[0][ks * 4 + 3]);
        pa[ks][3] = pack_bf16(sv[1][ks * 4 + 2], sv[1][ks * 4 + 3]);
      }
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= alpha[0];
        o[n][1] *= alpha[0];
        o[n][2] *= alpha[1];
        o[n][3] *= alpha[1];
      }
      // O[16 x 128 (this warp's latent slice)] += P V
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          const int n0 = warp * 128 + np * 16;
          const int mi = lane >> 3;
          const int row = ks * 16 + (mi & 1) * 8 + (lane & 7);
          const int cc = n0 + (mi >> 1) * 8;
          uint32_t v0, v1, v2, v3;
          ldmatrix_x4_trans(v0, v1, v2, v3, kv_base + swz(row, cc, kBoxBytes));
          mma_bf16_16816(o[np * 2], pa[ks], v0, v1);
          mma_bf16_16816(o[np * 2 + 1], pa[ks], v2, v3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[st]);
    }
    if (!ok) break;

    // ---- epilogue of the segment: the whole request here, or one chunk of it
    const int h_lo = hg * kHeads + r0;
    const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
    const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
    const int first_cta = p0 / W;
    const int n_chunks = (p1 - 1) / W - first_cta + 1;
    if (n_chunks == 1) {
      __nv_bfloat16* o0 = qo.out + (size_t)b * qo.out_sb + (size_t)h_lo * qo.out_sh;
      __nv_bfloat16* o1 = qo.out + (size_t)b * qo.out_sb + (size_t)(h_lo + 8) * qo.out_sh;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int col = warp * 128 + n * 8 + qd * 2;
        *reinterpret_cast<__nv_bfloat162*>(&o0[col]) = __floats2bfloat162_rn(o[n][0] * inv0, o[n][1] * inv0);
        *reinterpret_cast<__nv_bfloat162*>(&o1[col]) = __floats2bfloat162_rn(o[n][2] * inv1, o[n][3] * inv1);
      }
      continue;
    }
    const int slot = c * 2 + (seg == 0 ? 0 : 1);
    float* po = part_o + (size_t)slot * heads * kL;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int col = warp * 128 + n * 8 + qd * 2;
      *reinterpret_cast<float2*>(&po[(size_t)h_lo * kL + col]) = make_float2(o[n][0] * inv0, o[n][1] * inv0);
      *reinterpret_cast<float2*>(&po[(size_t)(h_lo + 8) * kL + col]) = make_float2(o[n][2] * inv1, o[n][3] * inv1);
    }
    if (warp == 0 && qd == 0) {
      float* pl = part_lse + (size_t)slot * heads;
      pl[h_lo] = l_run[0] > 0.f ? m_run[0] + log2f(l_run[0]) : -INFINITY;
      pl[h_lo + 8] = l_run[1] > 0.f ? m_run[1] + log2f(l_run[1]) : -INFINITY;
    }
    // release the partial and count it in; the request's last chunk to arrive merges
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
    if (tid == 0) {
      int* ctr = arrivals + (size_t)b * G + hg;
      const int prev = atomicAdd(ctr, 1);
      sm.last = prev == n_chunks - 1;
      if (sm.last) *ctr = 0;  // ready for the next launch (stream-ordered)
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
    if (sm.last) {
      __threadfence();
      merge_balanced(qo, part_o, part_lse, b, hg, heads, first_cta, n_chunks, p0 != first_cta * W, tid, bs.mx,
                     bs.inv);
    }
  }
}

}  // namespace mla


// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 get_tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

}  // namespace afd

using namespace afd;

int mla_decode_num_splits(int batch, int max_seq_len, int num_sms) {
  const int tiles = (max_seq_len + mla::kTile - 1) / mla::kTile;
  // Splitting costs a partial-O round trip through HBM (and a combine launch),
  // so split only when the batch alone leaves SMs idle.
  if (batch * 2 >= 3 * num_sms) return 1;
  // One wave of two resident CTAs per SM: a split count that overfills it
  // leaves a second, nearly empty wave that runs at a fraction of HBM.
  const int slots = 2 * num_sms;
  int s = slots / batch;
  s = s < 1 ? 1 : s;
  const int max_s = tiles / 2 > 0 ? tiles / 2 : 1;  // keep >= 2 tiles per split
  return s > max_s ? max_s : s;
}

// Opts the decode kernels into their dynamic shared memory on the current device.
cudaError_t mla_decode_prepare_device() {
  static PerDeviceOnce once;
  return once.run([] {
    const int smem = (int)sizeof(mla::Smem) + 1024;
    cudaError_t e =
        cudaFuncSetAttribute(mla::mla_decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(mla::mla_decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
}

cudaError_t launch_mla_decode(const MlaQO& qo, const void* cache, const int32_t* block_table,
                              const int32_t* seq_lens, float* partial_o, float* partial_lse, int* status, int batch,
                              int heads, int L, int R, int block_size, int num_blocks, int max_blocks_per_seq,
                              int num_splits, float scale, cudaStream_t s, int* arrivals) {
  if ((reinterpret_cast<uintptr_t>(cache) & 15u) != 0) return cudaErrorMisalignedAddress;
  cudaError_t e = mla_decode_prepare_device();
  if (e != cudaSuccess) return e;
  auto encode = get_tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)(L + R), (cuuint64_t)num_blocks * block_size};
  const cuuint64_t strides[1] = {(cuuint64_t)(L + R) * 2};
  const cuuint32_t box[2] = {mla::kBoxCols, mla::kTile};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(cache), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;  // the tensor map could not be encoded: launch nothing
  const int smem = (int)sizeof(mla::Smem) + 1024;
  dim3 grid(batch, heads / mla::kHeads, num_splits);
  const float scale_log2 = scale * 1.4426950408889634f;
  if (num_splits == 1 || num_splits > mla::kMergeMaxSplits) arrivals = nullptr;
  mla::mla_decode_kernel<false><<<grid, mla::kThreads, smem, s>>>(map, qo, block_table, seq_lens, partial_o, partial_lse,
                                                                   status, heads, block_size, max_blocks_per_seq,
                                                                   num_splits, scale_log2, nullptr, nullptr, 0,
                                                                   arrivals, (l2_hint_mask() & kL2HintMla) ? 1 : 0);
  if (num_splits > 1 && arrivals == nullptr) {
    mla::mla_combine_kernel<<<dim3(batch, heads), 128, 0, s>>>(qo, partial_o, partial_lse, heads, num_splits, L);
  }
  return cudaGetLastError();
}

int mla_decode_balanced_ctas(int heads, int num_sms) {
  // one wave of two resident CTAs per SM over all head groups
  const int groups = heads / mla::kHeads;
  const int c = (2 * num_sms) / (groups > 0 ? groups : 1);
  return c > 0 ? c : 1;
}

int mla_decode_balanced_max_batch() { return mla::kBalMaxBatch; }

cudaError_t launch_mla_decode_balanced(const MlaQO& qo, const void* cache, const int32_t* block_table,
                                       const int32_t* seq_lens, float* partial_o, float* partial_lse, int* status,
                                       int* arrivals, int batch, int heads, int block_size, int num_blocks,
                                       int max_blocks_per_seq, int ctas, float scale, cudaStream_t s) {
  if ((reinterpret_cast<uintptr_t>(cache) & 15u) != 0) return cudaErrorMisalignedAddress;
  if (batch > mla::kBalMaxBatch || heads % mla::kHeads != 0 || ctas < 1 || arrivals == nullptr)
    return cudaErrorNotSupported;
  static PerDeviceOnce once;
  const int smem = (int)sizeof(mla::BalSmem) + 1024;
  cudaError_t e = once.run([smem] {
    return cudaFuncSetAttribute(mla::mla_decode_bal_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  if (e != cudaSuccess) return e;
  auto encode = get_tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)mla::kD, (cuuint64_t)num_blocks * block_size};
  const cuuint64_t strides[1] = {(cuuint64_t)mla::kD * 2};
  const cuuint32_t box[2] = {mla::kBoxCols, mla::kTile};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(cache), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(ctas, heads / mla::kHeads);
  mla::mla_decode_bal_kernel<<<grid, mla::kThreads, smem, s>>>(
      map, qo, block_table, seq_lens, partial_o, partial_lse, status, arrivals, batch, heads, block_size,
      max_blocks_per_seq, scale_log2, (l2_hint_mask() & kL2HintMla) ? 1 : 0);
  return cudaGetLastError();
}

void launch_mla_decode_sparse(const MlaQO& qo, const void* cache, const int32_t* block_table, const int32_t* seq_lens,
                              const int32_t* keep_pos, int num_keep, float* partial_o, float* partial_lse, int* status,
                              int batch, int heads, int L, int block_size, int max_blocks_per_seq, int num_splits,
                              float scale, cudaStream_t s, int* arrivals) {
  CUtensorMap unused;
  memset(&unused, 0, sizeof(unused));
  const int smem = (int)sizeof(mla::Smem) + 1024;
  if (mla_decode_prepare_device() != cudaSuccess) return;
  dim3 grid(batch, heads / mla::kHeads, num_splits);
  const float scale_log2 = scale * 1.4426950408889634f;
  mla::mla_decode_kernel<true><<<grid, mla::kThreads, smem, s>>>(
      unused, qo, block_table, seq_lens, partial_o, partial_lse, status, heads, block_size, max_blocks_per_seq,
      num_splits, scale_log2, reinterpret_cast<const __nv_bfloat16*>(cache), keep_pos, num_keep,
      num_splits > 1 && num_splits <= mla::kMergeMaxSplits ? arrivals : nullptr, 0);
  if (num_splits > 1 && arrivals == nullptr) {
    mla::mla_combine_kernel<<<dim3(batch, heads), 128, 0, s>>>(qo, partial_o, partial_lse, heads, num_splits, L);
  }
}
