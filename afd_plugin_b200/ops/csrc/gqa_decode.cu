// Grouped-query paged decode for sm_100a (Qwen3-MoE: head_dim 128).
//
// One CTA = (request b, KV head h, KV split).  A producer warp loads 32-token
// K and V tiles of head h from the paged caches with TMA (3-D tensor maps over
// [tokens, kv_heads, head_dim], 128B swizzle), completing on mbarriers; four
// math warps run S = Q K^T for the head's query group (<= 16 query heads,
// padded to the MMA M of 16), an online softmax in the exp2 domain, and
// O += P V with tensor-core MMAs reading the swizzled tiles via ldmatrix.
// Several splits write normalised partials + log-sum-exp, merged by a
// combine kernel.  Waits are bounded and report through `status`.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "device_state.h"
#include "launchers.h"

namespace afd {
PFN_cuTensorMapEncodeTiled_v12000 get_tensor_map_encoder();

namespace gqa {

constexpr int kM = 16;         // query rows per CTA (group padded)
constexpr int kD = 128;        // head dim
constexpr int kTile = 32;
constexpr int kStages = 3;
constexpr int kMathWarps = 4;
constexpr int kThreads = (kMathWarps + 1) * 32;
constexpr int kBoxBytes = kTile * 128;           // 32 rows x 128 B
constexpr int kTileBytes = 2 * kBoxBytes;        // 128 dims = 2 swizzle boxes
constexpr int kQBoxBytes = kM * 128;
constexpr int kSStride = 36;

struct Smem {
  alignas(1024) uint8_t k[kStages][kTileBytes];
  alignas(1024) uint8_t v[kStages][kTileBytes];
  alignas(1024) uint8_t q[2 * kQBoxBytes];
  float s[2][kM * kSStride];
  uint64_t full[kStages];
  uint64_t empty[kStages];
};

AFD_DEVICE uint32_t swz(int row, int col, int box_bytes) {
  const int box = col >> 6;
  const int chunk = (col & 63) >> 3;
  return box * box_bytes + row * 128 + ((chunk ^ (row & 7)) << 4) + ((col & 7) << 1);
}

__global__ void __launch_bounds__(kThreads) gqa_decode_kernel(
    const __grid_constant__ CUtensorMap k_map, const __grid_constant__ CUtensorMap v_map,
    const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out, const int32_t* __restrict__ block_table,
    const int32_t* __restrict__ seq_lens, float* __restrict__ part_o, float* __restrict__ part_lse,
    int* __restrict__ status, int hq, int hkv, int block_size, int max_blocks, int num_splits, float scale_log2) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int group = hq / hkv;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int seq = seq_lens[b];
  const int n_total = (seq + kTile - 1) / kTile;
  const int per = (n_total + num_splits - 1) / num_splits;
  const int t_begin = split * per;
  const int n_tiles = max(0, min(n_total, t_begin + per) - t_begin);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kMathWarps);
    }
    fence_barrier_init();
  }
  // Q rows: the group's query heads; padding rows are zero.
  for (int c = threadIdx.x; c < kM * (kD / 8); c += kThreads) {
    const int r = c / (kD / 8), col = (c % (kD / 8)) * 8;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < group) val = *reinterpret_cast<const uint4*>(q + ((size_t)b * hq + h * group + r) * kD + col);
    *reinterpret_cast<uint4*>(sm.q + swz(r, col, kQBoxBytes)) = val;
  }
  __syncthreads();

  if (warp == kMathWarps) {
    if (lane == 0) {
      prefetch_tensormap(&k_map);
      prefetch_tensormap(&v_map);
      for (int i = 0; i < n_tiles; ++i) {
        const int st = i % kStages;
        if (!mbar_wait_bounded(&sm.empty[st], ((i / kStages) & 1) ^ 1)) {
          atomicExch(status, kStatusWaitTimeout);
          break;
        }
        const int t0 = (t_begin + i) * kTile;
        const int blk = block_table[(size_t)b * max_blocks + t0 / block_size];
        const int row = blk * block_size + (t0 % block_size);
        mbar_expect_tx(&sm.full[st], 2 * kTileBytes);
#pragma unroll
        for (int bx = 0; bx < 2; ++bx) {
          tma_load_3d(sm.k[st] + bx * kBoxBytes, &k_map, &sm.full[st], bx * 64, h, row);
          tma_load_3d(sm.v[st] + bx * kBoxBytes, &v_map, &sm.full[st], bx * 64, h, row);
        }
      }
    }
    return;
  }

  const int r0 = lane >> 2, qd = lane & 3;
  float o[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const uint32_t q_base = smem_u32(sm.q);
  for (int i = 0; i < n_tiles; ++i) {
    const int st = i % kStages;
    if (!mbar_wait_bounded(&sm.full[st], (i / kStages) & 1)) {
      atomicExch(status, kStatusWaitTimeout);
      break;
    }
    const uint32_t kb = smem_u32(sm.k[st]), vb = smem_u32(sm.v[st]);
    const int tok0 = (t_begin + i) * kTile;
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < kD / 16; kk += 2) {
      uint32_t a0[4], a1[4], b0, b1, b2, b3;
      const int qr = lane & 15, qc = kk * 16 + (lane >> 4) * 8;
      ldmatrix_x4(a0[0], a0[1], a0[2], a0[3], q_base + swz(qr, qc, kQBoxBytes));
      ldmatrix_x4(a1[0], a1[1], a1[2], a1[3], q_base + swz(qr, qc + 16, kQBoxBytes));
      ldmatrix_x4(b0, b1, b2, b3, kb + swz(warp * 8 + (lane & 7), kk * 16 + (lane >> 3) * 8, kBoxBytes));
      mma_bf16_16816(sacc, a0, b0, b1);
      mma_bf16_16816(sacc, a1, b2, b3);
    }
    float* sS = sm.s[i & 1];
    {
      const int tcol = warp * 8 + qd * 2;
#pragma unroll
      for (int j = 0; j < 4; ++j) sacc[j] = (tok0 + tcol + (j & 1) < seq) ? sacc[j] * scale_log2 : -INFINITY;
      *reinterpret_cast<float2*>(&sS[r0 * kSStride + tcol]) = make_float2(sacc[0], sacc[1]);
      *reinterpret_cast<float2*>(&sS[(r0 + 8) * kSStride + tcol]) = make_float2(sacc[2], sacc[3]);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kMathWarps * 32));
    float sv[2][8], alpha[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float* srow = &sS[(r0 + 8 * hh) * kSStride];
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const float2 lo = *reinterpret_cast<const float2*>(&srow[ks * 16 + qd * 2]);
        const float2 hi = *reinterpret_cast<const float2*>(&srow[ks * 16 + 8 + qd * 2]);
        sv[hh][ks * 4 + 0] = lo.x;
        sv[hh][ks * 4 + 1] = lo.y;
        sv[hh][ks * 4 + 2] = hi.x;
        sv[hh][ks * 4 + 3] = hi.y;
      }
      float mt = sv[hh][0];
#pragma unroll
      for (int j = 1; j < 8; ++j) mt = fmaxf(mt, sv[hh][j]);
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      const float m_new = fmaxf(m_run[hh], mt);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      alpha[hh] = exp2f(m_run[hh] - m_use);
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sv[hh][j] = exp2f(sv[hh][j] - m_use);
        ls += sv[hh][j];
      }
      ls += __shfl_xor_sync(0xffffffffu, ls, 1);
      ls += __shfl_xor_sync(0xffffffffu, ls, 2);
      l_run[hh] = l_run[hh] * alpha[hh] + ls;
      m_run[hh] = m_new;
    }
    uint32_t pa[2][4];
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      pa[ks][0] = pack_bf16(sv[0][ks * 4 + 0], sv[0][ks * 4 + 1]);
      pa[ks][1] = pack_bf16(sv[1][ks * 4 + 0], sv[1][ks * 4 + 1]);
      pa[ks][2] = pack_bf16(sv[0][ks * 4 + 2], sv[0][ks * 4 + 3]);
      pa[ks][3] = pack_bf16(sv[1][ks * 4 + 2], sv[1][ks * 4 + 3]);
    }
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int n0 = warp * 32 + np * 16;
        const int mi = lane >> 3;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3,
                          vb + swz(ks * 16 + (mi & 1) * 8 + (lane & 7), n0 + (mi >> 1) * 8, kBoxBytes));
        mma_bf16_16816(o[np * 2], pa[ks], b0, b1);
        mma_bf16_16816(o[np * 2 + 1], pa[ks], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[st]);
  }
  const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
  const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
  for (int hh = 0; hh < 2; ++hh) {
    const int r = r0 + 8 * hh;
    if (r >= group) continue;
    const float inv = hh ? inv1 : inv0;
    const int head = h * group + r;
    if (num_splits == 1) {
      __nv_bfloat16* ob = out + ((size_t)b * hq + head) * kD;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int col = warp * 32 + n * 8 + qd * 2;
        *reinterpret_cast<__nv_bfloat162*>(&ob[col]) =
            __floats2bfloat162_rn(o[n][hh * 2] * inv, o[n][hh * 2 + 1] * inv);
      }
    } else {
      float* po = part_o + (((size_t)b * num_splits + split) * hq + head) * kD;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int col = warp * 32 + n * 8 + qd * 2;
        *reinterpret_cast<float2*>(&po[col]) = make_float2(o[n][hh * 2] * inv, o[n][hh * 2 + 1] * inv);
      }
      if (warp == 0 && qd == 0)
        part_lse[((size_t)b * num_splits + split) * hq + head] =
            (hh ? l_run[1] : l_run[0]) > 0.f ? (hh ? m_run[1] : m_run[0]) + log2f(hh ? l_run[1] : l_run[0])
                                               : -INFINITY;
    }
  }
}

__global__ void gqa_combine_kernel(__nv_bfloat16* __restrict__ out, const float* __restrict__ part_o,
                                   const float* __restrict__ part_lse, int hq, int num_splits) {
  const int b = blockIdx.x, h = blockIdx.y, c = threadIdx.x;  // 128 threads = head dim
  const float* pl = part_lse + (size_t)b * num_splits * hq + h;
  float mx = -INFINITY;
  for (int s = 0; s < num_splits; ++s) mx = fmaxf(mx, pl[(size_t)s * hq]);
  float acc = 0.f, wsum = 0.f;
  for (int s = 0; s < num_splits; ++s) {
    const float v = pl[(size_t)s * hq];
    if (v == -INFINITY) continue;
    const float w = exp2f(v - mx);
    wsum += w;
    acc += w * part_o[(((size_t)b * num_splits + s) * hq + h) * kD + c];
  }
  out[((size_t)b * hq + h) * kD + c] = __float2bfloat16_rn(wsum > 0.f ? acc / wsum : 0.f);
}

static void encode_3d(CUtensorMap* map, const void* base, int tokens, int hkv) {
  const cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)hkv, (cuuint64_t)tokens};
  const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)hkv * kD * 2};
  const cuuint32_t box[3] = {64, 1, kTile};
  const cuuint32_t estr[3] = {1, 1, 1};
  get_tensor_map_encoder()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace gqa
}  // namespace afd

using namespace afd;

int gqa_decode_num_splits(int batch, int hkv, int max_seq_len, int num_sms) {
  const int tiles = (max_seq_len + gqa::kTile - 1) / gqa::kTile;
  const int ctas = batch * hkv;
  // One wave of the four resident CTAs per SM (shared memory allows four): a
  // split count that overfills it leaves a nearly empty second wave.
  int s = (4 * num_sms) / ctas;
  s = s < 1 ? 1 : s;
  const int max_s = tiles / 2 > 0 ? tiles / 2 : 1;
  return s > max_s ? max_s : s;
}

void launch_gqa_decode(void* out, const void* q, const void* kc, const void* vc, const int32_t* block_table,
                       const int32_t* seq_lens, float* partial_o, float* partial_lse, int* status, int batch, int hq,
                       int hkv, int d, int block_size, int num_blocks, int max_blocks_per_seq, int num_splits,
                       float scale, cudaStream_t s) {
  CUtensorMap kmap, vmap;
  gqa::encode_3d(&kmap, kc, num_blocks * block_size, hkv);
  gqa::encode_3d(&vmap, vc, num_blocks * block_size, hkv);
  const int smem = (int)sizeof(gqa::Smem) + 1024;
  static PerDeviceOnce attr;
  attr.run([&] { return cudaFuncSetAttribute(gqa::gqa_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); });
  gqa::gqa_decode_kernel<<<dim3(batch, hkv, num_splits), gqa::kThreads, smem, s>>>(
      kmap, vmap, (const __nv_bfloat16*)q, (__nv_bfloat16*)out, block_table, seq_lens, partial_o, partial_lse, status,
      hq, hkv, block_size, max_blocks_per_seq, num_splits, scale * 1.4426950408889634f);
  if (num_splits > 1)
    gqa::gqa_combine_kernel<<<dim3(batch, hq), gqa::kD, 0, s>>>((__nv_bfloat16*)out, partial_o, partial_lse, hq,
                                                               num_splits);
}
