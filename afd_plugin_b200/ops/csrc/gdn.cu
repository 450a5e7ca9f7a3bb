// Gated DeltaNet (linear attention of the Qwen3.5 / Qwen3-Next family).
//
// gdn_conv       depthwise causal convolution (kernel K <= 8) over the
//                q|k|v channels with a per-sequence rolling state of the last
//                K-1 inputs, SiLU fused.  One thread per (sequence, channel)
//                walks the sequence's tokens, so prefill and decode share it.
// gdn_recurrent  per (sequence, value head): L2-normalise q and k, gates
//                g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b),
//                the gated delta rule
//                    S = exp(g) S;  S += k (beta (v - S^T k))^T;  o = S^T q / sqrt(dk)
//                and the gated RMSNorm  o * rstd * w * silu(z).
//                Column j of the dk x dv fp32 state is held in registers by
//                one thread (two at dk = 128) across the sequence's tokens; the state is
//                read and written once per call (decode: 64 KB each way per
//                token and head at dk = dv = 128).
//
// Sequences are given by cu_seqlens [S + 1]; slots [S] pick each sequence's
// state row; reset [S] (optional) starts a sequence from a zero state.
#include "common.cuh"
#include "launchers.h"

namespace afd {
namespace gdn {

using bf16 = __nv_bfloat16;
constexpr int kMaxConvK = 8;

__global__ void conv_kernel(GdnConvParams p) {
  const int s = blockIdx.x;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= p.C) return;
  const int t0 = p.cu_seqlens[s], t1 = p.cu_seqlens[s + 1];
  const bool reset = p.reset != nullptr && p.reset[s] != 0;
  const int K = p.K;
  bf16* st = p.state + ((size_t)p.slots[s] * p.C + c) * (K - 1);
  float w[kMaxConvK], u[kMaxConvK];
#pragma unroll
  for (int j = 0; j < kMaxConvK; ++j) {
    w[j] = j < K ? __bfloat162float(p.weight[(size_t)c * K + j]) : 0.f;
    u[j] = (j < K - 1 && !reset) ? __bfloat162float(st[j]) : 0.f;
  }
  for (int t = t0; t < t1; ++t) {
    u[K - 1] = __bfloat162float(p.x[(size_t)t * p.ldx + c]);
    float y = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxConvK; ++j)
      if (j < K) y += w[j] * u[j];
    y = y / (1.f + __expf(-y));
    p.y[(size_t)t * p.C + c] = __float2bfloat16_rn(y);
#pragma unroll
    for (int j = 0; j + 1 < kMaxConvK; ++j)
      if (j < K - 1) u[j] = u[j + 1];
  }
  if (t1 > t0 || reset) {
#pragma unroll
    for (int j = 0; j < kMaxConvK - 1; ++j)
      if (j < K - 1) st[j] = __float2bfloat16_rn(u[j]);
  }
}

// SPLIT threads share one value column: thread (j, half) holds state rows
// [half * DK / SPLIT, (half + 1) * DK / SPLIT) of column j in registers.
template <int DK, int SPLIT>
__global__ void __launch_bounds__(256) recurrent_kernel(GdnRecurrentParams p) {
  constexpr int R = DK / SPLIT;
  __shared__ float s_q[DK], s_k[DK];
  __shared__ float s_red[2][8];
  __shared__ float s_gate[2];
  const int s = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x;
  const int j = tid / SPLIT, half = tid % SPLIT;  // value column, row block
  const int dv = p.dv;
  const int warp = tid / 32, lane = tid & 31, nwarps = (int)(blockDim.x + 31) / 32;
  const int hk = h / (p.nv / p.nk);
  const int t0 = p.cu_seqlens[s], t1 = p.cu_seqlens[s + 1];
  const bool reset = p.reset != nullptr && p.reset[s] != 0;
  float* S = p.state + (((size_t)p.slots[s] * p.nv + h) * DK + half * R) * dv + j;
  float col[R];
#pragma unroll
  for (int i = 0; i < R; ++i) col[i] = reset ? 0.f : S[(size_t)i * dv];
  const float A = -__expf(p.A_log[h]);
  const float dt_b = p.dt_bias[h];
  const float nw = __bfloat162float(p.norm_w[j]);
  const float scale = rsqrtf((float)DK);
  const float* kk = s_k + half * R;
  const float* qq = s_q + half * R;
  for (int t = t0; t < t1; ++t) {
    // q, k of this head (L2-normalised) into shared memory; gates by thread 0
    const bf16* qk = p.qkv + (size_t)t * p.ld_qkv;
    float qv = 0.f, kv = 0.f;
    if (tid < DK) {
      qv = __bfloat162float(qk[hk * DK + tid]);
      kv = __bfloat162float(qk[p.nk * DK + hk * DK + tid]);
    }
    const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
    if (lane == 0) {
      s_red[0][warp] = sq;
      s_red[1][warp] = sk;
    }
    if (tid == 0) {
      const float a = __bfloat162float(p.a[(size_t)t * p.ld_ab + h]) + dt_b;
      const float b = __bfloat162float(p.b[(size_t)t * p.ld_ab + h]);
      const float sp = a > 20.f ? a : log1pf(__expf(a));
      s_gate[0] = __expf(A * sp);            // exp(g)
      s_gate[1] = 1.f / (1.f + __expf(-b));  // beta
    }
    __syncthreads();
    float tq = 0.f, tk = 0.f;
    for (int w = 0; w < nwarps; ++w) {
      tq += s_red[0][w];
      tk += s_red[1][w];
    }
    if (tid < DK) {
      s_q[tid] = qv * rsqrtf(tq + 1e-6f) * scale;
      s_k[tid] = kv * rsqrtf(tk + 1e-6f);
    }
    __syncthreads();
    const float decay = s_gate[0], beta = s_gate[1];
    const float v = __bfloat162float(p.qkv[(size_t)t * p.ld_qkv + 2 * p.nk * DK + (size_t)h * dv + j]);
    float kvm = 0.f;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      col[i] *= decay;
      kvm += col[i] * kk[i];
    }
    if (SPLIT == 2) kvm += __shfl_xor_sync(0xffffffffu, kvm, 1);
    const float u = beta * (v - kvm);
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      col[i] += kk[i] * u;
      o += col[i] * qq[i];
    }
    if (SPLIT == 2) o += __shfl_xor_sync(0xffffffffu, o, 1);
    // gated RMSNorm over the dv outputs of this head (each column counted once)
    const float so = warp_sum(half == 0 ? o * o : 0.f);
    if (lane == 0) s_red[0][warp] = so;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < nwarps; ++w) tot += s_red[0][w];
    if (half == 0) {
      const float rstd = rsqrtf(tot / (float)dv + p.eps);
      const float z = __bfloat162float(p.z[(size_t)t * p.ld_z + (size_t)h * dv + j]);
      const float gz = z / (1.f + __expf(-z));
      p.out[(size_t)t * p.nv * dv + (size_t)h * dv + j] = __float2bfloat16_rn(o * rstd * nw * gz);
    }
    __syncthreads();  // shared buffers are rewritten by the next token
  }
  if (t1 > t0 || reset) {
#pragma unroll
    for (int i = 0; i < R; ++i) S[(size_t)i * dv] = col[i];
  }
}

}  // namespace gdn
}  // namespace afd

using namespace afd;

void launch_gdn_conv(const GdnConvParams& p, cudaStream_t s) {
  const int threads = 128;
  dim3 grid(p.num_seqs, (p.C + threads - 1) / threads);
  gdn::conv_kernel<<<grid, threads, 0, s>>>(p);
}

bool launch_gdn_recurrent(const GdnRecurrentParams& p, cudaStream_t s) {
  dim3 grid(p.num_seqs, p.nv);
  switch (p.dk) {
    case 32: gdn::recurrent_kernel<32, 1><<<grid, p.dv, 0, s>>>(p); return true;
    case 64: gdn::recurrent_kernel<64, 1><<<grid, p.dv, 0, s>>>(p); return true;
    case 128:
      if (p.dv * 2 > 256) return false;
      gdn::recurrent_kernel<128, 2><<<grid, p.dv * 2, 0, s>>>(p);
      return true;
    default: return false;
  }
}
