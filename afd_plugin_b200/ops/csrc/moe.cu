// MoE routing bookkeeping, token gather and weighted combine.
//
// moe_align   one CTA: per-expert histogram of the (token, k) assignments that
//             land on this rank's experts, exclusive prefix sum -> contiguous
//             row segments, and the row <-> (token, slot) maps.
// moe_gather  xs[row] = x[row_token[row]]  (expert-sorted activations)
// moe_combine out[t] = sum_j w[t, j] * ys[row(t, j)] (+ shared[t]), fp32 sums.
#include "common.cuh"
#include "device_state.h"
#include "launchers.h"

namespace afd {

constexpr int kMaxLocalExperts = 1024;

// Entries are (token, slot) pairs: the routed ones (slot < k, expert from
// `ids`) and, with n_shared > 0, every token's shared-expert chunks (slot
// k + c, virtual expert e_local + c, weight 1).  Segments of the virtual
// experts follow the routed ones.
__global__ void moe_align_kernel(const int32_t* __restrict__ ids, int tokens, int k, int n_shared, int e_local,
                                 int offset, int32_t* __restrict__ counts_out, int32_t* __restrict__ offsets_out,
                                 int32_t* __restrict__ row_token, int32_t* __restrict__ row_slot,
                                 int32_t* __restrict__ token_slot_row, int* __restrict__ total_rows) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  __shared__ int cnt[kMaxLocalExperts];
  __shared__ int cur[kMaxLocalExperts];
  const int ks = k + n_shared;
  const int e_all = e_local + n_shared;
  const int n = tokens * ks;
  auto expert_of = [&](int i) {
    const int t = i / ks, j = i % ks;
    return j < k ? ids[t * k + j] - offset : e_local + (j - k);
  };
  for (int e = threadIdx.x; e < e_all; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = expert_of(i);
    if (e >= 0 && e < e_all) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < e_all; ++e) {
      cur[e] = run;
      offsets_out[e] = run;
      counts_out[e] = cnt[e];
      run += cnt[e];
    }
    *total_rows = run;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = expert_of(i);
    if (e >= 0 && e < e_all) {
      const int r = atomicAdd(&cur[e], 1);
      row_token[r] = i / ks;
      row_slot[r] = i % ks;
      token_slot_row[i] = r;
    } else {
      token_slot_row[i] = -1;
    }
  }
}

template <typename T>
__global__ void moe_gather_kernel(T* __restrict__ xs, const T* __restrict__ x, const int32_t* __restrict__ row_token,
                                  int rows_cap, int hidden, const int* __restrict__ total_rows) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  constexpr int VN = Vec16<T>::N;
  const int nv = hidden / VN;
  const int total = *total_rows;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)rows_cap * nv;
       i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / nv);
    if (r >= total) continue;
    const int c = (int)(i % nv);
    store16(xs + (size_t)r * hidden + c * VN, load16(x + (size_t)row_token[r] * hidden + c * VN));
  }
}

// Slots j < k_routed carry routing weight w[t, j]; the remaining slots (shared
// chunks) have weight 1.
template <typename T>
__global__ void moe_combine_kernel(T* __restrict__ out, const T* __restrict__ ys, const float* __restrict__ w,
                                   const int32_t* __restrict__ tsr, int k, int k_routed, int hidden,
                                   const T* __restrict__ shared) {
  pdl_wait();  // launched with PDL: nothing global is touched before the predecessor completes
  pdl_launch_dependents();
  constexpr int VN = Vec16<T>::N;
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < hidden / VN; c += blockDim.x) {
    float acc[VN];
#pragma unroll
    for (int i = 0; i < VN; ++i) acc[i] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int r = tsr[t * k + j];
      if (r < 0) continue;
      const float wj = j < k_routed ? w[t * k_routed + j] : 1.f;
      Vec16<T> y = load16(ys + (size_t)r * hidden + c * VN);
#pragma unroll
      for (int i = 0; i < VN; ++i) acc[i] += wj * to_f32(y.v[i]);
    }
    if (shared) {
      Vec16<T> s = load16(shared + (size_t)t * hidden + c * VN);
#pragma unroll
      for (int i = 0; i < VN; ++i) acc[i] += to_f32(s.v[i]);
    }
    Vec16<T> o;
#pragma unroll
    for (int i = 0; i < VN; ++i) o.v[i] = from_f32<T>(acc[i]);
    store16(out + (size_t)t * hidden + c * VN, o);
  }
}

}  // namespace afd

using namespace afd;

#define AFD_DTYPE_SWITCH(dt, T, ...)                                \
  switch (dt) {                                                     \
    case kF32: { using T = float; __VA_ARGS__; break; }             \
    case kBF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }    \
    case kF16: { using T = __half; __VA_ARGS__; break; }            \
  }

void launch_moe_align(const int32_t* topk_ids, int tokens, int k, int n_shared, int e_local, int offset,
                      int32_t* expert_counts, int32_t* expert_offsets, int32_t* row_token, int32_t* row_slot,
                      int32_t* token_slot_row, int* total_rows, cudaStream_t s) {
  launch_pdl(moe_align_kernel, dim3(1), dim3(1024), 0, s, topk_ids, tokens, k, n_shared, e_local, offset, expert_counts,
             expert_offsets, row_token, row_slot, token_slot_row, total_rows);
}

void launch_moe_gather(void* xs, const void* x, const int32_t* row_token, int rows_cap, int hidden,
                       const int* total_rows, int dtype, cudaStream_t s) {
  AFD_DTYPE_SWITCH(dtype, T, {
    const size_t work = (size_t)rows_cap * hidden / Vec16<T>::N;
    int grid = (int)((work + 255) / 256);
    const int cap = device_sm_count() * 16;
    grid = grid > cap ? cap : (grid < 1 ? 1 : grid);
    launch_pdl(moe_gather_kernel<T>, dim3(grid), dim3(256), 0, s, (T*)xs, (const T*)x, row_token, rows_cap, hidden, total_rows);
  });
}

void launch_moe_combine(void* out, const void* ys, const float* topk_w, const int32_t* token_slot_row, int tokens,
                        int k, int k_routed, int hidden, const void* shared_out, int dtype, cudaStream_t s) {
  AFD_DTYPE_SWITCH(dtype, T, {
    const int threads = hidden / Vec16<T>::N < 256 ? hidden / Vec16<T>::N : 256;
    launch_pdl(moe_combine_kernel<T>, dim3(tokens), dim3(threads), 0, s, (T*)out, (const T*)ys, topk_w, token_slot_row, k,
               k_routed, hidden, (const T*)shared_out);
  });
}
