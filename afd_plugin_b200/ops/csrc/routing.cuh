// Warp-level MoE routing: scores, optional group limit, top-k selection.
// Shared by the standalone routing kernel and the fused AFD dispatch kernel.
#pragma once
#include "common.cuh"

namespace afd {

constexpr int kRouteMaxPerLane = 16;  // E <= 512

// `row` holds E fp32 logits (global or shared memory).  Lanes 0..k-1 receive
// (weight, expert id) of the r-th selected expert.  Ties break toward the
// lower expert id.  scoring: 0 softmax, 1 sigmoid, 2 sqrt(softplus) (1 and 2
// add the bias for selection only).  `forced` (hash routing) gives the k
// expert ids; only their weights come from the scores.
AFD_DEVICE void warp_route(const float* row, const float* bias, int E, int k, int scoring, bool renorm,
                           int n_group, int topk_group, float scale, float& out_w, int& out_id,
                           const int32_t* forced = nullptr) {
  const int lane = threadIdx.x & 31;
  float score[kRouteMaxPerLane], sel[kRouteMaxPerLane];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kRouteMaxPerLane; ++j) {
    const int e = j * 32 + lane;
    score[j] = (e < E) ? row[e] : -INFINITY;
    mx = fmaxf(mx, score[j]);
  }
  if (scoring == 0) {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kRouteMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      score[j] = (e < E) ? __expf(score[j] - mx) : 0.f;
      sum += score[j];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < kRouteMaxPerLane; ++j) {
      score[j] *= inv;
      sel[j] = (j * 32 + lane < E) ? score[j] : -INFINITY;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kRouteMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      const float x = score[j];
      const float act = scoring == 1 ? 1.f / (1.f + __expf(-x)) : sqrtf(x > 20.f ? x : log1pf(__expf(x)));
      score[j] = (e < E) ? act : 0.f;
      sel[j] = (e < E) ? score[j] + (bias ? bias[e] : 0.f) : -INFINITY;
    }
  }
  if (forced != nullptr) {
    float wsum = 0.f, my_w = 0.f;
    int my_id = 0;
    for (int r = 0; r < k; ++r) {
      const int id = forced[r];
      const int jj = id >> 5;
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < kRouteMaxPerLane; ++j)
        if (j == jj) v = score[j];
      const float wv = __shfl_sync(0xffffffffu, v, id & 31);
      wsum += wv;
      if (lane == r) {
        my_w = wv;
        my_id = id;
      }
    }
    out_w = (renorm ? my_w / wsum : my_w) * scale;
    out_id = my_id;
    return;
  }
  if (n_group > 1 && topk_group < n_group) {
    const int gsize = E / n_group;
    uint32_t keep = 0;
    float gmine = -INFINITY;
    for (int g = 0; g < n_group; ++g) {
      float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
      for (int j = 0; j < kRouteMaxPerLane; ++j) {
        const int e = j * 32 + lane;
        if (e < E && e / gsize == g) {
          const float v = sel[j];
          if (v > m1) {
            m2 = m1;
            m1 = v;
          } else if (v > m2) {
            m2 = v;
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float a1 = __shfl_xor_sync(0xffffffffu, m1, o);
        const float a2 = __shfl_xor_sync(0xffffffffu, m2, o);
        const float n1 = fmaxf(m1, a1);
        const float n2 = fmaxf(fminf(m1, a1), fmaxf(m2, a2));
        m1 = n1;
        m2 = n2;
      }
      const float gs = (scoring == 1) ? m1 + m2 : m1;
      if (lane == g) gmine = gs;
    }
    for (int r = 0; r < topk_group; ++r) {
      float v = gmine;
      int idx = (lane < n_group && !((keep >> lane) & 1u)) ? lane : (1 << 20);
      if (idx == (1 << 20)) v = -INFINITY;
      warp_argmax(v, idx);
      keep |= 1u << idx;
    }
#pragma unroll
    for (int j = 0; j < kRouteMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      if (e < E && !((keep >> (e / gsize)) & 1u)) sel[j] = -INFINITY;
    }
  }
  float wsum = 0.f, my_w = 0.f;
  int my_id = 0;
  for (int r = 0; r < k; ++r) {
    float v = -INFINITY;
    int idx = 1 << 20;
#pragma unroll
    for (int j = 0; j < kRouteMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      if (e < E && (sel[j] > v || (sel[j] == v && e < idx))) {
        v = sel[j];
        idx = e;
      }
    }
    warp_argmax(v, idx);
    float wv = 0.f;
#pragma unroll
    for (int j = 0; j < kRouteMaxPerLane; ++j) {
      if (j * 32 + lane == idx) {
        wv = score[j];
        sel[j] = -INFINITY;
      }
    }
    wv = warp_sum(wv);
    wsum += wv;
    if (lane == r) {
      my_w = wv;
      my_id = idx;
    }
  }
  out_w = (renorm ? my_w / wsum : my_w) * scale;
  out_id = my_id;
}

}  // namespace afd
