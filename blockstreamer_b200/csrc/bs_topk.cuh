// Warp-level top-k + softmax of one token's router logits (shared by the
// decode kernels).  transformers models/gpt_oss/modeling_gpt_oss.py:126-130:
// topk (sorted descending; ties go to the lower expert index, NaN counts as
// below everything) and softmax over the k selected logits.
#pragma once

#include <math.h>

namespace bs {

// One warp: top-k of E <= 32 PER values (ties -> lower index), softmax over
// the k (modeling_gpt_oss.py:126-130).  Lane l holds experts l + 32 i.
template <int PER, typename Get>
__device__ void warp_topk(Get get, int E, int k, float* scores, int* idx) {
  const int lane = threadIdx.x & 31;
  float v[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? get(e) : -INFINITY;
    if (v[i] != v[i]) v[i] = -INFINITY;
  }
  float sel_v = 0.f;
  int sel_e = 0;
  for (int j = 0; j < k; ++j) {
    float bv = __int_as_float(0x7fc00000u);  // NaN: below everything, never wins
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > bv || bv != bv || (v[i] == bv && e < be))) {
        if (v[i] == v[i]) {
          bv = v[i];
          be = e;
        }
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (ov == ov && (bv != bv || ov > bv || (ov == bv && oe < be))) {
        bv = ov;
        be = oe;
      }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == be) v[i] = __int_as_float(0x7fc00000u);  // removed: never selected again
    if (lane == j) {
      sel_v = bv;
      sel_e = be;
    }
  }
  const float mx = __shfl_sync(0xffffffffu, sel_v, 0);
  const float ex = (lane < k) ? expf(sel_v - mx) : 0.f;
  float sum = ex;
#pragma unroll
  for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane < k) {
    if (scores) scores[lane] = ex / sum;
    idx[lane] = sel_e;
  }
}

template <typename Get>
__device__ void warp_topk_any(Get get, int E, int k, float* scores, int* idx) {
  if (E <= 32) warp_topk<1>(get, E, k, scores, idx);
  else if (E <= 64) warp_topk<2>(get, E, k, scores, idx);
  else if (E <= 128) warp_topk<4>(get, E, k, scores, idx);
  else if (E <= 256) warp_topk<8>(get, E, k, scores, idx);
  else if (E <= 512) warp_topk<16>(get, E, k, scores, idx);
  else warp_topk<32>(get, E, k, scores, idx);
}

}  // namespace bs
