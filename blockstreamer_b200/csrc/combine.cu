// Weighted combine and un-permute.
//
// Replaces block_streamer/gptoss.py:175-176, where each expert's rows are scaled
// by their fp32 routing weight, rounded to bf16 and index_add_-ed into a bf16
// accumulator in ascending expert order.  Here every output row is produced once:
// out[t] = bf16( sum_s w[t,s] * y[row_of_slot[t*k+s]] ) with an fp32 sum in slot
// order — one rounding instead of k+1, and no atomics (deterministic).
// HBM-bound: k*H*2 bytes read + H*2 written per token.
#include "bs_common.cuh"

namespace bs {
namespace {

__global__ void __launch_bounds__(256) combine_kernel(const uint4* __restrict__ y,
                                                      const int* __restrict__ row_of_slot,
                                                      const float* __restrict__ w, int64_t T,
                                                      int k, int64_t vecs, const uint4* __restrict__ residual,
                                                      uint4* __restrict__ out) {
  const int64_t total = T * vecs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vecs, v = i - t * vecs;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < k; ++s) {
      const int r = row_of_slot[t * k + s];
      if (r < 0) continue;
      const float ws = w[t * k + s];
      const uint4 q = y[(int64_t)r * vecs + v];
      const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = fmaf(ws, bf16lo(u[j]), acc[2 * j]);
        acc[2 * j + 1] = fmaf(ws, bf16hi(u[j]), acc[2 * j + 1]);
      }
    }
    if (residual) {
      const uint4 q = residual[i];
      out[i] = make_uint4(add_residual_bf16x2(q.x, acc[0], acc[1]), add_residual_bf16x2(q.y, acc[2], acc[3]),
                          add_residual_bf16x2(q.z, acc[4], acc[5]), add_residual_bf16x2(q.w, acc[6], acc[7]));
    } else {
      out[i] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                          pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
    }
  }
}

}  // namespace

int combine_launch(const void* y, const int32_t* row_of_slot, const float* weights, int64_t T,
                   int64_t k, int64_t H, void* out, cudaStream_t st, const void* residual) {
  BS_ARG(y && row_of_slot && weights && out, "bs_combine: null pointer");
  BS_ARG(T >= 0 && k > 0 && H > 0, "bs_combine: bad sizes");
  BS_ARG(H % 8 == 0, "bs_combine: hidden size must be a multiple of 8");
  BS_ALIGNED16(y, "y");
  BS_ALIGNED16(out, "out");
  if (residual) BS_ALIGNED16(residual, "residual");
  if (T == 0) return BS_OK;
  BS_TRY(check_device());
  const int64_t vecs = H / 8;
  const int grid = (int)std::min<int64_t>(cdiv(T * vecs, 256), (int64_t)sm_count() * 16);
  combine_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(y), row_of_slot, weights, T,
                                       (int)k, vecs, static_cast<const uint4*>(residual),
                                       static_cast<uint4*>(out));
  BS_LAUNCHED();
  return BS_OK;
}

}  // namespace bs

extern "C" int bs_combine(const void* y, const int32_t* row_of_slot, const float* weights,
                          int64_t T, int64_t k, int64_t H, void* out, void* stream) {
  return bs::combine_launch(y, row_of_slot, weights, T, k, H, out,
                            reinterpret_cast<cudaStream_t>(stream), nullptr);
}
