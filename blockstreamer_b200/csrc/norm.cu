// RMSNorm of the gpt-oss decoder layer (transformers models/gpt_oss/
// modeling_gpt_oss.py, GptOssRMSNorm.forward):
//   v = float(x);  r = rsqrt(mean(v * v) + eps);  out = bf16(weight * (v * r))
// with weight in its own dtype (bf16 or fp32) promoted to fp32, as torch does.
// One warp per token row, 16-byte loads; HBM-bound (read H*2 bytes twice from
// L1/L2, write H*2).
#include "bs_common.cuh"

namespace bs {
namespace {

template <typename WT>
__device__ __forceinline__ float wget(const WT* w, int64_t i);
template <>
__device__ __forceinline__ float wget<float>(const float* w, int64_t i) { return w[i]; }
template <>
__device__ __forceinline__ float wget<__nv_bfloat16>(const __nv_bfloat16* w, int64_t i) {
  return __bfloat162float(w[i]);
}

template <typename WT>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint4* __restrict__ x, const WT* __restrict__ w,
                                                      int64_t T, int vecs, float H, float eps,
                                                      uint4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  for (int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; t < T;
       t += (int64_t)gridDim.x * blockDim.x / 32) {
    const uint4* row = x + t * vecs;
    float ss = 0.f;
    for (int v = lane; v < vecs; v += 32) {
      const uint4 q = row[v];
      const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf16lo(u[j]), b = bf16hi(u[j]);
        ss = fmaf(a, a, ss);
        ss = fmaf(b, b, ss);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / H + eps);
    uint4* orow = out + t * vecs;
    for (int v = lane; v < vecs; v += 32) {
      const uint4 q = row[v];
      const uint32_t u[4] = {q.x, q.y, q.z, q.w};
      uint32_t o4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t c = (int64_t)v * 8 + 2 * j;
        o4[j] = pack_bf16x2(wget(w, c) * (bf16lo(u[j]) * r), wget(w, c + 1) * (bf16hi(u[j]) * r));
      }
      orow[v] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  }
}

}  // namespace

int rmsnorm_launch(const void* x, int64_t T, int64_t H, const void* weight, int w_dtype, float eps, void* out,
                   cudaStream_t st) {
  BS_ARG(x && weight && out, "bs_rmsnorm: null pointer");
  BS_ARG(T >= 0 && H > 0 && H % 8 == 0, "bs_rmsnorm: hidden size must be a positive multiple of 8");
  BS_ARG(w_dtype == BS_BF16 || w_dtype == BS_F32, "bs_rmsnorm: weight dtype must be bf16 or f32");
  BS_ALIGNED16(x, "x");
  BS_ALIGNED16(out, "out");
  if (T == 0) return BS_OK;
  BS_TRY(check_device());
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(T, (int64_t)8), (int64_t)sm_count() * 8));
  if (w_dtype == BS_F32)
    rmsnorm_kernel<float><<<grid, 256, 0, st>>>(static_cast<const uint4*>(x), static_cast<const float*>(weight),
                                                T, (int)(H / 8), (float)H, eps, static_cast<uint4*>(out));
  else
    rmsnorm_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const uint4*>(x),
                                                        static_cast<const __nv_bfloat16*>(weight), T,
                                                        (int)(H / 8), (float)H, eps, static_cast<uint4*>(out));
  BS_LAUNCHED();
  return BS_OK;
}

}  // namespace bs

extern "C" int bs_rmsnorm(const void* x, int64_t T, int64_t H, const void* weight, int w_dtype, float eps,
                          void* out, void* stream) {
  return bs::rmsnorm_launch(x, T, H, weight, w_dtype, eps, out, reinterpret_cast<cudaStream_t>(stream));
}
