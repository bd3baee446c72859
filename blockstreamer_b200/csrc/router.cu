// Router: logits = x W^T + b (fp32 accumulate), top-k (descending), softmax over
// the k selected logits.  Replaces transformers models/gpt_oss/modeling_gpt_oss.py:
// 126-130 (GptOssTopKRouter.forward).
//
// Two forms:
//  * fused tiled kernel (any T): a CTA owns 32 tokens, computes their logits for
//    every expert into shared memory with a 4x4 register tile per thread, then
//    runs top-k + softmax per token with one warp per token;
//  * small-T form: one warp per expert streams W once for all (<= 16) tokens and
//    writes logits to global memory, then a top-k kernel (one warp per token).
// Top-k ties resolve to the lower expert index.
#include "bs_common.cuh"

namespace bs {
namespace {

constexpr int kTokTile = 32;    // tokens per CTA (fused kernel)
constexpr int kExpTile = 128;   // experts per pass (fused kernel)
constexpr int kKChunk = 32;     // K per shared-memory stage
constexpr int kMaxE = 512;
constexpr int kMaxK = 32;

template <typename T> __device__ __forceinline__ float ld_f32(const T* p);
template <> __device__ __forceinline__ float ld_f32<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// Eight consecutive elements (16-byte aligned) as floats.
__device__ __forceinline__ void ld8_f32(const float* p, float (&o)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
__device__ __forceinline__ void ld8_f32(const __nv_bfloat16* p, float (&o)[8]) {
  const uint4 q = *reinterpret_cast<const uint4*>(p);
  const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = __uint_as_float(u[i] << 16);
    o[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ float round_logit(float v, bool bf16_logits) {
  return bf16_logits ? __bfloat162float(__float2bfloat16_rn(v)) : v;
}

// One warp: top-k over `E` logits read by `get(e)`, softmax over the k values.
template <typename Get>
__device__ __forceinline__ void warp_topk_softmax(Get get, int E, int k, float* scores,
                                                  int32_t* idx32, int64_t* idx64) {
  const int lane = threadIdx.x & 31;
  constexpr int kPer = kMaxE / 32;
  float v[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? get(e) : -INFINITY;
    if (v[i] != v[i]) v[i] = -INFINITY;  // NaN logits are never selected first
  }
  float sel_v = 0.f;
  int sel_e = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > bv || (v[i] == bv && e < be))) { bv = v[i]; be = e; }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    // remove the winner: a NaN never compares greater or equal, so it is skipped
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == be) v[i] = __int_as_float(0x7fc00000u);
    if (lane == j) { sel_v = bv; sel_e = be; }
  }
  // softmax over the k selected (max is the first one)
  const float mx = __shfl_sync(0xffffffffu, sel_v, 0);
  const float ex = (lane < k) ? expf(sel_v - mx) : 0.f;
  float sum = ex;
#pragma unroll
  for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane < k) {
    scores[lane] = ex / sum;
    if (idx32) idx32[lane] = sel_e;
    if (idx64) idx64[lane] = sel_e;
  }
}

template <typename XT, typename WT>
__global__ void __launch_bounds__(256) router_fused_kernel(
    const XT* __restrict__ x, const WT* __restrict__ W, const WT* __restrict__ b, int T, int H,
    int E, int k, bool bf16_logits, float* __restrict__ logits_out, float* __restrict__ scores,
    int32_t* __restrict__ idx32, int64_t* __restrict__ idx64) {
  extern __shared__ float smem[];
  float* lg = smem;                                   // [kTokTile][E]
  float* xs = lg + kTokTile * E;                      // [kKChunk][kTokTile + 4]
  float* ws = xs + kKChunk * (kTokTile + 4);          // [kKChunk][kExpTile + 4]
  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * kTokTile;
  const int tx = tid % 32;  // expert group of 4
  const int ty = tid / 32;  // token group of 4
  for (int e0 = 0; e0 < E; e0 += kExpTile) {
    float acc[4][4] = {};
    for (int k0 = 0; k0 < H; k0 += kKChunk) {
      __syncthreads();
      // x chunk: kTokTile x kKChunk, stored transposed
      for (int i = tid; i < kTokTile * kKChunk; i += 256) {
        const int tt = i / kKChunk, kk = i % kKChunk;
        const int t = t0 + tt, kg = k0 + kk;
        xs[kk * (kTokTile + 4) + tt] = (t < T && kg < H) ? ld_f32(x + (int64_t)t * H + kg) : 0.f;
      }
      for (int i = tid; i < kExpTile * kKChunk; i += 256) {
        const int ee = i / kKChunk, kk = i % kKChunk;
        const int e = e0 + ee, kg = k0 + kk;
        ws[kk * (kExpTile + 4) + ee] = (e < E && kg < H) ? ld_f32(W + (int64_t)e * H + kg) : 0.f;
      }
      __syncthreads();
#pragma unroll 8
      for (int kk = 0; kk < kKChunk; ++kk) {
        const float4 a = *reinterpret_cast<const float4*>(&xs[kk * (kTokTile + 4) + ty * 4]);
        const float4 c = *reinterpret_cast<const float4*>(&ws[kk * (kExpTile + 4) + tx * 4]);
        const float av[4] = {a.x, a.y, a.z, a.w};
        const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], cv[j], acc[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = e0 + tx * 4 + j;
        if (e < E) lg[(ty * 4 + i) * E + e] = round_logit(acc[i][j] + ld_f32(b + e), bf16_logits);
      }
  }
  __syncthreads();
  const int warp = tid / 32;
  for (int tt = warp; tt < kTokTile; tt += 8) {
    const int t = t0 + tt;
    if (t >= T) break;
    const float* row = lg + tt * E;
    if (logits_out)
      for (int e = tx; e < E; e += 32) logits_out[(int64_t)t * E + e] = row[e];
    warp_topk_softmax([&](int e) { return row[e]; }, E, k, scores + (int64_t)t * k,
                      idx32 ? idx32 + (int64_t)t * k : nullptr, idx64 ? idx64 + (int64_t)t * k : nullptr);
  }
}

// Small T: warp per expert, MaxT tokens per CTA; each lane takes 8
// consecutive elements of H per step as 16-byte loads (H a multiple of 8,
// 16-byte aligned x and W), so every load feeds 8 FMAs per token.
template <typename XT, typename WT, int MaxT>
__global__ void __launch_bounds__(256) router_logits_small_vec_kernel(
    const XT* __restrict__ x, const WT* __restrict__ W, const WT* __restrict__ b, int T, int H,
    int E, bool bf16_logits, float* __restrict__ logits) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (warp >= E) return;
  const int t0 = blockIdx.y * MaxT;
  x += (int64_t)t0 * H;
  logits += (int64_t)t0 * E;
  T = min(T - t0, MaxT);
  const WT* w = W + (int64_t)warp * H;
  float acc[MaxT];
#pragma unroll
  for (int t = 0; t < MaxT; ++t) acc[t] = 0.f;
  for (int h = lane * 8; h < H; h += 256) {
    float wv[8];
    ld8_f32(w + h, wv);
#pragma unroll
    for (int t = 0; t < MaxT; ++t) {
      if (t < T) {
        float xv[8];
        ld8_f32(x + (int64_t)t * H + h, xv);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[t] = fmaf(xv[i], wv[i], acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MaxT; ++t) {
    float v = acc[t];
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0 && t < T) logits[(int64_t)t * E + warp] = round_logit(v + ld_f32(b + warp), bf16_logits);
  }
}

// Small T, any H or alignment: warp per expert; lane strides over H.
template <typename XT, typename WT, int MaxT>
__global__ void __launch_bounds__(256) router_logits_small_kernel(
    const XT* __restrict__ x, const WT* __restrict__ W, const WT* __restrict__ b, int T, int H,
    int E, bool bf16_logits, float* __restrict__ logits) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (warp >= E) return;
  // blockIdx.y: this CTA's chunk of MaxT tokens
  const int t0 = blockIdx.y * MaxT;
  x += (int64_t)t0 * H;
  logits += (int64_t)t0 * E;
  T = min(T - t0, MaxT);
  const WT* w = W + (int64_t)warp * H;
  float acc[MaxT];
#pragma unroll
  for (int t = 0; t < MaxT; ++t) acc[t] = 0.f;
  for (int h = lane; h < H; h += 32) {
    const float wv = ld_f32(w + h);
#pragma unroll
    for (int t = 0; t < MaxT; ++t)
      if (t < T) acc[t] = fmaf(ld_f32(x + (int64_t)t * H + h), wv, acc[t]);
  }
#pragma unroll
  for (int t = 0; t < MaxT; ++t) {
    float v = acc[t];
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0 && t < T) logits[(int64_t)t * E + warp] = round_logit(v + ld_f32(b + warp), bf16_logits);
  }
}

__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, int T,
                                                          int E, int k, float* __restrict__ scores,
                                                          int32_t* __restrict__ idx32,
                                                          int64_t* __restrict__ idx64) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  if (t >= T) return;
  const float* row = logits + (int64_t)t * E;
  warp_topk_softmax([&](int e) { return row[e]; }, E, k, scores + (int64_t)t * k,
                    idx32 ? idx32 + (int64_t)t * k : nullptr, idx64 ? idx64 + (int64_t)t * k : nullptr);
}

// Sum the K-split partial logits of the tensor-core form, add the bias, then
// top-k + softmax with one warp per token.
__global__ void __launch_bounds__(256) router_finish_kernel(
    const float* __restrict__ partial, int ns, int T, int Ep, int E, const void* __restrict__ bias,
    int bias_f32, int bf16_logits, int k, float* __restrict__ logits, float* __restrict__ scores,
    int32_t* __restrict__ idx32, int64_t* __restrict__ idx64) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  if (t >= T) return;
  auto get = [&](int e) {
    float v = 0.f;
    for (int s = 0; s < ns; ++s) v += partial[((int64_t)s * T + t) * Ep + e];
    v += bias_f32 ? static_cast<const float*>(bias)[e]
                  : __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[e]);
    v = round_logit(v, bf16_logits);
    if (logits) logits[(int64_t)t * E + e] = v;
    return v;
  };
  warp_topk_softmax(get, E, k, scores + (int64_t)t * k, idx32 ? idx32 + (int64_t)t * k : nullptr,
                    idx64 ? idx64 + (int64_t)t * k : nullptr);
}

template <typename XT, typename WT>
int launch_router(const void* x, const void* w, const void* b, int T, int H, int E, int k,
                  bool bf16_logits, float* logits, float* scores, int32_t* i32, int64_t* i64,
                  cudaStream_t st) {
  const XT* xp = static_cast<const XT*>(x);
  const WT* wp = static_cast<const WT*>(w);
  const WT* bp = static_cast<const WT*>(b);
  if (logits && T <= 64) {
    // one warp per (expert, 8 tokens): E/8 x T/8 CTAs, so that even a few
    // tokens spread over the SMs
    const dim3 grid((unsigned)cdiv(E, 8), (unsigned)cdiv(T, 8));
    if (H % 8 == 0 && (((uintptr_t)x | (uintptr_t)w) & 15) == 0)
      router_logits_small_vec_kernel<XT, WT, 8><<<grid, 256, 0, st>>>(xp, wp, bp, T, H, E, bf16_logits, logits);
    else
      router_logits_small_kernel<XT, WT, 8><<<grid, 256, 0, st>>>(xp, wp, bp, T, H, E, bf16_logits, logits);
    BS_LAUNCHED();
    router_topk_kernel<<<(unsigned)cdiv(T, 8), 256, 0, st>>>(logits, T, E, k, scores, i32, i64);
    BS_LAUNCHED();
    return BS_OK;
  }
  const size_t smem = sizeof(float) * ((size_t)kTokTile * E + kKChunk * (kTokTile + 4) +
                                       kKChunk * (kExpTile + 4));
  auto kern = router_fused_kernel<XT, WT>;
  BS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<(unsigned)cdiv(T, kTokTile), 256, smem, st>>>(xp, wp, bp, T, H, E, k, bf16_logits, logits,
                                                       scores, i32, i64);
  BS_LAUNCHED();
  return BS_OK;
}

}  // namespace

int router_finish_launch(const float* partial, int ns, int64_t T, int64_t Ep, int64_t E,
                         const void* bias, int bias_f32, int bf16_logits, int64_t k,
                         float* logits, float* scores, void* indices, int index_dtype,
                         cudaStream_t st) {
  int32_t* i32 = index_dtype == BS_I32 ? static_cast<int32_t*>(indices) : nullptr;
  int64_t* i64 = index_dtype == BS_I64 ? static_cast<int64_t*>(indices) : nullptr;
  router_finish_kernel<<<(unsigned)cdiv(T, 8), 256, 0, st>>>(partial, ns, (int)T, (int)Ep, (int)E,
                                                              bias, bias_f32, bf16_logits, (int)k,
                                                              logits, scores, i32, i64);
  BS_LAUNCHED();
  return BS_OK;
}

size_t router_tc_workspace_bytes(int64_t T, int64_t H, int64_t E, int w_dtype);
bool router_tc_supported(int x_dtype, int64_t T, int64_t H, int64_t E, int64_t k, const void* x);
int router_tc_launch(const void* x, const void* weight, const void* bias, int w_dtype, int64_t T,
                     int64_t H, int64_t E, int64_t k, float* logits, float* scores, void* indices,
                     int index_dtype, void* ws, size_t ws_bytes, cudaStream_t st);

// Workspace: the tensor-core form's split weight, and logits scratch for the
// small-T form.
size_t router_workspace_bytes(int64_t T, int64_t H, int64_t E, int w_dtype) {
  return router_tc_workspace_bytes(T, H, E, w_dtype) + align_up((size_t)std::max<int64_t>(T, 1) * E * 4, 256);
}

int router_launch(const void* x, int x_dtype, const void* weight, const void* bias, int w_dtype,
                  int64_t T, int64_t H, int64_t E, int64_t k, float* logits, float* scores,
                  void* indices, int index_dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  BS_ARG(x && weight && bias && scores && indices, "bs_router: null pointer");
  BS_ARG(x_dtype == BS_BF16 || x_dtype == BS_F32, "bs_router: x dtype must be bf16 or f32");
  BS_ARG(w_dtype == BS_BF16 || w_dtype == BS_F32, "bs_router: weight dtype must be bf16 or f32");
  BS_ARG(index_dtype == BS_I32 || index_dtype == BS_I64, "bs_router: indices must be int32/int64");
  BS_ARG(T >= 0 && H > 0 && E > 0 && k > 0, "bs_router: bad sizes");
  BS_ARG(E <= kMaxE, "bs_router: at most %d experts", kMaxE);
  BS_ARG(k <= E && k <= kMaxK, "bs_router: top_k must be <= experts and <= %d", kMaxK);
  BS_ARG(T <= (int64_t)INT32_MAX / 32 && H <= INT32_MAX, "bs_router: too many tokens");
  if (T == 0) return BS_OK;
  BS_TRY(check_device());
  const size_t tc_bytes = router_tc_workspace_bytes(T, H, E, w_dtype);
  if (ws && ws_bytes >= tc_bytes && router_tc_supported(x_dtype, T, H, E, k, x))
    return router_tc_launch(x, weight, bias, w_dtype, T, H, E, k, logits, scores, indices,
                            index_dtype, ws, ws_bytes, st);
  // the small-T form needs a logits buffer: the caller's, or the workspace's
  float* lg = logits;
  if (!lg && ws && ws_bytes >= router_workspace_bytes(T, H, E, w_dtype))
    lg = reinterpret_cast<float*>(static_cast<char*>(ws) + tc_bytes);
  int32_t* i32 = index_dtype == BS_I32 ? static_cast<int32_t*>(indices) : nullptr;
  int64_t* i64 = index_dtype == BS_I64 ? static_cast<int64_t*>(indices) : nullptr;
  const bool bl = w_dtype == BS_BF16;
  const int Ti = (int)T, Hi = (int)H, Ei = (int)E, ki = (int)k;
  if (x_dtype == BS_BF16 && w_dtype == BS_F32)
    return launch_router<__nv_bfloat16, float>(x, weight, bias, Ti, Hi, Ei, ki, bl, lg, scores, i32, i64, st);
  if (x_dtype == BS_BF16 && w_dtype == BS_BF16)
    return launch_router<__nv_bfloat16, __nv_bfloat16>(x, weight, bias, Ti, Hi, Ei, ki, bl, lg, scores, i32, i64, st);
  if (x_dtype == BS_F32 && w_dtype == BS_F32)
    return launch_router<float, float>(x, weight, bias, Ti, Hi, Ei, ki, bl, lg, scores, i32, i64, st);
  return launch_router<float, __nv_bfloat16>(x, weight, bias, Ti, Hi, Ei, ki, bl, lg, scores, i32, i64, st);
}

}  // namespace bs

extern "C" size_t bs_router_workspace_bytes(int64_t T, int64_t H, int64_t E, int w_dtype) {
  return bs::router_workspace_bytes(T, H, E, w_dtype);
}

extern "C" int bs_router(const void* x, int x_dtype, const void* weight, const void* bias,
                         int w_dtype, int64_t T, int64_t H, int64_t E, int64_t k, float* logits,
                         float* scores, void* indices, int index_dtype, void* workspace,
                         size_t workspace_bytes, void* stream) {
  return bs::router_launch(x, x_dtype, weight, bias, w_dtype, T, H, E, k, logits, scores, indices,
                           index_dtype, workspace, workspace_bytes,
                           reinterpret_cast<cudaStream_t>(stream));
}
