// Backward of the MoE layer (dL/dx, dL/d routing weights, and through the
// router), with no host synchronization.
//
// Replaces autograd through block_streamer/gptoss.py:137-177 with
// _MXFP4Matmul.backward (gptoss.py:64-71), where the reference re-runs its
// per-expert loop (host syncs per expert) and multiplies by a densely
// dequantized weight.  Here, for S = T * k routed rows:
//   1. dispatch (the forward's grouping) and x_perm;
//   2. g = x_perm @ W_gu^T + b_gu  (forward grouped GEMM, plain epilogue, fp32:
//      the clamps of the SwiGLU decide which elements pass a gradient, and
//      with bf16 g the decisions near +-limit flip against an fp32
//      evaluation -- at saturating shapes that alone moves dL/dx by ~4%);
//   3. h = SwiGLU(g)               (swiglu_rows_kernel, bf16 h);
//   4. y = h @ W_d^T + b_d         (forward grouped GEMM);
//   5. dw[t,s] = <dout[t], y[row]>, dy[row] = w[t,s] * dout[t]
//      (combine_backward_kernel: the backward of out = sum_s w * y);
//   6. dg = SwiGLU'(g) * (dy @ W_d)   (transposed grouped GEMM, SwiGLU-backward
//      epilogue, bf16 dg);
//   7. dx_perm = dg @ W_gu            (transposed grouped GEMM);
//   8. dx[t] = sum_s dx_perm[row(t,s)] (unpermute_sum_kernel, fp32).
// The router's part (GptOssTopKRouter, modeling_gpt_oss.py:126-130: logits,
// top-k, softmax over the k) is router_backward_kernel.
#include "bs_common.cuh"

namespace bs {

size_t dispatch_workspace_bytes(int64_t T, int64_t k, int64_t E);
int dispatch_launch(const void* indices, int index_dtype, int64_t T, int64_t k, int64_t E, const void* x, int64_t H,
                    int32_t* offsets, int32_t* row_of_slot, int32_t* token_of_row, void* x_perm, void* ws,
                    size_t ws_bytes, cudaStream_t st);
int tc_grouped_launch(int mode, const void* x, const int32_t* offsets, int64_t rows_total,
                      int64_t max_rows_per_expert, int64_t E, int64_t K, int64_t N, const void* blocks,
                      const void* scales, const void* bias, int bias_f32, float alpha, float limit, void* out,
                      cudaStream_t st);
bool tc_supported(const void* scales, int64_t K, int64_t N);
size_t tc_t_scales_bytes(int64_t E, int64_t Nw, int64_t Kw);
bool tc_t_supported(int64_t Nw, int64_t Kw);
int tc_grouped_t_launch(int epi, const void* dy, const int32_t* offsets, int64_t rows_total, int64_t E, int64_t Nw,
                        int64_t Kw, const void* blocks, const void* scales, void* scales_t, const void* g,
                        float alpha, float limit, void* out, cudaStream_t st);

namespace {

// h[r, i] = (clamp(up) + 1) * min(gate, L) * sigmoid(alpha * min(gate, L)),
// gate = g[r, 2i], up = g[r, 2i + 1] (gptoss.py:130-135), from fp32 g.
__device__ __forceinline__ float swiglu_exact(float gate, float up, float alpha, float limit) {
  gate = fminf(gate, limit);
  up = fminf(fmaxf(up, -limit), limit);
  return (up + 1.0f) * (gate / (1.0f + expf(-alpha * gate)));
}

// Two outputs per thread (16-byte loads of g, 4-byte stores of h); n_pairs even.
__global__ void __launch_bounds__(256) swiglu_rows_kernel(const float4* __restrict__ g, int64_t n_pairs,
                                                          float alpha, float limit, uint32_t* __restrict__ h) {
  const int64_t n2 = n_pairs / 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n2; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = g[i];
    h[i] = pack_bf16x2(swiglu_exact(v.x, v.y, alpha, limit), swiglu_exact(v.z, v.w, alpha, limit));
  }
}

// One warp per routed slot (t, s): dw[t,s] = sum_f dout[t,f] * y[row,f] and
// dy[row, :] = bf16(w[t,s] * dout[t, :]) -- the backward of
// out[t] = sum_s w[t,s] * y[row(t,s)] (gptoss.py:175-176).
template <typename GT>
__global__ void __launch_bounds__(256) combine_backward_kernel(const GT* __restrict__ dout, const uint16_t* __restrict__ y,
                                                               const int* __restrict__ row_of_slot,
                                                               const float* __restrict__ w, int64_t T, int k, int H,
                                                               float* __restrict__ dw, uint16_t* __restrict__ dy) {
  const int lane = threadIdx.x & 31;
  const int64_t nslots = T * k;
  for (int64_t sl = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; sl < nslots;
       sl += (int64_t)gridDim.x * blockDim.x / 32) {
    const int64_t t = sl / k;
    const int r = row_of_slot[sl];
    if (r < 0) {
      if (lane == 0) dw[sl] = 0.f;
      continue;
    }
    const float ws = w[sl];
    const GT* go = dout + t * H;
    const uint16_t* yr = y + (int64_t)r * H;
    uint16_t* dr = dy + (int64_t)r * H;
    float acc = 0.f;
    for (int f = lane * 2; f < H; f += 64) {
      float g0, g1;
      if constexpr (sizeof(GT) == 4) {
        const float2 q = *reinterpret_cast<const float2*>(go + f);
        g0 = q.x, g1 = q.y;
      } else {
        const uint32_t q = *reinterpret_cast<const uint32_t*>(go + f);
        g0 = bf16lo(q), g1 = bf16hi(q);
      }
      const uint32_t yv = *reinterpret_cast<const uint32_t*>(yr + f);
      acc = fmaf(g0, bf16lo(yv), fmaf(g1, bf16hi(yv), acc));
      *reinterpret_cast<uint32_t*>(dr + f) = pack_bf16x2(ws * g0, ws * g1);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) dw[sl] = acc;
  }
}

// dx[t, :] = sum_s src[row(t,s), :] in fp32 (the backward of the gather x_perm[row] = x[t]).
__global__ void __launch_bounds__(256) unpermute_sum_kernel(const uint32_t* __restrict__ src,
                                                            const int* __restrict__ row_of_slot, int64_t T, int k,
                                                            int pairs, float2* __restrict__ dx) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < T * pairs; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / pairs, c = i - t * pairs;
    float a = 0.f, b = 0.f;
    for (int s = 0; s < k; ++s) {
      const int r = row_of_slot[t * k + s];
      if (r < 0) continue;
      const uint32_t v = src[(int64_t)r * pairs + c];
      a += bf16lo(v);
      b += bf16hi(v);
    }
    dx[i] = make_float2(a, b);
  }
}

template <typename T>
__device__ __forceinline__ float ld_as_f32(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_as_f32<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_as_f32<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

// Router backward, one CTA per token (modeling_gpt_oss.py:126-130): scores =
// softmax over the k selected logits, so dlogit_j = s_j (ds_j - sum_i s_i ds_i);
// the selected logits are x . W[e_j] + b[e_j]: dx[t] += sum_j dlogit_j W[e_j],
// dW[e_j] += dlogit_j x[t], db[e_j] += dlogit_j (fp32 atomics).
template <typename XT, typename WT>
__global__ void __launch_bounds__(256) router_backward_kernel(const XT* __restrict__ x, const WT* __restrict__ W, int H,
                                                              int E, int k, const float* __restrict__ scores,
                                                              const int* __restrict__ idx,
                                                              const float* __restrict__ dscores, float* __restrict__ dx,
                                                              float* __restrict__ dW, float* __restrict__ db) {
  __shared__ float dl[32];
  __shared__ int ex[32];
  const int64_t t = blockIdx.x;
  if (threadIdx.x == 0) {
    float dot = 0.f;
    for (int j = 0; j < k; ++j) dot += scores[t * k + j] * dscores[t * k + j];
    for (int j = 0; j < k; ++j) {
      dl[j] = scores[t * k + j] * (dscores[t * k + j] - dot);
      const int e = idx[t * k + j];
      ex[j] = (e >= 0 && e < E) ? e : -1;
    }
  }
  __syncthreads();
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float a = 0.f;
    const float xv = ld_as_f32(x, t * H + h);
    for (int j = 0; j < k; ++j) {
      const int e = ex[j];
      if (e < 0) continue;
      a = fmaf(dl[j], ld_as_f32(W, (int64_t)e * H + h), a);
      if (dW) atomicAdd(dW + (int64_t)e * H + h, dl[j] * xv);
    }
    dx[t * H + h] += a;
  }
  if (db && threadIdx.x < k && ex[threadIdx.x] >= 0) atomicAdd(db + ex[threadIdx.x], dl[threadIdx.x]);
}

struct BwdWS {
  void* dispatch;
  size_t dispatch_bytes;
  int32_t* offsets;
  int32_t* row_of_slot;
  int32_t* token_of_row;
  uint16_t* xp;   // x_perm, later dy
  float* g;       // gate_up pre-activation (fp32)
  uint16_t* dg;   // its gradient
  uint16_t* h;
  uint16_t* y;    // down output, later dx_perm
  uint8_t* scales_t;
  size_t total;
};

BwdWS bwd_carve(void* base, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  BwdWS w{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return base ? static_cast<char*>(base) + at : nullptr;
  };
  const int64_t S = T * k;
  w.dispatch_bytes = dispatch_workspace_bytes(T, k, E);
  w.dispatch = take(w.dispatch_bytes);
  w.offsets = reinterpret_cast<int32_t*>(take((size_t)(E + 1) * 4));
  w.row_of_slot = reinterpret_cast<int32_t*>(take((size_t)S * 4));
  w.token_of_row = reinterpret_cast<int32_t*>(take((size_t)S * 4));
  w.xp = reinterpret_cast<uint16_t*>(take((size_t)S * H * 2));
  w.g = reinterpret_cast<float*>(take((size_t)S * 2 * I * 4));
  w.dg = reinterpret_cast<uint16_t*>(take((size_t)S * 2 * I * 2));
  w.h = reinterpret_cast<uint16_t*>(take((size_t)S * I * 2));
  w.y = reinterpret_cast<uint16_t*>(take((size_t)S * H * 2));
  w.scales_t = reinterpret_cast<uint8_t*>(take(std::max(tc_t_scales_bytes(E, H, I), tc_t_scales_bytes(E, 2 * I, H))));
  w.total = o;
  return w;
}

int grid_for(int64_t work) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(work, 256), (int64_t)sm_count() * 8));
}

}  // namespace

size_t moe_backward_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  return bwd_carve(nullptr, T, H, I, E, k).total;
}

}  // namespace bs

using namespace bs;

extern "C" size_t bs_moe_backward_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  return moe_backward_workspace_bytes(T, H, I, E, k);
}

extern "C" int bs_moe_backward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                               const int32_t* indices, const float* weights, const void* grad_out, int grad_dtype,
                               const void* gate_up_blocks, const void* gate_up_scales, const void* gate_up_bias,
                               const void* down_blocks, const void* down_scales, const void* down_bias,
                               int bias_dtype, float alpha, float limit, float* grad_x, float* grad_weights,
                               void* workspace, size_t workspace_bytes, void* stream) {
  BS_ARG(x && indices && weights && grad_out && gate_up_blocks && gate_up_scales && down_blocks && down_scales &&
             grad_x && grad_weights,
         "bs_moe_backward: null pointer");
  BS_ARG(T >= 0 && H > 0 && I > 0 && E > 0 && k > 0 && k <= E, "bs_moe_backward: bad sizes");
  BS_ARG(grad_dtype == BS_BF16 || grad_dtype == BS_F32, "bs_moe_backward: grad_out must be bf16 or f32");
  BS_ARG(bias_dtype == BS_BF16 || bias_dtype == BS_F32, "bs_moe_backward: bias dtype must be bf16 or f32");
  BS_ARG(tc_t_supported(H, I) && tc_t_supported(2 * I, H),
         "bs_moe_backward: H and 2I must be multiples of 64, H and I of 32");
  BS_ARG(E <= 1024, "bs_moe_backward: at most 1024 experts");
  BS_REQUIRE(tc_supported(gate_up_scales, H, 2 * I) && tc_supported(down_scales, I, H), BS_ERR_MISALIGNED,
             "bs_moe_backward: scales must be 16-byte aligned with rows*groups a multiple of 16");
  BS_ALIGNED16(x, "x");
  BS_ALIGNED16(grad_out, "grad_out");
  if (T == 0) return BS_OK;
  BS_ARG(workspace, "bs_moe_backward: null workspace");
  BS_ALIGNED16(workspace, "workspace");
  const BwdWS w = bwd_carve(workspace, T, H, I, E, k);
  BS_REQUIRE(workspace_bytes >= w.total, BS_ERR_CAPACITY,
             "bs_moe_backward: workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, w.total);
  BS_TRY(check_device());
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t S = T * k;
  const int bf32 = bias_dtype == BS_F32;
  // 1-4: the forward's intermediates, recomputed
  BS_TRY(dispatch_launch(indices, BS_I32, T, k, E, x, H, w.offsets, w.row_of_slot, w.token_of_row, w.xp, w.dispatch,
                         w.dispatch_bytes, st));
  BS_TRY(tc_grouped_launch(2, w.xp, w.offsets, S, S, E, H, 2 * I, gate_up_blocks, gate_up_scales, gate_up_bias, bf32,
                           0.f, 0.f, w.g, st));
  swiglu_rows_kernel<<<grid_for(S * I / 2), 256, 0, st>>>(reinterpret_cast<const float4*>(w.g), S * I, alpha,
                                                          limit, reinterpret_cast<uint32_t*>(w.h));
  BS_LAUNCHED();
  BS_TRY(tc_grouped_launch(1, w.h, w.offsets, S, S, E, I, H, down_blocks, down_scales, down_bias, bf32, 0.f, 0.f,
                           w.y, st));
  // 5: dL/dw and dy (into the x_perm buffer)
  const int cgrid = grid_for(S * 32);
  if (grad_dtype == BS_F32)
    combine_backward_kernel<float><<<cgrid, 256, 0, st>>>(static_cast<const float*>(grad_out), w.y, w.row_of_slot,
                                                          weights, T, (int)k, (int)H, grad_weights, w.xp);
  else
    combine_backward_kernel<uint16_t><<<cgrid, 256, 0, st>>>(static_cast<const uint16_t*>(grad_out), w.y,
                                                             w.row_of_slot, weights, T, (int)k, (int)H, grad_weights,
                                                             w.xp);
  BS_LAUNCHED();
  // 6: dg = SwiGLU'(g) * (dy @ W_d)
  BS_TRY(tc_grouped_t_launch(1, w.xp, w.offsets, S, E, H, I, down_blocks, down_scales, w.scales_t, w.g, alpha, limit,
                             w.dg, st));
  // 7: dx_perm = dg @ W_gu (into the y buffer)
  BS_TRY(tc_grouped_t_launch(0, w.dg, w.offsets, S, E, 2 * I, H, gate_up_blocks, gate_up_scales, w.scales_t, nullptr,
                             0.f, 0.f, w.y, st));
  // 8: dx[t] = sum over the token's slots
  unpermute_sum_kernel<<<grid_for(T * H / 2), 256, 0, st>>>(reinterpret_cast<const uint32_t*>(w.y), w.row_of_slot, T,
                                                            (int)k, (int)(H / 2), reinterpret_cast<float2*>(grad_x));
  BS_LAUNCHED();
  return BS_OK;
}

extern "C" int bs_router_backward(const void* x, int x_dtype, int64_t T, int64_t H, int64_t E, int64_t k,
                                  const void* weight, int w_dtype, const float* scores, const int32_t* indices,
                                  const float* grad_scores, float* grad_x, float* grad_weight, float* grad_bias,
                                  void* stream) {
  BS_ARG(x && weight && scores && indices && grad_scores && grad_x, "bs_router_backward: null pointer");
  BS_ARG(T >= 0 && H > 0 && E > 0 && k > 0 && k <= 32 && k <= E, "bs_router_backward: bad sizes");
  BS_ARG((x_dtype == BS_BF16 || x_dtype == BS_F32) && (w_dtype == BS_BF16 || w_dtype == BS_F32),
         "bs_router_backward: x and weight must be bf16 or f32");
  if (T == 0) return BS_OK;
  BS_TRY(check_device());
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)T);
#define BS_RB(XT, WT)                                                                                              \
  router_backward_kernel<XT, WT><<<grid, 256, 0, st>>>(static_cast<const XT*>(x), static_cast<const WT*>(weight),  \
                                                       (int)H, (int)E, (int)k, scores, indices, grad_scores,       \
                                                       grad_x, grad_weight, grad_bias)
  if (x_dtype == BS_F32 && w_dtype == BS_F32) BS_RB(float, float);
  else if (x_dtype == BS_F32) BS_RB(float, __nv_bfloat16);
  else if (w_dtype == BS_F32) BS_RB(__nv_bfloat16, float);
  else BS_RB(__nv_bfloat16, __nv_bfloat16);
#undef BS_RB
  BS_LAUNCHED();
  return BS_OK;
}

extern "C" size_t bs_mxfp4_matmul_backward_workspace_bytes(int64_t N, int64_t K) {
  return tc_t_scales_bytes(1, N, K);
}

extern "C" int bs_mxfp4_matmul_backward(const void* grad_out, int64_t m, int64_t N, const void* blocks,
                                        const void* scales, int64_t K, void* grad_x, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  BS_ARG(grad_out && blocks && scales && grad_x, "bs_mxfp4_matmul_backward: null pointer");
  BS_ARG(m >= 0 && N > 0 && K > 0, "bs_mxfp4_matmul_backward: bad sizes");
  BS_ARG(tc_t_supported(N, K), "bs_mxfp4_matmul_backward: N must be a multiple of 64 and K of 32");
  if (m == 0) return BS_OK;
  BS_ARG(workspace, "bs_mxfp4_matmul_backward: null workspace");
  BS_REQUIRE(workspace_bytes >= tc_t_scales_bytes(1, N, K), BS_ERR_CAPACITY,
             "bs_mxfp4_matmul_backward: workspace of %zu bytes is smaller than the %zu needed", workspace_bytes,
             tc_t_scales_bytes(1, N, K));
  BS_TRY(check_device());
  return tc_grouped_t_launch(0, grad_out, nullptr, m, 1, N, K, blocks, scales, workspace, nullptr, 0.f, 0.f, grad_x,
                             reinterpret_cast<cudaStream_t>(stream));
}
