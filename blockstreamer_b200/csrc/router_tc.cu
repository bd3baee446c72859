// Router on the tensor cores (tcgen05): logits = x W^T + b, top-k, softmax.
//
// Same contract as the CUDA-core router in router.cu (transformers
// models/gpt_oss/modeling_gpt_oss.py:126-130), for prefill-sized T.
//   * The fp32 router weight is split exactly into three bf16 terms
//     (W = W1 + W2 + W3: each term takes the next 8 significand bits, and 24
//     bits cover fp32), so x (bf16) times each term is exact and the MMA's fp32
//     accumulation gives fp32-grade logits.  A bf16 weight needs one term.
//   * MMA: M = 128 tokens (TMEM lanes), N = experts (padded to 16), K = H in
//     steps of 64; A = x and B = the split weight, both 128B-swizzled TMA tiles.
//   * Precision: the tensor core's fp32 accumulation loses low bits at every
//     step into a large accumulator (measured: 4-6e-5 on these logits after
//     the 540 steps of one accumulator).  So every two K steps of 64 go into a
//     fresh TMEM accumulator pair — the W1 products apart from the small W2+W3
//     corrections — which the epilogue warps drain into fp32 registers while
//     the MMA fills the other pair (double buffered).  Measured logit error is
//     then below the reference's own CPU fp32 GEMM.
//   * Parallelism: a token tile of 128 is split over K across up to 16 CTAs
//     so the grid fills the SMs at any token count; each CTA writes fp32 partial logits and a
//     warp-per-token kernel (router.cu) adds the partials and the bias, then
//     runs top-k (ties go to the lower expert index) and the softmax.
#include "bs_common.cuh"
#include "bs_ptx.cuh"

namespace bs {
namespace {

constexpr int kRBM = 128;   // tokens per CTA
constexpr int kRBK = 64;    // K per stage
constexpr int kRMaxK = 8;   // top-k handled in registers
constexpr int kREMax = 128; // experts (padded) held in registers per token
constexpr int kRChunk = 2;  // K steps summed in TMEM before each drain to registers
constexpr int kRThreads = 192;
constexpr int kRABytes = kRBM * kRBK * 2;  // 16 KiB

template <typename WT>
__global__ void router_split_kernel(const WT* __restrict__ W, int E, int Ep, int H, int nterms,
                                    uint16_t* __restrict__ out) {
  const int64_t n = (int64_t)Ep * H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i / H;
    float r = 0.f;
    if (e < E) {
      if constexpr (sizeof(WT) == 4) r = W[i]; else r = __bfloat162float(W[i]);
    }
    for (int t = 0; t < nterms; ++t) {
      const __nv_bfloat16 b = __float2bfloat16_rn(r);
      out[t * n + i] = __bfloat16_as_ushort(b);
      r -= __bfloat162float(b);  // exact: the rounding residue of r
    }
  }
}

template <int NTERMS>
__global__ void __launch_bounds__(kRThreads, 1) router_tc_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, int T,
    int H, int Ep, int stages, uint32_t tmem_cols, float* __restrict__ partial, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int SB = kRABytes + NTERMS * Ep * 128;
  constexpr int kParts = NTERMS == 3 ? 2 : 1;  // accumulators per buffer: W1, W2+W3
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + stages * SB);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * stages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  auto full = [&](int s) { return ptx::smem_addr(bars + s); };
  auto empty = [&](int s) { return ptx::smem_addr(bars + stages + s); };
  auto accfull = [&](int b) { return ptx::smem_addr(bars + 2 * stages + b); };
  auto accempty = [&](int b) { return ptx::smem_addr(bars + 2 * stages + 2 + b); };
  const uint32_t drain = ptx::smem_addr(bars + 2 * stages + 4);
  const int m0 = blockIdx.x * kRBM;
  // this CTA's share of the K steps
  const int KS = (H + kRBK - 1) / kRBK;
  const int ns = gridDim.y, split = blockIdx.y;
  const int ks0 = (int)((int64_t)KS * split / ns), ks1 = (int)((int64_t)KS * (split + 1) / ns);
  const int nks = ks1 - ks0;
  const int nch = (nks + kRChunk - 1) / kRChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      ptx::mbar_init(full(s), 1);
      ptx::mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(accfull(b), 1);
      ptx::mbar_init(accempty(b), 4);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_holder), tmem_cols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  // TMEM column of accumulator (buffer b, part p)
  auto acc_col = [&](int b, int p) { return (uint32_t)((b * kParts + p) * Ep); };

  if (warp == 0) {
    if (lane == 0) {
      ptx::tma_prefetch_desc(&tm_x);
      ptx::tma_prefetch_desc(&tm_w);
      int last_round[4] = {-1, -1, -1, -1};
      bool ok = true;
      for (int j = 0; j < nks; ++j) {
        const int s = j % stages, r = j / stages, ks = ks0 + j;
        if (!ptx::mbar_wait(empty(s), (r & 1) ^ 1, abort_flag)) { ok = false; break; }
        uint8_t* st = smem + s * SB;
        ptx::mbar_arrive_expect_tx(full(s), (uint32_t)SB);
        ptx::tma_load_2d(ptx::smem_addr(st), &tm_x, full(s), ks * kRBK, m0);
        for (int t = 0; t < NTERMS; ++t)
          ptx::tma_load_2d(ptx::smem_addr(st + kRABytes + t * Ep * 128), &tm_w, full(s), ks * kRBK, t * Ep);
        last_round[s] = r;
      }
      if (!ok)
        for (int s = 0; s < stages; ++s)
          if (last_round[s] >= 0) ptx::mbar_wait(full(s), last_round[s] & 1, abort_flag, 200000000LL);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_bf16_f32(kRBM, Ep);
      bool ok = true, issued = false;
      for (int j = 0; j < nks && ok; ++j) {
        const int s = j % stages, c = j / kRChunk, b = c & 1;
        const bool first = (j % kRChunk) == 0;
        const bool last = (j % kRChunk) == kRChunk - 1 || j == nks - 1;
        if (!ptx::mbar_wait(full(s), (j / stages) & 1, abort_flag) ||
            (first && !ptx::mbar_wait(accempty(b), ((c >> 1) & 1) ^ 1, abort_flag))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t a = ptx::smem_addr(smem + s * SB);
#pragma unroll
        for (int kk = 0; kk < kRBK / 16; ++kk) {
          const uint64_t ad = ptx::sdesc_kmajor_sw128(a + kk * 32);
          const uint32_t acc = (!first || kk) ? 1u : 0u;
          ptx::mma_ss_bf16(tbase + acc_col(b, 0), ad, ptx::sdesc_kmajor_sw128(a + kRABytes + kk * 32),
                           idesc, acc);
#pragma unroll
          for (int t = 1; t < NTERMS; ++t)
            ptx::mma_ss_bf16(tbase + acc_col(b, 1), ad,
                             ptx::sdesc_kmajor_sw128(a + kRABytes + t * Ep * 128 + kk * 32), idesc,
                             (acc || t > 1) ? 1u : 0u);
        }
        ptx::tc_commit(empty(s));
        if (last) ptx::tc_commit(accfull(b));
        issued = true;
      }
      if (!ok && issued) {
        ptx::tc_commit(drain);
        ptx::mbar_wait(drain, 0, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else {
    // drain each chunk's accumulators into fp32 registers (one token per thread)
    const int q = warp & 3;
    const int t = m0 + q * 32 + lane;
    const uint32_t lane_base = tbase + ((uint32_t)(q * 32) << 16);
    float sum[kREMax];
#pragma unroll
    for (int i = 0; i < kREMax; ++i) sum[i] = 0.f;
    bool ok = true;
    for (int c = 0; c < nch; ++c) {
      const int b = c & 1;
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(accfull(b), (c >> 1) & 1, abort_flag));
      if (!ok) break;
      ptx::tc_fence_after();
#pragma unroll
      for (int cb = 0; cb < kREMax / 32; ++cb) {
        if (cb * 32 < Ep) {
          uint32_t hv[32], lv[32];
          ptx::tmem_ld_32x32b_x32(lane_base + acc_col(b, 0) + cb * 32, hv);
          if (kParts == 2) ptx::tmem_ld_32x32b_x32(lane_base + acc_col(b, 1) + cb * 32, lv);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            sum[cb * 32 + i] += kParts == 2 ? __uint_as_float(hv[i]) + __uint_as_float(lv[i])
                                            : __uint_as_float(hv[i]);
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(accempty(b));
    }
    if (ok && t < T) {
      float4* dst = reinterpret_cast<float4*>(partial + ((int64_t)split * T + t) * Ep);
#pragma unroll
      for (int i = 0; i < kREMax / 4; ++i)
        if (i * 4 < Ep) dst[i] = make_float4(sum[4 * i], sum[4 * i + 1], sum[4 * i + 2], sum[4 * i + 3]);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) record_status(status, BS_ERR_TIMEOUT);
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, tmem_cols);
  }
}

int64_t padded_experts(int64_t E) { return (E + 15) / 16 * 16; }

// K splits per token tile, so that the grid fills the SMs even with few
// token tiles (an expert-parallel rank routes T / R tokens): up to 16, each
// split keeping at least two K steps.  split_cap bounds it independently of
// the device, for the workspace size.
constexpr int kMaxSplits = 16;
int64_t split_cap(int64_t T) {
  const int64_t tiles = std::max<int64_t>(cdiv(T, kRBM), 1);
  return std::max<int64_t>(1, std::min<int64_t>(kMaxSplits, 256 / tiles));
}
int router_splits(int64_t T, int64_t H) {
  const int64_t tiles = std::max<int64_t>(cdiv(T, kRBM), 1);
  const int64_t ks = cdiv(H, kRBK);
  return (int)std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(split_cap(T), ks / 2), sm_count() / tiles));
}

}  // namespace

int router_finish_launch(const float* partial, int ns, int64_t T, int64_t Ep, int64_t E,
                         const void* bias, int bias_f32, int bf16_logits, int64_t k,
                         float* logits, float* scores, void* indices, int index_dtype,
                         cudaStream_t st);

size_t router_tc_workspace_bytes(int64_t T, int64_t H, int64_t E, int w_dtype) {
  const int nterms = w_dtype == BS_F32 ? 3 : 1;
  const int64_t Ep = padded_experts(E);
  return align_up((size_t)nterms * Ep * H * 2, 256) +
         align_up((size_t)split_cap(T) * std::max<int64_t>(T, 1) * Ep * 4, 256);
}

bool router_tc_supported(int x_dtype, int64_t T, int64_t H, int64_t E, int64_t k, const void* x) {
  return x_dtype == BS_BF16 && T > 64 && E <= kREMax && k <= 32 && H % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(x) & 15) == 0 && T < (int64_t)INT32_MAX - kRBM;
}

int router_tc_launch(const void* x, const void* weight, const void* bias, int w_dtype, int64_t T,
                     int64_t H, int64_t E, int64_t k, float* logits, float* scores, void* indices,
                     int index_dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  const int nterms = w_dtype == BS_F32 ? 3 : 1;
  const int64_t Ep = padded_experts(E);
  BS_REQUIRE(ws && ws_bytes >= router_tc_workspace_bytes(T, H, E, w_dtype), BS_ERR_CAPACITY,
             "router: workspace too small");
  BS_ALIGNED16(ws, "router workspace");
  uint16_t* wsplit = static_cast<uint16_t*>(ws);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(ws) +
                                            align_up((size_t)nterms * Ep * H * 2, 256));
  const int grid_split = (int)std::min<int64_t>(cdiv(Ep * H, 256), (int64_t)sm_count() * 8);
  if (w_dtype == BS_F32)
    router_split_kernel<float><<<grid_split, 256, 0, st>>>(static_cast<const float*>(weight), (int)E,
                                                           (int)Ep, (int)H, nterms, wsplit);
  else
    router_split_kernel<__nv_bfloat16><<<grid_split, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(weight), (int)E, (int)Ep, (int)H, nterms, wsplit);
  BS_LAUNCHED();
  CUtensorMap tm_x, tm_w;
  BS_TRY(make_map_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)H, (uint64_t)T,
                     (uint64_t)H * 2, kRBK, kRBM, CU_TENSOR_MAP_SWIZZLE_128B));
  BS_TRY(make_map_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, wsplit, (uint64_t)H,
                     (uint64_t)(nterms * Ep), (uint64_t)H * 2, kRBK, (uint32_t)Ep,
                     CU_TENSOR_MAP_SWIZZLE_128B));
  const int SB = kRABytes + nterms * (int)Ep * 128;
  const int stages = (int)std::min<int64_t>(4, (200 * 1024) / SB);
  BS_REQUIRE(stages >= 2, BS_ERR_CAPACITY, "router: too many experts for the tensor-core path");
  const size_t smem = 1024 + (size_t)stages * SB + (2 * stages + 5) * 8 + 16;
  uint32_t cols = 32;
  while (cols < (uint32_t)(2 * (nterms == 3 ? 2 : 1) * Ep)) cols <<= 1;
  auto kern = nterms == 3 ? router_tc_kernel<3> : router_tc_kernel<1>;
  BS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int ns = router_splits(T, H);
  dim3 grid((unsigned)cdiv(T, kRBM), (unsigned)ns);
  kern<<<grid, kRThreads, smem, st>>>(tm_x, tm_w, (int)T, (int)H, (int)Ep, stages, cols, partial,
                                      device_status_ptr());
  BS_LAUNCHED();
  return router_finish_launch(partial, ns, T, Ep, E, bias, w_dtype == BS_F32, w_dtype == BS_BF16, k,
                              logits, scores, indices, index_dtype, st);
}

}  // namespace bs
