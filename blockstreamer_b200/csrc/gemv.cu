// Decode-shape expert projections: MXFP4 dequant-GEMV on CUDA cores.
//
// At a few tokens per expert the layer is bound by streaming the packed
// weights from HBM (0.53 bytes per weight), so each weight row is read once
// with 128-bit loads — one 16-byte load is exactly one 32-element MX group
// with one scale byte — decoded in registers and dotted with up to kNT tokens
// held in shared memory.  Work items are (expert, token chunk, 32 output
// columns); the item list is derived on the device from expert_offsets, so no
// host synchronization is needed.
//
//  gemv_gate_up:  h = SwiGLU(x @ W_gu[e] + b_gu[e])  (block_streamer/gptoss.py:158-166, 130-135)
//  gemv_plain:    y = h @ W_d[e] + b_d[e]            (gptoss.py:167-174; also mxfp4_matmul)
#include "bs_common.cuh"

namespace bs {
namespace {

constexpr int kNT = 8;          // tokens per chunk
constexpr int kWarps = 8;       // warps per CTA
constexpr int kColsPerWarp = 4; // output columns per warp per item
constexpr int kColsPerItem = kWarps * kColsPerWarp;

// Per-CTA schedule: expert row offsets and the prefix of token chunks.
struct Schedule {
  int* off;   // [E+1]
  int* cpre;  // [E+1]
};

__device__ void build_schedule(const int* __restrict__ offsets, int64_t rows_total, int E,
                               Schedule s) {
  const int tid = threadIdx.x;
  for (int e = tid; e <= E; e += blockDim.x)
    s.off[e] = offsets ? offsets[e] : (e == 0 ? 0 : (int)rows_total);
  __syncthreads();
  if (tid < 32) {
    const int per = (E + 31) / 32;
    const int e0 = tid * per;
    int sum = 0;
    for (int e = e0; e < min(E, e0 + per); ++e) sum += (s.off[e + 1] - s.off[e] + kNT - 1) / kNT;
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += v;
    }
    int run = incl - sum;
    for (int e = e0; e < min(E, e0 + per); ++e) {
      s.cpre[e] = run;
      run += (s.off[e + 1] - s.off[e] + kNT - 1) / kNT;
    }
    if (tid == 31) s.cpre[E] = incl;
  }
  __syncthreads();
}

__device__ __forceinline__ int find_expert(const int* cpre, int E, int c) {
  int lo = 0, hi = E - 1;  // largest e with cpre[e] <= c
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cpre[mid] <= c) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float load_bias(const void* bias, int f32, int64_t i) {
  if (!bias) return 0.f;
  return f32 ? static_cast<const float*>(bias)[i]
             : __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[i]);
}

// Load rows [r0, r0+nt) of a [*, K] bf16 matrix into xs [kNT][K].
__device__ __forceinline__ void load_rows(const uint16_t* __restrict__ src, int64_t r0, int nt, int K,
                                          uint16_t* xs) {
  const int vecs = K / 8;
  for (int i = threadIdx.x; i < nt * vecs; i += blockDim.x) {
    const int t = i / vecs, v = i - t * vecs;
    reinterpret_cast<uint4*>(xs + (int64_t)t * K)[v] =
        reinterpret_cast<const uint4*>(src + (r0 + t) * (int64_t)K)[v];
  }
}

// acc[t] += dot(32 weights in w[16] (bf16x2), xs[t][k0 .. k0+31])
__device__ __forceinline__ void dot32(const uint32_t w[16], const uint16_t* xs, int K, int k0, int nt,
                                      float acc[kNT]) {
#pragma unroll
  for (int t = 0; t < kNT; ++t) {
    if (t < nt) {
      const uint4* xp = reinterpret_cast<const uint4*>(xs + (int64_t)t * K + k0);
      float a = acc[t];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 xv = xp[q];
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          a = fmaf(bf16lo(w[q * 4 + p]), bf16lo(xw[p]), a);
          a = fmaf(bf16hi(w[q * 4 + p]), bf16hi(xw[p]), a);
        }
      }
      acc[t] = a;
    }
  }
}

__device__ __forceinline__ void decode_group(uint4 b, uint32_t s, uint32_t w[16]) {
  const E2M1Pool pool = make_e2m1_pool(s);
  e2m1x8_decode(b.x, s, pool, w + 0);
  e2m1x8_decode(b.y, s, pool, w + 4);
  e2m1x8_decode(b.z, s, pool, w + 8);
  e2m1x8_decode(b.w, s, pool, w + 12);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kWarps * 32) gemv_gate_up_kernel(
    const uint16_t* __restrict__ x, const int* __restrict__ offsets, int64_t rows_total, int E,
    int H, int I, const uint4* __restrict__ blocks, const uint8_t* __restrict__ scales,
    const void* __restrict__ bias, int bias_f32, float alpha, float limit,
    uint16_t* __restrict__ h) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);
  int* off = reinterpret_cast<int*>(smem_raw + (size_t)kNT * H * 2);
  Schedule sch{off, off + E + 1};
  build_schedule(offsets, rows_total, E, sch);
  const int G = H / 32;
  const int JB = (I + kColsPerItem - 1) / kColsPerItem;
  const int64_t items = (int64_t)sch.cpre[E] * JB;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  int loaded = -1;
  for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
    const int c = (int)(item / JB), jb = (int)(item - (int64_t)c * JB);
    const int e = find_expert(sch.cpre, E, c);
    const int64_t r0 = sch.off[e] + (int64_t)(c - sch.cpre[e]) * kNT;
    const int nt = (int)min64(kNT, sch.off[e + 1] - r0);
    if (c != loaded) {
      __syncthreads();
      load_rows(x, r0, nt, H, xs);
      __syncthreads();
      loaded = c;
    }
    for (int jj = 0; jj < kColsPerWarp; ++jj) {
      const int j = jb * kColsPerItem + warp * kColsPerWarp + jj;
      if (j >= I) break;
      const int64_t rg = (int64_t)e * 2 * I + 2 * j;  // gate row; up row = rg + 1
      float ag[kNT], au[kNT];
#pragma unroll
      for (int t = 0; t < kNT; ++t) ag[t] = au[t] = 0.f;
      for (int g = lane; g < G; g += 32) {
        const uint4 bg = blocks[rg * G + g];
        const uint4 bu = blocks[(rg + 1) * G + g];
        const uint32_t sg = scales[rg * G + g];
        const uint32_t su = scales[(rg + 1) * G + g];
        uint32_t w[16];
        decode_group(bg, sg, w);
        dot32(w, xs, H, g * 32, nt, ag);
        decode_group(bu, su, w);
        dot32(w, xs, H, g * 32, nt, au);
      }
      const float bgv = load_bias(bias, bias_f32, rg), buv = load_bias(bias, bias_f32, rg + 1);
#pragma unroll
      for (int t = 0; t < kNT; ++t) {
        if (t < nt) {
          const float gsum = warp_sum(ag[t]);
          const float usum = warp_sum(au[t]);
          if (lane == t) {
            const float hv = swiglu(gsum + bgv, usum + buv, alpha, limit);
            h[(r0 + t) * I + j] = __bfloat16_as_ushort(__float2bfloat16_rn(hv));
          }
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kWarps * 32) gemv_plain_kernel(
    const uint16_t* __restrict__ x, const int* __restrict__ offsets, int64_t rows_total, int E,
    int K, int N, const uint4* __restrict__ blocks, const uint8_t* __restrict__ scales,
    const void* __restrict__ bias, int bias_f32, uint16_t* __restrict__ y) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);
  int* off = reinterpret_cast<int*>(smem_raw + (size_t)kNT * K * 2);
  Schedule sch{off, off + E + 1};
  build_schedule(offsets, rows_total, E, sch);
  const int G = K / 32;
  const int NB = (N + kColsPerItem - 1) / kColsPerItem;
  const int64_t items = (int64_t)sch.cpre[E] * NB;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  int loaded = -1;
  for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
    const int c = (int)(item / NB), nb = (int)(item - (int64_t)c * NB);
    const int e = find_expert(sch.cpre, E, c);
    const int64_t r0 = sch.off[e] + (int64_t)(c - sch.cpre[e]) * kNT;
    const int nt = (int)min64(kNT, sch.off[e + 1] - r0);
    if (c != loaded) {
      __syncthreads();
      load_rows(x, r0, nt, K, xs);
      __syncthreads();
      loaded = c;
    }
    for (int nn = 0; nn < kColsPerWarp; ++nn) {
      const int n = nb * kColsPerItem + warp * kColsPerWarp + nn;
      if (n >= N) break;
      const int64_t row = (int64_t)e * N + n;
      float acc[kNT];
#pragma unroll
      for (int t = 0; t < kNT; ++t) acc[t] = 0.f;
      for (int g = lane; g < G; g += 32) {
        const uint4 b = blocks[row * G + g];
        const uint32_t s = scales[row * G + g];
        uint32_t w[16];
        decode_group(b, s, w);
        dot32(w, xs, K, g * 32, nt, acc);
      }
      const float bv = load_bias(bias, bias_f32, row);
#pragma unroll
      for (int t = 0; t < kNT; ++t) {
        if (t < nt) {
          const float sum = warp_sum(acc[t]);
          if (lane == t) y[(r0 + t) * N + n] = __bfloat16_as_ushort(__float2bfloat16_rn(sum + bv));
        }
      }
    }
  }
}

int gemv_grid(int64_t rows_total, int E, int per_item_cols, int cols) {
  const int64_t chunks = cdiv(rows_total, kNT) + E;
  const int64_t items = chunks * cdiv(cols, per_item_cols);
  return (int)std::max<int64_t>(1, std::min<int64_t>(items, (int64_t)sm_count() * 4));
}

}  // namespace

int gemv_gate_up_launch(const void* x, const int32_t* offsets, int64_t rows_total, int64_t E,
                        int64_t H, int64_t I, const void* blocks, const void* scales,
                        const void* bias, int bias_f32, float alpha, float limit, void* h,
                        cudaStream_t st) {
  const size_t smem = (size_t)kNT * H * 2 + (size_t)(2 * (E + 1)) * sizeof(int);
  BS_REQUIRE(smem <= 200 * 1024, BS_ERR_CAPACITY, "gemv: hidden size too large");
  BS_CUDA(cudaFuncSetAttribute(gemv_gate_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
  const int grid = gemv_grid(rows_total, (int)E, kColsPerItem, (int)I);
  gemv_gate_up_kernel<<<grid, kWarps * 32, smem, st>>>(
      static_cast<const uint16_t*>(x), offsets, rows_total, (int)E, (int)H, (int)I,
      static_cast<const uint4*>(blocks), static_cast<const uint8_t*>(scales), bias, bias_f32,
      alpha, limit, static_cast<uint16_t*>(h));
  BS_LAUNCHED();
  return BS_OK;
}

int gemv_plain_launch(const void* x, const int32_t* offsets, int64_t rows_total, int64_t E,
                      int64_t K, int64_t N, const void* blocks, const void* scales,
                      const void* bias, int bias_f32, void* y, cudaStream_t st) {
  const size_t smem = (size_t)kNT * K * 2 + (size_t)(2 * (E + 1)) * sizeof(int);
  BS_REQUIRE(smem <= 200 * 1024, BS_ERR_CAPACITY, "gemv: contraction size too large");
  BS_CUDA(cudaFuncSetAttribute(gemv_plain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
  const int grid = gemv_grid(rows_total, (int)E, kColsPerItem, (int)N);
  gemv_plain_kernel<<<grid, kWarps * 32, smem, st>>>(
      static_cast<const uint16_t*>(x), offsets, rows_total, (int)E, (int)K, (int)N,
      static_cast<const uint4*>(blocks), static_cast<const uint8_t*>(scales), bias, bias_f32,
      static_cast<uint16_t*>(y));
  BS_LAUNCHED();
  return BS_OK;
}

}  // namespace bs
