// Standalone MXFP4 -> bf16 dequantization (bs_dequant_mxfp4).
//
// Replaces block_streamer/gptoss.py:24-42 (dequantize_expert) ->
// transformers integrations/mxfp4.py:279-355.  HBM-bound: 16.5 bytes read and
// 64 bytes written per 32-element group.
#include "bs_common.cuh"

namespace bs {
namespace {

constexpr int kTileRows = 64;  // rows (N) per CTA tile
constexpr int kTileGroups = 2; // groups per CTA tile (64 K elements)

// Natural orientation out[e, r, g*32 + j]: one thread per group.
__global__ void dequant_natural_kernel(const uint4* __restrict__ blocks,
                                       const uint8_t* __restrict__ scales, int64_t n_groups,
                                       uint4* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_groups;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 b = blocks[i];
    const uint32_t s = scales[i];
    const E2M1Pool pool = make_e2m1_pool(s);
    uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t o[4];
      e2m1x8_decode(w[q], s, pool, o);
      out[i * 4 + q] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Transposed orientation out[e, k, r] (the reference's [G*32, rows]): a CTA
// dequantizes a 64-row x 64-k tile into shared memory and writes it out along r.
__global__ void __launch_bounds__(128) dequant_transposed_kernel(
    const uint4* __restrict__ blocks, const uint8_t* __restrict__ scales, int64_t rows,
    int64_t groups, uint16_t* __restrict__ out) {
  __shared__ uint16_t tile[kTileGroups * 32][kTileRows + 2];
  const int64_t e = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.x * kTileRows;
  const int64_t g0 = (int64_t)blockIdx.y * kTileGroups;
  const int tid = threadIdx.x;
  {
    const int rl = tid % kTileRows;
    const int gl = tid / kTileRows;  // 0..1
    const int64_t r = r0 + rl, g = g0 + gl;
    if (r < rows && g < groups) {
      const int64_t gi = (e * rows + r) * groups + g;
      const uint4 b = blocks[gi];
      const uint32_t s = scales[gi];
      const E2M1Pool pool = make_e2m1_pool(s);
      uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t o[4];
        e2m1x8_decode(w[q], s, pool, o);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          tile[gl * 32 + q * 8 + p * 2][rl] = (uint16_t)(o[p] & 0xFFFF);
          tile[gl * 32 + q * 8 + p * 2 + 1][rl] = (uint16_t)(o[p] >> 16);
        }
      }
    }
  }
  __syncthreads();
  const int64_t K = groups * 32;
  const int64_t k0 = g0 * 32;
  const int kmax = (int)min64(kTileGroups * 32, K - k0);
  const int rmax = (int)min64(kTileRows, rows - r0);
  uint16_t* base = out + e * K * rows;
  for (int i = tid; i < kmax * kTileRows; i += blockDim.x) {
    const int kl = i / kTileRows, rl = i % kTileRows;
    if (rl < rmax) base[(k0 + kl) * rows + r0 + rl] = tile[kl][rl];
  }
}

}  // namespace
}  // namespace bs

extern "C" int bs_dequant_mxfp4(const void* blocks, const void* scales, int64_t experts,
                                int64_t rows, int64_t groups, int transpose, void* out,
                                void* stream) {
  using namespace bs;
  BS_ARG(blocks && scales && out, "bs_dequant_mxfp4: null pointer");
  BS_ARG(experts >= 0 && rows >= 0 && groups >= 0, "bs_dequant_mxfp4: negative size");
  BS_ALIGNED16(blocks, "blocks");
  BS_ALIGNED16(out, "out");
  if (experts == 0 || rows == 0 || groups == 0) return BS_OK;
  BS_TRY(check_device());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!transpose) {
    const int64_t n = experts * rows * groups;
    const int grid = (int)std::min<int64_t>(cdiv(n, 256), (int64_t)sm_count() * 16);
    dequant_natural_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const uint4*>(blocks),
                                                 reinterpret_cast<const uint8_t*>(scales), n,
                                                 reinterpret_cast<uint4*>(out));
  } else {
    BS_ARG(experts <= 65535, "bs_dequant_mxfp4: at most 65535 experts per call");
    dim3 grid((unsigned)cdiv(rows, kTileRows), (unsigned)cdiv(groups, kTileGroups),
              (unsigned)experts);
    BS_ARG(grid.y <= 65535, "bs_dequant_mxfp4: too many groups");
    dequant_transposed_kernel<<<grid, 128, 0, st>>>(reinterpret_cast<const uint4*>(blocks),
                                                    reinterpret_cast<const uint8_t*>(scales),
                                                    rows, groups,
                                                    reinterpret_cast<uint16_t*>(out));
  }
  BS_LAUNCHED();
  return BS_OK;
}
