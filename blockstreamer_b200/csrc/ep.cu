// Expert-parallel row movement: regroup rows received from an all-to-all into
// expert order, and gather them back.
//
// After the dispatch all-to-all a rank holds, for each source rank s and each
// of its local experts e, a contiguous segment of counts[s][e] rows, laid out
// [s][e] (source-major).  The grouped GEMMs want expert-major rows, so
//   dest(s, e, j) = expert_offsets[e] + sum_{s' < s} counts[s'][e] + j
// and row_map[i] records, for received row i, its expert-major row.  The
// reverse gather restores the [s][e] order for the combine all-to-all.  Every
// CTA recomputes the small R x E scans in shared memory (no extra launch).
#include "bs_common.cuh"

namespace bs {
namespace {

constexpr int kMaxSeg = 4096;  // R * E_local

__global__ void __launch_bounds__(256) ep_regroup_kernel(const int* __restrict__ counts, int R, int El,
                                                         const uint4* __restrict__ x_recv,
                                                         int64_t vecs, int64_t rows,
                                                         uint4* __restrict__ x_grouped,
                                                         int* __restrict__ expert_offsets,
                                                         int* __restrict__ row_map) {
  __shared__ int seg_start[kMaxSeg + 1];  // source-major start of segment (s, e)
  __shared__ int dst_start[kMaxSeg];      // expert-major start of segment (s, e)
  const int nseg = R * El;
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < nseg; ++i) {
      seg_start[i] = run;
      run += counts[i];
    }
    seg_start[nseg] = run;
    int eo = 0;
    for (int e = 0; e < El; ++e) {
      if (blockIdx.x == 0) expert_offsets[e] = eo;
      for (int s = 0; s < R; ++s) {
        dst_start[s * El + e] = eo;
        eo += counts[s * El + e];
      }
    }
    if (blockIdx.x == 0) expert_offsets[El] = eo;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; r < rows;
       r += (int64_t)gridDim.x * blockDim.x / 32) {
    int lo = 0, hi = nseg - 1;  // last segment with seg_start <= r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (seg_start[mid] <= r) lo = mid; else hi = mid - 1;
    }
    const int64_t d = dst_start[lo] + (r - seg_start[lo]);
    if (lane == 0) row_map[r] = (int)d;
    if (x_recv) {
      const uint4* src = x_recv + r * vecs;
      uint4* dst = x_grouped + d * vecs;
      for (int64_t v = lane; v < vecs; v += 32) dst[v] = src[v];
    }
  }
}

__global__ void __launch_bounds__(256) gather_by_map_kernel(const uint4* __restrict__ src,
                                                            const int* __restrict__ row_map,
                                                            int64_t rows, int64_t vecs,
                                                            uint4* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; r < rows;
       r += (int64_t)gridDim.x * blockDim.x / 32) {
    const uint4* s = src + (int64_t)row_map[r] * vecs;
    uint4* d = dst + r * vecs;
    for (int64_t v = lane; v < vecs; v += 32) d[v] = s[v];
  }
}

}  // namespace
}  // namespace bs

extern "C" int bs_ep_regroup(const int32_t* recv_counts, int64_t R, int64_t El, const void* x_recv,
                             int64_t rows, int64_t H, void* x_grouped, int32_t* expert_offsets,
                             int32_t* row_map, void* stream) {
  using namespace bs;
  BS_ARG(recv_counts && expert_offsets && row_map, "bs_ep_regroup: null pointer");
  BS_ARG(R > 0 && El > 0 && R * El <= kMaxSeg, "bs_ep_regroup: need 0 < ranks*experts <= %d", kMaxSeg);
  BS_ARG(rows >= 0 && rows < (int64_t)INT32_MAX, "bs_ep_regroup: bad row count");
  BS_ARG((x_recv == nullptr) == (x_grouped == nullptr), "bs_ep_regroup: x_recv and x_grouped go together");
  if (x_recv) {
    BS_ARG(H > 0 && H % 8 == 0, "bs_ep_regroup: hidden size must be a multiple of 8");
    BS_ALIGNED16(x_recv, "x_recv");
    BS_ALIGNED16(x_grouped, "x_grouped");
  }
  BS_TRY(check_device());
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(rows, 8), (int64_t)sm_count() * 8));
  ep_regroup_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      recv_counts, (int)R, (int)El, static_cast<const uint4*>(x_recv), H / 8, rows,
      static_cast<uint4*>(x_grouped), expert_offsets, row_map);
  BS_LAUNCHED();
  return BS_OK;
}

extern "C" int bs_gather_rows(const void* src, const int32_t* row_map, int64_t rows, int64_t H,
                              void* dst, void* stream) {
  using namespace bs;
  BS_ARG(src && row_map && dst, "bs_gather_rows: null pointer");
  BS_ARG(rows >= 0 && H > 0 && H % 8 == 0, "bs_gather_rows: bad sizes");
  BS_ALIGNED16(src, "src");
  BS_ALIGNED16(dst, "dst");
  if (rows == 0) return BS_OK;
  BS_TRY(check_device());
  const int grid = (int)std::min<int64_t>(cdiv(rows, 8), (int64_t)sm_count() * 8);
  gather_by_map_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), row_map, rows, H / 8, static_cast<uint4*>(dst));
  BS_LAUNCHED();
  return BS_OK;
}
