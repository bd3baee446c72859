// Token permutation (dispatch) without host synchronization.
//
// Replaces block_streamer/gptoss.py:143-154: the reference builds a one-hot
// [E, k, T] mask, calls nonzero() (a device->host sync) and then torch.where()
// per hit expert (one more sync each) before gathering hidden_states[token_idx].
// Here four kernels produce the same grouping on the device:
//   1. count    per token block, per-expert counts (shared-memory atomics);
//   2. scan     per-expert prefix over blocks + exclusive scan over experts;
//   3. scatter  each slot's permuted row: warps rank equal experts with
//               __match_any_sync / __popc, warps and blocks are ordered by scans,
//               so rows of an expert keep (token, slot) order (deterministic);
//   4. gather   x_perm[row] = x[token_of_row[row]] with 16-byte copies.
#include <mutex>

#include "bs_common.cuh"

namespace bs {
namespace {

constexpr int kTokBlock = 256;  // tokens per dispatch block
constexpr int kWarps = 8;

template <typename IdxT>
__device__ __forceinline__ int load_expert(const IdxT* idx, int64_t i, int E, int* status) {
  const int64_t v = (int64_t)idx[i];
  if (v < 0 || v >= E) {
    record_status(status, BS_ERR_INVALID_ARGUMENT);
    return -1;
  }
  return (int)v;
}

template <typename IdxT>
__global__ void __launch_bounds__(256) dispatch_count_kernel(const IdxT* __restrict__ idx,
                                                             int64_t n_slots, int k, int E,
                                                             int* __restrict__ block_counts,
                                                             int* status) {
  extern __shared__ int cnt[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int64_t s0 = (int64_t)blockIdx.x * kTokBlock * k;
  const int64_t s1 = min(n_slots, s0 + (int64_t)kTokBlock * k);
  for (int64_t i = s0 + threadIdx.x; i < s1; i += blockDim.x) {
    const int e = load_expert(idx, i, E, status);
    if (e >= 0) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_counts[(int64_t)blockIdx.x * E + e] = cnt[e];
}

// One CTA: block_prefix[b][e] = sum_{b' < b} counts[b'][e]; offsets = exclusive scan of totals.
__global__ void __launch_bounds__(1024) dispatch_scan_kernel(const int* __restrict__ block_counts,
                                                             int nblk, int E,
                                                             int* __restrict__ block_prefix,
                                                             int* __restrict__ offsets) {
  __shared__ int tot[1024];
  __shared__ int warp_sums[32];
  const int e = threadIdx.x;
  int run = 0;
  if (e < E) {
    for (int b = 0; b < nblk; ++b) {
      const int c = block_counts[(int64_t)b * E + e];
      block_prefix[(int64_t)b * E + e] = run;
      run += c;
    }
  }
  // block-wide exclusive scan of `run` over threads (experts)
  const int lane = e & 31, warp = e >> 5;
  int v = run;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += o;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < (int)(blockDim.x / 32)) ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += o;
    }
    warp_sums[lane] = w;  // inclusive
  }
  __syncthreads();
  const int incl = v + (warp > 0 ? warp_sums[warp - 1] : 0);
  tot[e] = incl;
  if (e < E) offsets[e] = incl - run;
  __syncthreads();
  if (e == 0) offsets[E] = tot[E - 1];
}

template <typename IdxT>
__global__ void __launch_bounds__(256) dispatch_scatter_kernel(
    const IdxT* __restrict__ idx, int64_t n_slots, int k, int E, const int* __restrict__ offsets,
    const int* __restrict__ block_prefix, int* __restrict__ row_of_slot,
    int* __restrict__ token_of_row) {
  extern __shared__ int sm[];
  int* base = sm;        // [E]
  int* wc = sm + E;      // [kWarps][E]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t s0 = (int64_t)blockIdx.x * kTokBlock * k;
  const int n = (int)min(n_slots - s0, (int64_t)kTokBlock * k);
  for (int e = tid; e < E; e += blockDim.x) {
    base[e] = offsets[e] + block_prefix[(int64_t)blockIdx.x * E + e];
    for (int w = 0; w < kWarps; ++w) wc[w * E + e] = 0;
  }
  __syncthreads();
  const int per = (int)cdiv(cdiv(n, kWarps), 32) * 32;
  const int lo = warp * per, hi = min(n, lo + per);
  const unsigned lt_mask = (1u << lane) - 1u;
  // phase 1: per-warp counts
  for (int i0 = lo; i0 < hi; i0 += 32) {
    const int i = i0 + lane;
    int e = -1;
    if (i < hi) {
      const int64_t v = (int64_t)idx[s0 + i];
      e = (v >= 0 && v < E) ? (int)v : -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) wc[warp * E + e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // phase 2: exclusive scan over warps, per expert
  for (int e = tid; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kWarps; ++w) {
      const int c = wc[w * E + e];
      wc[w * E + e] = run;
      run += c;
    }
  }
  __syncthreads();
  // phase 3: positions
  for (int i0 = lo; i0 < hi; i0 += 32) {
    const int i = i0 + lane;
    int e = -1;
    if (i < hi) {
      const int64_t v = (int64_t)idx[s0 + i];
      e = (v >= 0 && v < E) ? (int)v : -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      const int pos = base[e] + wc[warp * E + e] + __popc(peers & lt_mask);
      row_of_slot[s0 + i] = pos;
      token_of_row[pos] = (int)((s0 + i) / k);
    } else if (i < hi) {
      row_of_slot[s0 + i] = -1;
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) wc[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

__global__ void __launch_bounds__(256) gather_rows_kernel(const uint4* __restrict__ x,
                                                          int64_t vecs_per_row,
                                                          const int* __restrict__ token_of_row,
                                                          const int* __restrict__ offsets, int E,
                                                          uint4* __restrict__ x_perm) {
  const int64_t rows = offsets[E];
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; r < rows;
       r += (int64_t)gridDim.x * blockDim.x / 32) {
    const int64_t t = token_of_row[r];
    const uint4* src = x + t * vecs_per_row;
    uint4* dst = x_perm + r * vecs_per_row;
    for (int64_t v = lane; v < vecs_per_row; v += 32) dst[v] = src[v];
  }
}

template <typename IdxT>
int launch_dispatch(const IdxT* idx, int64_t T, int64_t k, int64_t E, const void* x, int64_t H,
                    int32_t* offsets, int32_t* row_of_slot, int32_t* token_of_row, void* x_perm,
                    void* ws, cudaStream_t st) {
  const int64_t n_slots = T * k;
  const int nblk = (int)cdiv(T, kTokBlock);
  int* block_counts = static_cast<int*>(ws);
  int* block_prefix = block_counts + (int64_t)nblk * E;
  int* status = device_status_ptr();
  dispatch_count_kernel<IdxT><<<nblk, 256, E * sizeof(int), st>>>(idx, n_slots, (int)k, (int)E,
                                                                  block_counts, status);
  BS_LAUNCHED();
  dispatch_scan_kernel<<<1, 1024, 0, st>>>(block_counts, nblk, (int)E, block_prefix, offsets);
  BS_LAUNCHED();
  const size_t smem = (size_t)E * (1 + kWarps) * sizeof(int);
  dispatch_scatter_kernel<IdxT><<<nblk, 256, smem, st>>>(idx, n_slots, (int)k, (int)E, offsets,
                                                         block_prefix, row_of_slot, token_of_row);
  BS_LAUNCHED();
  if (x && x_perm) {
    const int64_t vecs = H * 2 / 16;
    const int grid = (int)std::min<int64_t>(cdiv(n_slots, 8), (int64_t)sm_count() * 8);
    gather_rows_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(x), vecs, token_of_row,
                                             offsets, (int)E, static_cast<uint4*>(x_perm));
    BS_LAUNCHED();
  }
  return BS_OK;
}

}  // namespace

// Sizes the dispatch accepts; checked before any size arithmetic, so that
// nothing below can overflow (nblk * E * 8 <= 2^23 * 1024 * 8 bytes).
bool dispatch_sizes_ok(int64_t T, int64_t k, int64_t E) {
  return T >= 0 && k > 0 && k <= 65536 / kTokBlock && E > 0 && E <= 1024 &&
         T <= ((int64_t)INT32_MAX - 1) / k;
}

size_t dispatch_workspace_bytes(int64_t T, int64_t k, int64_t E) {
  if (!dispatch_sizes_ok(T, k, E)) return 0;  // rejected by the entry points anyway
  const int64_t nblk = cdiv(std::max<int64_t>(T, 1), kTokBlock);
  return align_up((size_t)(2 * nblk * E) * sizeof(int), 256);
}

int dispatch_launch(const void* indices, int index_dtype, int64_t T, int64_t k, int64_t E,
                    const void* x, int64_t H, int32_t* offsets, int32_t* row_of_slot,
                    int32_t* token_of_row, void* x_perm, void* ws, size_t ws_bytes,
                    cudaStream_t st) {
  BS_ARG(indices && offsets && row_of_slot && token_of_row, "bs_dispatch: null pointer");
  BS_ARG(index_dtype == BS_I32 || index_dtype == BS_I64, "bs_dispatch: indices must be int32/int64");
  BS_ARG(dispatch_sizes_ok(T, k, E),
         "bs_dispatch: need 0 < E <= 1024, 0 < k <= %d and T * k < 2^31 (T=%lld k=%lld E=%lld)",
         65536 / kTokBlock, (long long)T, (long long)k, (long long)E);
  if (x || x_perm) {
    BS_ARG(x && x_perm && H > 0, "bs_dispatch: x and x_perm go together");
    BS_ARG((H * 2) % 16 == 0, "bs_dispatch: hidden size must be a multiple of 8");
    BS_ALIGNED16(x, "x");
    BS_ALIGNED16(x_perm, "x_perm");
  }
  BS_ARG(ws || T == 0, "bs_dispatch: null workspace");
  BS_REQUIRE(ws_bytes >= dispatch_workspace_bytes(T, k, E), BS_ERR_CAPACITY,
             "bs_dispatch: workspace of %zu bytes is smaller than the %zu needed", ws_bytes,
             dispatch_workspace_bytes(T, k, E));
  BS_TRY(check_device());
  if (T == 0) {
    BS_CUDA(cudaMemsetAsync(offsets, 0, (E + 1) * sizeof(int32_t), st));
    return BS_OK;
  }
  if (index_dtype == BS_I32)
    return launch_dispatch(static_cast<const int32_t*>(indices), T, k, E, x, H, offsets,
                           row_of_slot, token_of_row, x_perm, ws, st);
  return launch_dispatch(static_cast<const int64_t*>(indices), T, k, E, x, H, offsets, row_of_slot,
                         token_of_row, x_perm, ws, st);
}

}  // namespace bs

extern "C" size_t bs_dispatch_workspace_bytes(int64_t T, int64_t k, int64_t E) {
  return bs::dispatch_workspace_bytes(T, k, E);
}

extern "C" int bs_dispatch(const void* indices, int index_dtype, int64_t T, int64_t k, int64_t E,
                           const void* x, int64_t H, int32_t* expert_offsets,
                           int32_t* row_of_slot, int32_t* token_of_row, void* x_perm,
                           void* workspace, size_t workspace_bytes, void* stream) {
  return bs::dispatch_launch(indices, index_dtype, T, k, E, x, H, expert_offsets, row_of_slot,
                             token_of_row, x_perm, workspace, workspace_bytes,
                             reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Allocation-free dispatch (bs_dispatch_noalloc).
//
// Some callers cannot allocate device memory at the point where they dispatch
// tokens: serving loops that must not stall on the device-wide
// synchronization cudaMalloc/cudaFree imply, runtimes that pre-reserve all
// device memory in their own pools, and foreign-language callers (ctypes, cgo,
// JNI) that have no allocator to hand a workspace from.  For them this entry
// point keeps its scratch (the per-block expert counts and their prefix) in a
// fixed device array owned by the library, so the caller passes only inputs
// and outputs.
namespace bs {
namespace {

// Scratch limit: 2 * ceil(T/256) * E ints <= 512 KiB, e.g. T <= 65536 tokens
// with E <= 256 experts.  Every GPU that loads this library holds this array
// until the process exits.
constexpr size_t kNoAllocScratchBytes = 512 * 1024;
static __device__ __align__(256) int g_dispatch_scratch[kNoAllocScratchBytes / sizeof(int)];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of the scratch array on the current device.  The array's name
// is only a host-side handle, so the address is looked up once per device, with
// that device current, on the first call made on it, and cached for the
// process (a cudaDeviceReset would make the cached address stale).
int noalloc_scratch(void** out) {
  int dev = 0;
  BS_CUDA(cudaGetDevice(&dev));
  BS_REQUIRE(dev >= 0 && dev < 64, BS_ERR_UNSUPPORTED, "bs_dispatch_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    BS_CUDA(cudaGetSymbolAddress(&p, g_dispatch_scratch));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return BS_OK;
}

}  // namespace
}  // namespace bs

extern "C" int bs_dispatch_noalloc(const void* indices, int index_dtype, int64_t T, int64_t k,
                                   int64_t E, const void* x, int64_t H, int32_t* expert_offsets,
                                   int32_t* row_of_slot, int32_t* token_of_row, void* x_perm,
                                   void* stream) {
  using namespace bs;
  BS_ARG(dispatch_sizes_ok(T, k, E),
         "bs_dispatch_noalloc: need 0 < E <= 1024, 0 < k <= %d and T * k < 2^31 (T=%lld k=%lld E=%lld)",
         65536 / kTokBlock, (long long)T, (long long)k, (long long)E);
  const size_t need = dispatch_workspace_bytes(T, k, E);
  BS_REQUIRE(need <= kNoAllocScratchBytes, BS_ERR_CAPACITY,
             "bs_dispatch_noalloc: T=%lld, E=%lld needs %zu bytes of scratch, above the fixed %zu "
             "(2 * ceil(T/256) * E * 4 bytes must fit; use bs_dispatch with a workspace)",
             (long long)T, (long long)E, need, kNoAllocScratchBytes);
  BS_TRY(check_device());
  void* scratch = nullptr;
  BS_TRY(noalloc_scratch(&scratch));
  // The scratch is fully rewritten by every call (counts, then prefixes), so
  // nothing has to start at zero.
  return dispatch_launch(indices, index_dtype, T, k, E, x, H, expert_offsets, row_of_slot,
                         token_of_row, x_perm, scratch, kNoAllocScratchBytes,
                         reinterpret_cast<cudaStream_t>(stream));
}
