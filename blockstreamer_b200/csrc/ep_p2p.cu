// Expert-parallel exchange over peer memory (NVLink through NVSwitch), with
// no host synchronization and no library collective on the data path.
//
// Every rank owns one exchange buffer, allocated once and mapped into every
// other rank's address space through CUDA IPC (plain peer loads and stores;
// no multicast object, no TMA multicast).  Its layout (ep_layout):
//   flags   [3][kMaxRanks] u32: counts / rows / results from source s arrived
//           (each holds the epoch of the last layer call that set it), two
//           local launch counters, this rank's epoch (layer calls so far,
//           advanced on the device, so a captured CUDA graph replays correctly)
//           and this rank's buffer sizes (cap_rows, src_rows), published so
//           that every peer can bound the stores it makes into this buffer;
//   counts  [R][E] i32: row s = source s's rows per global expert;
//   recv    [cap_rows][H] bf16: rows this rank's experts process, expert-major
//           and, within an expert, source-major (the grouped GEMMs read them
//           in place);
//   yback   [src_rows][H] bf16: this rank's own dispatched rows' results,
//           in its dispatch order (the combine reads them in place).
// One layer call with epoch n (the same on every rank, increasing):
//   1. ep_counts_kernel   advance the epoch; publish this rank's per-expert
//                         row counts into every rank's counts row `me`, then
//                         raise flags.counts[me] there (release, system scope);
//   2. ep_scatter_kernel  wait for every source's counts (bounded), compute
//                         where each of this rank's rows lands in its
//                         destination's recv (expert-major), copy x[token] there
//                         (16-byte peer stores), and the last CTA raises
//                         flags.rows[me] on every rank;
//   3. ep_arrived_kernel  wait for every source's rows; write the local expert
//                         offsets for the grouped GEMMs;
//   (the rank's gate_up + SwiGLU and down run on recv)
//   4. ep_return_kernel   copy each result row to its source's yback at the
//                         source's dispatch row; the last CTA raises
//                         flags.results[me] on every rank;
//   5. ep_arrived_kernel  wait for every destination's results (then the
//                         combine kernel reads yback).
// Capacity: a rank whose dispatched rows exceed its src_rows sends nothing
// (its counts go out as zeros) and records BS_ERR_CAPACITY; a sender skips any
// row that would land at or beyond its destination's published cap_rows, and a
// result row beyond its source's published src_rows, recording the same code;
// a receiver clamps its local offsets to its cap_rows.  So no argument can
// make a kernel write outside a peer's buffer.
// Reuse across calls is safe without extra handshakes: a rank starts call n+1
// only after its combine of call n, which follows every destination's step 4
// of call n, which follows that destination's GEMMs over recv (stream order).
// Every wait is bounded (~2 s of SM clock): on timeout the kernel records
// BS_ERR_TIMEOUT in the status word and returns.
#include "bs_common.cuh"

#include <cstring>

namespace bs {
namespace {

constexpr int kMaxRanks = 64;
constexpr int kMaxExperts = 1024;
constexpr long long kWaitCycles = 4000000000LL;
constexpr int kCounts = 0, kRows = 1, kResults = 2;  // flag groups
constexpr int kCtrScatter = 3 * kMaxRanks, kCtrReturn = 3 * kMaxRanks + 1, kEpoch = 3 * kMaxRanks + 2;
constexpr int kCapRows = 3 * kMaxRanks + 3, kSrcRows = 3 * kMaxRanks + 4;  // this buffer's sizes
constexpr int kNumFlags = 3 * kMaxRanks + 5;

struct EPLayout {
  size_t flags, counts, recv, yback, total;
};

__host__ __device__ inline EPLayout ep_layout(int64_t R, int64_t E, int64_t H, int64_t cap_rows,
                                              int64_t src_rows) {
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  EPLayout L;
  size_t o = 0;
  L.flags = o;
  o = al(o + 4 * kNumFlags);
  L.counts = o;
  o = al(o + (size_t)R * E * 4);
  L.recv = o;
  o = al(o + (size_t)cap_rows * H * 2);
  L.yback = o;
  o = al(o + (size_t)src_rows * H * 2);
  L.total = o;
  return L;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0: wait until flags[s] has reached `epoch` for every s < R.
__device__ bool wait_all(const uint32_t* flags, int R, uint32_t epoch, int* status) {
  const long long t0 = clock64();
  for (int s = 0; s < R; ++s) {
    while ((int)(ld_acquire_sys(flags + s) - epoch) < 0) {
      if (clock64() - t0 > kWaitCycles) {
        record_status(status, BS_ERR_TIMEOUT);
        return false;
      }
      __nanosleep(100);
    }
  }
  return true;
}

template <typename T>
__device__ __forceinline__ T* at(uint64_t base, size_t off) {
  return reinterpret_cast<T*>(base + off);
}

// One warp copies a row of `vecs` 16-byte words (src local, dst possibly a
// peer's memory): four loads in flight per lane before its stores, so the
// row's load latency is paid once per four words rather than per word.
__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int64_t vecs,
                                         int lane) {
  int64_t v = lane;
  for (; v + 96 < vecs; v += 128) {
    const uint4 a = src[v], b = src[v + 32], c = src[v + 64], d = src[v + 96];
    dst[v] = a;
    dst[v + 32] = b;
    dst[v + 64] = c;
    dst[v + 96] = d;
  }
  for (; v < vecs; v += 32) dst[v] = src[v];
}

// Last index i in [0, n) with a[i] <= v (a ascending, a[0] <= v).
__device__ __forceinline__ int last_le(const int* a, int n, int v) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a[mid] <= v) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(256) ep_counts_kernel(const int* __restrict__ offsets,
                                                        const uint64_t* __restrict__ bases, int R, int E,
                                                        int me, EPLayout L, int cap_rows, int src_rows,
                                                        int* status) {
  __shared__ uint32_t epoch;
  __shared__ int over;
  if (threadIdx.x == 0) {
    uint32_t* fl = at<uint32_t>(bases[me], L.flags);
    epoch = fl[kEpoch] + 1;
    fl[kEpoch] = epoch;
    // sizes of this rank's buffer, for the peers' bounds checks (ordered
    // before the counts flags below by the fence and the release)
    fl[kCapRows] = (uint32_t)cap_rows;
    fl[kSrcRows] = (uint32_t)src_rows;
    over = offsets[E] > src_rows;
    if (over) record_status(status, BS_ERR_CAPACITY);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * E; i += blockDim.x) {
    const int d = i / E, e = i - d * E;
    at<int>(bases[d], L.counts)[me * E + e] = over ? 0 : offsets[e + 1] - offsets[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < R) st_release_sys(at<uint32_t>(bases[threadIdx.x], L.flags) + kCounts * kMaxRanks + me, epoch);
}

// Dynamic shared memory: counts [R][E], pos [E], off [E + 1] (ints).
__global__ void __launch_bounds__(256) ep_scatter_kernel(const uint4* __restrict__ x, int64_t vecs,
                                                         const int* __restrict__ offsets,
                                                         const int* __restrict__ token_of_row,
                                                         const uint64_t* __restrict__ bases, int R, int E,
                                                         int me, EPLayout L, int src_rows, int* status) {
  extern __shared__ int sm[];
  int* cm = sm;            // [R][E]
  int* pos = cm + R * E;   // [E]: first recv row of this rank's rows of expert e at its destination
  int* off = pos + E;      // [E + 1]: this rank's dispatch offsets
  __shared__ int ok;
  __shared__ int cap[kMaxRanks];  // every destination's published cap_rows
  const uint64_t mine = bases[me];
  uint32_t* flags = at<uint32_t>(mine, L.flags);
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(flags + kEpoch);
  if (threadIdx.x == 0) ok = wait_all(flags + kCounts * kMaxRanks, R, epoch, status);
  __syncthreads();
  if (!ok) return;
  const volatile int* cmg = at<int>(mine, L.counts);
  for (int i = threadIdx.x; i < R * E; i += blockDim.x) cm[i] = cmg[i];
  for (int i = threadIdx.x; i <= E; i += blockDim.x) off[i] = offsets[i];
  // the destinations published their sizes before raising their counts flags
  for (int d = threadIdx.x; d < R; d += blockDim.x)
    cap[d] = (int)*reinterpret_cast<const volatile uint32_t*>(at<uint32_t>(bases[d], L.flags) + kCapRows);
  __syncthreads();
  const int El = E / R;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int d0 = (e / El) * El;
    int p = 0;
    for (int e2 = d0; e2 < e; ++e2)
      for (int s = 0; s < R; ++s) p += cm[s * E + e2];
    for (int s = 0; s < me; ++s) p += cm[s * E + e];
    pos[e] = p;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  // more rows than the exchange was sized for: ep_counts_kernel sent zero
  // counts and recorded the error; send nothing (the flags below still rise)
  const int rows = off[E] > src_rows ? 0 : off[E];
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) / 32; r < rows; r += gridDim.x * blockDim.x / 32) {
    const int e = last_le(off, E + 1, r);
    const int d = e / El;
    const int64_t dst_row = pos[e] + (r - off[e]);
    if (dst_row >= cap[d]) {  // the destination's buffer is smaller than this rank assumed
      if (lane == 0) record_status(status, BS_ERR_CAPACITY);
      continue;
    }
    const uint4* src = x + (int64_t)token_of_row[r] * vecs;
    uint4* dst = at<uint4>(bases[d], L.recv) + dst_row * vecs;
    copy_row(dst, src, vecs, lane);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* ctr = reinterpret_cast<unsigned int*>(flags + kCtrScatter);
    if (atomicAdd(ctr, 1u) == gridDim.x - 1) {
      *ctr = 0;
      __threadfence_system();
      for (int d = 0; d < R; ++d) st_release_sys(at<uint32_t>(bases[d], L.flags) + kRows * kMaxRanks + me, epoch);
    }
  }
}

// Wait for every rank's flag of `group`; with El > 0 also write the local
// expert offsets of recv (expert-major over the counts matrix).
__global__ void ep_arrived_kernel(uint64_t mine, EPLayout L, int group, int R, int E, int me, int El,
                                  int cap_rows, int* __restrict__ local_offsets, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const uint32_t* flags = at<uint32_t>(mine, L.flags);
    ok = wait_all(flags + group * kMaxRanks, R, *reinterpret_cast<const volatile uint32_t*>(flags + kEpoch), status);
  }
  __syncthreads();
  if (!ok || El == 0 || threadIdx.x != 0) return;
  const volatile int* cm = at<int>(mine, L.counts);
  int run = 0;
  for (int e = 0; e < El; ++e) {
    local_offsets[e] = min(run, cap_rows);
    for (int s = 0; s < R; ++s) run += cm[s * E + me * El + e];
  }
  if (run > cap_rows) record_status(status, BS_ERR_CAPACITY);  // the GEMMs then stop at cap_rows
  local_offsets[El] = min(run, cap_rows);
}

// Dynamic shared memory: counts [R][E], loc [El + 1], seg [El][R + 1], src [El][R] (ints).
__global__ void __launch_bounds__(256) ep_return_kernel(const uint4* __restrict__ y, int64_t vecs,
                                                        const uint64_t* __restrict__ bases, int R, int E,
                                                        int me, EPLayout L, int cap_rows, int* status) {
  extern __shared__ int sm[];
  __shared__ int srcmax[kMaxRanks];  // every source's published src_rows
  const int El = E / R;
  int* cm = sm;                    // [R][E]
  int* loc = cm + R * E;           // [El + 1]: expert-major start of local expert e
  int* seg = loc + El + 1;         // [El][R + 1]: start of source s's rows within expert e
  int* src = seg + El * (R + 1);   // [El][R]: source s's dispatch row of its first row of expert e
  const uint64_t mine = bases[me];
  const volatile int* cmg = at<int>(mine, L.counts);
  for (int i = threadIdx.x; i < R * E; i += blockDim.x) cm[i] = cmg[i];
  for (int s = threadIdx.x; s < R; s += blockDim.x)
    srcmax[s] = (int)*reinterpret_cast<const volatile uint32_t*>(at<uint32_t>(bases[s], L.flags) + kSrcRows);
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < El; ++e) {
      loc[e] = run;
      int rs = 0;
      for (int s = 0; s < R; ++s) {
        seg[e * (R + 1) + s] = rs;
        rs += cm[s * E + me * El + e];
      }
      seg[e * (R + 1) + R] = rs;
      run += rs;
    }
    loc[El] = run;
  }
  for (int i = threadIdx.x; i < El * R; i += blockDim.x) {
    const int e = i / R, s = i - e * R;
    int p = 0;
    for (int e2 = 0; e2 < me * El + e; ++e2) p += cm[s * E + e2];
    src[e * R + s] = p;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int rows = min(loc[El], cap_rows);  // the GEMMs produced at most cap_rows rows
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) / 32; r < rows; r += gridDim.x * blockDim.x / 32) {
    const int e = last_le(loc, El + 1, r);
    const int within = r - loc[e];
    const int s = last_le(seg + e * (R + 1), R + 1, within);
    const int64_t dst_row = src[e * R + s] + (within - seg[e * (R + 1) + s]);
    if (dst_row >= srcmax[s]) {  // beyond the source's yback
      if (lane == 0) record_status(status, BS_ERR_CAPACITY);
      continue;
    }
    const uint4* a = y + (int64_t)r * vecs;
    uint4* b = at<uint4>(bases[s], L.yback) + dst_row * vecs;
    copy_row(b, a, vecs, lane);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* ctr = reinterpret_cast<unsigned int*>(at<uint32_t>(mine, L.flags) + kCtrReturn);
    if (atomicAdd(ctr, 1u) == gridDim.x - 1) {
      const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(at<uint32_t>(mine, L.flags) + kEpoch);
      *ctr = 0;
      __threadfence_system();
      for (int s = 0; s < R; ++s) st_release_sys(at<uint32_t>(bases[s], L.flags) + kResults * kMaxRanks + me, epoch);
    }
  }
}

int check_shape(int64_t R, int64_t E, int64_t H, int64_t me) {
  BS_TRY(check_device());
  BS_ARG(R >= 1 && R <= kMaxRanks, "expert parallel: 1 <= ranks <= %d", kMaxRanks);
  BS_ARG(E >= R && E <= kMaxExperts && E % R == 0, "expert parallel: experts (%lld) must split over ranks",
         (long long)E);
  BS_ARG(me >= 0 && me < R, "expert parallel: rank %lld of %lld", (long long)me, (long long)R);
  BS_ARG(H > 0 && H % 8 == 0, "expert parallel: hidden size must be a multiple of 8");
  return BS_OK;
}

int grid_rows(int64_t rows) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, 4 * (int64_t)sm_count()));
}

}  // namespace
}  // namespace bs

using namespace bs;

extern "C" {

size_t bs_ep_p2p_bytes(int64_t R, int64_t E, int64_t H, int64_t cap_rows, int64_t src_rows) {
  return ep_layout(R, E, H, cap_rows, src_rows).total;
}

int bs_ep_p2p_layout(int64_t R, int64_t E, int64_t H, int64_t cap_rows, int64_t src_rows, size_t* recv_offset,
                     size_t* yback_offset) {
  const EPLayout L = ep_layout(R, E, H, cap_rows, src_rows);
  if (recv_offset) *recv_offset = L.recv;
  if (yback_offset) *yback_offset = L.yback;
  return BS_OK;
}

int bs_ep_p2p_alloc(size_t bytes, void** base, void* ipc_handle) {
  BS_ARG(base && ipc_handle && bytes > 0, "bs_ep_p2p_alloc: null argument");
  BS_TRY(check_device());
  void* p = nullptr;
  BS_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    set_error("bs_ep_p2p_alloc: %s", cudaGetErrorString(e));
    return BS_ERR_CUDA;
  }
  *base = p;
  return BS_OK;
}

int bs_ep_p2p_open(const void* ipc_handle, void** peer_base) {
  BS_ARG(ipc_handle && peer_base, "bs_ep_p2p_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  BS_CUDA(cudaIpcOpenMemHandle(peer_base, h, cudaIpcMemLazyEnablePeerAccess));
  return BS_OK;
}

int bs_ep_p2p_close(void* peer_base) {
  BS_CUDA(cudaIpcCloseMemHandle(peer_base));
  return BS_OK;
}

int bs_ep_p2p_free(void* base) {
  BS_CUDA(cudaFree(base));
  return BS_OK;
}

int bs_ep_p2p_dispatch(const void* x, int64_t H, const int32_t* expert_offsets, const int32_t* token_of_row,
                       void* my_base, const uint64_t* peer_bases, int64_t R, int64_t E, int64_t me,
                       int64_t cap_rows, int64_t src_rows, int32_t* local_offsets, void* stream) {
  // every check comes before the first launch: once ep_counts_kernel runs,
  // the peers expect this rank's rows for this epoch
  BS_TRY(check_shape(R, E, H, me));
  BS_ARG(x && expert_offsets && token_of_row && my_base && peer_bases && local_offsets,
         "bs_ep_p2p_dispatch: null pointer");
  BS_ALIGNED16(x, "x");
  BS_ARG(src_rows >= 0 && cap_rows >= R * src_rows && cap_rows < (int64_t)INT32_MAX,
         "bs_ep_p2p_dispatch: cap_rows must hold every rank's rows (>= R * src_rows)");
  const size_t smem = (size_t)(R * E + 2 * E + 1) * 4;
  BS_REQUIRE(smem <= 48 * 1024, BS_ERR_UNSUPPORTED, "bs_ep_p2p_dispatch: %lld ranks x %lld experts too large",
             (long long)R, (long long)E);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const EPLayout L = ep_layout(R, E, H, cap_rows, src_rows);
  int* status = device_status_ptr();
  ep_counts_kernel<<<1, 256, 0, st>>>(expert_offsets, peer_bases, (int)R, (int)E, (int)me, L, (int)cap_rows,
                                      (int)src_rows, status);
  BS_CUDA(cudaGetLastError());
  ep_scatter_kernel<<<grid_rows(src_rows), 256, smem, st>>>(
      static_cast<const uint4*>(x), H / 8, expert_offsets, token_of_row, peer_bases, (int)R, (int)E, (int)me,
      L, (int)src_rows, status);
  BS_CUDA(cudaGetLastError());
  ep_arrived_kernel<<<1, 32, 0, st>>>(reinterpret_cast<uint64_t>(my_base), L, kRows, (int)R, (int)E, (int)me,
                                      (int)(E / R), (int)cap_rows, local_offsets, status);
  BS_CUDA(cudaGetLastError());
  return BS_OK;
}

int bs_ep_p2p_return(const void* y, int64_t H, void* my_base, const uint64_t* peer_bases, int64_t R, int64_t E,
                     int64_t me, int64_t cap_rows, int64_t src_rows, void* stream) {
  BS_TRY(check_shape(R, E, H, me));
  BS_ARG(y && my_base && peer_bases, "bs_ep_p2p_return: null pointer");
  BS_ALIGNED16(y, "y");
  BS_ARG(src_rows >= 0 && cap_rows >= R * src_rows && cap_rows < (int64_t)INT32_MAX,
         "bs_ep_p2p_return: cap_rows must hold every rank's rows (>= R * src_rows)");
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const EPLayout L = ep_layout(R, E, H, cap_rows, src_rows);
  int* status = device_status_ptr();
  const int El = (int)(E / R);
  const size_t smem = (size_t)(R * E + (El + 1) + El * (R + 1) + El * R) * 4;
  BS_REQUIRE(smem <= 48 * 1024, BS_ERR_UNSUPPORTED, "bs_ep_p2p_return: %lld ranks x %lld experts too large",
             (long long)R, (long long)E);
  ep_return_kernel<<<grid_rows(cap_rows), 256, smem, st>>>(static_cast<const uint4*>(y), H / 8, peer_bases,
                                                            (int)R, (int)E, (int)me, L, (int)cap_rows, status);
  BS_CUDA(cudaGetLastError());
  ep_arrived_kernel<<<1, 32, 0, st>>>(reinterpret_cast<uint64_t>(my_base), L, kResults, (int)R, (int)E, (int)me, 0,
                                      (int)cap_rows, nullptr, status);
  BS_CUDA(cudaGetLastError());
  return BS_OK;
}

}  // extern "C"
