// Grouped expert GEMM run by CTA pairs (tcgen05.mma.cta_group::2, sm_100a):
// BS_ALGO_TCGEN05_PAIR, an alternative to the one-CTA kernel of
// grouped_gemm.cu that the library chooses only on request.
//
// Same product as grouped_gemm.cu (block_streamer/gptoss.py:149-176: for every
// expert e, out[rows of e] = epilogue(X[rows of e] @ W[e]^T), W[e] the MXFP4
// weight [Nw, K] in checkpoint layout), but the MMA's M side is 256 WEIGHT
// rows, 128 in each CTA of a cluster pair, and its N side (up to 320 TOKEN
// rows of one expert) is split in halves between the pair, so every token
// tile crosses L2 once per 256 weight rows instead of once per 128.  One
// thread of the pair's even CTA issues the MMAs (one 256 x 256 and, past 256
// rows, one 256 x <= 64 per K16 step) over both CTAs' tensor and shared
// memory.
//   * A (weights): per CTA, TMA brings 128 rows x 128 bytes of packed e2m1
//     codes (four K steps, 128B-swizzled) and a bulk copy the tile's e8m0
//     scale rows; eight dequant warps (two groups taking alternate K steps,
//     each decoding its two steps of a packed stage together) write bf16
//     straight into TENSOR MEMORY with tcgen05.st ("TS" MMA).
//   * B (tokens): each CTA loads its half of every step's rows (128B-swizzled
//     TMA boxes of 64 and 8 rows) into its own shared memory; the copies of
//     both CTAs count on the even CTA's barrier.
//   * D: fp32 accumulators in each CTA's TMEM (its 128 weight rows x the
//     chunk's columns), drained by the epilogue warps with tcgen05.ld.
// Measured on B200 (gpt-oss-120b, 8192 tokens): slower than the one-CTA
// kernel (gate_up 1.39 vs 1.08 ms, down 0.80 vs 0.53 ms).  Halving the token
// traffic does not pay here because the drain of the single TMEM accumulator
// (~10K cycles per tile; TMEM holds the 320-column accumulator and the six
// dequantized-weight slots, so it cannot be double-buffered) stalls both CTAs
// of a pair, and a 256-row tile pair wastes 6% of the down projection's MMA
// work (2880 rows = 11.25 pairs).
// Warp roles (480 threads per CTA): 0 token TMA, 1 MMA issuer (even CTA) +
// TMEM owner, 2-5 epilogue, 6-13 dequant, 14 weight TMA.  Barriers that
// collect both CTAs' work (token tiles, dequantized slots, accumulator
// release) live in the even CTA; the MMA's completions are multicast to both
// CTAs by tcgen05.commit.  No TMA or bulk copy uses cluster multicast.  Every
// wait is bounded (timeout -> status word, the peer CTA told, clean exit with
// TMEM freed).
// MODE 0: gate_up — bias + clamped interleaved SwiGLU (gptoss.py:130-135,158-166).
// MODE 1: plain   — bias (gptoss.py:167-174) / mxfp4_matmul.
// MODE 2: plain   — bias, fp32 output.
#include <cudaTypedefs.h>

#include "bs_common.cuh"
#include "bs_ptx.cuh"

namespace bs {
namespace {

constexpr int kBM = 128;                       // weight rows per CTA (TMEM lanes); a pair covers 256
constexpr int kBK = 64;                        // K per pipeline step
constexpr int kNMax = 320;                     // token rows per chunk
constexpr int kStagesB = 8;                    // token ring (each CTA holds half of a step's rows)
constexpr int kStagesA = 6;                    // dequantized weight slots (bf16 in TMEM), one per K step
constexpr int kStagesW = 3;                    // packed weight ring (e2m1 bytes in shared memory)
constexpr int kScaleBufs = 1;                  // per-tile scale rows (the next tile's load waits for this one)
constexpr int kWSteps = 4;                     // K steps per packed weight stage
constexpr int kRow = kBK * 2;                  // 128 bytes: one token row of a step
constexpr int kBHalfBytes = kNMax / 2 * kRow;  // 20 KiB: a CTA's half of a token stage
constexpr int kWRow = kWSteps * kBK / 2;       // 128 bytes of one weight row per packed stage
constexpr int kWBytes = kBM * kWRow;           // 16 KiB per packed stage (128B-swizzled)
constexpr int kMaxGroups = 128;                // K <= 4096
constexpr int kACol = 320;                     // TMEM: accumulator columns 0..319, then the weight slots
constexpr int kTmemCols = 512;
constexpr int kDeqGroups = 2;                  // dequant groups of 4 warps, alternating K steps
constexpr int kEpiWarps = 4;                   // epilogue warps (4 or 8: two per TMEM lane quarter)
constexpr int kPerGroup = kWSteps / kDeqGroups;  // K steps per packed stage and dequant group
constexpr int kWarpTMA = 0, kWarpMMA = 1, kWarpEpi0 = 2, kWarpDeq0 = kWarpEpi0 + kEpiWarps;
constexpr int kWarpTMA_A = kWarpDeq0 + 4 * kDeqGroups;  // weight-ring producer
constexpr int kThreads = (kWarpTMA_A + 1) * 32;
// barriers: fullB per token stage (even CTA: both halves' bytes); wfull,
// wempty per packed weight stage; adone (even CTA: both CTAs' dequant warps),
// emptyP / emptyBP (multicast commits after every second step: free the TMEM
// slots / token stages of both steps) per pair of slots / stages; sfull,
// sempty per scale buffer; accfull (multicast commit),
// accempty (even CTA: both CTAs' epilogue warps), drain
constexpr int kPairs = kStagesA / 2;            // MMA completions are committed per two K steps
constexpr int kPairsB = kStagesB / 2;
constexpr int kNumBars = kStagesB + 2 * kStagesW + kStagesA + kPairs + kPairsB + 2 * kScaleBufs + 3;

static_assert(kBHalfBytes % 1024 == 0, "token stages must keep 1024-byte alignment for SW128");
static_assert(kWBytes % 1024 == 0 && kWRow == 128, "packed weight stages are 128B-swizzled rows");
static_assert(kStagesB % 2 == 0 && kStagesA % 2 == 0, "slots and stages are freed per pair of steps");
static_assert(kACol + kStagesA * (kBK / 2) <= kTmemCols, "TMEM budget");
static_assert(kNMax - 256 <= 64 && kNMax % 16 == 0, "chunks are one 256-row and at most one 64-row MMA");

struct Tile {
  int e, mp, nrows, nmma;
  int64_t r0;
};

__device__ __forceinline__ int nchunks_of(int n) { return n > 0 ? (n + kNMax - 1) / kNMax : 0; }

__device__ void build_sched(const int* __restrict__ offsets, int64_t rows_total, int E, int MT,
                            int* off, int* ipre) {
  const int tid = threadIdx.x;
  for (int e = tid; e <= E; e += blockDim.x)
    off[e] = offsets ? offsets[e] : (e == 0 ? 0 : (int)rows_total);
  __syncthreads();
  if (tid < 32) {
    const int per = (E + 31) / 32;
    const int e0 = tid * per, e1 = min(E, e0 + per);
    int sum = 0;
    for (int e = e0; e < e1; ++e) sum += nchunks_of(off[e + 1] - off[e]) * MT;
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += v;
    }
    int run = incl - sum;
    for (int e = e0; e < e1; ++e) {
      ipre[e] = run;
      run += nchunks_of(off[e + 1] - off[e]) * MT;
    }
    if (tid == 31) ipre[E] = incl;
  }
  __syncthreads();
}

__device__ __forceinline__ Tile decode_item(const int* off, const int* ipre, int E, int MT, int item) {
  int lo = 0, hi = E - 1;  // largest e with ipre[e] <= item (skips experts without rows)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (ipre[mid] <= item) lo = mid; else hi = mid - 1;
  }
  Tile t;
  t.e = lo;
  const int local = item - ipre[lo];
  const int c = local / MT;
  t.mp = local - c * MT;
  const int n = off[lo + 1] - off[lo];
  const int nch = nchunks_of(n);
  const int a = (int)(((int64_t)c * n) / nch), b = (int)(((int64_t)(c + 1) * n) / nch);
  t.r0 = off[lo] + a;
  t.nrows = b - a;
  t.nmma = (t.nrows + 15) & ~15;
  return t;
}

__device__ __forceinline__ float bias_at(const void* bias, int f32, int64_t i) {
  if (!bias) return 0.f;
  return f32 ? static_cast<const float*>(bias)[i]
             : __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[i]);
}

// all lanes wait; the warp proceeds only if every lane saw the phase complete
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  const bool ok = ptx::mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// SwiGLU of the reference (gptoss.py:130-135) with the hardware exponential;
// its few-ulp error is far below the bf16 rounding of the output.
__device__ __forceinline__ float swiglu_fast(float gate, float up, float alpha, float limit) {
  gate = fminf(gate, limit);
  up = fminf(fmaxf(up, -limit), limit);
  return (up + 1.0f) * __fdividef(gate, 1.0f + __expf(-alpha * gate));
}

// One 16-column chunk of the accumulator (one token per column) for the lane's
// weight row: bias, then SwiGLU across the (gate, up) lane pair (MODE 0) or the
// plain projection (MODE 1: bf16; MODE 2: fp32).
template <int MODE>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&v)[16], int c0, const Tile& t, int row_w,
                                               bool rv, float bv, float bp, int lane, int Nw,
                                               float alpha, float limit, uint16_t* __restrict__ out) {
  if (MODE == 0) {
    // Lane pair (2i, 2i+1) holds the gate and up rows of one output column.
    // The even lane produces the pair's even token columns, the odd lane the
    // odd ones; each sends its partner the value the partner lacks.
    const int odd = lane & 1;
    const int Iout = Nw >> 1;
    uint16_t* orow = out + (row_w >> 1);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const uint32_t e0 = v[2 * jj], e1 = v[2 * jj + 1];
      const uint32_t mine = odd ? e1 : e0;  // my row at my column
      const uint32_t give = odd ? e0 : e1;  // my row at the partner's column
      const uint32_t got = __shfl_xor_sync(0xffffffffu, give, 1);  // partner's row at my column
      const float own = __uint_as_float(mine) + bv;
      const float oth = __uint_as_float(got) + bp;
      const float hv = odd ? swiglu_fast(oth, own, alpha, limit) : swiglu_fast(own, oth, alpha, limit);
      const int n = c0 + 2 * jj + odd;
      if (n < t.nrows && rv) orow[(t.r0 + n) * Iout] = __bfloat16_as_ushort(__float2bfloat16_rn(hv));
    }
  } else if (MODE == 1) {
    uint16_t* ocol = out + row_w;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int n = c0 + i;
      if (n < t.nrows && rv)
        ocol[(t.r0 + n) * Nw] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[i]) + bv));
    }
  } else {
    float* ocol = reinterpret_cast<float*>(out) + row_w;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int n = c0 + i;
      if (n < t.nrows && rv) ocol[(t.r0 + n) * Nw] = __uint_as_float(v[i]) + bv;
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) tc_grouped_kernel(
    const __grid_constant__ CUtensorMap tm_b64, const __grid_constant__ CUtensorMap tm_b8,
    const __grid_constant__ CUtensorMap tm_a, const uint8_t* __restrict__ scales,
    const int* __restrict__ offsets, int64_t rows_total, int E, int K, int Nw,
    const void* __restrict__ bias, int bias_f32, float alpha, float limit, uint16_t* __restrict__ out,
    int* status) {
  extern __shared__ uint8_t smem_raw[];
  // the dynamic shared window starts at the same offset in both CTAs, so the
  // aligned layout below is identical in the pair (the MMA relies on it)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* wring = smem + kStagesB * kBHalfBytes;            // [kStagesW][kWBytes]
  uint8_t* sbuf = wring + kStagesW * kWBytes;                 // [kScaleBufs][scale_buf]
  const int scale_buf = (kBM * (K / 32) + 127) & ~127;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbuf + kScaleBufs * scale_buf);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* off = reinterpret_cast<int*>(tmem_holder + 2);
  int* ipre = off + (E + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();   // 0: the pair's even CTA, which issues the MMAs
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  auto bar = [&](int i) { return ptx::smem_addr(bars + i); };
  auto fullB = [&](int s) { return bar(s); };
  auto wfull = [&](int s) { return bar(kStagesB + s); };
  auto wempty = [&](int s) { return bar(kStagesB + kStagesW + s); };
  auto adone = [&](int s) { return bar(kStagesB + 2 * kStagesW + s); };
  auto emptyP = [&](int p) { return bar(kStagesB + 2 * kStagesW + kStagesA + p); };
  auto emptyBP = [&](int p) { return bar(kStagesB + 2 * kStagesW + kStagesA + kPairs + p); };
  constexpr int kB0 = kStagesB + 2 * kStagesW + kStagesA + kPairs + kPairsB;
  auto sfull = [&](int b) { return bar(kB0 + b); };
  auto sempty = [&](int b) { return bar(kB0 + kScaleBufs + b); };
  const uint32_t accfull = bar(kB0 + 2 * kScaleBufs), accempty = bar(kB0 + 2 * kScaleBufs + 1),
                 drain = bar(kB0 + 2 * kScaleBufs + 2);
  auto lead = [&](uint32_t a) { return ptx::mapa(a, 0); };   // the even CTA's copy of a barrier
  // a timed-out wait also stops the peer CTA's waits
  const uint32_t peer_abort = ptx::mapa(ptx::smem_addr((const void*)abort_flag), rank ^ 1u);
  auto fail = [&]() { asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory"); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesB; ++s) ptx::mbar_init(fullB(s), 1);
    for (int s = 0; s < kStagesW; ++s) {
      ptx::mbar_init(wfull(s), 1);
      ptx::mbar_init(wempty(s), 4 * kDeqGroups);
    }
    for (int s = 0; s < kStagesA; ++s) ptx::mbar_init(adone(s), 2 * 4);  // the owning group's 4 warps, both CTAs
    for (int p = 0; p < kPairs; ++p) ptx::mbar_init(emptyP(p), 1);
    for (int p = 0; p < kPairsB; ++p) ptx::mbar_init(emptyBP(p), 1);
    for (int b = 0; b < kScaleBufs; ++b) {
      ptx::mbar_init(sfull(b), 1);
      ptx::mbar_init(sempty(b), 4 * kDeqGroups);
    }
    ptx::mbar_init(accfull, 1);
    ptx::mbar_init(accempty, 2 * kEpiWarps);
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kWarpTMA && lane == 0) {
    ptx::tma_prefetch_desc(&tm_b64);
    ptx::tma_prefetch_desc(&tm_b8);
    ptx::tma_prefetch_desc(&tm_a);
  }
  if (warp == kWarpMMA) {
    ptx::tmem_alloc_pair(ptx::smem_addr(tmem_holder), kTmemCols);
    ptx::tmem_relinquish_pair();
  }
  const int MP = (Nw + 2 * kBM - 1) / (2 * kBM);   // 256-row weight tile pairs per expert
  build_sched(offsets, rows_total, E, MP, off, ipre);  // contains __syncthreads
  ptx::tc_fence_before();
  ptx::cluster_sync();        // both CTAs' barriers initialized before any cross-CTA signal
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const int KS = (K + kBK - 1) / kBK;
  const int WS = (KS + kWSteps - 1) / kWSteps;  // packed weight stages per tile
  const int G = K / 32;
  const int total = ipre[E];

  if (warp == kWarpTMA) {
    // ------------------------------------------------------------ token producer (both CTAs)
    if (lane == 0) {
      int last_round[kStagesB];
      for (int s = 0; s < kStagesB; ++s) last_round[s] = -1;
      uint32_t g = 0;
      bool ok = true;
      for (int item = pair; ok && item < total; item += npairs) {
        const Tile t = decode_item(off, ipre, E, MP, item);
        const int h1 = min(t.nmma, 256) / 2, h2 = t.nmma / 2 - h1;   // this CTA's rows of each MMA
        const int row1 = (int)t.r0 + (int)rank * h1;
        const int row2 = (int)t.r0 + 2 * h1 + (int)rank * h2;
        for (int ks = 0; ks < KS; ++ks, ++g) {
          const int s = g % kStagesB;
          // stage s last held step g - kStagesB, whose MMAs are complete once
          // the commit of that step's pair arrived (multicast to both CTAs)
          if (g >= (uint32_t)kStagesB) {
            const uint32_t gp = (g - kStagesB) >> 1;
            if (!ptx::mbar_wait(emptyBP(gp % kPairsB), (gp / kPairsB) & 1, abort_flag)) {
              ok = false;
              fail();
              break;
            }
          }
          const uint32_t fb = lead(fullB(s));
          if (rank == 0) ptx::mbar_arrive_expect_tx(fullB(s), (uint32_t)(t.nmma * kRow));
          uint8_t* st = smem + s * kBHalfBytes;
          const int x = ks * kBK;
          int i = 0;
          for (; i + 64 <= h1; i += 64) ptx::tma_load_2d_pair(ptx::smem_addr(st + i * kRow), &tm_b64, fb, x, row1 + i);
          for (; i < h1; i += 8) ptx::tma_load_2d_pair(ptx::smem_addr(st + i * kRow), &tm_b8, fb, x, row1 + i);
          for (int i2 = 0; i2 < h2; i2 += 8)
            ptx::tma_load_2d_pair(ptx::smem_addr(st + (h1 + i2) * kRow), &tm_b8, fb, x, row2 + i2);
          last_round[s] = g / kStagesB;
        }
      }
      if (!ok && rank == 0) {  // let issued copies (both halves count here) land before the CTA exits
        for (int s = 0; s < kStagesB; ++s)
          if (last_round[s] >= 0) ptx::mbar_wait(fullB(s), last_round[s] & 1, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else if (warp == kWarpTMA_A) {
    // ------------------------------------------------------------ weight producer (both CTAs, own rows)
    if (lane == 0) {
      int last_round[kStagesW];
      for (int s = 0; s < kStagesW; ++s) last_round[s] = -1;
      int last_srnd[kScaleBufs];
      for (int b = 0; b < kScaleBufs; ++b) last_srnd[b] = -1;
      uint32_t g = 0, j = 0;
      bool ok = true;
      for (int item = pair; ok && item < total; item += npairs, ++j) {
        const Tile t = decode_item(off, ipre, E, MP, item);
        const int mt = 2 * t.mp + (int)rank;
        const int arow = t.e * Nw + mt * kBM;
        const int b = j % kScaleBufs, sr = j / kScaleBufs;
        if (!ptx::mbar_wait(sempty(b), (sr & 1) ^ 1, abort_flag)) { ok = false; fail(); break; }
        // the tile's scale rows: one contiguous run of valid_rows * G bytes
        const int vrows = min(kBM, Nw - mt * kBM);
        if (vrows > 0) {
          ptx::mbar_arrive_expect_tx(sfull(b), (uint32_t)(vrows * G));
          ptx::bulk_load(ptx::smem_addr(sbuf + b * scale_buf), scales + (int64_t)arow * G,
                         (uint32_t)(vrows * G), sfull(b));
          last_srnd[b] = sr;
        } else {
          ptx::mbar_arrive(sfull(b));   // a tile past the expert's rows: computed, never stored
        }
        for (int w = 0; w < WS; ++w, ++g) {
          const int s = g % kStagesW, r = g / kStagesW;
          // freed once all eight dequant warps have read their K steps of it
          if (!ptx::mbar_wait(wempty(s), (r & 1) ^ 1, abort_flag)) { ok = false; fail(); break; }
          ptx::mbar_arrive_expect_tx(wfull(s), kWBytes);
          ptx::tma_load_2d(ptx::smem_addr(wring + s * kWBytes), &tm_a, wfull(s), w * kWRow, arow);
          last_round[s] = r;
        }
      }
      if (!ok) {
        for (int s = 0; s < kStagesW; ++s)
          if (last_round[s] >= 0) ptx::mbar_wait(wfull(s), last_round[s] & 1, abort_flag, 200000000LL);
        for (int b = 0; b < kScaleBufs; ++b)
          if (last_srnd[b] >= 0) ptx::mbar_wait(sfull(b), last_srnd[b] & 1, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else if (warp == kWarpMMA) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      uint32_t g = 0, j = 0;
      bool ok = true;
      bool issued = false;
      const uint64_t bdesc0 = ptx::sdesc_kmajor_sw128(ptx::smem_addr(smem));
      const uint32_t a_t0 = tbase + kACol;
      for (int item = pair; ok && item < total; item += npairs, ++j) {
        const Tile t = decode_item(off, ipre, E, MP, item);
        const uint32_t n1 = t.nmma < 256 ? t.nmma : 256, n2 = t.nmma - n1;
        const uint32_t id1 = ptx::idesc_bf16_f32(2 * kBM, n1);
        const uint32_t id2 = n2 ? ptx::idesc_bf16_f32(2 * kBM, n2) : 0u;
        // the B rows of the second MMA follow this CTA's n1 / 2 rows of the first
        const uint64_t b2off = (uint64_t)(((n1 / 2) * kRow) >> 4);
        if (!ptx::mbar_wait(accempty, (j & 1) ^ 1, abort_flag)) { ok = false; fail(); break; }
        ptx::tc_fence_after();
        for (int ks = 0; ks < KS; ++ks, ++g) {
          const int sb = g % kStagesB, sa = g % kStagesA;
          if (!ptx::mbar_wait(adone(sa), (g / kStagesA) & 1, abort_flag) ||
              !ptx::mbar_wait(fullB(sb), (g / kStagesB) & 1, abort_flag)) {
            ok = false;
            fail();
            break;
          }
          ptx::tc_fence_after();
          // descriptors advance by adding to the 16-byte start-address field
          const uint64_t bd = bdesc0 + (uint64_t)((sb * kBHalfBytes) >> 4);
          const uint32_t at = a_t0 + sa * (kBK / 2);
          const uint32_t acc0 = ks > 0 ? 1u : 0u;
          if (n2) {
            // two independent accumulators (columns [0, n1) and [n1, n1 + n2)),
            // issued alternately
            const uint64_t bd2 = bd + b2off;
            ptx::mma_ts_bf16_pair(tbase, at + 0, bd + 0, id1, acc0);
            ptx::mma_ts_bf16_pair(tbase + n1, at + 0, bd2 + 0, id2, acc0);
            ptx::mma_ts_bf16_pair(tbase, at + 8, bd + 2, id1, 1u);
            ptx::mma_ts_bf16_pair(tbase + n1, at + 8, bd2 + 2, id2, 1u);
            ptx::mma_ts_bf16_pair(tbase, at + 16, bd + 4, id1, 1u);
            ptx::mma_ts_bf16_pair(tbase + n1, at + 16, bd2 + 4, id2, 1u);
            ptx::mma_ts_bf16_pair(tbase, at + 24, bd + 6, id1, 1u);
            ptx::mma_ts_bf16_pair(tbase + n1, at + 24, bd2 + 6, id2, 1u);
          } else {
            ptx::mma_ts_bf16_pair(tbase, at + 0, bd + 0, id1, acc0);
            ptx::mma_ts_bf16_pair(tbase, at + 8, bd + 2, id1, 1u);
            ptx::mma_ts_bf16_pair(tbase, at + 16, bd + 4, id1, 1u);
            ptx::mma_ts_bf16_pair(tbase, at + 24, bd + 6, id1, 1u);
          }
          if (g & 1) {
            ptx::tc_commit_pair(emptyP((g >> 1) % kPairs), 0x3);
            ptx::tc_commit_pair(emptyBP((g >> 1) % kPairsB), 0x3);
          }
          issued = true;
        }
        if (!ok) break;
        ptx::tc_commit_pair(accfull, 0x3);
      }
      if (issued) {  // every issued MMA completes before either CTA frees its TMEM
        ptx::tc_commit_pair(drain, 0x3);
        ptx::mbar_wait(drain, 0, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else if (warp < kWarpDeq0) {
    // ------------------------------------------------------------ epilogue (both CTAs, own rows)
    const int q = warp & 3;                           // TMEM lane quarter (warp % 4 rule)
    const int half = (warp - kWarpEpi0) >> 2;         // with 8 warps: alternate 16-column chunks
    const uint32_t accempty_lead = lead(accempty);
    uint32_t j = 0;
    for (int item = pair; item < total; item += npairs, ++j) {
      Tile t = decode_item(off, ipre, E, MP, item);
      if (!warp_wait(accfull, j & 1, abort_flag)) {
        if (lane == 0) fail();
        break;
      }
      ptx::tc_fence_after();
      const int row_w = (2 * t.mp + (int)rank) * kBM + q * 32 + lane;
      const bool rv = row_w < Nw;
      const float bv = rv ? bias_at(bias, bias_f32, (int64_t)t.e * Nw + row_w) : 0.f;
      const float bp = __shfl_xor_sync(0xffffffffu, bv, 1);
      const uint32_t taddr = tbase + ((uint32_t)(q * 32) << 16);
      // One 16-column load per wait: keeping a second load in flight while a
      // chunk is computed made this loop slower on B200 (measured), so the
      // loads stay single.
      for (int c0 = half * 16; c0 < t.nmma; c0 += 16 * (kEpiWarps / 4)) {
        uint32_t v[16];
        ptx::tmem_ld_32x32b_x16(taddr + c0, v);
        ptx::tmem_wait_ld();
        epilogue_chunk<MODE>(v, c0, t, row_w, rv, bv, bp, lane, Nw, alpha, limit, out);
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(accempty_lead);
    }
  } else {
    // ------------------------------------------------------------ dequant (A -> TMEM, both CTAs)
    const int dg = (warp - kWarpDeq0) >> 2;  // dequant group: K steps dg, dg + kDeqGroups, ... of every packed stage
    const int q = warp & 3;
    const int r = q * 32 + lane;            // TMEM lane == row within the weight tile
    const int x = r & 7;                    // 128B swizzle: 16-byte chunk c of row r sits at c ^ (r % 8)
    const uint32_t taddr = tbase + ((uint32_t)(q * 32) << 16) + kACol;
    uint32_t gbase = 0, gw = 0, j = 0;
    bool ok = true;
    for (int item = pair; ok && item < total; item += npairs, ++j, gbase += KS) {
      const int b = j % kScaleBufs;
      if (!warp_wait(sfull(b), (j / kScaleBufs) & 1, abort_flag)) { ok = false; if (lane == 0) fail(); break; }
      const uint8_t* srow = sbuf + b * scale_buf + r * G;
      for (int w = 0; w < WS; ++w, ++gw) {
        const int sw = gw % kStagesW;
        const int kb = w * kWSteps;
        // read this group's K steps of the stage, then release it at once
        uint4 raw[kPerGroup][2] = {};
        if (kb + dg < KS) {
          if (!warp_wait(wfull(sw), (gw / kStagesW) & 1, abort_flag)) { ok = false; if (lane == 0) fail(); break; }
          const uint8_t* row = wring + sw * kWBytes + r * kWRow;
#pragma unroll
          for (int i = 0; i < kPerGroup; ++i) {
            const int kk = dg + i * kDeqGroups;
            raw[i][0] = *reinterpret_cast<const uint4*>(row + (((2 * kk) ^ x) << 4));
            raw[i][1] = *reinterpret_cast<const uint4*>(row + (((2 * kk + 1) ^ x) << 4));
          }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(wempty(sw));
        // decode the steps together (independent work for the scheduler); the
        // byte-table form covers scales 2..252, the general form the rest
        int nst = 0;
        uint32_t sc[kPerGroup][2];
        bool fast = true;
#pragma unroll
        for (int i = 0; i < kPerGroup; ++i) {
          const int ks = kb + dg + i * kDeqGroups;
          nst += ks < KS;
          sc[i][0] = 2 * ks < G ? srow[2 * ks] : 127u;
          sc[i][1] = 2 * ks + 1 < G ? srow[2 * ks + 1] : 127u;
          fast = fast && sc[i][0] - 2u <= 250u && sc[i][1] - 2u <= 250u;
        }
        uint32_t v[kPerGroup][32];
        if (fast) {
#pragma unroll
          for (int i = 0; i < kPerGroup; ++i) {
            const E2M1Pool p0 = make_e2m1_pool(sc[i][0]), p1 = make_e2m1_pool(sc[i][1]);
            e2m1x8_to_bf16x8(raw[i][0].x, p0, v[i] + 0);
            e2m1x8_to_bf16x8(raw[i][0].y, p0, v[i] + 4);
            e2m1x8_to_bf16x8(raw[i][0].z, p0, v[i] + 8);
            e2m1x8_to_bf16x8(raw[i][0].w, p0, v[i] + 12);
            e2m1x8_to_bf16x8(raw[i][1].x, p1, v[i] + 16);
            e2m1x8_to_bf16x8(raw[i][1].y, p1, v[i] + 20);
            e2m1x8_to_bf16x8(raw[i][1].z, p1, v[i] + 24);
            e2m1x8_to_bf16x8(raw[i][1].w, p1, v[i] + 28);
          }
        } else {
#pragma unroll
          for (int i = 0; i < kPerGroup; ++i) {
            const E2M1Pool p0 = make_e2m1_pool(sc[i][0]), p1 = make_e2m1_pool(sc[i][1]);
            e2m1x8_decode(raw[i][0].x, sc[i][0], p0, v[i] + 0);
            e2m1x8_decode(raw[i][0].y, sc[i][0], p0, v[i] + 4);
            e2m1x8_decode(raw[i][0].z, sc[i][0], p0, v[i] + 8);
            e2m1x8_decode(raw[i][0].w, sc[i][0], p0, v[i] + 12);
            e2m1x8_decode(raw[i][1].x, sc[i][1], p1, v[i] + 16);
            e2m1x8_decode(raw[i][1].y, sc[i][1], p1, v[i] + 20);
            e2m1x8_decode(raw[i][1].z, sc[i][1], p1, v[i] + 24);
            e2m1x8_decode(raw[i][1].w, sc[i][1], p1, v[i] + 28);
          }
        }
        // a TMEM slot is free once the MMAs of step g - kStagesA (this group's
        // own earlier step) and of its partner step have completed
#pragma unroll
        for (int i = 0; i < kPerGroup; ++i) {
          const uint32_t g = gbase + kb + dg + i * kDeqGroups;
          if (i < nst && ok && !warp_wait(emptyP((g >> 1) % kPairs), (((g >> 1) / kPairs) & 1) ^ 1, abort_flag))
            ok = false;
        }
        if (!ok) {
          if (lane == 0) fail();
          break;
        }
        ptx::tc_fence_after();
#pragma unroll
        for (int i = 0; i < kPerGroup; ++i) {
          const uint32_t g = gbase + kb + dg + i * kDeqGroups;
          if (i < nst) ptx::tmem_st_32x32b_x32(taddr + (g % kStagesA) * (kBK / 2), v[i]);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int i = 0; i < kPerGroup; ++i) {
            const uint32_t g = gbase + kb + dg + i * kDeqGroups;
            if (i < nst) ptx::mbar_arrive_cluster(lead(adone(g % kStagesA)));
          }
        }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(sempty(b));
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();        // the pair's MMAs, copies and cross-CTA signals are all finished
  if (threadIdx.x == 0 && *abort_flag) record_status(status, BS_ERR_TIMEOUT);
  if (warp == kWarpMMA) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tbase, kTmemCols);
  }
}

}  // namespace

bool tc_supported(const void* scales, int64_t K, int64_t N);

int tc_pair_launch(int mode, const void* x, const int32_t* offsets, int64_t rows_total,
                      int64_t max_rows_per_expert, int64_t E, int64_t K, int64_t N,
                      const void* blocks, const void* scales, const void* bias, int bias_f32,
                      float alpha, float limit, void* out, cudaStream_t st) {
  (void)max_rows_per_expert;
  BS_ARG(E * N < (int64_t)INT32_MAX && rows_total + kNMax < (int64_t)INT32_MAX,
         "tcgen05 pair GEMM: sizes exceed 32-bit TMA coordinates");
  BS_ARG(mode == 1 || N % 2 == 0, "tcgen05 pair GEMM: gate_up rows must be even");
  BS_ARG(offsets || E == 1, "tcgen05 pair GEMM: expert_offsets required");
  BS_ARG(K / 32 <= kMaxGroups, "tcgen05 pair GEMM: contraction size above %d", kMaxGroups * 32);
  BS_REQUIRE(tc_supported(scales, K, N), BS_ERR_MISALIGNED,
             "tcgen05 pair GEMM: scales must be 16-byte aligned with rows*groups a multiple of 16");
  const int64_t G = K / 32;
  CUtensorMap tm_b64, tm_b8, tm_a;
  BS_TRY(make_map_2d(&tm_b64, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)rows_total,
                     (uint64_t)K * 2, kBK, 64, CU_TENSOR_MAP_SWIZZLE_128B));
  BS_TRY(make_map_2d(&tm_b8, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)rows_total,
                     (uint64_t)K * 2, kBK, 8, CU_TENSOR_MAP_SWIZZLE_128B));
  BS_TRY(make_map_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, blocks, (uint64_t)G * 16, (uint64_t)(E * N),
                     (uint64_t)G * 16, kWRow, kBM, CU_TENSOR_MAP_SWIZZLE_128B));
  const size_t scale_buf = (size_t)((kBM * G + 127) & ~127);
  const size_t smem = 1024 + (size_t)kStagesB * kBHalfBytes + (size_t)kStagesW * kWBytes + kScaleBufs * scale_buf +
                      kNumBars * 8 + 16 + (size_t)2 * (E + 1) * sizeof(int);
  BS_REQUIRE(smem <= 227 * 1024, BS_ERR_CAPACITY, "tcgen05 pair GEMM: too many experts for shared memory");
  auto kern = mode == 0 ? tc_grouped_kernel<0> : mode == 1 ? tc_grouped_kernel<1> : tc_grouped_kernel<2>;
  BS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent: one CTA pair per resident SM pair
  cfg.gridDim = dim3((unsigned)(sm_count() & ~1));
  int clusters = 0;
  BS_CUDA(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
  BS_REQUIRE(clusters > 0, BS_ERR_UNSUPPORTED, "tcgen05 pair GEMM: no CTA pair fits on the device");
  cfg.gridDim = dim3((unsigned)(2 * min(clusters, sm_count() / 2)));
  BS_CUDA(cudaLaunchKernelEx(&cfg, kern, tm_b64, tm_b8, tm_a, static_cast<const uint8_t*>(scales), offsets,
                             rows_total, (int)E, (int)K, (int)N, bias, bias_f32, alpha, limit,
                             static_cast<uint16_t*>(out), device_status_ptr()));
  BS_LAUNCHED();
  return BS_OK;
}

}  // namespace bs
