// Grouped expert GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces the per-expert loop of block_streamer/gptoss.py:149-176 at prefill
// shapes: for every expert e, out[rows of e] = epilogue(X[rows of e] @ W[e]^T)
// with W[e] the MXFP4 weight [Nw, K] (checkpoint layout, K-contiguous).
//
// Formulation ("swap AB"): the MMA's M side is 128 WEIGHT rows, its N side is up
// to 320 TOKEN rows of one expert, so at uniform routing every weight byte is
// fetched and dequantized once per layer.
//   * A (weights): TMA brings the packed e2m1 bytes of a 128x64 slice into
//     shared memory and a bulk copy brings the tile's e8m0 scale rows; eight
//     dequant warps (two groups taking alternate K steps) decode them bit-exactly
//     and write bf16 straight into TENSOR MEMORY with tcgen05.st — the MMA reads
//     A from TMEM ("TS" form), so dequantized weights never touch shared memory.
//   * B (tokens): 128B-swizzled TMA tiles of 64 x 64 bf16 in shared memory.
//   * D: fp32 accumulators in TMEM (up to 320 columns: one 128x256 and one
//     128x64 MMA per K16 step), drained by four epilogue warps with tcgen05.ld.
// Warp roles (512 threads): 0 token-tile TMA producer, 1 MMA issuer (+TMEM
// owner), 2-5 epilogue, 6-13 dequant, 14 weight TMA producer, 15 second MMA
// issuer.  MMA issue is on the critical path (one thread issues a tcgen05.mma
// every ~115 cycles at N <= 128, ~160 at N = 256, whatever other threads
// issue), so each issuer's loop is kept minimal -- one barrier wait, four MMAs
// with precomputed descriptors, one commit -- and the 128x64 MMAs of tiles
// above 256 token rows have their own issuer.  The token tiles
// (4 x 40 KiB stages) and the weights (6 x 4 KiB e2m1 stages, 6 x 32 TMEM
// columns) have separate rings so the dequant can run further ahead than the
// large token stages allow.  Every wait is bounded (timeout -> status word +
// clean exit, TMEM freed).
// MODE 0: gate_up — bias + clamped interleaved SwiGLU (gptoss.py:130-135,158-166).
// MODE 1: plain   — bias (gptoss.py:167-174) / mxfp4_matmul.
// MODE 2: plain   — bias, fp32 output (the backward's recomputed gate_up
//                   pre-activation, whose clamp masks must match fp32).
#include <cudaTypedefs.h>

#include "bs_common.cuh"
#include "bs_ptx.cuh"

namespace bs {
namespace {

constexpr int kBM = 128;                       // weight rows per tile (MMA M)
constexpr int kBK = 64;                        // K per pipeline stage
constexpr int kNMax = 320;                     // token rows per tile
constexpr int kStagesB = 4;                    // token-tile ring (shared memory)
constexpr int kStagesA = 6;                    // weight ring (e2m1 bytes in smem, bf16 in TMEM)
constexpr int kBoxRows = 64;                   // token rows per TMA box
constexpr int kBoxBytes = kBoxRows * kBK * 2;  // 8 KiB
constexpr int kBBytes = kNMax * kBK * 2;       // 40 KiB per token stage
constexpr int kABytes = kBM * kBK / 2;         // 4 KiB of e2m1 bytes per weight stage
constexpr int kMaxGroups = 128;                // K <= 4096
constexpr int kACol = 320;                   constexpr int kTmemCols = 512;
constexpr int kDeqGroups = 2;
constexpr int kWarpTMA = 0, kWarpMMA = 1, kWarpEpi0 = 2, kWarpDeq0 = 6;
constexpr int kWarpTMA_A = kWarpDeq0 + 4 * kDeqGroups;  // weight-ring producer
constexpr int kWarpMMA2 = kWarpTMA_A + 1;              // second MMA issuer: the 128x64 MMAs of tiles above 256 rows
constexpr int kThreads = (kWarpMMA2 + 1) * 32;
// barriers: fullB per token stage; fullA, adone, emptyA per weight stage (emptyA
// also frees the token stage of the same K step); sfull, sempty per scale
// buffer; accfull, accempty, drain
constexpr int kNumBars = kStagesB + 3 * kStagesA + 4 + 3;

static_assert(kBBytes % 1024 == 0, "token stages must keep 1024-byte alignment for SW128");
static_assert(kACol + kStagesA * (kBK / 2) <= kTmemCols, "TMEM budget");

struct Tile {
  int e, mt, nrows, nmma;
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
  t.mt = local - c * MT;
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
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_a,
    const uint8_t* __restrict__ scales, const int* __restrict__ offsets, int64_t rows_total,
    int E, int K, int Nw, const void* __restrict__ bias, int bias_f32, float alpha, float limit,
    uint16_t* __restrict__ out, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* asm_ring = smem + kStagesB * kBBytes;            // [kStagesA][kABytes]
  uint8_t* sbuf = asm_ring + kStagesA * kABytes;            // [2][scale_buf]
  const int scale_buf = (kBM * (K / 32) + 127) & ~127;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbuf + 2 * scale_buf);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* off = reinterpret_cast<int*>(tmem_holder + 2);
  int* ipre = off + (E + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return ptx::smem_addr(bars + i); };
  auto fullB = [&](int s) { return bar(s); };
  auto fullA = [&](int s) { return bar(kStagesB + s); };
  auto adone = [&](int s) { return bar(kStagesB + kStagesA + s); };
  auto emptyA = [&](int s) { return bar(kStagesB + 2 * kStagesA + s); };
  constexpr int kB0 = kStagesB + 3 * kStagesA;
  auto sfull = [&](int b) { return bar(kB0 + b); };
  auto sempty = [&](int b) { return bar(kB0 + 2 + b); };
  const uint32_t accfull = bar(kB0 + 4), accempty = bar(kB0 + 5), drain = bar(kB0 + 6);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesB; ++s) ptx::mbar_init(fullB(s), 1);
    for (int s = 0; s < kStagesA; ++s) {
      ptx::mbar_init(fullA(s), 1);
      ptx::mbar_init(adone(s), 4);
      ptx::mbar_init(emptyA(s), 2);  // a commit from each MMA issuer
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(sfull(b), 1);
      ptx::mbar_init(sempty(b), 4 * kDeqGroups);
    }
    ptx::mbar_init(accfull, 2);
    ptx::mbar_init(accempty, 4);
    ptx::mbar_init(drain, 2);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kWarpTMA && lane == 0) {
    ptx::tma_prefetch_desc(&tm_b);
    ptx::tma_prefetch_desc(&tm_a);
  }
  if (warp == kWarpMMA) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_holder), kTmemCols);
    ptx::tmem_relinquish();
  }
  const int MT = (Nw + kBM - 1) / kBM;
  build_sched(offsets, rows_total, E, MT, off, ipre);  // contains __syncthreads
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const int KS = (K + kBK - 1) / kBK;
  const int G = K / 32;
  const int total = ipre[E];

  if (warp == kWarpTMA) {
    // ------------------------------------------------------------ token-tile producer
    if (lane == 0) {
      int last_round[kStagesB];
      for (int s = 0; s < kStagesB; ++s) last_round[s] = -1;
      uint32_t g = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x) {
        const Tile t = decode_item(off, ipre, E, MT, item);
        const int nbox = (t.nmma + kBoxRows - 1) / kBoxRows;
        for (int ks = 0; ks < KS; ++ks, ++g) {
          const int s = g % kStagesB, r = g / kStagesB;
          // stage s last held K step g - kStagesB; its MMAs are complete once the
          // weight-ring barrier of that step has flipped (one commit per step)
          if (g >= (uint32_t)kStagesB) {
            const uint32_t gp = g - kStagesB;
            if (!ptx::mbar_wait(emptyA(gp % kStagesA), (gp / kStagesA) & 1, abort_flag)) { ok = false; break; }
          }
          uint8_t* st = smem + s * kBBytes;
          ptx::mbar_arrive_expect_tx(fullB(s), nbox * kBoxBytes);
          for (int jb = 0; jb < nbox; ++jb)
            ptx::tma_load_2d(ptx::smem_addr(st + jb * kBoxBytes), &tm_b, fullB(s), ks * kBK,
                             (int)(t.r0 + jb * kBoxRows));
          last_round[s] = r;
        }
      }
      if (!ok) {  // let issued copies land before the CTA exits
        for (int s = 0; s < kStagesB; ++s)
          if (last_round[s] >= 0) ptx::mbar_wait(fullB(s), last_round[s] & 1, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else if (warp == kWarpTMA_A) {
    // ------------------------------------------------------------ weight producer (e2m1 + scales)
    if (lane == 0) {
      int last_round[kStagesA];
      for (int s = 0; s < kStagesA; ++s) last_round[s] = -1;
      int last_srnd[2] = {-1, -1};
      uint32_t g = 0, j = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x, ++j) {
        const Tile t = decode_item(off, ipre, E, MT, item);
        const int arow = t.e * Nw + t.mt * kBM;
        // the tile's scale rows: one contiguous run of valid_rows * G bytes
        const int b = j & 1, sr = j >> 1;
        if (!ptx::mbar_wait(sempty(b), (sr & 1) ^ 1, abort_flag)) { ok = false; break; }
        const int vrows = min(kBM, Nw - t.mt * kBM);
        ptx::mbar_arrive_expect_tx(sfull(b), (uint32_t)(vrows * G));
        ptx::bulk_load(ptx::smem_addr(sbuf + b * scale_buf), scales + (int64_t)arow * G,
                       (uint32_t)(vrows * G), sfull(b));
        last_srnd[b] = sr;
        for (int ks = 0; ks < KS; ++ks, ++g) {
          const int s = g % kStagesA, r = g / kStagesA;
          if (!ptx::mbar_wait(emptyA(s), (r & 1) ^ 1, abort_flag)) { ok = false; break; }
          ptx::mbar_arrive_expect_tx(fullA(s), kABytes);
          ptx::tma_load_2d(ptx::smem_addr(asm_ring + s * kABytes), &tm_a, fullA(s), ks * (kBK / 2), arow);
          last_round[s] = r;
        }
      }
      if (!ok) {
        for (int s = 0; s < kStagesA; ++s)
          if (last_round[s] >= 0) ptx::mbar_wait(fullA(s), last_round[s] & 1, abort_flag, 200000000LL);
        for (int b = 0; b < 2; ++b)
          if (last_srnd[b] >= 0) ptx::mbar_wait(sfull(b), last_srnd[b] & 1, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else if (warp == kWarpMMA || warp == kWarpMMA2) {
    // ------------------------------------------------------------ MMA issuers
    // One thread issues a tcgen05.mma every ~115 cycles (N <= 128; ~160 at
    // N = 256) whatever other threads issue, so the second accumulator of a
    // tile above 256 rows (its 128x64 MMAs) has its own issuer: warp
    // kWarpMMA issues the N <= 256 MMAs, warp kWarpMMA2 the rest; both wait
    // for the same operands and both commit every stage and tile.
    if (lane == 0) {
      const bool second = warp == kWarpMMA2;
      uint32_t g = 0, j = 0;
      bool ok = true;
      bool issued = false;
      const uint64_t bdesc0 = ptx::sdesc_kmajor_sw128(ptx::smem_addr(smem));
      const uint32_t a_t0 = tbase + kACol;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x, ++j) {
        const Tile t = decode_item(off, ipre, E, MT, item);
        const uint32_t n1 = t.nmma < 256 ? t.nmma : 256, n2 = t.nmma - n1;
        const uint32_t id = second ? (n2 ? ptx::idesc_bf16_f32(kBM, n2) : 0u) : ptx::idesc_bf16_f32(kBM, n1);
        const bool any = !second || n2 > 0;  // the second issuer has nothing to do for tiles of <= 256 rows
        const uint32_t dacc = second ? tbase + 256 : tbase;
        if (!ptx::mbar_wait(accempty, (j & 1) ^ 1, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        for (int ks = 0; ks < KS; ++ks, ++g) {
          const int sb = g % kStagesB, sa = g % kStagesA;
          // adone(sa) is signalled by the dequant warps only after they also saw
          // this step's token tile land (fullB), so one wait covers both operands
          if (!ptx::mbar_wait(adone(sa), (g / kStagesA) & 1, abort_flag)) {
            ok = false;
            break;
          }
          if (any) {
            ptx::tc_fence_after();
            // descriptors advance by adding to the 16-byte start-address field
            const uint64_t bd = bdesc0 + (uint64_t)((sb * kBBytes) >> 4) + (second ? (uint64_t)((256 * 128) >> 4) : 0u);
            const uint32_t at = a_t0 + sa * (kBK / 2);
            const uint32_t acc0 = ks > 0 ? 1u : 0u;
            ptx::mma_ts_bf16(dacc, at + 0, bd + 0, id, acc0);
            ptx::mma_ts_bf16(dacc, at + 8, bd + 2, id, 1u);
            ptx::mma_ts_bf16(dacc, at + 16, bd + 4, id, 1u);
            ptx::mma_ts_bf16(dacc, at + 24, bd + 6, id, 1u);
            issued = true;
          }
          ptx::tc_commit(emptyA(sa));
        }
        if (!ok) break;
        ptx::tc_commit(accfull);
      }
      if (!ok) {  // every issued MMA must finish before TMEM is freed: both issuers commit
        ptx::tc_commit(drain);
        if (issued) ptx::mbar_wait(drain, 0, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else if (warp < kWarpDeq0) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    uint32_t j = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++j) {
      const Tile t = decode_item(off, ipre, E, MT, item);
      if (!warp_wait(accfull, j & 1, abort_flag)) break;
      ptx::tc_fence_after();
      const int row_w = t.mt * kBM + q * 32 + lane;
      const bool rv = row_w < Nw;
      const float bv = rv ? bias_at(bias, bias_f32, (int64_t)t.e * Nw + row_w) : 0.f;
      const float bp = __shfl_xor_sync(0xffffffffu, bv, 1);
      const uint32_t taddr = tbase + ((uint32_t)(q * 32) << 16);
      // One 16-column load per wait: issuing two loads before the wait made
      // this loop ~3x slower on B200 (measured), so the loads stay single.
      for (int c0 = 0; c0 < t.nmma; c0 += 16) {
        uint32_t v[16];
        ptx::tmem_ld_32x32b_x16(taddr + c0, v);
        ptx::tmem_wait_ld();
        epilogue_chunk<MODE>(v, c0, t, row_w, rv, bv, bp, lane, Nw, alpha, limit, out);
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(accempty);
    }
  } else {
    // ------------------------------------------------------------ dequant (A -> TMEM)
    const int dg = (warp - kWarpDeq0) >> 2;  // dequant group: takes K steps ks = dg, dg+2, ...
    const int q = warp & 3;
    const int r = q * 32 + lane;            // TMEM lane == row within the weight tile
    const uint32_t taddr = tbase + ((uint32_t)(q * 32) << 16) + kACol;
    uint32_t gbase = 0, j = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < total; item += gridDim.x, ++j, gbase += KS) {
      (void)decode_item(off, ipre, E, MT, item);
      const int b = j & 1;
      if (!warp_wait(sfull(b), (j >> 1) & 1, abort_flag)) { ok = false; break; }
      const uint8_t* srow = sbuf + b * scale_buf + r * G;
      for (int ks = dg; ks < KS; ks += kDeqGroups) {
        const uint32_t g = gbase + ks;
        const int s = g % kStagesA;
        const uint32_t ph = (g / kStagesA) & 1;
        const int g0 = 2 * ks;
        const uint32_t s0 = srow[g0];
        const uint32_t s1 = (g0 + 1 < G) ? srow[g0 + 1] : 127u;
        if (!warp_wait(fullA(s), ph, abort_flag)) { ok = false; break; }
        const uint4* src = reinterpret_cast<const uint4*>(asm_ring + s * kABytes + r * 32);
        const uint4 b0 = src[0], b1 = src[1];
        const E2M1Pool p0 = make_e2m1_pool(s0), p1 = make_e2m1_pool(s1);
        uint32_t v[32];
        e2m1x8_decode(b0.x, s0, p0, v + 0);
        e2m1x8_decode(b0.y, s0, p0, v + 4);
        e2m1x8_decode(b0.z, s0, p0, v + 8);
        e2m1x8_decode(b0.w, s0, p0, v + 12);
        e2m1x8_decode(b1.x, s1, p1, v + 16);
        e2m1x8_decode(b1.y, s1, p1, v + 20);
        e2m1x8_decode(b1.z, s1, p1, v + 24);
        e2m1x8_decode(b1.w, s1, p1, v + 28);
        ptx::tmem_st_32x32b_x32(taddr + s * (kBK / 2), v);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        if (!warp_wait(fullB(g % kStagesB), (g / kStagesB) & 1, abort_flag)) { ok = false; break; }
        if (lane == 0) ptx::mbar_arrive(adone(s));
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(sempty(b));
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) record_status(status, BS_ERR_TIMEOUT);
  if (warp == kWarpMMA) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace

// Whether the tcgen05 path can take these weights: the per-tile scale rows are
// bulk-copied, which needs 16-byte aligned, 16-byte multiple runs.
bool tc_supported(const void* scales, int64_t K, int64_t N) {
  const int64_t G = K / 32;
  return (reinterpret_cast<uintptr_t>(scales) & 15) == 0 && (N * G) % 16 == 0 && G <= kMaxGroups;
}

int tc_grouped_launch(int mode, const void* x, const int32_t* offsets, int64_t rows_total,
                      int64_t max_rows_per_expert, int64_t E, int64_t K, int64_t N,
                      const void* blocks, const void* scales, const void* bias, int bias_f32,
                      float alpha, float limit, void* out, cudaStream_t st) {
  (void)max_rows_per_expert;
  BS_ARG(E * N < (int64_t)INT32_MAX && rows_total + kNMax < (int64_t)INT32_MAX,
         "tcgen05 GEMM: sizes exceed 32-bit TMA coordinates");
  BS_ARG(mode == 1 || N % 2 == 0, "tcgen05 GEMM: gate_up rows must be even");
  BS_ARG(offsets || E == 1, "tcgen05 GEMM: expert_offsets required");
  BS_ARG(K / 32 <= kMaxGroups, "tcgen05 GEMM: contraction size above %d", kMaxGroups * 32);
  BS_REQUIRE(tc_supported(scales, K, N), BS_ERR_MISALIGNED,
             "tcgen05 GEMM: scales must be 16-byte aligned with rows*groups a multiple of 16");
  const int64_t G = K / 32;
  CUtensorMap tm_b, tm_a;
  BS_TRY(make_map_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)rows_total,
                     (uint64_t)K * 2, kBK, kBoxRows, CU_TENSOR_MAP_SWIZZLE_128B));
  BS_TRY(make_map_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, blocks, (uint64_t)G * 16, (uint64_t)(E * N),
                     (uint64_t)G * 16, kBK / 2, kBM, CU_TENSOR_MAP_SWIZZLE_NONE));
  const size_t scale_buf = (size_t)((kBM * G + 127) & ~127);
  const size_t smem = 1024 + (size_t)kStagesB * kBBytes + (size_t)kStagesA * kABytes + 2 * scale_buf +
                      kNumBars * 8 + 16 + (size_t)2 * (E + 1) * sizeof(int);
  BS_REQUIRE(smem <= 227 * 1024, BS_ERR_CAPACITY, "tcgen05 GEMM: too many experts for shared memory");
  auto kern = mode == 0 ? tc_grouped_kernel<0> : mode == 1 ? tc_grouped_kernel<1> : tc_grouped_kernel<2>;
  BS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int grid = sm_count();
  kern<<<grid, kThreads, smem, st>>>(tm_b, tm_a, static_cast<const uint8_t*>(scales), offsets,
                                     rows_total, (int)E, (int)K, (int)N, bias, bias_f32, alpha,
                                     limit, static_cast<uint16_t*>(out), device_status_ptr());
  BS_LAUNCHED();
  return BS_OK;
}

}  // namespace bs
