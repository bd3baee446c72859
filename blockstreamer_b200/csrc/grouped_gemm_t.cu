// Transposed grouped expert GEMM on tcgen05 (sm_100a): the backward of the
// expert projections.
//
// Forward (grouped_gemm.cu) computes y[rows of e] = x[rows of e] @ W[e]^T
// with W[e] the MXFP4 weight [Nw, Kw] as stored (Kw contiguous).  Its input
// gradient is
//     dx[rows of e] = dy[rows of e] @ W[e]          (contraction over Nw)
// -- block_streamer/gptoss.py:64-71 (_MXFP4Matmul.backward), where the
// reference dequantizes W densely and calls a library GEMM per expert.  Here
// the same swap-AB tcgen05 pipeline as the forward kernel runs with A = W^T:
// the MMA's M side is 128 OUTPUT features (Kw), its N side the expert's token
// rows, K the Nw weight rows, 64 per stage.
//   * A (W^T): TMA brings a [64 weight rows x 128 features] slice of the codes
//     (64 bytes of each row) and the matching e8m0 scales from a transposed
//     copy of the scale tensor ([E][G padded to 4][Nw], built per call); four
//     dequant warps decode the 64 rows bit-exactly (byte-table path, one row
//     half per thread), pair rows (n, n+1) per feature through a shuffle, and
//     write the pairs into a shared staging tile whose words are XOR-swizzled
//     so that both the row-wise writes and the column-wise reads are
//     bank-conflict free; each lane then reads its feature's 32 pairs and
//     stores them into tensor memory with tcgen05.st.  Two dequant groups take
//     alternate stages.  The MMA reads A from tensor memory ("TS" form).
//   * B (dy rows): 128B-swizzled TMA tiles, as in the forward kernel.
//   * D: fp32 accumulators in TMEM, drained by four epilogue warps.
// EPI 0: plain bf16 store (dx of the gate_up projection, mxfp4_matmul's dx).
// EPI 1: the SwiGLU backward of gptoss.py:130-135 fused in: the accumulator is
//   dh for intermediate feature i; with the gate_up pre-activation g (fp32,
//   so that the clamp masks match an fp32 evaluation) it writes dg[:, 2i]
//   (gate) and dg[:, 2i+1] (up) in bf16 -- the gradient the gate_up backward
//   consumes.
// Every wait is bounded (timeout -> status word + clean exit, TMEM freed).
// No TMA multicast.
#include <cudaTypedefs.h>

#include "bs_common.cuh"
#include "bs_ptx.cuh"

namespace bs {
namespace {

constexpr int kBM = 128;                       // output features per tile (MMA M)
constexpr int kBK = 64;                        // weight rows (contraction) per stage
constexpr int kNMax = 320;                     // token rows per tile
constexpr int kStagesB = 3;                    // token-tile ring
constexpr int kStagesA = 6;                    // weight ring
constexpr int kBoxRows = 64;
constexpr int kBoxBytes = kBoxRows * kBK * 2;  // 8 KiB
constexpr int kBBytes = kNMax * kBK * 2;       // 40 KiB per token stage
constexpr int kACodes = kBK * kBM / 2;         // 4 KiB of codes per weight stage
constexpr int kAScales = 4 * kBK;              // 4 scale groups x 64 rows
constexpr int kABytes = kACodes + kAScales;
constexpr int kStageWords = (kBK / 2) * kBM;   // staging tile: 32 row pairs x 128 features (u32)
constexpr int kACol = 320;
constexpr int kTmemCols = 512;
constexpr int kDeqGroups = 2;
constexpr int kWarpTMA = 0, kWarpMMA = 1, kWarpDeq0 = 6;
constexpr int kWarpTMA_A = kWarpDeq0 + 4 * kDeqGroups;
constexpr int kWarpMMA2 = kWarpTMA_A + 1;  // second MMA issuer: the 128x64 MMAs of tiles above 256 rows
constexpr int kThreads = (kWarpMMA2 + 1) * 32;
// barriers: fullB per token stage; fullA, adone, emptyA per weight stage;
// accfull, accempty, drain
constexpr int kNumBars = kStagesB + 3 * kStagesA + 3;

static_assert(kBBytes % 1024 == 0, "token stages keep 1024-byte alignment for SW128");
static_assert(kACol + kStagesA * (kBK / 2) <= kTmemCols, "TMEM budget");

struct Tile {
  int e, mt, nrows, nmma;
  int64_t r0;
};

__device__ __forceinline__ int nchunks_of(int n) { return n > 0 ? (n + kNMax - 1) / kNMax : 0; }

// Per-expert work-item prefix (items = token chunks x feature tiles), as the forward kernel.
__device__ void build_sched(const int* __restrict__ offsets, int64_t rows_total, int E, int MT, int* off,
                            int* ipre) {
  const int tid = threadIdx.x;
  for (int e = tid; e <= E; e += blockDim.x) off[e] = offsets ? offsets[e] : (e == 0 ? 0 : (int)rows_total);
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
  int lo = 0, hi = E - 1;
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

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  const bool ok = ptx::mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Barrier over n threads that also returns true iff every participant passed
// true: a decision to stop is taken by the whole group at once.
__device__ __forceinline__ bool named_and(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// Staging-tile word index of (row pair p, feature c): the words a writer warp
// stores for one column step and the 32 a reader warp loads for one row pair
// land in distinct banks.
__device__ __forceinline__ int swz(int p, int c) {
  return p * kBM + (c ^ (((p & 7) << 1) | (((c >> 6) & 1) << 4)));
}

// dL/dgate and dL/dup of h = (clamp(up) + 1) * min(gate, L) * sigmoid(alpha * min(gate, L))
// (gptoss.py:130-135), torch clamp semantics (gradient 1 inside the closed range).
__device__ __forceinline__ void swiglu_backward(float gate, float up, float dh, float alpha, float limit,
                                                float& dgate, float& dup) {
  const float gc = fminf(gate, limit);
  const float uc = fminf(fmaxf(up, -limit), limit);
  // the hardware exponential and division, as the forward epilogue: their
  // few-ulp error is far below the bf16 rounding of dg
  const float sg = __fdividef(1.0f, 1.0f + __expf(-alpha * gc));
  const float glu = gc * sg;
  dup = (up >= -limit && up <= limit) ? dh * glu : 0.f;
  dgate = (gate <= limit) ? dh * (uc + 1.0f) * (sg + gc * alpha * sg * (1.0f - sg)) : 0.f;
}

// tm_b: dy [rows_total][Nw] bf16, box {64, 64}, SW128.  tm_a: codes as
// [E*Nw rows][Kw/2 bytes], box {64 bytes, 64 rows}.  tm_s: transposed scales
// [E*Gp rows][Nw bytes], box {64 bytes, 4 rows}.
template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) tc_grouped_t_kernel(
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_a,
    const __grid_constant__ CUtensorMap tm_s, const int* __restrict__ offsets, int64_t rows_total, int E,
    int Nw, int Kw, int Gp, const float* __restrict__ g, float alpha, float limit, uint16_t* __restrict__ out,
    int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* a_ring = smem + kStagesB * kBBytes;                                   // [kStagesA][kABytes]
  uint32_t* staging = reinterpret_cast<uint32_t*>(a_ring + kStagesA * kABytes);  // [kDeqGroups][kStageWords]
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + kDeqGroups * kStageWords);
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
  const uint32_t accfull = bar(kB0), accempty = bar(kB0 + 1), drain = bar(kB0 + 2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesB; ++s) ptx::mbar_init(fullB(s), 1);
    for (int s = 0; s < kStagesA; ++s) {
      ptx::mbar_init(fullA(s), 1);
      ptx::mbar_init(adone(s), 4);
      ptx::mbar_init(emptyA(s), 2);  // a commit from each MMA issuer
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
    ptx::tma_prefetch_desc(&tm_s);
  }
  if (warp == kWarpMMA) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_holder), kTmemCols);
    ptx::tmem_relinquish();
  }
  const int MT = (Kw + kBM - 1) / kBM;
  build_sched(offsets, rows_total, E, MT, off, ipre);  // contains __syncthreads
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const int KS = Nw / kBK;
  const int total = ipre[E];

  if (warp == kWarpTMA) {
    // ------------------------------------------------------------ token-tile producer (dy rows)
    if (lane == 0) {
      int last_round[kStagesB];
      for (int s = 0; s < kStagesB; ++s) last_round[s] = -1;
      uint32_t gi = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x) {
        const Tile t = decode_item(off, ipre, E, MT, item);
        const int nbox = (t.nmma + kBoxRows - 1) / kBoxRows;
        for (int ks = 0; ks < KS; ++ks, ++gi) {
          const int s = gi % kStagesB, r = gi / kStagesB;
          if (gi >= (uint32_t)kStagesB) {  // the stage's previous K step's MMAs are complete
            const uint32_t gp = gi - kStagesB;
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
      if (!ok) {
        for (int s = 0; s < kStagesB; ++s)
          if (last_round[s] >= 0) ptx::mbar_wait(fullB(s), last_round[s] & 1, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else if (warp == kWarpTMA_A) {
    // ------------------------------------------------------------ weight producer (codes + scales)
    if (lane == 0) {
      int last_round[kStagesA];
      for (int s = 0; s < kStagesA; ++s) last_round[s] = -1;
      uint32_t gi = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x) {
        const Tile t = decode_item(off, ipre, E, MT, item);
        for (int ks = 0; ks < KS; ++ks, ++gi) {
          const int s = gi % kStagesA, r = gi / kStagesA;
          if (!ptx::mbar_wait(emptyA(s), (r & 1) ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* st = a_ring + s * kABytes;
          ptx::mbar_arrive_expect_tx(fullA(s), kABytes);
          ptx::tma_load_2d(ptx::smem_addr(st), &tm_a, fullA(s), t.mt * (kBM / 2), t.e * Nw + ks * kBK);
          ptx::tma_load_2d(ptx::smem_addr(st + kACodes), &tm_s, fullA(s), ks * kBK, t.e * Gp + t.mt * 4);
          last_round[s] = r;
        }
      }
      if (!ok) {
        for (int s = 0; s < kStagesA; ++s)
          if (last_round[s] >= 0) ptx::mbar_wait(fullA(s), last_round[s] & 1, abort_flag, 200000000LL);
      }
    }
    __syncwarp();
  } else if (warp == kWarpMMA || warp == kWarpMMA2) {
    // ------------------------------------------------------------ MMA issuers (as the forward kernel)
    // warp kWarpMMA issues the N <= 256 MMAs, kWarpMMA2 the 128x64 ones of
    // tiles above 256 rows (one thread's issue rate is the limit); both wait
    // for the same operands and commit every stage and tile.
    if (lane == 0) {
      const bool second = warp == kWarpMMA2;
      uint32_t gi = 0, j = 0;
      bool ok = true, issued = false;
      const uint64_t bdesc0 = ptx::sdesc_kmajor_sw128(ptx::smem_addr(smem));
      const uint32_t a_t0 = tbase + kACol;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x, ++j) {
        const Tile t = decode_item(off, ipre, E, MT, item);
        const uint32_t n1 = t.nmma < 256 ? t.nmma : 256, n2 = t.nmma - n1;
        const uint32_t id = second ? (n2 ? ptx::idesc_bf16_f32(kBM, n2) : 0u) : ptx::idesc_bf16_f32(kBM, n1);
        const bool any = !second || n2 > 0;
        const uint32_t dacc = second ? tbase + 256 : tbase;
        if (!ptx::mbar_wait(accempty, (j & 1) ^ 1, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        for (int ks = 0; ks < KS; ++ks, ++gi) {
          const int sb = gi % kStagesB, sa = gi % kStagesA;
          // the weight slot (dequant) and the token tile (TMA) of this step
          if (!ptx::mbar_wait(adone(sa), (gi / kStagesA) & 1, abort_flag) ||
              !ptx::mbar_wait(fullB(sb), (gi / kStagesB) & 1, abort_flag)) {
            ok = false;
            break;
          }
          if (any) {
            ptx::tc_fence_after();
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
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;
    uint32_t j = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++j) {
      const Tile t = decode_item(off, ipre, E, MT, item);
      if (EPI == 1 && t.mt * kBM + q * 32 < Kw) {
        // while the tile's MMAs run: pull this warp's 32 features (256 bytes)
        // of every row's pre-activation into L2 for the drain below
        const float* gq = g + 2 * (t.mt * kBM + q * 32);
        for (int n = lane; n < t.nrows; n += 32) {
          const float* pr = gq + (t.r0 + n) * 2 * Kw;
          asm volatile("prefetch.global.L2 [%0];" ::"l"(pr));
          asm volatile("prefetch.global.L2 [%0];" ::"l"(pr + 32));
        }
      }
      if (!warp_wait(accfull, j & 1, abort_flag)) break;
      ptx::tc_fence_after();
      const int feat = t.mt * kBM + q * 32 + lane;
      const bool fv = feat < Kw;
      const uint32_t taddr = tbase + ((uint32_t)(q * 32) << 16);
      for (int c0 = 0; c0 < t.nmma; c0 += 16) {
        // EPI 1: the chunk's 16 pre-activation pairs are requested before the
        // accumulator load, so their HBM latency is paid once per chunk
        float2 gp[16];
        if (EPI == 1) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c0 + i;
            gp[i] = (n < t.nrows && fv) ? *reinterpret_cast<const float2*>(g + (t.r0 + n) * 2 * Kw + 2 * feat)
                                        : make_float2(0.f, 0.f);
          }
        }
        uint32_t v[16];
        ptx::tmem_ld_32x32b_x16(taddr + c0, v);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int n = c0 + i;
          if (n >= t.nrows || !fv) continue;
          const int64_t row = t.r0 + n;
          const float acc = __uint_as_float(v[i]);
          if (EPI == 0) {
            out[row * Kw + feat] = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
          } else {
            float dgate, dup;
            swiglu_backward(gp[i].x, gp[i].y, acc, alpha, limit, dgate, dup);
            *reinterpret_cast<uint32_t*>(out + row * 2 * Kw + 2 * feat) = pack_bf16x2(dgate, dup);
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(accempty);
    }
  } else {
    // ------------------------------------------------------------ dequant (W^T -> TMEM)
    const int dg = (warp - kWarpDeq0) >> 2;  // group: takes K steps ks = dg, dg + 2, ...
    const int q = warp & 3;
    const int tg = q * 32 + lane;            // 0..127 within the group
    const int jrow = tg >> 1, half = tg & 1; // step 1: weight row jrow, features half*64 .. +63
    const int feat = tg;                     // step 2: this lane's feature (TMEM lane)
    uint32_t* stg = staging + dg * kStageWords;
    const uint32_t taddr = tbase + ((uint32_t)(q * 32) << 16) + kACol;
    const int bar_id = 2 + dg;
    uint32_t gbase = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < total; item += gridDim.x, gbase += KS) {
      (void)decode_item(off, ipre, E, MT, item);
      for (int ks = dg; ks < KS; ks += kDeqGroups) {
        const uint32_t gi = gbase + ks;
        const int s = gi % kStagesA;
        // every decision to stop is taken by the whole group at once: the
        // group's named barriers below must always see all 128 threads
        ok = named_and(bar_id, 128, warp_wait(fullA(s), (gi / kStagesA) & 1, abort_flag));
        if (!ok) break;
        const uint8_t* A = a_ring + s * kABytes;
        uint32_t v[32];
        {
          const uint4* src = reinterpret_cast<const uint4*>(A + jrow * 64 + half * 32);
          const uint4 b0 = src[0], b1 = src[1];
          const uint32_t s0 = A[kACodes + (2 * half) * 64 + jrow];
          const uint32_t s1 = A[kACodes + (2 * half + 1) * 64 + jrow];
          const E2M1Pool p0 = make_e2m1_pool(s0), p1 = make_e2m1_pool(s1);
          if (s0 - 2u <= 250u && s1 - 2u <= 250u) {   // byte-table form for both scales: branch-free
            e2m1x8_to_bf16x8(b0.x, p0, v + 0);
            e2m1x8_to_bf16x8(b0.y, p0, v + 4);
            e2m1x8_to_bf16x8(b0.z, p0, v + 8);
            e2m1x8_to_bf16x8(b0.w, p0, v + 12);
            e2m1x8_to_bf16x8(b1.x, p1, v + 16);
            e2m1x8_to_bf16x8(b1.y, p1, v + 20);
            e2m1x8_to_bf16x8(b1.z, p1, v + 24);
            e2m1x8_to_bf16x8(b1.w, p1, v + 28);
          } else {
            e2m1x8_decode(b0.x, s0, p0, v + 0);
            e2m1x8_decode(b0.y, s0, p0, v + 4);
            e2m1x8_decode(b0.z, s0, p0, v + 8);
            e2m1x8_decode(b0.w, s0, p0, v + 12);
            e2m1x8_decode(b1.x, s1, p1, v + 16);
            e2m1x8_decode(b1.y, s1, p1, v + 20);
            e2m1x8_decode(b1.z, s1, p1, v + 24);
            e2m1x8_decode(b1.w, s1, p1, v + 28);
          }
        }
        // rows (2p, 2p + 1) of one feature into one word; staging[p][feature]
        const int odd = jrow & 1, pr = jrow >> 1;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t other = __shfl_xor_sync(0xffffffffu, v[i], 2);
          const uint32_t w = odd ? prmt(other, v[i], 0x7632u) : prmt(v[i], other, 0x5410u);
          stg[swz(pr, half * 64 + 2 * i + odd)] = w;
        }
        named_sync(bar_id, 128);
#pragma unroll
        for (int p = 0; p < 32; ++p) v[p] = stg[swz(p, feat)];
        ptx::tmem_st_32x32b_x32(taddr + s * (kBK / 2), v);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        // the staging tile may be overwritten once the whole group passed here
        named_sync(bar_id, 128);
        if (lane == 0) ptx::mbar_arrive(adone(s));
      }
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

// scales [E][Nw][G] -> [E][Gp][Nw] (rows G..Gp-1 zero): 32 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256) transpose_scales_kernel(const uint8_t* __restrict__ in, int E, int Nw, int G,
                                                               int Gp, uint8_t* __restrict__ out) {
  __shared__ uint8_t tile[32][33];
  const int e = blockIdx.z, n0 = blockIdx.x * 32, g0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += 8) {
    const int n = n0 + r, gg = g0 + tx;
    tile[r][tx] = (n < Nw && gg < G) ? in[((int64_t)e * Nw + n) * G + gg] : 0;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int gg = g0 + r, n = n0 + tx;
    if (gg < Gp && n < Nw) out[((int64_t)e * Gp + gg) * Nw + n] = tile[tx][r];
  }
}

}  // namespace

// Bytes of the transposed scale copy the transposed GEMM reads.
size_t tc_t_scales_bytes(int64_t E, int64_t Nw, int64_t Kw) {
  const int64_t Gp = ((Kw / 32) + 3) / 4 * 4;
  return align_up((size_t)(E * Gp * Nw), 256);
}

// Shapes the transposed GEMM takes: contraction (weight rows) a multiple of
// 64, output features a multiple of 32.
bool tc_t_supported(int64_t Nw, int64_t Kw) { return Nw % 64 == 0 && Kw % 32 == 0 && Kw / 32 <= 1024; }

// dx[rows, Kw] = dy[rows, Nw] @ dequant(W[e]) per expert segment (epi 0), or
// with the SwiGLU backward fused (epi 1: Kw = I, g [rows, 2I] fp32, out
// [rows, 2I] bf16).
// `scales_t` is a workspace of tc_t_scales_bytes; it is rebuilt from `scales`.
int tc_grouped_t_launch(int epi, const void* dy, const int32_t* offsets, int64_t rows_total, int64_t E, int64_t Nw,
                        int64_t Kw, const void* blocks, const void* scales, void* scales_t, const void* g,
                        float alpha, float limit, void* out, cudaStream_t st) {
  BS_ARG(dy && blocks && scales && scales_t && out, "transposed GEMM: null pointer");
  BS_ARG(offsets || E == 1, "transposed GEMM: expert_offsets required");
  BS_ARG(epi == 0 || g, "transposed GEMM: the SwiGLU backward needs the gate_up pre-activation");
  BS_ARG(tc_t_supported(Nw, Kw), "transposed GEMM: weight rows must be a multiple of 64 and K of 32");
  BS_ARG(E * Nw < (int64_t)INT32_MAX && rows_total + kNMax < (int64_t)INT32_MAX, "transposed GEMM: sizes too large");
  BS_ALIGNED16(dy, "dy");
  BS_ALIGNED16(blocks, "blocks");
  BS_ALIGNED16(scales_t, "scales workspace");
  if (rows_total == 0) return BS_OK;
  const int64_t G = Kw / 32, Gp = (G + 3) / 4 * 4;
  {
    const dim3 grid((unsigned)cdiv(Nw, 32), (unsigned)cdiv(Gp, 32), (unsigned)E);
    transpose_scales_kernel<<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(scales), (int)E, (int)Nw, (int)G,
                                                  (int)Gp, static_cast<uint8_t*>(scales_t));
    BS_LAUNCHED();
  }
  CUtensorMap tm_b, tm_a, tm_s;
  BS_TRY(make_map_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dy, (uint64_t)Nw, (uint64_t)rows_total,
                     (uint64_t)Nw * 2, kBK, kBoxRows, CU_TENSOR_MAP_SWIZZLE_128B));
  BS_TRY(make_map_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, blocks, (uint64_t)G * 16, (uint64_t)(E * Nw),
                     (uint64_t)G * 16, kBM / 2, kBK, CU_TENSOR_MAP_SWIZZLE_NONE));
  BS_TRY(make_map_2d(&tm_s, CU_TENSOR_MAP_DATA_TYPE_UINT8, scales_t, (uint64_t)Nw, (uint64_t)(E * Gp),
                     (uint64_t)Nw, kBK, 4, CU_TENSOR_MAP_SWIZZLE_NONE));
  const size_t smem = 1024 + (size_t)kStagesB * kBBytes + (size_t)kStagesA * kABytes +
                      (size_t)kDeqGroups * kStageWords * 4 + kNumBars * 8 + 16 + (size_t)2 * (E + 1) * sizeof(int);
  BS_REQUIRE(smem <= 227 * 1024, BS_ERR_CAPACITY, "transposed GEMM: too many experts for shared memory");
  auto kern = epi == 0 ? tc_grouped_t_kernel<0> : tc_grouped_t_kernel<1>;
  BS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<sm_count(), kThreads, smem, st>>>(tm_b, tm_a, tm_s, offsets, rows_total, (int)E, (int)Nw, (int)Kw, (int)Gp,
                                           static_cast<const float*>(g), alpha, limit,
                                           static_cast<uint16_t*>(out), device_status_ptr());
  BS_LAUNCHED();
  return BS_OK;
}

}  // namespace bs
