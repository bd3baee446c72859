// Decode-shape MoE layer (T <= 8 tokens) as ONE cooperative persistent kernel.
//
// At a few tokens the layer is the stream of the routed experts' packed
// weights (13.2 MB per expert at gpt-oss-120b shape) plus fixed latency.  The
// four-launch decode path (decode.cu) spends most of its time in launch
// chaining and per-item prologues; this kernel runs the whole layer in a
// single launch with one CTA per SM, so every SM starts streaming weights a
// few microseconds after launch and never stops until the last byte:
//
//   R  router (transformers modeling_gpt_oss.py:126-130): every CTA loads the
//      tokens; CTA c computes the fp32 logits of experts c, c + grid, ...;
//      grid barrier.
//   K  every CTA computes top-k + softmax of every token (warp per token) and
//      the dispatch (block_streamer/gptoss.py:143-154) in shared memory: the
//      sorted list of distinct routed experts and, per expert, its tokens.
//   G  gate_up + bias + clamped SwiGLU (gptoss.py:130-135, 158-166): CTA c
//      owns intermediate features [i0, i1) of EVERY routed expert -- rows
//      [2 i0, 2 i1) of each expert's gate_up weight, one contiguous run of
//      the checkpoint layout -- and writes h for those features; grid barrier.
//   D  down + bias, weighted combine (gptoss.py:167-176): CTA c owns output
//      features [f0, f1) of every routed expert (rows [f0, f1) of each down
//      weight), so the k-way combine of a token's experts is local: out is
//      written once, summed in fp32 in ascending expert order (one rounding).
//
// Streaming: one producer thread issues 1-D bulk copies (cp.async.bulk, no
// multicast) of each (expert, phase) run -- codes, then its e8m0 scales --
// into a byte ring of shared memory with one mbarrier per run; the down runs
// are issued as soon as ring space frees during phase G, so they have landed
// by the time phase D starts.  Every weight byte is read from HBM once.
//
// Math: mma.sync m16n8k16 (f16 in, f32 accumulate) per 16-row tile and
// 32-element scale block.  A = the e2m1 codes converted with
// cvt.rn.f16x2.e2m1x2 (exact); B = the tokens (all <= 8 of them) in f16,
// each token pre-scaled by a power of two so its largest element sits in
// [2^14, 2^15) (bf16 -> f16 is then exact down to 2^-29 of the token's
// maximum); h is bounded by (limit + 1) * limit for alpha > 0, so it is held
// in f16 under one fixed power-of-two scale.  Each block's product is scaled
// by its row's 2^(s-127) in fp32.  The K order inside a block is permuted
// identically for A and B so that every thread's operands are contiguous.
// The tensor-core rate is irrelevant here (the layer moves ~1 byte per FMA);
// what matters is that every SM keeps up with its share of HBM.
//
// Safety: cooperative launch (all CTAs co-resident); every wait -- grid
// barrier, mbarrier -- is bounded (~1 s of SM clock) and on expiry records
// BS_ERR_TIMEOUT in the status word, stops the work and lets in-flight bulk
// copies land (bounded) before the CTA exits.  No __trap, no multicast.
#include <cooperative_groups.h>

#include "bs_common.cuh"
#include "bs_ptx.cuh"
#include "bs_topk.cuh"

namespace bs {
namespace {

constexpr int kFT = 8;            // tokens (mma N = 8)
constexpr int kFK = 8;            // top-k
constexpr int kMaxD = kFT * kFK;  // distinct routed experts
constexpr int kCW = 16;           // compute warps
constexpr int kFThreads = (kCW + 1) * 32;  // + the producer warp
constexpr int kSlots = 8;         // runs in flight (mbarrier pairs)
constexpr int kMaxTiles = 4;      // 16-row tiles per run
constexpr int kMaxBPW = 8;        // K blocks per compute warp (K <= 32 * kCW * kMaxBPW)
constexpr long long kWaitLimit = 2000000000LL;  // ~1 s at 1.9 GHz

struct FusedArgs {
  const __nv_bfloat16* x;  // [T][H]
  const void* rw;          // router weight [E][H] (f32 or bf16) or NULL: idx/scores are inputs
  const void* rb;          // router bias [E]
  int router_bf16;
  float* scores;           // [T][k]
  int32_t* idx;            // [T][k]
  const uint8_t* gu_b;     // [E][2I][H/32][16]
  const uint8_t* gu_s;     // [E][2I][H/32]
  const void* gu_bias;     // [E][2I]
  const uint8_t* dn_b;     // [E][H][I/32][16]
  const uint8_t* dn_s;     // [E][H][I/32]
  const void* dn_bias;     // [E][H]
  int bias_f32;
  float alpha, limit;
  int h_shift;             // h is stored in f16 as h * 2^h_shift
  __nv_bfloat16* out;      // [T][H]
  const __nv_bfloat16* residual;  // [T][H] or NULL
  unsigned* bar;           // workspace: grid barrier {count, generation}
  float* logits;           // workspace: [T][E]
  uint8_t* hbuf;           // workspace: [kMaxD][T] rows of hrow_bytes (f16 h, padded)
  int* status;
  int T, H, I, E, k;
  int ring_bytes;          // dynamic shared memory layout: x rows, reduction, ring
  int xrow_bytes;          // pitch of a token row of x in shared memory (H * 2 + 64)
  int hrow_bytes;          // pitch of a token row of h, in hbuf and in shared memory (I * 2 + 64)
};

// 2^n exactly, for -126 <= n <= 127.
__device__ __forceinline__ float pow2i(int n) { return __uint_as_float((uint32_t)(n + 127) << 23); }

// 2^(s-127) for an e8m0 byte, in one shift: exact for s >= 1 (255 -> inf, as
// the reference's ldexp); s = 0 (2^-127) becomes 0, a weight below 6 * 2^-127
// whose products are far below every output's rounding.
__device__ __forceinline__ float e8m0_fast(uint32_t s) { return __uint_as_float(s << 23); }

__device__ __forceinline__ void cvt_e2m1x8_f16(uint32_t w, uint32_t& o0, uint32_t& o1, uint32_t& o2,
                                               uint32_t& o3) {
  asm("{\n\t.reg .b8 t0, t1, t2, t3;\n\tmov.b32 {t0, t1, t2, t3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, t0;\n\tcvt.rn.f16x2.e2m1x2 %1, t1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, t2;\n\tcvt.rn.f16x2.e2m1x2 %3, t3;\n\t}"
      : "=r"(o0), "=r"(o1), "=r"(o2), "=r"(o3)
      : "r"(w));
}

// D = A(16x16, row) * B(16x8, col) + C, f16 inputs, f32 accumulate.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1, float c0, float c1, float c2, float c3) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread per CTA: arrive and wait until every CTA arrived.  bar[0] counts
// arrivals (0 between barriers), bar[1] is the generation.  Bounded: false
// after ~kWaitLimit cycles (status recorded) or when *abort is raised.
__device__ bool grid_sync(unsigned* bar, unsigned nblocks, int* status, volatile int* abort) {
  const unsigned gen = ld_acquire_gpu(bar + 1);
  __threadfence();
  if (atomicAdd(bar, 1u) == nblocks - 1) {
    bar[0] = 0;
    st_release_gpu(bar + 1, gen + 1);
    return true;
  }
  const long long t0 = clock64();
  while (ld_acquire_gpu(bar + 1) == gen) {
    if (*abort) return false;
    if (clock64() - t0 > kWaitLimit) {
      record_status(status, BS_ERR_TIMEOUT);
      *abort = 1;
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void st_release_cta_shared(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(ptx::smem_addr(p)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_cta_shared(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(ptx::smem_addr(p)) : "memory");
  return v;
}
// Generic-proxy writes (other CTAs' h, ordered by the grid barrier) before
// this thread's async-proxy (bulk copy) reads of them.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float load_bias(const void* b, int f32, int64_t i) {
  return f32 ? static_cast<const float*>(b)[i] : __bfloat162float(static_cast<const __nv_bfloat16*>(b)[i]);
}

// One (expert, phase) run of contiguous weight rows.
struct Run {
  const uint8_t* codes;   // rows * kb bytes
  const uint8_t* senv;    // 16-byte aligned envelope of the rows' scales
  int code_bytes, env_bytes, s_skew;  // s_skew: first scale byte's offset in the envelope
  int rows, d, phase;     // phase 0 = gate_up, 1 = down
  int ring_off;           // placement in the ring (producer)
};

// Shared-memory state of the kernel (static part).
struct FusedShared {
  uint64_t full[kSlots];    // run j landed (slot j % kSlots)
  uint64_t freed[kSlots];   // run j consumed by every compute warp
  int place[kSlots];        // ring offset of run j
  int idx[kFT * kFK];       // routing, [T][k]
  float w[kFT * kFK];
  int dist[kMaxD];          // distinct routed experts, ascending
  unsigned mask[kMaxD];     // tokens routed to dist[d]
  float wd[kMaxD][kFT];     // routing weight of (dist[d], token)
  int D;
  int xsh[kFT];             // token t's f16 pre-scale 2^xsh
  unsigned xmax[kFT];       // bits of max |x[t]|
  unsigned bits[32];        // routed-expert bitmap (E <= 1024)
  float rred[kCW + 1][kFT]; // router reduction
  float out[kFT][kMaxTiles * 16];  // this CTA's output features, fp32
  int abort;
  int phase2;               // set once the grid barrier before phase D passed
};

// Run j of this CTA: j < nG gate_up of expert dist[j], else down of dist[j - nG].
__device__ __forceinline__ Run run_of(const FusedArgs& p, const FusedShared& s, int j, int nG, int i0, int gRows,
                                      int f0, int dRows) {
  Run r;
  const bool g = j < nG;
  r.d = g ? j : j - nG;
  r.phase = g ? 0 : 1;
  const int64_t e = s.dist[r.d];
  const int K = g ? p.H : p.I;
  const int64_t kb = K / 2, G = K / 32;
  const int64_t row0 = g ? e * 2 * p.I + 2 * (int64_t)i0 : e * p.H + f0;
  r.rows = g ? gRows : dRows;
  r.codes = (g ? p.gu_b : p.dn_b) + row0 * kb;
  r.code_bytes = (int)(r.rows * kb);
  const int64_t sa = row0 * G, sb = sa + (int64_t)r.rows * G;
  const int64_t ea = sa & ~(int64_t)15, eb = (sb + 15) & ~(int64_t)15;
  r.senv = (g ? p.gu_s : p.dn_s) + ea;
  r.env_bytes = (int)(eb - ea);
  r.s_skew = (int)(sa - ea);
  r.ring_off = 0;
  return r;
}

// Sum over the compute warps of the partial result of (row, token).
__device__ __forceinline__ float red_sum(const float* red, int row, int t) {
  const int tile = row >> 4, rr = row & 15;
  const int ib = ((rr >> 3) << 1) | (t & 1);
  const int ln = ((rr & 7) << 2) | (t >> 1);
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) v += red[((w * kMaxTiles + tile) * 4 + ib) * 32 + ln];
  return v;
}

// Byte offset of a down run's h rows behind its weights in the ring.
__device__ __forceinline__ int h_offset(const Run& r) { return (r.code_bytes + r.env_bytes + 127) & ~127; }

// The compute warps' work on one run: wait for its bytes, multiply its rows
// with the tokens (gate_up: x; down: h, both in shared memory), reduce over
// the warps, epilogue.  `dry` runs the same code on in-bounds shared memory
// without waiting, loading from or storing to global memory: executed once
// before the weights stream, it brings this code into the instruction cache
// while HBM is idle (instruction fetches that miss while the weight stream
// saturates HBM cost microseconds each).  Kept out of line: one copy of the
// code serves every call.
__device__ __noinline__ void consume(const FusedArgs& p, FusedShared& s, uint8_t* ring, const uint8_t* xs, float* red,
                                     const Run r, int j, bool dry, int i0, int f0) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int T = p.T;
  const int slot = j % kSlots;
  const int K = r.phase ? p.I : p.H;
  const int kb = K / 2, G = K / 32;
  const int ntile = (r.rows + 15) >> 4;
  volatile int* abort = &s.abort;
  bool ok = true;
  if (!dry) {
    ok = !*abort && ptx::mbar_wait(ptx::smem_addr(&s.full[slot]), (j / kSlots) & 1, abort, kWaitLimit);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && lane == 0) record_status(p.status, BS_ERR_TIMEOUT);
  }
  if (ok) {
    const uint8_t* codes = ring + (dry ? 0 : s.place[slot]);
    const uint8_t* scl = codes + r.code_bytes + r.s_skew;
    const uint8_t* bb = r.phase ? codes + h_offset(r) : xs;
    const int bp = r.phase ? p.hrow_bytes : p.xrow_bytes;
    float tot[kMaxTiles][4];
#pragma unroll
    for (int tl = 0; tl < kMaxTiles; ++tl) tot[tl][0] = tot[tl][1] = tot[tl][2] = tot[tl][3] = 0.f;
    // two K blocks per iteration (blk, blk + kCW) so that two independent
    // chains (loads -> cvt -> mma -> mma -> scale) are in flight per tile; a
    // missing second block reuses the first block's operands under a zero
    // scale.  Rows past the run's end read its last row (in bounds, finite)
    // and their results are never used.
    const int nblk_iter = dry ? kCW : G;
#pragma unroll 1
    for (int blk = warp; blk < nblk_iter; blk += 2 * kCW) {
      const bool two = blk + kCW < nblk_iter;
      const int blk2 = two ? blk + kCW : blk;
      uint4 bv = make_uint4(0u, 0u, 0u, 0u), bw = make_uint4(0u, 0u, 0u, 0u);
      if (g < T) {
        bv = *reinterpret_cast<const uint4*>(bb + g * bp + blk * 64 + 16 * q);
        bw = *reinterpret_cast<const uint4*>(bb + g * bp + blk2 * 64 + 16 * q);
      }
#pragma unroll
      for (int tl = 0; tl < kMaxTiles; ++tl) {
        if (tl < ntile) {
          const int r0 = min(tl * 16 + g, r.rows - 1), r1 = min(tl * 16 + g + 8, r.rows - 1);
          const uint8_t* c0p = codes + r0 * kb + 4 * q;
          const uint8_t* c1p = codes + r1 * kb + 4 * q;
          const uint32_t wa = *reinterpret_cast<const uint32_t*>(c0p + blk * 16);
          const uint32_t wb = *reinterpret_cast<const uint32_t*>(c1p + blk * 16);
          const uint32_t wc = *reinterpret_cast<const uint32_t*>(c0p + blk2 * 16);
          const uint32_t wd = *reinterpret_cast<const uint32_t*>(c1p + blk2 * 16);
          const float sa = e8m0_fast(scl[r0 * G + blk]), sb = e8m0_fast(scl[r1 * G + blk]);
          const float sc = two ? e8m0_fast(scl[r0 * G + blk2]) : 0.f;
          const float sd = two ? e8m0_fast(scl[r1 * G + blk2]) : 0.f;
          uint32_t a0, a1, a2, a3, b0, b1, b2, b3, c0, c1, c2, c3, d0, d1, d2, d3;
          cvt_e2m1x8_f16(wa, a0, a1, a2, a3);
          cvt_e2m1x8_f16(wb, b0, b1, b2, b3);
          cvt_e2m1x8_f16(wc, c0, c1, c2, c3);
          cvt_e2m1x8_f16(wd, d0, d1, d2, d3);
          float acc[4], acd[4];
          mma_f16_16816(acc, a0, b0, a1, b1, bv.x, bv.y, 0.f, 0.f, 0.f, 0.f);
          mma_f16_16816(acd, c0, d0, c1, d1, bw.x, bw.y, 0.f, 0.f, 0.f, 0.f);
          mma_f16_16816(acc, a2, b2, a3, b3, bv.z, bv.w, acc[0], acc[1], acc[2], acc[3]);
          mma_f16_16816(acd, c2, d2, c3, d3, bw.z, bw.w, acd[0], acd[1], acd[2], acd[3]);
          tot[tl][0] = fmaf(acc[0], sa, fmaf(acd[0], sc, tot[tl][0]));
          tot[tl][1] = fmaf(acc[1], sa, fmaf(acd[1], sc, tot[tl][1]));
          tot[tl][2] = fmaf(acc[2], sb, fmaf(acd[2], sd, tot[tl][2]));
          tot[tl][3] = fmaf(acc[3], sb, fmaf(acd[3], sd, tot[tl][3]));
        }
      }
    }
#pragma unroll
    for (int tl = 0; tl < kMaxTiles; ++tl)
      if (tl < ntile)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[((warp * kMaxTiles + tl) * 4 + i) * 32 + lane] = tot[tl][i];
  }
  __syncwarp();
  if (!dry && lane == 0) ptx::mbar_arrive(ptx::smem_addr(&s.freed[slot]));  // the run's bytes may be overwritten
  if (!dry) named_sync(1, kCW * 32);
  if (!*abort) {
    const unsigned msk = dry ? 0xFFu : s.mask[r.d];
    const int64_t e = dry ? 0 : s.dist[r.d];
    if (r.phase == 0) {
      // gate_up epilogue: bias, clamped SwiGLU; h in f16 for the routed tokens
      const int np = r.rows >> 1;
      for (int it = tid; it < np * T; it += kCW * 32) {
        const int pr = it / T, t = it - pr * T;
        if (!((msk >> t) & 1u)) continue;
        const float xs_inv = pow2i(-s.xsh[t]);
        const int64_t brow = e * 2 * p.I + 2 * (i0 + pr);
        float gate = red_sum(red, 2 * pr, t) * xs_inv, up = red_sum(red, 2 * pr + 1, t) * xs_inv;
        if (!dry) {
          gate += load_bias(p.gu_bias, p.bias_f32, brow);
          up += load_bias(p.gu_bias, p.bias_f32, brow + 1);
        }
        gate = fminf(gate, p.limit);
        up = fminf(fmaxf(up, -p.limit), p.limit);
        const float hv = (up + 1.0f) * __fdividef(gate, 1.0f + __expf(-p.alpha * gate));
        const __half hh = __float2half_rn(hv * pow2i(p.h_shift));
        if (!dry)
          *reinterpret_cast<__half*>(p.hbuf + (int64_t)(r.d * T + t) * p.hrow_bytes + 2 * (int64_t)(i0 + pr)) = hh;
      }
    } else {
      // down epilogue: bias, times the routing weight, summed per token in
      // ascending expert order (each (token, feature) has one owner thread)
      for (int it = tid; it < r.rows * T; it += kCW * 32) {
        const int lf = it / T, t = it - lf * T;
        if (!((msk >> t) & 1u)) continue;
        float v = red_sum(red, lf, t) * pow2i(-p.h_shift);
        if (!dry) {
          v += load_bias(p.dn_bias, p.bias_f32, e * p.H + f0 + lf);
          s.out[t][lf] = fmaf(s.wd[r.d][t], v, s.out[t][lf]);
        }
      }
    }
  }
  if (!dry) named_sync(1, kCW * 32);
}

__global__ void __launch_bounds__(kFThreads, 1) decode_fused_kernel(const __grid_constant__ FusedArgs p) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ FusedShared s;
  volatile int* abort = &s.abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.T, H = p.H, I = p.I, E = p.E, k = p.k;
  const int nblk = gridDim.x, c = blockIdx.x;
  uint8_t* xs = dsm;
  float* red = reinterpret_cast<float*>(dsm + ((T * p.xrow_bytes + 127) & ~127));
  uint8_t* ring = reinterpret_cast<uint8_t*>(red) + kCW * kMaxTiles * 128 * 4;

  if (tid == 0) {
    s.abort = 0;
    s.phase2 = 0;
    for (int i = 0; i < kSlots; ++i) {
      ptx::mbar_init(ptx::smem_addr(&s.full[i]), 1);
      ptx::mbar_init(ptx::smem_addr(&s.freed[i]), kCW);
    }
    ptx::fence_mbar_init();
  }
  if (tid < kFT) s.xmax[tid] = 0;
  if (tid < 32) s.bits[tid] = 0;
  for (int i = tid; i < kFT * kMaxTiles * 16; i += kFThreads) (&s.out[0][0])[i] = 0.f;
  __syncthreads();

  // ---------------------------------------------------------------- R: tokens, router logits
  const int vpr = H / 8;  // 16-byte vectors per token row
  for (int i = tid; i < T * vpr; i += kFThreads) {
    const int t = i / vpr, v = i - t * vpr;
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(p.x + (int64_t)t * H) + v);
    *reinterpret_cast<uint4*>(xs + t * p.xrow_bytes + v * 16) = q;
    const uint32_t m = (q.x | q.y | q.z | q.w);  // not the max: the bf16 pairs' largest exponent below
    (void)m;
    float mx = fmaxf(fmaxf(fmaxf(fabsf(bf16lo(q.x)), fabsf(bf16hi(q.x))), fmaxf(fabsf(bf16lo(q.y)), fabsf(bf16hi(q.y)))),
                     fmaxf(fmaxf(fabsf(bf16lo(q.z)), fabsf(bf16hi(q.z))), fmaxf(fabsf(bf16lo(q.w)), fabsf(bf16hi(q.w)))));
    atomicMax(&s.xmax[t], __float_as_uint(mx));
  }
  __syncthreads();
  if (p.rw) {
    for (int e = c; e < E; e += nblk) {
      float acc[kFT];
#pragma unroll
      for (int t = 0; t < kFT; ++t) acc[t] = 0.f;
      for (int h = tid * 4; h < H; h += kFThreads * 4) {
        float w4[4];
        if (p.router_bf16) {
          const uint2 q = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.rw) + (int64_t)e * H + h));
          w4[0] = bf16lo(q.x), w4[1] = bf16hi(q.x), w4[2] = bf16lo(q.y), w4[3] = bf16hi(q.y);
        } else {
          const float4 q = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.rw) + (int64_t)e * H + h));
          w4[0] = q.x, w4[1] = q.y, w4[2] = q.z, w4[3] = q.w;
        }
#pragma unroll
        for (int t = 0; t < kFT; ++t) {
          if (t < T) {
            const uint2 xv = *reinterpret_cast<const uint2*>(xs + t * p.xrow_bytes + h * 2);
            acc[t] = fmaf(bf16lo(xv.x), w4[0], acc[t]);
            acc[t] = fmaf(bf16hi(xv.x), w4[1], acc[t]);
            acc[t] = fmaf(bf16lo(xv.y), w4[2], acc[t]);
            acc[t] = fmaf(bf16hi(xv.y), w4[3], acc[t]);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kFT; ++t) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) s.rred[warp][t] = v;
      }
      __syncthreads();
      if (tid < T) {
        float v = 0.f;
        for (int w = 0; w <= kCW; ++w) v += s.rred[w][tid];
        v += p.router_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.rb)[e])
                           : static_cast<const float*>(p.rb)[e];
        if (p.router_bf16) v = __bfloat162float(__float2bfloat16_rn(v));
        p.logits[(int64_t)tid * E + e] = v;
      }
      __syncthreads();
    }
  }
  // tokens -> f16 in place, each under its power-of-two scale (max in [2^14, 2^15))
  if (tid < T) {
    const int ef = (int)((s.xmax[tid] >> 23) & 0xFF);
    s.xsh[tid] = (ef == 0 || ef == 255) ? 0 : min(141 - ef, 126);
  }
  __syncthreads();
  for (int i = tid; i < T * vpr; i += kFThreads) {
    const int t = i / vpr, v = i - t * vpr;
    uint4* a = reinterpret_cast<uint4*>(xs + t * p.xrow_bytes + v * 16);
    const uint4 q = *a;
    const float sc = pow2i(s.xsh[t]);
    uint4 o;
    const uint32_t in[4] = {q.x, q.y, q.z, q.w};
    uint32_t outw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 hh = __floats2half2_rn(bf16lo(in[j]) * sc, bf16hi(in[j]) * sc);
      outw[j] = *reinterpret_cast<const uint32_t*>(&hh);
    }
    o.x = outw[0], o.y = outw[1], o.z = outw[2], o.w = outw[3];
    *a = o;
  }
  __syncthreads();
  if (tid == 0) {
    if (p.rw) grid_sync(p.bar, nblk, p.status, abort);
  } else if (warp != 0 && warp < kCW) {
    // while thread 0 waits for every CTA's logits, the other compute warps
    // run the run-processing and top-k code once on in-bounds shared memory
    // (no global access, results discarded): their instruction fetches miss
    // while HBM is idle instead of once the weights saturate it
    Run dry{};
    dry.rows = 16;
    dry.code_bytes = 16 * (H / 2);
    dry.env_bytes = 16 * (H / 32);
    consume(p, s, ring, xs, red, dry, 0, true, 0, 0);
    dry.phase = 1;
    dry.code_bytes = 16 * (I / 2);
    dry.env_bytes = 16 * (I / 32);
    consume(p, s, ring, xs, red, dry, 0, true, 0, 0);
    if (warp == 1) {
      float* junk = red + 64 * 32;  // scratch for the discarded top-k
      warp_topk_any([&](int e) { return red[e]; }, E, k, junk, reinterpret_cast<int*>(junk + 32));
    }
  }
  __syncthreads();

  // ---------------------------------------------------------------- K: top-k, dispatch (every CTA)
  if (warp < T) {
    if (p.rw) {
      const float* lg = p.logits + (int64_t)warp * E;
      warp_topk_any([&](int e) { return __ldcg(lg + e); }, E, k, s.w + warp * k, s.idx + warp * k);
    } else if (lane < k) {
      s.idx[warp * k + lane] = p.idx[warp * k + lane];
      s.w[warp * k + lane] = p.scores[warp * k + lane];
    }
  }
  __syncthreads();
  if (tid < T * k) {
    const int e = s.idx[tid];
    if (c == 0 && p.rw) {
      p.idx[tid] = e;
      p.scores[tid] = s.w[tid];
    }
    if (e >= 0 && e < E) atomicOr(&s.bits[e >> 5], 1u << (e & 31));
    else if (c == 0) record_status(p.status, BS_ERR_INVALID_ARGUMENT);
  }
  __syncthreads();
  if (tid == 0) {
    int D = 0;
    for (int wd = 0; wd < 32; ++wd) {
      unsigned b = s.bits[wd];
      while (b) {
        const int bit = __ffs(b) - 1;
        b &= b - 1;
        s.dist[D++] = wd * 32 + bit;
      }
    }
    s.D = D;
  }
  __syncthreads();
  const int D = s.D;
  if (tid < D) {
    const int e = s.dist[tid];
    unsigned m = 0;
    for (int t = 0; t < kFT; ++t) s.wd[tid][t] = 0.f;
    for (int i = 0; i < T * k; ++i)
      if (s.idx[i] == e) {
        m |= 1u << (i / k);
        s.wd[tid][i / k] = s.w[i];
      }
    s.mask[tid] = m;
  }
  __syncthreads();

  // this CTA's slices: intermediate features [i0, i1), output features [f0, f1)
  const int i0 = (int)((int64_t)c * I / nblk), i1 = (int)((int64_t)(c + 1) * I / nblk);
  const int f0 = (int)((int64_t)c * H / nblk), f1 = (int)((int64_t)(c + 1) * H / nblk);
  const int gRows = 2 * (i1 - i0), dRows = f1 - f0;
  const int nG = gRows > 0 ? D : 0, nD = dRows > 0 ? D : 0, nRuns = nG + nD;
  const int hbytes = T * p.hrow_bytes;  // a down run's h rows (all T tokens)

  if (warp == kCW) {
    // ---------------------------------------------------------------- producer
    // Places run j's weights in the ring as soon as space frees (down runs
    // included, long before phase D), and a down run's h rows once the grid
    // barrier before phase D has passed.  Never blocks: it polls the
    // consumers' release barriers and the phase flag, bounded overall.
    if (lane == 0) {
      int j = 0, hn = nG, lo = 0, head = 0;
      int start[kSlots];
      bool ph2 = false;
      long long t_last = clock64();
      while ((j < nRuns || hn < j) && !*abort) {
        bool progress = false;
        while (lo < j && mbar_test(ptx::smem_addr(&s.freed[lo % kSlots]), (lo / kSlots) & 1)) {
          ++lo;
          progress = true;
        }
        if (!ph2) ph2 = ld_acquire_cta_shared(&s.phase2) != 0;
        if (ph2 && hn < j) {
          fence_proxy_async_global();
          const Run r = run_of(p, s, hn, nG, i0, gRows, f0, dRows);
          ptx::bulk_load(ptx::smem_addr(ring + s.place[hn % kSlots] + h_offset(r)),
                         p.hbuf + (int64_t)r.d * hbytes, (uint32_t)hbytes, ptx::smem_addr(&s.full[hn % kSlots]));
          ++hn;
          progress = true;
        } else if (j < nRuns && j - lo < kSlots) {
          const Run r = run_of(p, s, j, nG, i0, gRows, f0, dRows);
          const int need = h_offset(r) + (r.phase ? ((hbytes + 127) & ~127) : 0);
          int pos = -1;
          if (j == lo) {
            pos = 0;
          } else {
            // head == tail only when the ring is empty: a placement never
            // ends exactly at the tail
            const int tail = start[lo % kSlots];
            if (head > tail) {
              if (head + need <= p.ring_bytes) pos = head;
              else if (need < tail) pos = 0;
            } else if (head + need < tail) {
              pos = head;
            }
          }
          if (pos >= 0) {
            start[j % kSlots] = pos;
            head = pos + need;
            s.place[j % kSlots] = pos;
            const uint32_t fb = ptx::smem_addr(&s.full[j % kSlots]);
            ptx::mbar_arrive_expect_tx(fb, (uint32_t)(r.code_bytes + r.env_bytes + (r.phase ? hbytes : 0)));
            ptx::bulk_load(ptx::smem_addr(ring + pos), r.codes, (uint32_t)r.code_bytes, fb);
            ptx::bulk_load(ptx::smem_addr(ring + pos + r.code_bytes), r.senv, (uint32_t)r.env_bytes, fb);
            ++j;
            progress = true;
          }
        }
        if (progress) {
          t_last = clock64();
        } else if (clock64() - t_last > kWaitLimit) {
          record_status(p.status, BS_ERR_TIMEOUT);
          *abort = 1;
        } else {
          __nanosleep(32);
        }
      }
      // on an abort, complete every placed run's transaction count (their h
      // rows may be stale then) so that the wait below finds every copy landed
      for (; hn < j; ++hn) {
        const Run r = run_of(p, s, hn, nG, i0, gRows, f0, dRows);
        ptx::bulk_load(ptx::smem_addr(ring + s.place[hn % kSlots] + h_offset(r)), p.hbuf + (int64_t)r.d * hbytes,
                       (uint32_t)hbytes, ptx::smem_addr(&s.full[hn % kSlots]));
      }
      // copies still in flight must land before the CTA exits
      volatile int quiet = 0;
      for (int jj = max(0, j - kSlots); jj < j; ++jj)
        ptx::mbar_wait(ptx::smem_addr(&s.full[jj % kSlots]), (jj / kSlots) & 1, &quiet, 200000000LL);
    }
    __syncwarp();
    return;
  }

  // ---------------------------------------------------------------- consumers (compute warps)
  for (int j = 0; j <= nRuns; ++j) {
    if (j == nG) {
      // every CTA's h is written before any CTA reads it
      named_sync(1, kCW * 32);
      if (tid == 0) {
        __threadfence();
        grid_sync(p.bar, nblk, p.status, abort);
        st_release_cta_shared(&s.phase2, 1);
      }
      named_sync(1, kCW * 32);
    }
    if (j == nRuns) break;
    consume(p, s, ring, xs, red, run_of(p, s, j, nG, i0, gRows, f0, dRows), j, false, i0, f0);
  }
  named_sync(1, kCW * 32);
  for (int it = tid; it < T * dRows; it += kCW * 32) {
    const int t = it / dRows, lf = it - t * dRows;
    float v = __bfloat162float(__float2bfloat16_rn(s.out[t][lf]));
    const int64_t o = (int64_t)t * H + f0 + lf;
    if (p.residual) v += __bfloat162float(p.residual[o]);
    p.out[o] = __float2bfloat16_rn(v);
  }
}

// ------------------------------------------------------------------ host side

struct FusedWS {
  unsigned* bar;
  float* logits;
  uint8_t* hbuf;
  size_t total;
};

// Pitch of a token row of x (H) or h (I) in shared memory and of h in the
// workspace: 64 bytes of padding spread the 8 token rows over the banks.
inline int64_t token_row_bytes(int64_t n) { return n * 2 + 64; }

FusedWS fused_carve(void* base, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  (void)H;
  FusedWS w{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return base ? static_cast<char*>(base) + at : nullptr;
  };
  const int64_t dmax = std::min<int64_t>(E, T * k);
  w.bar = reinterpret_cast<unsigned*>(take(64));
  w.logits = reinterpret_cast<float*>(take((size_t)T * E * 4));
  w.hbuf = reinterpret_cast<uint8_t*>(take((size_t)dmax * T * token_row_bytes(I)));
  w.total = o;
  return w;
}

// Power of two under which h = (up + 1) * gate * sigmoid(alpha * gate) fits
// f16: |up + 1| <= limit + 1 and, for alpha > 0, |gate * sigmoid(alpha gate)|
// <= max(limit, 0.2785 / alpha) (the minimum of g * sigmoid(a g) is -0.2785 / a).
int h_shift_for(float alpha, float limit) {
  const double bound = ((double)limit + 1.0) * std::max((double)limit, 0.2785 / (double)alpha);
  int sh = 0;
  while (bound * std::ldexp(1.0, sh + 1) <= 32768.0 && sh < 24) ++sh;
  while (bound * std::ldexp(1.0, sh) > 32768.0 && sh > -24) --sh;
  return sh;
}

struct FusedPlan {
  int grid, dyn_smem, ring_bytes, xrow_bytes, hrow_bytes;
};

// Whether the fused decode kernel takes this layer, and its launch shape;
// `why` receives the reason when it does not.
bool fused_plan(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k, float alpha, float limit,
                const void* gu_b, const void* gu_s, const void* dn_b, const void* dn_s, FusedPlan* pl,
                const char** why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (T < 1 || T > kFT) return no("needs 1 <= T <= 8 tokens");
  if (k < 1 || k > kFK || E < k || E > 1024) return no("needs k <= 8 and k <= E <= 1024");
  if (H % 64 || I % 64 || H / 32 > kCW * kMaxBPW || I / 32 > kCW * kMaxBPW)
    return no("needs H and I multiples of 64, at most 4096");
  if (!(alpha > 0.f) || !(limit > 0.f) || !(limit <= 180.f)) return no("needs alpha > 0 and 0 < limit <= 180");
  if (((uintptr_t)gu_b | (uintptr_t)gu_s | (uintptr_t)dn_b | (uintptr_t)dn_s) & 15)
    return no("needs 16-byte aligned expert blocks and scales");
  if ((E * 2 * I * (H / 32)) % 16 || (E * H * (I / 32)) % 16)
    return no("needs scale tensors whose sizes are multiples of 16 bytes");
  int dev = 0, coop = 0, optin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return no("no device");
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (!coop) return no("device without cooperative launch");
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, decode_fused_kernel) != cudaSuccess) return no("kernel attributes unavailable");
  const int grid = sm_count();
  const int xrow = (int)token_row_bytes(H), hrow = (int)token_row_bytes(I);
  const int xbytes = (int)align_up((size_t)T * xrow, 128);
  const int red = kCW * kMaxTiles * 128 * 4;
  const int ring = ((optin - (int)fa.sharedSizeBytes - 1024 - xbytes - red) / 128) * 128;
  const int64_t g_rows = 2 * ((I + grid - 1) / grid), d_rows = (H + grid - 1) / grid;
  if (g_rows > kMaxTiles * 16 || d_rows > kMaxTiles * 16) return no("too many rows per CTA");
  // largest run: codes + a 16-byte aligned envelope of its scales (+32 for
  // the alignment), rounded to 128; a down run also holds its tokens' h rows
  // (the dry warm-up passes use 16 rows, fewer than any real run's bound)
  const int64_t run_g = ((g_rows * (H / 2) + g_rows * (H / 32) + 32 + 127) / 128) * 128;
  const int64_t run_d = ((d_rows * (I / 2) + d_rows * (I / 32) + 32 + 127) / 128) * 128 + ((T * hrow + 127) / 128) * 128;
  const int64_t dry_d = ((16 * (I / 2) + 16 * (I / 32) + 127) / 128) * 128 + T * hrow;
  const int64_t dry_g = 16 * (H / 2) + 16 * (H / 32);
  if (ring <= 0 || std::max(std::max(run_g, run_d), std::max(dry_g, dry_d)) > ring)
    return no("shared memory too small for one run");
  pl->grid = grid;
  pl->xrow_bytes = xrow;
  pl->hrow_bytes = hrow;
  pl->ring_bytes = ring;
  pl->dyn_smem = xbytes + red + ring;
  return true;
}

}  // namespace

size_t fused_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  return fused_carve(nullptr, T, H, I, E, k).total;
}

bool fused_supported(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k, float alpha, float limit,
                     const void* gu_b, const void* gu_s, const void* dn_b, const void* dn_s) {
  FusedPlan pl;
  return fused_plan(T, H, I, E, k, alpha, limit, gu_b, gu_s, dn_b, dn_s, &pl, nullptr);
}

// The whole layer in one cooperative launch (plus a memset of the grid
// barrier's two words).  router weight NULL: scores/indices are inputs.
int fused_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k, const void* rw,
                  const void* rb, int rdt, float* scores, int32_t* indices, const void* gu_b, const void* gu_s,
                  const void* gu_bias, const void* dn_b, const void* dn_s, const void* dn_bias, int bias_f32,
                  float alpha, float limit, void* out, void* ws, cudaStream_t st, const void* residual) {
  FusedPlan pl;
  const char* why = "";
  BS_REQUIRE(fused_plan(T, H, I, E, k, alpha, limit, gu_b, gu_s, dn_b, dn_s, &pl, &why), BS_ERR_UNSUPPORTED,
             "fused decode path: %s", why);
  BS_ALIGNED16(x, "x");
  BS_ALIGNED16(out, "out");
  if (residual) BS_ALIGNED16(residual, "residual");
  if (rw) BS_REQUIRE(((uintptr_t)rw & 15) == 0, BS_ERR_MISALIGNED, "router weight must be 16-byte aligned");
  const FusedWS w = fused_carve(ws, T, H, I, E, k);
  FusedArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.rw = rw;
  a.rb = rb;
  a.router_bf16 = rw && rdt == BS_BF16;
  a.scores = scores;
  a.idx = indices;
  a.gu_b = static_cast<const uint8_t*>(gu_b);
  a.gu_s = static_cast<const uint8_t*>(gu_s);
  a.gu_bias = gu_bias;
  a.dn_b = static_cast<const uint8_t*>(dn_b);
  a.dn_s = static_cast<const uint8_t*>(dn_s);
  a.dn_bias = dn_bias;
  a.bias_f32 = bias_f32;
  a.alpha = alpha;
  a.limit = limit;
  a.h_shift = h_shift_for(alpha, limit);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.bar = w.bar;
  a.logits = w.logits;
  a.hbuf = w.hbuf;
  a.status = device_status_ptr();
  a.T = (int)T, a.H = (int)H, a.I = (int)I, a.E = (int)E, a.k = (int)k;
  a.ring_bytes = pl.ring_bytes;
  a.xrow_bytes = pl.xrow_bytes;
  a.hrow_bytes = pl.hrow_bytes;
  BS_CUDA(cudaFuncSetAttribute(decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.dyn_smem));
  int per_sm = 0;
  BS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_fused_kernel, kFThreads, pl.dyn_smem));
  BS_REQUIRE(per_sm >= 1, BS_ERR_UNSUPPORTED, "fused decode path: the kernel does not fit on an SM");
  BS_CUDA(cudaMemsetAsync(w.bar, 0, 2 * sizeof(unsigned), st));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.grid);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = (size_t)pl.dyn_smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  BS_CUDA(cudaLaunchKernelEx(&cfg, decode_fused_kernel, a));
  return BS_OK;
}

}  // namespace bs
