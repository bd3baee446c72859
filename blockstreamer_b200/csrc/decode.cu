// Decode-shape MoE layer (<= 64 tokens) on tcgen05 block-scaled MMAs.
//
// At decode sizes the layer streams the packed weights of the experts the
// tokens picked and does little arithmetic with them.  Turning e2m1 codes into
// bf16 on CUDA cores costs about as long as streaming them, so the tensor
// cores consume the checkpoint's codes and e8m0 scales directly with
// `kind::mxf4` (K = 64 per instruction).  The other operand must then be e2m1
// too: each activation is split into four e2m1 terms, each with its own e8m0
// scale per 32 values,
//     v ~= sum_t q_t * 2^(s_t - 127),   q_t in {0, +-0.5, ..., +-6},
// every term taking the residual of the ones before (the block maximum of the
// residual sets the next scale).  Four terms keep the dot products within
// ~1e-4 relative of exact, far inside the layer's 5e-3 bar; the terms are
// separate B rows (N = 4 x tokens), whose products are summed in the epilogue.
// At these N the cost of an M=128 block-scaled MMA does not depend on N, so
// the instruction count -- weights / (128 x 64) -- sets the tensor-core time;
// K = 64 per instruction keeps it under the HBM time of the weights.
//
// The layer runs as four launches chained with programmatic dependent launch:
//  1. decode_route_kernel  x -> four e2m1 terms; router logits with one CTA per
//     (expert, 16 tokens) (modeling_gpt_oss.py:126-130).
//  2. decode_mx_kernel<0>  every CTA first computes top-k + softmax over the k
//     (modeling_gpt_oss.py:126-130) and the dispatch (gptoss.py:143-154) into
//     its shared memory, CTA 0 writing them out; then gate_up + bias +
//     clamped SwiGLU (gptoss.py:130-135, 158-166); h is written as four e2m1
//     terms for the next projection.
//  3. decode_mx_kernel<1>  down + bias, times the routing weight (167-175),
//     fp32 rows.
//  4. decode_combine_kernel out[t] = bf16(sum over the k slots), fp32 sum.
//
// Work item of 2/3: 128 weight rows of one expert and a group of up to 16 of
// its tokens, K in stages of 256.  The items' stages are cut into equal
// contiguous ranges, one per CTA (stream-K): at one token the gate_up
// projection is 180 items of 12 stages on 148 SMs, which whole items would
// leave 32 SMs doing two.  An item split across CTAs is finished by the CTA
// holding its last stage, which adds the others' partial sums (written to
// the workspace, counted by a flag per CTA) before its epilogue.
//
// One CTA per SM (512 threads), two pipelines that take alternate stages of
// every piece, each with a TMA warp (weight tiles [128 rows x 256 codes] as
// stored, the B term rows; pipeline 0's also the per-item scale blocks and B
// tiles), an MMA thread with its own accumulator, and two scale-factor warps
// (a stage's scales laid out in shared memory, copied into TMEM by
// tcgen05.cp); two epilogue groups of four warps drain alternate accumulator
// buffers, adding the two pipelines' accumulators.  Measured on this GPU: one
// thread issues a block-scaled MMA every ~115 cycles and a commit in ~90,
// whatever other threads of the SM issue, so the issuing threads' own
// instructions set the stage rate; two pipelines double it.  The loops have
// no divisions and advance descriptors by addition.

#include "bs_common.cuh"
#include "bs_ptx.cuh"
#include "bs_topk.cuh"

#include <initializer_list>

namespace bs {
namespace {

constexpr int kMaxDecodeT = 64;
constexpr int kTerms = 4;       // e2m1 terms per activation
constexpr int kRTok = 16;       // tokens per router CTA
constexpr int kKC = 256;        // K elements per pipeline stage: 128 bytes of codes per row, 4 MMAs
constexpr int kBM = 128;        // weight rows per item (MMA M)
constexpr int kThreads = 512;   // pipeline 0: warps 4 TMA, 5 MMA, 6-7 scale factors; pipeline 1: 8-11; epilogues 0-3, 12-15
constexpr int kAtomBytes = 2048; // a stage's scale factors as tcgen05.cp sources: SFA, SFB x 2 groups x 32 x 16 B
constexpr int kSfWarps = 2;      // scale-factor warps a pipeline, each with one atom buffer
constexpr int kTmemCols = 512;
constexpr int kSfStageCols = 24;  // per stage: SFA 2 groups x 4 columns, SFB 2 groups x 4 or 8 columns
constexpr int kMaxStages = 12;
constexpr int kMaxRing = 4;       // per-item buffers
constexpr int kGroupTok = 16;     // tokens per group: an item's B is 4 x 16 = 64 rows at most
constexpr int kMaxGroups = 1024 + 2048 / kGroupTok;
constexpr int kMaxCtas = 256;     // grid of the expert launches (one CTA per SM, at most this)
constexpr long long kFlagWait = 2000000000LL;  // ~1 s of SM clock: bound of a wait on another CTA
constexpr int64_t kPrefetchMax = 48ll << 20;  // the next projection's weights pulled into L2 at most

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Uniform vote over a named barrier: true iff every participant passed true.
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

// Bounded wait until *f >= target (acquire, GPU scope); raises *abort and
// returns false after ~kFlagWait cycles or when another thread raised it.
__device__ __forceinline__ bool wait_flag(const unsigned* f, unsigned target, volatile int* abort) {
  if (ptx::ld_acquire_gpu(f) >= target) return true;
  const long long t0 = clock64();
  while (ptx::ld_acquire_gpu(f) < target) {
    if (*abort) return false;
    if (clock64() - t0 > kFlagWait) {
      *abort = 1;
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

struct DecodeMeta {  // lives in the workspace
  unsigned ticket;   // zeroed before the router launch
  int n_groups;      // (expert, token group) pairs with work
  int pad[2];
};

// ------------------------------------------------------------------ e2m1 terms
// e8m0 scale of a term whose block maximum is m: m / 2^(s-127) in [4, 8)
// (the top of e2m1 is 6; what saturates is left for the next term).
__device__ __forceinline__ uint32_t e8m0_for_max(float m) {
  const int ef = (int)((__float_as_uint(m) >> 23) & 0xFF);
  return (uint32_t)min(max(ef - 2, 1), 253);
}
__device__ __forceinline__ float exp2_neg(uint32_t s) { return __uint_as_float((254u - s) << 23); }  // 2^(127-s)
__device__ __forceinline__ float exp2_pos(uint32_t s) { return __uint_as_float(s << 23); }         // 2^(s-127)

template <int W>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = W / 2; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <typename WT> __device__ __forceinline__ float ldf(const WT* p);
template <> __device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

__device__ __forceinline__ void load4(const float* p, float (&w)[4]) {
  const float4 q = *reinterpret_cast<const float4*>(p);
  w[0] = q.x, w[1] = q.y, w[2] = q.z, w[3] = q.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&w)[4]) {
  const uint2 q = *reinterpret_cast<const uint2*>(p);
  w[0] = bf16lo(q.x), w[1] = bf16hi(q.x), w[2] = bf16lo(q.y), w[3] = bf16hi(q.y);
}

// ------------------------------------------------------------------ 1. route
// x -> four e2m1 terms and, with router weights, the router logits
// (modeling_gpt_oss.py:126: linear + bias in the weights' dtype); top-k and
// the dispatch run in the prologue of every gate_up CTA (route_dispatch).
// xq: rows (4 t + term) of H/2 bytes (two codes per byte, low nibble first);
// xs: rows (4 t + term) of gp bytes (one e8m0 scale per 32 values).
template <typename WT>
__global__ void __launch_bounds__(256) decode_route_kernel(
    const __nv_bfloat16* __restrict__ x, const WT* __restrict__ W, const WT* __restrict__ b,
    int T, int H, int E, int bf16_logits, float* __restrict__ logits, uint8_t* __restrict__ xq,
    uint8_t* __restrict__ xs, int gp, unsigned* __restrict__ flags, int nflags) {
  __shared__ float red[8][kRTok];
  pdl_wait();  // x comes from the previous kernel in the stream
  pdl_launch();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the expert launches' partial-sum flags start at zero every layer
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = tid; i < nflags; i += blockDim.x) flags[i] = 0u;
  // this CTA's router row on its way into L2 while the terms are computed
  if (W && blockIdx.x < E && tid * 128 < H * (int)sizeof(WT))
    for (int o = tid * 128; o < H * (int)sizeof(WT); o += 256 * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(W + (int64_t)blockIdx.x * H) + o));

  // x -> four e2m1 terms; 16 lanes per 32-value block, two values a lane
  {
    const int G = H / 32, t_in = tid >> 4, pr = tid & 15;
    for (int blk = blockIdx.x; blk < G; blk += gridDim.x)
      for (int t0 = blockIdx.y * kRTok; t0 < T; t0 += gridDim.y * kRTok) {
        const int t = t0 + t_in;
        float r0 = 0.f, r1 = 0.f;
        if (t < T) {
          const uint32_t xv = *reinterpret_cast<const uint32_t*>(x + (int64_t)t * H + blk * 32 + 2 * pr);
          r0 = bf16lo(xv);
          r1 = bf16hi(xv);
        }
#pragma unroll
        for (int term = 0; term < kTerms; ++term) {
          const uint32_t sb = e8m0_for_max(group_max<16>(fmaxf(fabsf(r0), fabsf(r1))));
          const float inv = exp2_neg(sb), sc = exp2_pos(sb);
          const uint32_t byte = ptx::e2m1x2_from_f32(r0 * inv, r1 * inv);
          r0 -= ptx::e2m1_lo_to_f32(byte) * sc;
          r1 -= ptx::e2m1_lo_to_f32(byte >> 4) * sc;
          if (t < T) {
            const int64_t row = (int64_t)t * kTerms + term;
            xq[row * (H / 2) + blk * 16 + pr] = (uint8_t)byte;
            if (pr == 0) xs[row * gp + blk] = (uint8_t)sb;
          }
        }
      }
  }

  if (W) {  // logits of expert blockIdx.x for 16 tokens: all weight loads issued first
    const int e = blockIdx.x, t0 = blockIdx.y * kRTok;
    if (e < E) {
      const int nt = min(kRTok, T - t0);
      float acc[kRTok];
#pragma unroll
      for (int t = 0; t < kRTok; ++t) acc[t] = 0.f;
      const WT* w = W + (int64_t)e * H;
      for (int h0 = 0; h0 < H; h0 += 4 * 1024) {
        float wv[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int h = h0 + (tid + 256 * j) * 4;
          if (h < H) load4(w + h, wv[j]);
          else wv[j][0] = wv[j][1] = wv[j][2] = wv[j][3] = 0.f;
        }
#pragma unroll
        for (int t = 0; t < kRTok; ++t) {
          if (t < nt) {
            float a = acc[t];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int h = h0 + (tid + 256 * j) * 4;
              if (h < H) {
                const uint2 xv = *reinterpret_cast<const uint2*>(x + (int64_t)(t0 + t) * H + h);
                a = fmaf(bf16lo(xv.x), wv[j][0], a);
                a = fmaf(bf16hi(xv.x), wv[j][1], a);
                a = fmaf(bf16lo(xv.y), wv[j][2], a);
                a = fmaf(bf16hi(xv.y), wv[j][3], a);
              }
            }
            acc[t] = a;
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kRTok; ++t) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp][t] = v;
      }
      __syncthreads();
      if (tid < nt) {
        float v = 0.f;
#pragma unroll
        for (int w8 = 0; w8 < 8; ++w8) v += red[w8][tid];
        v += ldf(b + e);
        if (bf16_logits) v = __bfloat162float(__float2bfloat16_rn(v));
        logits[(int64_t)(t0 + tid) * E + e] = v;
      }
    }
  }
}

// ------------------------------------------------------------------ 2/3. experts
struct MxArgs {
  CUtensorMap tm_a;   // weight codes [E*Nw rows][K/2 bytes], box {128 B, 128 rows}, 128B swizzle
  CUtensorMap tm_b;   // B term rows [R][K/2 bytes], box {128 B, nb rows}: a stage's tile or the tail chunk
  CUtensorMap tm_b3;  // the same rows as {128 B, R rows, nfull chunks}, box {128, nb, nfull}
  const uint8_t* scales;  // [E][Nw][K/32] e8m0
  const void* bias;       // [E][Nw]
  int bias_f32;
  const uint8_t* bsf;     // B scales: rows (4 r + term) of gp bytes
  int gp;
  // routing: MODE 0 computes it (route_dispatch) and CTA 0 writes it out;
  // MODE 1 reads it
  const float* logits;    // [T][E] router logits, or NULL: idx / scores are the caller's
  int32_t* idx;           // [T][k]
  float* scores;          // [T][k]
  int* offsets;           // [E + 1] first dispatch row of each expert
  int* row_of_slot;       // [T k]
  int* slot_of_row;       // [T k]
  int2* groups;           // (expert | tokens << 16, first row) per group of an expert's tokens
  DecodeMeta* meta;
  int E, Nw, K, k, T;
  int nb;                 // B rows of a tile (multiple of 16)
  int b_mode;             // where B comes from: kBStage, kBItem, kBResident
  int stages, nsc, nacc;  // pipeline stages, per-item buffers, accumulator buffers
  float alpha, limit;
  uint8_t* hq;            // MODE 0 out: rows (4 r + term) of Nw/4 bytes (codes of h, Nw/2 values)
  uint8_t* hs;            //             rows (4 r + term) of gp_out bytes
  int gp_out;
  float* y;               // MODE 1 out: [rows][Nw] fp32
  // items split across CTAs: the partial sums of every piece but the last,
  // [CTA][token of the group][row], and per CTA a count of the epilogue warps
  // that wrote theirs (zeroed by the route kernel)
  float* part;
  unsigned* flags;
  // MODE 0: the down projection's weights, pulled into L2 once the routing
  // is known (NULL: not pulled); bytes of codes and of scales per expert
  const uint8_t* pf_codes;
  const uint8_t* pf_scales;
  int64_t pf_cb, pf_sb;
  int* status;
};
constexpr int kBStage = 0;     // one B tile per pipeline stage
constexpr int kBItem = 1;      // an item's B tiles for all of K in one copy (per-item buffers)
constexpr int kBResident = 2;  // MODE 0, few tokens: every token's B tiles and scales, loaded once
constexpr int kBGather = 3;    // MODE 0, many tokens: the group's tokens' rows, one 4-row box each per stage

// Shared-memory plan of decode_mx_kernel (bytes; regions 1024-aligned).
struct MxSmem {
  int stage, ring_b, ring_sa, ring, res_b, res, total;
};
__host__ __device__ inline MxSmem mx_smem(int K, int nb, int b_mode, int gp, int S, int nsc) {
  const int G = K / 32, nkc = (K + kKC - 1) / kKC;
  auto al = [](int v) { return (v + 1023) & ~1023; };
  MxSmem m;
  m.stage = kBM * 128 + ((b_mode == kBStage || b_mode == kBGather) ? nb * 128 : 0);
  m.ring_b = b_mode == kBItem ? nkc * nb * 128 : 0;        // B tiles of every chunk
  m.ring_sa = (kBM * G + 15) & ~15;                         // A scale rows [128][G]
  m.ring = al(m.ring_b + m.ring_sa + (b_mode == kBResident ? 0 : nb * gp));  // + B scale rows [nb][gp]
  m.res_b = b_mode == kBResident ? nkc * nb * 128 : 0;
  m.res = b_mode == kBResident ? al(m.res_b + nb * gp) : 0;
  m.total = 2 * kSfWarps * kAtomBytes + S * m.stage + nsc * m.ring + m.res + 1024;
  return m;
}

// Top-k + softmax of every token (from the logits; modeling_gpt_oss.py:126-130)
// and the dispatch (gptoss.py:143-154: rows grouped by expert, (token, slot)
// order within an expert, groups of <= kGroupTok tokens), computed by every
// CTA of the gate_up launch into shared memory -- the same result everywhere,
// no cross-CTA handoff; CTA 0 writes it out for the later launches and the
// caller.  `scratch` holds T k + E ints and, for the rank method, T E + T k floats.
__device__ void route_dispatch(const MxArgs& p, int* scratch, int* s_slot, int2* s_grp, int* s_ngrp,
                               int (*wsum)[2]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = p.T, E = p.E, k = p.k, n = T * k;
  const bool writer = blockIdx.x == 0;
  int* s_idx = scratch;
  int* cnt = scratch + n;
  if (p.logits && T * E <= kThreads) {
    // rank every (token, expert), one per thread: the number of experts ahead
    // of it (higher logit, or equal and lower index; NaN counts as -inf);
    // ranks < k are the top-k in order.  Measured faster than the warp top-k
    // below when every pair has its own thread, slower otherwise.
    float* lg = reinterpret_cast<float*>(scratch + n + E);
    float* sv = lg + T * E;  // [T][k] selected logits
    for (int i = tid; i < T * E; i += kThreads) {
      const float v = __ldcg(p.logits + i);
      lg[i] = v != v ? -INFINITY : v;
    }
    __syncthreads();
    for (int i = tid; i < T * E; i += kThreads) {
      const int t = i / E, e = i - t * E;
      const float* row = lg + t * E;
      const float v = row[e];
      int r = 0;
      if ((E & 3) == 0) {
        const float4* row4 = reinterpret_cast<const float4*>(row);
        int r1 = 0, r2 = 0, r3 = 0;
#pragma unroll 8
        for (int e4 = 0; e4 < E / 4; ++e4) {
          const float4 w = row4[e4];
          const int b2 = 4 * e4;
          r += (w.x > v) | ((w.x == v) & (b2 < e));
          r1 += (w.y > v) | ((w.y == v) & (b2 + 1 < e));
          r2 += (w.z > v) | ((w.z == v) & (b2 + 2 < e));
          r3 += (w.w > v) | ((w.w == v) & (b2 + 3 < e));
        }
        r += r1 + r2 + r3;
      } else {
        for (int e2 = 0; e2 < E; ++e2) r += (row[e2] > v) | ((row[e2] == v) & (e2 < e));
      }
      if (r < k) {
        s_idx[t * k + r] = e;
        sv[t * k + r] = v;
      }
    }
    __syncthreads();
    if (writer)  // softmax over the k selected logits: a warp per token, a lane per slot (k <= 32)
      for (int t = warp; t < T; t += kThreads / 32) {
        const float ev = lane < k ? expf(sv[t * k + lane] - sv[t * k]) : 0.f;
        float sum = ev;
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane < k) p.scores[t * k + lane] = ev / sum;
      }
  } else if (p.logits) {  // a warp per token
    for (int t = warp; t < T; t += kThreads / 32)
      warp_topk_any([&](int e2) { return __ldcg(p.logits + (int64_t)t * E + e2); }, E, k,
                    writer ? p.scores + (int64_t)t * k : nullptr, s_idx + t * k);
  } else {
    for (int i = tid; i < n; i += kThreads) s_idx[i] = p.idx[i];
  }
  if (n <= 32 && T <= kGroupTok) {
    // Few slots: one warp dispatches them (every expert then has <= T <=
    // kGroupTok tokens, one group).  Slot j's row: the valid slots with a
    // lower expert, or the same expert and a lower slot index; its group: the
    // distinct experts below.  Same tables as the general path below.
    __syncthreads();  // s_idx complete
    int* lead = scratch + n;  // [n]: slot j is its expert's first slot (cnt's space and, past E, the rank scratch, both unused now)
    if (warp == 0) {
      const int e = lane < n ? s_idx[lane] : -1;
      const bool valid = lane < n && e >= 0 && e < E;
      if (lane < n && writer && p.logits) p.idx[lane] = e;
      if (lane < n && !valid && writer) record_status(p.status, BS_ERR_INVALID_ARGUMENT);
      int below = 0, same = 0, same_before = 0;
      for (int j = 0; j < n; ++j) {
        const int ej = s_idx[j];
        const bool vj = ej >= 0 && ej < E;
        below += vj && ej < e;
        same += vj && ej == e;
        same_before += vj && ej == e && j < lane;
      }
      const bool first = valid && same_before == 0;
      if (lane < n) lead[lane] = first;
      __syncwarp();
      int grank = 0;
      for (int j = 0; j < n; ++j) grank += lead[j] && s_idx[j] < e;
      const int pos = below + same_before;
      if (first) {
        const int2 gr = make_int2(e | (same << 16), below);
        s_grp[grank] = gr;
        if (writer) p.groups[grank] = gr;
      }
      if (valid) s_slot[pos] = lane;
      if (writer && lane < n) {
        p.row_of_slot[lane] = valid ? pos : -1;
        if (valid) p.slot_of_row[pos] = lane;
      }
      const int ng = __popc(__ballot_sync(0xffffffffu, first));
      if (lane == 0) {
        *s_ngrp = ng;
        if (writer) p.meta->n_groups = ng;
      }
    }
    if (writer)  // first row of every expert (and the total)
      for (int e = tid; e <= E; e += kThreads) {
        int r = 0;
        for (int j = 0; j < n; ++j) {
          const int ej = s_idx[j];
          r += ej >= 0 && ej < E && ej < e;
        }
        p.offsets[e] = r;
      }
    __syncthreads();
    return;
  }
  for (int e = tid; e < E; e += kThreads) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) {
    const int e = s_idx[i];
    if (writer && p.logits) p.idx[i] = e;
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    else if (writer) record_status(p.status, BS_ERR_INVALID_ARGUMENT);
  }
  __syncthreads();
  // exclusive scans of rows and groups over the experts: threads 0-255, four each
  int c[4], lc = 0, lg = 0, ic = 0, ig = 0;
  if (tid < 256) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = tid * 4 + q;
      c[q] = e < E ? cnt[e] : 0;
      lc += c[q];
      lg += (c[q] + kGroupTok - 1) / kGroupTok;
    }
    ic = lc, ig = lg;  // inclusive within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int uc = __shfl_up_sync(0xffffffffu, ic, o), ug = __shfl_up_sync(0xffffffffu, ig, o);
      if (lane >= o) ic += uc, ig += ug;
    }
    if (lane == 31) wsum[warp][0] = ic, wsum[warp][1] = ig;
  }
  __syncthreads();
  if (tid < 256) {
    int rc = ic - lc, rg = ig - lg;
    for (int w8 = 0; w8 < warp; ++w8) rc += wsum[w8][0], rg += wsum[w8][1];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = tid * 4 + q;
      if (e < E) {
        if (writer) p.offsets[e] = rc;
        cnt[e] = rc;  // now the expert's first row
        for (int c0 = 0; c0 < c[q]; c0 += kGroupTok) {
          const int2 gr = make_int2(e | (min(kGroupTok, c[q] - c0) << 16), rc + c0);
          s_grp[rg] = gr;
          if (writer) p.groups[rg] = gr;
          ++rg;
        }
        rc += c[q];
      }
      if (e == E - 1) {
        *s_ngrp = rg;
        if (writer) {
          p.offsets[E] = rc;
          p.meta->n_groups = rg;
        }
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) {
    const int e = s_idx[i];
    if (e < 0 || e >= E) {
      if (writer) p.row_of_slot[i] = -1;
      continue;
    }
    int r = 0;
#pragma unroll 8
    for (int j = 0; j < i; ++j) r += (s_idx[j] == e);
    const int pos = cnt[e] + r;
    s_slot[pos] = i;
    if (writer) {
      p.row_of_slot[i] = pos;
      p.slot_of_row[pos] = i;
    }
  }
  __syncthreads();
}

// MODE 0 epilogue of four tokens (chunk c) once their accumulators are read,
// by one epilogue group (four warps, warp q holding tile rows 32 q..32 q+31):
// clamped SwiGLU of the (gate, up) row pairs, then h re-split into four e2m1
// terms with their e8m0 scales for the down projection.  Rows alternate gate
// / up, so lanes 2m, 2m+1 of warp q give h index 16 q + m of the tile's 64;
// the values go through shared memory so that each 32-value block of h (the
// unit of an e8m0 scale) sits in one warp, which then computes the four terms
// with shuffles alone: warp q takes (token, block) pairs q and q + 4.
// i0: the tile's first h index; hb: the group's [4 tokens][64] buffer.
__device__ __forceinline__ void h_terms(const MxArgs& p, const float (&acc)[4], int c, int ntok, int row_lo, int i0,
                                        int q, int lane, float (*hb)[64], int ebar) {
  const int I = p.Nw >> 1;
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const float other = __shfl_xor_sync(0xffffffffu, acc[jj], 1);
    const float gate = (lane & 1) ? other : acc[jj], up = (lane & 1) ? acc[jj] : other;
    // the reference's clamped SwiGLU (gptoss.py:130-135) with the hardware
    // exponential and division: a few ulp, far below the e2m1 terms' error
    const float gc = fminf(gate, p.limit), uc = fminf(fmaxf(up, -p.limit), p.limit);
    const float hv = (uc + 1.0f) * __fdividef(gc, 1.0f + __expf(-p.alpha * gc));
    if (!(lane & 1)) hb[jj][16 * q + (lane >> 1)] = hv;
  }
  named_sync(ebar, 128);
#pragma unroll 1
  for (int pr = q; pr < 8; pr += 4) {
    const int jj = pr & 3, blk = pr >> 2, tok = c * 4 + jj;
    if (tok >= ntok) continue;  // uniform over the warp
    float r = hb[jj][32 * blk + lane];
    const int i = i0 + 32 * blk + lane;  // h index of this lane
#pragma unroll 1
    for (int term = 0; term < kTerms; ++term) {
      const uint32_t sb = e8m0_for_max(group_max<32>(fabsf(r)));
      const float qv = r * exp2_neg(sb);
      const float qn = __shfl_down_sync(0xffffffffu, qv, 1);  // h_{i+1}
      const uint32_t byte = ptx::e2m1x2_from_f32(qv, qn);    // low nibble: this lane's value
      r -= ptx::e2m1_lo_to_f32(byte) * exp2_pos(sb);
      const int64_t hr = (int64_t)(row_lo + tok) * kTerms + term;
      if (!(lane & 1)) p.hq[hr * (I / 2) + (i >> 1)] = (uint8_t)byte;
      if (lane == 0) p.hs[hr * p.gp_out + (i >> 5)] = (uint8_t)sb;
    }
  }
  named_sync(ebar, 128);  // hb is rewritten by the next chunk
}

// MODE 0: B = the four term rows of tokens (every token's when resident or
// per stage; the MMA computes them all and the epilogue keeps the expert's);
// MODE 1: B = the group's own rows of h.
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) decode_mx_kernel(const __grid_constant__ MxArgs pa) {
  extern __shared__ uint8_t smem_raw[];
  // The roles read the arguments from a shared-memory copy; the tensor maps
  // stay in parameter space for the TMA unit.
  __shared__ MxArgs p;
  // data[s] a stage's copies landed, empty[s] its MMAs are done, sffull[s] its
  // scale factors are in TMEM; item[b] an item's scales (and B tiles) landed in
  // ring buffer b, bfree[b] that item's MMAs are done; accfull / accempty:
  // accumulator handoff; res: resident B landed; drain: teardown.  A waiter is
  // never two phases ahead of a barrier it waits on.
  __shared__ uint64_t bars[3 * kMaxStages + 2 * kMaxRing + 6 + 2 * kSfWarps];
  __shared__ uint32_t tmem_holder;
  __shared__ volatile int abort_flag;
  __shared__ float hbuf[2][4][64];  // MODE 0 epilogue: h of four tokens, per epilogue group
  __shared__ int2 s_grp[kMaxGroups];  // (expert | tokens << 16, first row)
  __shared__ int s_ngrp;
  __shared__ int s_slot[MODE == 0 ? kMaxDecodeT * 32 : 1];  // MODE 0: slot of each dispatch row
  __shared__ int wsum[8][2];
  uint8_t* smem = smem_raw + ((1024u - (ptx::smem_addr(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  {
    static_assert(sizeof(MxArgs) % 16 == 0, "MxArgs is copied in 16-byte words");
    const int4* src = reinterpret_cast<const int4*>(&pa);
    int4* dst = reinterpret_cast<int4*>(&p);
    for (int i = tid; i < (int)(sizeof(MxArgs) / 16); i += kThreads) dst[i] = src[i];
    __syncthreads();
  }
  const int S = p.stages, NR = p.nsc;
  const int K = p.K, G = K / 32, Nw = p.Nw, nb = p.nb;
  const int nkc = (K + kKC - 1) / kKC, nfull = K / kKC;
  const int nbk = nb > 128 ? 2 : 1;
  const MxSmem L = mx_smem(K, nb, p.b_mode, p.gp, S, NR);
  // [scale-factor atoms | S stages | NR per-item buffers | resident B]; the
  // atoms come first, so that every tcgen05.cp source lies well inside the
  // allocation
  uint8_t* atoms = smem;
  uint8_t* stages = smem + 2 * kSfWarps * kAtomBytes;
  uint8_t* ring0 = stages + S * L.stage;
  uint8_t* res = ring0 + NR * L.ring;
  auto data = [&](int s) { return ptx::smem_addr(bars + s); };
  auto empty = [&](int s) { return ptx::smem_addr(bars + kMaxStages + s); };
  auto sffull = [&](int s) { return ptx::smem_addr(bars + 2 * kMaxStages + s); };
  auto itemb = [&](int b) { return ptx::smem_addr(bars + 3 * kMaxStages + b); };
  auto bfree = [&](int b) { return ptx::smem_addr(bars + 3 * kMaxStages + kMaxRing + b); };
  auto accfull = [&](int b) { return ptx::smem_addr(bars + 3 * kMaxStages + 2 * kMaxRing + b); };
  auto accempty = [&](int b) { return ptx::smem_addr(bars + 3 * kMaxStages + 2 * kMaxRing + 2 + b); };
  const uint32_t resb = ptx::smem_addr(bars + 3 * kMaxStages + 2 * kMaxRing + 4);
  const uint32_t drain = ptx::smem_addr(bars + 3 * kMaxStages + 2 * kMaxRing + 5);
  auto atomfree = [&](int i) { return ptx::smem_addr(bars + 3 * kMaxStages + 2 * kMaxRing + 6 + i); };
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(data(s), 1);
      ptx::mbar_init(empty(s), 1);
      ptx::mbar_init(sffull(s), 1);  // the commit of the stage's tcgen05.cp
    }
    for (int b = 0; b < NR; ++b) {
      ptx::mbar_init(itemb(b), 1);
      ptx::mbar_init(bfree(b), 2);  // a commit from each pipeline's MMA thread
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(accfull(b), 2);
      ptx::mbar_init(accempty(b), 4);
    }
    ptx::mbar_init(resb, 1);
    ptx::mbar_init(drain, 2);
    for (int i = 0; i < 2 * kSfWarps; ++i) ptx::mbar_init(atomfree(i), 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 5) {
    ptx::tmem_alloc(ptx::smem_addr(&tmem_holder), kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    ptx::tma_prefetch_desc(&pa.tm_a);
    ptx::tma_prefetch_desc(&pa.tm_b);
    if (p.b_mode != kBStage && nfull > 0) ptx::tma_prefetch_desc(&pa.tm_b3);
  }
  pdl_wait();  // the logits / routing and the B operands come from the previous kernels
  pdl_launch();
  __syncthreads();  // barriers initialized, tensor memory allocated
  if (p.b_mode == kBResident && warp == 4 && lane == 0) {
    // every token's B tiles and scale rows, once, while the routing runs
    // (they do not depend on it); the TMA warp waits for them before it exits
    const uint32_t rb = ptx::smem_addr(res);
    ptx::mbar_arrive_expect_tx(resb, (uint32_t)(nkc * nb * 128 + kTerms * p.T * p.gp));
    if (nfull > 0) ptx::tma_load_3d(rb, &pa.tm_b3, resb, 0, 0, 0);
    if (nfull < nkc) ptx::tma_load_2d(rb + nfull * nb * 128, &pa.tm_b, resb, nfull * 128, 0);
    ptx::bulk_load(rb + L.res_b, p.bsf, (uint32_t)(kTerms * p.T * p.gp), resb);
  }
  if (MODE == 0) {
    // the stages' space is free until the pipeline starts
    route_dispatch(p, reinterpret_cast<int*>(smem), s_slot, s_grp, &s_ngrp, wsum);
  } else {
    if (tid == 0) s_ngrp = p.meta->n_groups;
    __syncthreads();
    for (int i = tid; i < s_ngrp; i += kThreads) s_grp[i] = p.groups[i];
    __syncthreads();
  }
  ptx::tc_fence_after();
  const uint32_t tmem = tmem_holder;

  const int per_e = (Nw + kBM - 1) / kBM;
  const int n_items = s_ngrp * per_e;
  // Stream-K: the items' K stages, item after item, cut into gridDim.x equal
  // ranges of consecutive stages.  CTA c takes range c and works through its
  // pieces (the parts of items inside the range) from the top down, so that
  // the head pieces of an item split across CTAs finish first, on lower CTAs,
  // and its tail piece -- the owner, which adds their partial sums before the
  // epilogue -- runs last, on the highest of them.  Every CTA holds at most
  // one head piece: its first.
  // 32-bit arithmetic (stages x grid < 2^31, checked by decode_supported):
  // a 64-bit division costs about a microsecond of one thread's time here
  const int G_ = (int)gridDim.x;
  const int n_st = n_items * nkc;
  auto range_lo = [&](int c) { return n_st * c / G_; };
  auto nonempty = [&](int c) { return n_st >= G_ || range_lo(c) < range_lo(c + 1); };
  const int lo = range_lo(blockIdx.x), hi = range_lo(blockIdx.x + 1);
  const int top = hi > lo ? (hi - 1) / nkc : 0;
  const int n_pc = hi > lo ? top - lo / nkc + 1 : 0;
  struct Piece {
    int item, kc0, kc1;
  };
  auto piece = [&](int pc) {
    Piece q;
    q.item = top - pc;
    const int s0 = q.item * nkc;
    q.kc0 = lo > s0 ? lo - s0 : 0;
    q.kc1 = hi - s0 < nkc ? hi - s0 : nkc;
    return q;
  };
  const uint32_t smem0 = ptx::smem_addr(stages);
  const uint32_t sf_base = (uint32_t)(2 * p.nacc * nb);  // TMEM column of stage 0's scale factors

  // MODE 0: the down projection's weights of the routed experts into L2 once
  // this CTA's own copies are issued (HBM would otherwise idle from the end
  // of this launch's stream to the first copies of the next); CTA c pulls
  // slice c of their concatenation.  One warp.
  auto prefetch_next = [&]() {
    if (MODE != 0 || !p.pf_codes || s_ngrp > 32) return;
    const uint32_t full = 0xffffffffu;
    const int ex = lane < s_ngrp ? (s_grp[lane].x & 0xFFFF) : -1;
    const int prev = __shfl_up_sync(full, ex, 1);
    const uint32_t firsts = __ballot_sync(full, lane < s_ngrp && (lane == 0 || prev != ex));
    const int D = __popc(firsts);
    if ((int64_t)D * (p.pf_cb + p.pf_sb) <= kPrefetchMax) {
      for (int part = 0; part < 2; ++part) {
        const int64_t per = part == 0 ? p.pf_cb : p.pf_sb;
        const uint8_t* base = part == 0 ? p.pf_codes : p.pf_scales;
        const int64_t a = ((int64_t)D * per * blockIdx.x / G_) & ~(int64_t)15;
        const int64_t b = ((int64_t)D * per * (blockIdx.x + 1) / G_) & ~(int64_t)15;
        for (int d = 0; d < D; ++d) {
          const int e = __shfl_sync(full, ex, __fns(firsts, 0, d + 1));
          const int64_t u0 = a > d * per ? a : d * per, u1 = b < (d + 1) * per ? b : (d + 1) * per;
          constexpr int64_t kChunk = 16384;
          for (int64_t o = u0 + lane * kChunk; o < u1; o += 32 * kChunk)
            ptx::bulk_prefetch_l2(base + (int64_t)e * per + (o - d * per),
                                  (uint32_t)(u1 - o < kChunk ? u1 - o : kChunk));
        }
      }
    }
  };
  // B rows of an item: MODE 0 every token's (or, gathered, the group's
  // tokens'), MODE 1 the group's
  const bool gather = p.b_mode == kBGather;
  auto brow0 = [&](int2 gr) { return MODE == 0 ? 0 : gr.y * kTerms; };
  auto nbrows = [&](int2 gr) { return (MODE == 0 && !gather) ? kTerms * p.T : kTerms * (gr.x >> 16); };

  // Two pipelines split every piece's stages (pipeline pl takes stages kc0 +
  // pl, kc0 + pl + 2, ...): each has its own TMA warp, MMA thread, group of
  // scale-factor warps, Sp stage slots and accumulator; the epilogue adds the
  // two accumulators.  One thread issues a block-scaled MMA every ~115
  // cycles whatever other threads of the SM issue, so two issuers double the
  // tensor pipe's work per SM.
  const int pl = (warp >= 8 && warp < 12) ? 1 : 0;
  // the warp's role in pipeline 0's numbering; 0-3: epilogue (both groups)
  const int rw = (warp >= 8 && warp < 12) ? warp - 4 : (warp >= 12 ? warp - 12 : warp);
  const int Sp = S / 2;
  if (rw == 4) {
    // ---------------------------------------------------------- TMA producer (one warp a pipeline)
    // Lane 0 waits and issues the weight tiles; with gathered B, lane j
    // issues token j's boxes (one thread issuing 17 copies a stage was the
    // limit at 64 tokens).  Pipeline 0's warp also loads the per-item blocks.
    const uint32_t full = 0xffffffffu;
    int g = 0, n_issued = 0;  // g: this pipeline's stages
    int s = 0, ph = 0;        // their slot and parity: g % Sp, (g / Sp) & 1 (no divisions in the loop)
    bool ok = true;
    // Per-item blocks (A scale rows, B scale rows, kBItem's B tiles) of piece
    // pi, once its ring buffer is free (the MMAs of the piece NR earlier
    // finished).  False on a timeout.  With three buffers the next piece's
    // blocks are issued at the start of this piece (with two, the buffer it
    // needs frees only as this piece begins, which measured no faster).
    auto issue_items = [&](int pi) {
      const int b = pi % NR;
      bool fr = pi < NR;
      if (!fr) {
        if (lane == 0) fr = ptx::mbar_wait(bfree(b), ((pi / NR) - 1) & 1, &abort_flag);
        fr = __shfl_sync(full, fr, 0);
      }
      if (!fr) return false;
      const Piece qi = piece(pi);
      const int2 gi = s_grp[qi.item / per_e];
      const int ei = gi.x & 0xFFFF, ri = (qi.item % per_e) * kBM, nti = gi.x >> 16;
      const int nri = min(kBM, Nw - ri), nbi = nbrows(gi), bi0 = brow0(gi);
      const uint32_t sbt = ptx::smem_addr(ring0 + b * L.ring), sca = sbt + L.ring_b, scb = sca + L.ring_sa;
      if (lane == 0) {
        // the item's scale rows (A contiguous [rows][G], B [nbv][gp]) and, per
        // item, its B tiles for all of K
        uint32_t tx = nri * G;
        if (p.b_mode != kBResident) tx += nbi * p.gp;
        if (p.b_mode == kBItem) tx += nkc * nb * 128;
        ptx::mbar_arrive_expect_tx(itemb(b), tx);
        ptx::bulk_load(sca, p.scales + ((int64_t)ei * Nw + ri) * G, (uint32_t)(nri * G), itemb(b));
        if (!gather && p.b_mode != kBResident)
          ptx::bulk_load(scb, p.bsf + (int64_t)bi0 * p.gp, (uint32_t)(nbi * p.gp), itemb(b));
        if (p.b_mode == kBItem) {
          if (nfull > 0) ptx::tma_load_3d(sbt, &pa.tm_b3, itemb(b), 0, bi0, 0);
          if (nfull < nkc) ptx::tma_load_2d(sbt + nfull * nb * 128, &pa.tm_b, itemb(b), nfull * 128, bi0);
        }
      }
      __syncwarp();
      if (gather && lane < nti) {
        const int tr = (s_slot[gi.y + lane] / p.k) * kTerms;  // the lane's token: its first term row
        ptx::bulk_load(scb + lane * kTerms * p.gp, p.bsf + (int64_t)tr * p.gp, (uint32_t)(kTerms * p.gp), itemb(b));
      }
      ++n_issued;
      return true;
    };
    for (int pc = 0; pc < n_pc && ok; ++pc) {
      const Piece q = piece(pc);
      const int item = q.item;
      const int2 gr = s_grp[item / per_e];
      const int e = gr.x & 0xFFFF, r0 = (item % per_e) * kBM, ntok = gr.x >> 16;
      const int nrows = min(kBM, Nw - r0), nbv = nbrows(gr), b0 = brow0(gr);
      // gathered B: this lane's token (its first term row)
      const int trow = (gather && lane < ntok) ? (s_slot[gr.y + lane] / p.k) * kTerms : 0;
      bool w = true;
      // pipeline 0: this piece's per-item blocks, once their buffer is free
      if (pl == 0 && n_issued <= pc && !issue_items(pc)) break;
      for (int kc = q.kc0 + pl; kc < q.kc1; kc += 2, ++g) {
        const int sl = pl * Sp + s;
        // with three or more per-item buffers the next piece's blocks go out
        // a piece ahead (its buffer was freed by the piece NR back, long done)
        if (pl == 0 && NR >= 3 && kc == q.kc0 && n_issued == pc + 1 && pc + 1 < n_pc) {
          bool fr = true;
          if (lane == 0 && pc + 1 >= NR) fr = ptx::mbar_test(bfree((pc + 1) % NR), (((pc + 1) / NR) - 1) & 1);
          if (__shfl_sync(full, fr, 0)) issue_items(pc + 1);
        }
        if (lane == 0 && g >= Sp) w = ptx::mbar_wait(empty(sl), ph ^ 1, &abort_flag);
        if (!__shfl_sync(full, w, 0)) {
          ok = false;
          break;
        }
        const uint32_t sa = smem0 + sl * L.stage;
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(data(sl), (uint32_t)(gather ? kBM * 128 + nbv * 128 : L.stage));
          ptx::tma_load_2d(sa, &pa.tm_a, data(sl), kc * 128, e * Nw + r0);
          if (p.b_mode == kBStage) ptx::tma_load_2d(sa + kBM * 128, &pa.tm_b, data(sl), kc * 128, b0);
        }
        __syncwarp();
        // one 4-row box per token of the group (the stage's count covers exactly these)
        if (gather && lane < ntok)
          ptx::tma_load_2d(sa + kBM * 128 + lane * kTerms * 128, &pa.tm_b, data(sl), kc * 128, trow);
        if (++s == Sp) s = 0, ph ^= 1;
      }
    }
    if (lane == 0 && abort_flag) {
      // after a timeout elsewhere: let this warp's copies in flight land
      // (bounded) before the CTA exits
      volatile int quiet = 0;
      for (int gg = max(0, g - Sp); gg < g; ++gg)
        ptx::mbar_wait(data(pl * Sp + gg % Sp), (gg / Sp) & 1, &quiet, 100000000LL);
      for (int i2 = max(0, n_issued - NR); i2 < n_issued; ++i2)
        ptx::mbar_wait(itemb(i2 % NR), (i2 / NR) & 1, &quiet, 100000000LL);
    }
    if (pl == 0 && lane == 0 && p.b_mode == kBResident) {
      // the resident B copies must have landed before the CTA exits (bounded)
      volatile int quiet = 0;
      ptx::mbar_wait(resb, 0, &quiet, 100000000LL);
    }
    __syncwarp();
    if (pl == 0 && !abort_flag) prefetch_next();
  } else if (rw == 5) {
    // ---------------------------------------------------------- MMA issue (one thread a pipeline)
    if (lane == 0) {
      // one thread whose per-stage instructions are the issue rate: no
      // divisions in the loop, descriptors advanced by addition
      int g = 0, s = 0, ph = 0;
      bool ok = true;
      if (p.b_mode == kBResident && n_pc > 0) ok = ptx::mbar_wait(resb, 0, &abort_flag);
      for (int pc = 0; pc < n_pc && ok; ++pc) {
        const Piece q = piece(pc);
        const int2 gr = s_grp[q.item / per_e];
        const int N = ((nbrows(gr) + 15) / 16) * 16;
        const int ab = pc % p.nacc, b = pc % NR;
        if (pc >= p.nacc && !ptx::mbar_wait(accempty(ab), ((pc / p.nacc) - 1) & 1, &abort_flag)) break;
        if (p.b_mode == kBItem && !ptx::mbar_wait(itemb(b), (pc / NR) & 1, &abort_flag)) break;
        ptx::tc_fence_after();
        const uint32_t acc = tmem + (pl * p.nacc + ab) * nb;
        const uint32_t bt = p.b_mode == kBItem ? ptx::smem_addr(ring0 + b * L.ring) : ptx::smem_addr(res);
        const uint32_t id0 = ptx::idesc_mxf4(N, 0, 0), id2 = ptx::idesc_mxf4(N, 2, 2);
        const bool b_in_stage = p.b_mode == kBStage || gather;
        // smem descriptors' address field is (address >> 4): advancing a
        // descriptor by a 16-byte multiple adds to it
        const uint64_t ad0 = ptx::sdesc_kmajor_sw128(smem0);
        const uint64_t bd_item = ptx::sdesc_kmajor_sw128(bt) + (uint64_t)((q.kc0 * nb * 128) >> 4);
        for (int kc = q.kc0 + pl; kc < q.kc1; kc += 2, ++g) {
          const int sl = pl * Sp + s;
          if (!ptx::mbar_wait(data(sl), ph, &abort_flag) || !ptx::mbar_wait(sffull(sl), ph, &abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint64_t ad = ad0 + (uint64_t)((sl * L.stage) >> 4);
          const uint64_t bd = b_in_stage ? ad + (kBM * 128 >> 4) : bd_item + (uint64_t)(((kc - q.kc0) * nb * 128) >> 4);
          // scale factors (written by the pipeline's scale-factor warps): SFA
          // at columns 4q, SFB at 8 + 4 nbk q for groups q = 0, 1 of four k-blocks
          const uint32_t sf = tmem + sf_base + sl * kSfStageCols;
          const int nm = (K - kc * kKC) >= kKC ? 4 : (K - kc * kKC) / 64;
          const bool acc0 = kc != q.kc0 + pl;  // this pipeline's first stage of the piece
          ptx::mma_mxf4_ss(acc, ad, bd, id0, sf, sf + 8, acc0);
          if (nm > 1) ptx::mma_mxf4_ss(acc, ad + 2, bd + 2, id2, sf, sf + 8, 1);
          if (nm > 2) ptx::mma_mxf4_ss(acc, ad + 4, bd + 4, id0, sf + 4, sf + 8 + 4 * nbk, 1);
          if (nm > 3) ptx::mma_mxf4_ss(acc, ad + 6, bd + 6, id2, sf + 4, sf + 8 + 4 * nbk, 1);
          ptx::tc_commit(empty(sl));
          if (++s == Sp) s = 0, ph ^= 1;
        }
        if (ok) {  // both pipelines arrive (a commit with no MMAs of this piece arrives once earlier ones finish)
          ptx::tc_commit(accfull(ab));
          ptx::tc_commit(bfree(b));
        }
      }
    }
    __syncwarp();
  } else if (rw >= 6) {
    // ---------------------------------------------------------- scale factors into TMEM
    // kSfWarps warps a pipeline take its stages in turn.  A warp lays out a
    // stage's scale factors in shared memory as 32 rows of 16 bytes -- row l
    // holds the words of rows l + 32 j, j = 0..3, each word four k-blocks'
    // scales; SFA then SFB, k-block groups q = 0, 1 -- and lane 0 copies each
    // 512-byte block into the stage's four columns of all four TMEM
    // subpartitions (tcgen05.cp ... warpx4).  The commit of the copies
    // completes sffull (for the MMA thread) and atomfree (the warp's own
    // buffer may be rewritten); nothing waits on the TMEM writes themselves.
    const int sw = rw - 6;
    const uint32_t atom_s = ptx::smem_addr(atoms + (pl * kSfWarps + sw) * kAtomBytes);
    uint8_t* atom = atoms + (pl * kSfWarps + sw) * kAtomBytes;
    const uint32_t afree = atomfree(pl * kSfWarps + sw);
    int g = 0, s = 0, ph = 0;  // this pipeline's stage g: slot and parity
    int used = 0;              // stages this warp laid out
    bool ok = true;
    if (p.b_mode == kBResident && n_pc > 0) {
      bool w = true;
      if (lane == 0) w = ptx::mbar_wait(resb, 0, &abort_flag);
      ok = __shfl_sync(0xffffffffu, w, 0);
    }
    for (int pc = 0; pc < n_pc && ok; ++pc) {
      const Piece q = piece(pc);
      const int2 gr = s_grp[q.item / per_e];
      const int r0 = (q.item % per_e) * kBM;
      const int nrows = min(kBM, Nw - r0), nbv = nbrows(gr);
      const int b = pc % NR;
      bool w = true;
      if (lane == 0) w = ptx::mbar_wait(itemb(b), (pc / NR) & 1, &abort_flag);
      if (!__shfl_sync(0xffffffffu, w, 0)) break;
      const uint8_t* sca = ring0 + b * L.ring + L.ring_b;
      const uint8_t* scb = p.b_mode == kBResident ? res + L.res_b : sca + L.ring_sa;
      for (int kc = q.kc0 + pl; kc < q.kc1; kc += 2, ++g) {
        const int sl = pl * Sp + s;
        if ((g & (kSfWarps - 1)) == sw) {
          // the slot's columns are free once the MMAs of its previous stage
          // finished; this warp's buffer once its previous copies finished
          if (lane == 0 && g >= Sp) w = ptx::mbar_wait(empty(sl), ph ^ 1, &abort_flag);
          if (lane == 0 && w && used > 0) w = ptx::mbar_wait(afree, (used - 1) & 1, &abort_flag);
          if (!__shfl_sync(0xffffffffu, w, 0)) {
            ok = false;
            break;
          }
          uint32_t wa[8], wb[8];
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            const int gq = 2 * kc + qq;
            const bool gv = 4 * gq < G;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int r = lane + 32 * j;
              uint32_t v = 0;
              if (gv && r < nrows) {
                const uint16_t* row = reinterpret_cast<const uint16_t*>(sca + r * G);
                v = row[2 * gq] | ((4 * gq + 2 < G) ? (uint32_t)row[2 * gq + 1] << 16 : 0u);
              }
              wa[4 * qq + j] = v;
              wb[4 * qq + j] = (gv && r < nbv) ? *reinterpret_cast<const uint32_t*>(scb + r * p.gp + 4 * gq) : 0u;
            }
          }
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            *reinterpret_cast<uint4*>(atom + qq * 512 + lane * 16) = make_uint4(wa[4 * qq], wa[4 * qq + 1], wa[4 * qq + 2], wa[4 * qq + 3]);
            *reinterpret_cast<uint4*>(atom + 1024 + qq * 512 + lane * 16) =
                make_uint4(wb[4 * qq], wb[4 * qq + 1], wb[4 * qq + 2], wb[4 * qq + 3]);
          }
          ptx::fence_proxy_async_smem();  // the rows, written by this warp, to the copy's (async) reads
          __syncwarp();
          if (lane == 0) {
            ptx::tc_fence_after();
            // columns: SFA group q at 4 q, SFB group q at 8 + 4 q (one 128-row block of B)
            const uint32_t sf = tmem + sf_base + sl * kSfStageCols;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
              ptx::tc_cp_32x128b_warpx4(sf + 4 * c4, ptx::sdesc_rows16(atom_s + 512 * c4));
            ptx::tc_commit(sffull(sl));
            ptx::tc_commit(afree);
          }
          __syncwarp();
          ++used;
        }
        if (++s == Sp) s = 0, ph ^= 1;
      }
    }
    if (lane == 0 && used > 0) {
      // copies still in flight must finish before the tensor memory is freed (bounded)
      volatile int quiet = 0;
      ptx::mbar_wait(afree, (used - 1) & 1, &quiet, 100000000LL);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- epilogue
    // Two groups of four warps (one per TMEM subpartition each), group eg
    // draining accumulator buffer eg: pieces alternate between them, so two
    // epilogues run at once (at a few tokens one epilogue outlasts a piece's
    // MMAs).  With a single buffer group 1 has nothing to do.
    const int eg = warp >= 12 ? 1 : 0, ew = eg * 4 + (warp & 3);
    const int ebar = eg ? 2 : 1;  // the group's named barrier
    const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
    bool ok = true;
    for (int pc = eg; pc < n_pc && ok && eg < p.nacc; pc += p.nacc) {
      const Piece q = piece(pc);
      const int item = q.item;
      const int2 gr = s_grp[item / per_e];
      const int e = gr.x & 0xFFFF, ntok = gr.x >> 16, row_lo = gr.y, r0 = (item % per_e) * kBM;
      const int nrows = min(kBM, Nw - r0);
      const int ab = pc % p.nacc;
      const int lrow = 32 * (warp & 3) + lane;
      const bool rv = lrow < nrows;
      const int64_t grow = (int64_t)e * Nw + r0 + lrow;
      // a head piece of a split item leaves its sums to the item's tail piece
      // (the owner), which adds those of CTAs [c_first, this one)
      const bool owner = q.kc1 == nkc;
      const int c_first = (owner && q.kc0 > 0) ? ((item * nkc + 1) * G_ - 1) / n_st : (int)blockIdx.x;
      float bv = 0.f;
      if (owner && rv && p.bias)
        bv = p.bias_f32 ? static_cast<const float*>(p.bias)[grow]
                        : __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[grow]);
      // per token j of the group: its accumulator column (MODE 0: the token's
      // row among all tokens) and, MODE 1, its routing weight
      int col = 0;
      float wt = 0.f;
      if (lane < ntok) {
        const int sl = MODE == 0 ? s_slot[row_lo + lane] : p.slot_of_row[row_lo + lane];
        col = (MODE == 0 && !gather) ? kTerms * (sl / p.k) : kTerms * lane;
        if (MODE == 1) wt = p.scores[sl];
      }
      // the head pieces' partial sums (written early by the CTAs below, which
      // process them first) of the first four tokens: loaded while this
      // piece's MMAs finish
      bool got = true;
      float pre[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c2 = c_first; got && c2 < (int)blockIdx.x; ++c2)
        if (nonempty(c2)) {
          got = wait_flag(p.flags + c2, 4u, &abort_flag);
          const float* pp = p.part + (int64_t)c2 * kGroupTok * kBM + lrow;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) pre[jj] += __ldcg(pp + jj * kBM);
        }
      got = got && ptx::mbar_wait(accfull(ab), (pc / p.nacc) & 1, &abort_flag);
      if (!named_and(ebar, 128, got)) break;
      ptx::tc_fence_after();
      const uint32_t tl = tmem + lanes + ab * nb;     // pipeline 0's accumulator
      const uint32_t tl1 = tl + p.nacc * nb;           // pipeline 1's, written if the piece has two stages
      const bool two = q.kc1 - q.kc0 >= 2;
      const int nchunk = (ntok + 3) / 4;
      for (int c = 0; c < nchunk; ++c) {
        // the head pieces' sums of these four tokens (the first four's are loaded)
        float acc[4] = {c ? 0.f : pre[0], c ? 0.f : pre[1], c ? 0.f : pre[2], c ? 0.f : pre[3]};
        for (int c2 = c_first; c > 0 && c2 < (int)blockIdx.x; ++c2)
          if (nonempty(c2)) {
            const float* pp = p.part + ((int64_t)c2 * kGroupTok + c * 4) * kBM + lrow;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[jj] += __ldcg(pp + jj * kBM);
          }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int cj = __shfl_sync(0xffffffffu, col, (c * 4 + jj) & 31);
          uint32_t u[4], v[4] = {0u, 0u, 0u, 0u};
          ptx::tmem_ld_32x32b_x4(tl + cj, u);  // tokens past ntok read column 0, unused
          if (two) ptx::tmem_ld_32x32b_x4(tl1 + cj, v);
          ptx::tmem_wait_ld();
          acc[jj] += ((__uint_as_float(u[0]) + __uint_as_float(u[1])) + (__uint_as_float(u[2]) + __uint_as_float(u[3]))) +
                     ((__uint_as_float(v[0]) + __uint_as_float(v[1])) + (__uint_as_float(v[2]) + __uint_as_float(v[3]))) + bv;
        }
        if (c == nchunk - 1) {
          // accumulator drained: the MMAs of a later item may use it
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(accempty(ab));
        }
        if (!owner) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj)
            if (c * 4 + jj < ntok && rv) p.part[((int64_t)blockIdx.x * kGroupTok + c * 4 + jj) * kBM + lrow] = acc[jj];
          continue;
        }
        if (MODE == 1) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int tok = c * 4 + jj;
            const float w = __shfl_sync(0xffffffffu, wt, tok & 31);
            if (tok < ntok && rv) p.y[(int64_t)(row_lo + tok) * Nw + r0 + lrow] = acc[jj] * w;
          }
        } else {
          h_terms(p, acc, c, ntok, row_lo, r0 >> 1, warp & 3, lane, hbuf[eg], ebar);
        }
      }
      if (!owner) {
        // this warp's partial sums are out: count it for the owner
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.flags + blockIdx.x, 1u);
      }
    }
  }
  __syncthreads();
  // MMAs may still be in flight after a timeout: both MMA threads commit to
  // `drain`, whose completion warp 5 waits for (bounded) before the tensor
  // memory is released
  if ((warp == 5 || warp == 9) && lane == 0 && abort_flag) ptx::tc_commit(drain);
  if (warp == 5) {
    if (lane == 0 && abort_flag) {
      record_status(p.status, BS_ERR_TIMEOUT);
      volatile int quiet = 0;
      ptx::mbar_wait(drain, 0, &quiet, 100000000LL);
    }
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ 4. combine
__global__ void __launch_bounds__(256) decode_combine_kernel(const float4* __restrict__ y,
                                                             const int* __restrict__ row_of_slot,
                                                             int T, int k, int vecs,
                                                             const uint2* __restrict__ residual,
                                                             uint2* __restrict__ out) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T * vecs; i += gridDim.x * blockDim.x) {
    const int t = i / vecs, v = i - t * vecs;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int s = 0; s < k; ++s) {
      const int r = row_of_slot[t * k + s];
      if (r < 0) continue;
      const float4 q = y[(int64_t)r * vecs + v];
      a0 += q.x;
      a1 += q.y;
      a2 += q.z;
      a3 += q.w;
    }
    if (residual) {
      const uint2 q = residual[i];
      out[i] = make_uint2(add_residual_bf16x2(q.x, a0, a1), add_residual_bf16x2(q.y, a2, a3));
    } else {
      out[i] = make_uint2(pack_bf16x2(a0, a1), pack_bf16x2(a2, a3));
    }
  }
}

template <typename Kern, typename... Args>
int launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  BS_CUDA(cudaLaunchKernelEx(&cfg, kern, args...));
  return BS_OK;
}

// Pitch of a row of per-32 scales (16-byte multiple: rows are bulk-copied).
int gp_of(int64_t K) { return (int)align_up((size_t)(K / 32), 16); }

// Pipeline shape of one expert projection: where B comes from, stages,
// per-item buffers and accumulator buffers that fit in shared and tensor
// memory.  Resident B (MODE 0, few tokens) or per-item B when that leaves at
// least four stages; else a B tile per stage.
int plan_mx(MxArgs& a, std::initializer_list<int> modes) {
  const int budget = 198 * 1024;  // dynamic shared memory (the static arrays take ~18 KB)
  a.stages = 0;
  for (int b_mode : modes) {
    // an even count: the two pipelines hold half each
    for (int S = kMaxStages; S >= ((b_mode == kBStage || b_mode == kBGather) ? 2 : 4); S -= 2) {
      if (mx_smem(a.K, a.nb, b_mode, a.gp, S, 2).total <= budget) {
        // a third per-item buffer (the next piece's blocks a piece ahead) if it costs no stage
        const int nsc = mx_smem(a.K, a.nb, b_mode, a.gp, S, 3).total <= budget ? 3 : 2;
        a.b_mode = b_mode, a.stages = S, a.nsc = nsc;
        break;
      }
    }
    if (a.stages) break;
  }
  BS_REQUIRE(a.stages >= 2, BS_ERR_UNSUPPORTED, "decode path: B tile of %d rows does not fit", a.nb);
  // one 128-row block of B scale factors per k-block group (the tcgen05.cp layout)
  BS_REQUIRE(a.nb <= 128, BS_ERR_UNSUPPORTED, "decode path: B tile of %d rows", a.nb);
  // accumulators: two pipelines x (two buffers if they fit, else one)
  a.nacc = (4 * a.nb + a.stages * kSfStageCols <= kTmemCols) ? 2 : 1;
  BS_REQUIRE(2 * a.nacc * a.nb + a.stages * kSfStageCols <= kTmemCols, BS_ERR_UNSUPPORTED,
             "decode path: tensor memory plan does not fit");
  return BS_OK;
}

// Maps of B: per-stage / tail boxes of nb rows, and the item's full chunks in one 3-D box.
int make_b_maps(MxArgs& a, const void* rows_base, int64_t rows) {
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const int64_t pitch = a.K / 2, nfull = a.K / kKC;
  const uint32_t box_rows = a.b_mode == kBGather ? kTerms : (uint32_t)a.nb;
  BS_TRY(make_map_2d(&a.tm_b, u8, rows_base, (uint64_t)pitch, (uint64_t)rows, (uint64_t)pitch, 128, box_rows, sw));
  if (a.b_mode != kBStage && nfull > 0) {
    const uint64_t dims[3] = {128, (uint64_t)rows, (uint64_t)nfull};
    const uint64_t strides[2] = {(uint64_t)pitch, 128};
    const uint32_t box[3] = {128, (uint32_t)a.nb, (uint32_t)nfull};
    BS_TRY(make_map_3d(&a.tm_b3, u8, rows_base, dims, strides, box, sw));
  }
  return BS_OK;
}

template <int MODE>
int launch_mx(const MxArgs& a, cudaStream_t st) {
  const size_t smem = mx_smem(a.K, a.nb, a.b_mode, a.gp, a.stages, a.nsc).total;
  BS_CUDA(cudaFuncSetAttribute(decode_mx_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return launch_pdl(decode_mx_kernel<MODE>, dim3((unsigned)std::min(sm_count(), kMaxCtas)), dim3(kThreads), smem, st,
                    a);
}

}  // namespace

struct DecodeWS {
  DecodeMeta* meta;
  float* logits;
  int* offsets;
  int* row_of_slot;
  int* slot_of_row;
  int2* groups;
  uint8_t* xq;
  uint8_t* xs;
  uint8_t* hq;
  uint8_t* hs;
  float* y;
  float* part;
  unsigned* flags;
  size_t total;
};

DecodeWS decode_carve(void* base, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  DecodeWS w{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return base ? static_cast<char*>(base) + at : nullptr;
  };
  const int64_t S = T * k;
  w.meta = reinterpret_cast<DecodeMeta*>(take(sizeof(DecodeMeta)));
  w.logits = reinterpret_cast<float*>(take((size_t)T * E * 4));
  w.offsets = reinterpret_cast<int*>(take((size_t)(E + 1) * 4));
  w.row_of_slot = reinterpret_cast<int*>(take((size_t)S * 4));
  w.slot_of_row = reinterpret_cast<int*>(take((size_t)S * 4));
  w.groups = reinterpret_cast<int2*>(take((size_t)kMaxGroups * sizeof(int2)));
  w.xq = reinterpret_cast<uint8_t*>(take((size_t)T * kTerms * H / 2));
  w.xs = reinterpret_cast<uint8_t*>(take((size_t)T * kTerms * gp_of(H)));
  w.hq = reinterpret_cast<uint8_t*>(take((size_t)S * kTerms * I / 2));
  w.hs = reinterpret_cast<uint8_t*>(take((size_t)S * kTerms * gp_of(I)));
  w.y = reinterpret_cast<float*>(take((size_t)S * H * 4));
  w.part = reinterpret_cast<float*>(take((size_t)kMaxCtas * kGroupTok * kBM * 4));
  w.flags = reinterpret_cast<unsigned*>(take((size_t)2 * kMaxCtas * 4));
  w.total = o;
  return w;
}

size_t decode_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  return decode_carve(nullptr, T, H, I, E, k).total;
}

bool decode_supported(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  // the expert launches split (item, K stage) pairs over the grid in 32-bit arithmetic
  const int64_t stages = kMaxGroups * std::max(cdiv(2 * I, (int64_t)kBM) * cdiv(H, (int64_t)kKC),
                                               cdiv(H, (int64_t)kBM) * cdiv(I, (int64_t)kKC));
  return T >= 1 && T <= kMaxDecodeT && E <= 1024 && k <= 32 && H % 64 == 0 && I % 64 == 0 &&
         (2 * I) % kBM == 0 && stages * kMaxCtas < ((int64_t)1 << 31);
}

// The four-launch decode forward.  router_weight NULL: scores/indices are inputs.
int decode_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                   const void* rw, const void* rb, int rdt, float* scores, int32_t* indices,
                   const void* gu_b, const void* gu_s, const void* gu_bias, const void* dn_b,
                   const void* dn_s, const void* dn_bias, int bias_f32, float alpha, float limit,
                   void* out, void* ws, cudaStream_t st, const void* residual) {
  BS_ARG(decode_supported(T, H, I, E, k),
         "decode path: need 1 <= T <= %d, E <= 1024, k <= 32, H and I multiples of 64", kMaxDecodeT);
  BS_REQUIRE(((uintptr_t)gu_b | (uintptr_t)dn_b | (uintptr_t)gu_s | (uintptr_t)dn_s) % 16 == 0,
             BS_ERR_MISALIGNED, "decode path: expert blocks and scales must be 16-byte aligned");
  const DecodeWS w = decode_carve(ws, T, H, I, E, k);
  int* status = device_status_ptr();
  const int64_t G = H / 32;
  const dim3 rgrid((unsigned)std::max<int64_t>(rw ? E : 1, std::min<int64_t>(G, 128)),
                   (unsigned)cdiv(T, (int64_t)kRTok));
  if (!rw || rdt == BS_F32) {
    BS_TRY(launch_pdl(decode_route_kernel<float>, rgrid, dim3(256), 0, st,
                      static_cast<const __nv_bfloat16*>(x), static_cast<const float*>(rw),
                      static_cast<const float*>(rb), (int)T, (int)H, (int)E, 0, w.logits, w.xq, w.xs,
                      gp_of(H), w.flags, 2 * kMaxCtas));
  } else {
    BS_TRY(launch_pdl(decode_route_kernel<__nv_bfloat16>, rgrid, dim3(256), 0, st,
                      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(rw),
                      static_cast<const __nv_bfloat16*>(rb), (int)T, (int)H, (int)E, 1, w.logits, w.xq,
                      w.xs, gp_of(H), w.flags, 2 * kMaxCtas));
  }
  MxArgs a{};
  a.logits = rw ? w.logits : nullptr;
  a.idx = indices;
  a.scores = scores;
  a.offsets = w.offsets;
  a.row_of_slot = w.row_of_slot;
  a.slot_of_row = w.slot_of_row;
  a.groups = w.groups;
  a.meta = w.meta;
  a.E = (int)E;
  a.k = (int)k;
  a.T = (int)T;
  a.alpha = alpha;
  a.limit = limit;
  a.bias_f32 = bias_f32;
  a.status = status;
  a.part = w.part;
  a.flags = w.flags;
  // the routed experts' down weights are pulled into L2 during gate_up
  a.pf_codes = static_cast<const uint8_t*>(dn_b);
  a.pf_scales = static_cast<const uint8_t*>(dn_s);
  a.pf_cb = H * (I / 2);
  a.pf_sb = H * (I / 32);
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  // gate_up: A = [E][2I][H/32][16], B = x terms of every token, out = h terms
  a.scales = static_cast<const uint8_t*>(gu_s);
  a.bias = gu_bias;
  a.bsf = w.xs;
  a.gp = gp_of(H);
  a.Nw = (int)(2 * I);
  a.K = (int)H;
  a.hq = w.hq;
  a.hs = w.hs;
  a.gp_out = gp_of(I);
  BS_TRY(make_map_2d(&a.tm_a, u8, gu_b, (uint64_t)(H / 2), (uint64_t)(E * 2 * I), (uint64_t)(H / 2), 128, kBM, sw));
  if (T <= kGroupTok) {  // every token's terms as B
    a.nb = (int)((kTerms * T + 15) / 16 * 16);
    BS_TRY(plan_mx(a, {kBResident, kBStage}));
  } else {  // the group's tokens' terms, gathered
    a.nb = kTerms * kGroupTok;
    BS_TRY(plan_mx(a, {kBGather}));
  }
  BS_TRY(make_b_maps(a, w.xq, T * kTerms));
  BS_TRY(launch_mx<0>(a, st));
  // down: A = [E][H][I/32][16], B = h terms (contiguous per expert), out = weighted fp32 rows
  a.scales = static_cast<const uint8_t*>(dn_s);
  a.bias = dn_bias;
  a.bsf = w.hs;
  a.gp = gp_of(I);
  a.Nw = (int)H;
  a.K = (int)I;
  a.y = w.y;
  a.flags = w.flags + kMaxCtas;
  a.pf_codes = nullptr;
  a.pf_scales = nullptr;
  BS_TRY(make_map_2d(&a.tm_a, u8, dn_b, (uint64_t)(I / 2), (uint64_t)(E * H), (uint64_t)(I / 2), 128, kBM, sw));
  a.nb = (int)((kTerms * std::min<int64_t>(T, kGroupTok) + 15) / 16 * 16);  // a group's tokens
  BS_TRY(plan_mx(a, {kBItem, kBStage}));
  BS_TRY(make_b_maps(a, w.hq, T * k * kTerms));
  BS_TRY(launch_mx<1>(a, st));
  const int vecs = (int)(H / 4);
  const int cgrid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(T * vecs, (int64_t)256), sm_count() * 4));
  BS_TRY(launch_pdl(decode_combine_kernel, dim3(cgrid), dim3(256), 0, st, (const float4*)w.y,
                    (const int*)w.row_of_slot, (int)T, (int)k, vecs, static_cast<const uint2*>(residual),
                    static_cast<uint2*>(out)));
  return BS_OK;
}

}  // namespace bs
