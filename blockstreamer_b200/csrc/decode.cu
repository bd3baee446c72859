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
// On this GPU an M=128 block-scaled MMA costs ~143 cycles whatever N is, so
// the instruction count -- weights / (128 x 64) -- sets the tensor-core time;
// K = 64 per instruction keeps it under the HBM time of the weights.
//
// The layer runs as four launches chained with programmatic dependent launch:
//  1. decode_route_kernel  x -> four e2m1 terms; router logits with one CTA per
//     (expert, 16 tokens) (modeling_gpt_oss.py:126-130); the last CTA to finish
//     (ticket counter) runs top-k + softmax over the k and the dispatch
//     (gptoss.py:143-154) and writes the list of experts that received tokens.
//  2. decode_mx_kernel<0>  gate_up + bias + clamped SwiGLU (gptoss.py:130-135,
//     158-166); h is written as four e2m1 terms for the next projection.
//  3. decode_mx_kernel<1>  down + bias, times the routing weight (167-175),
//     fp32 rows.
//  4. decode_combine_kernel out[t] = bf16(sum over the k slots), fp32 sum.
//
// Work item of 2/3: 128 weight rows of one expert and a group of up to 16 of
// its tokens (an expert with more tokens has several groups; the route
// kernel lists them).
// One CTA per SM: warp 4 issues the TMA copies (weight tiles [128 rows x 256
// codes] as stored, the B term rows, per-item scale blocks); warps 0-3 repack
// each item's scales into the 32-row blocks tcgen05.cp reads and drain the
// accumulators; warp 5 copies every stage's scale factors into TMEM
// (tcgen05.cp, ordered with its MMAs) and issues the MMAs.
#include "bs_common.cuh"
#include "bs_ptx.cuh"

namespace bs {
namespace {

constexpr int kMaxDecodeT = 64;
constexpr int kTerms = 4;       // e2m1 terms per activation
constexpr int kRTok = 16;       // tokens per router CTA
constexpr int kKC = 256;        // K elements per pipeline stage: 128 bytes of codes per row, 4 MMAs
constexpr int kBM = 128;        // weight rows per item (MMA M)
constexpr int kThreads = 192;   // warps 0-3 scale repack + epilogue, 4 TMA, 5 MMA
constexpr int kTmemCols = 512;
constexpr int kSfStageCols = 16;  // per stage: SFA and SFB, 2 groups of four k-blocks x 4 columns
constexpr int kMaxStages = 12;
constexpr int kGroupTok = 16;     // tokens per group: B = 4 terms x 16 = 64 rows at most
constexpr int kMaxGroups = 1024 + 2048 / kGroupTok;

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

// One warp: top-k of E values (ties -> lower index), softmax over the k.
template <typename Get>
__device__ void warp_topk(Get get, int E, int k, float* scores, int32_t* idx) {
  const int lane = threadIdx.x & 31;
  constexpr int kPer = 1024 / 32;
  float v[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? get(e) : -INFINITY;
    if (v[i] != v[i]) v[i] = -INFINITY;
  }
  float sel_v = 0.f;
  int sel_e = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > bv || (v[i] == bv && e < be))) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == be) v[i] = __int_as_float(0x7fc00000u);  // removed: never selected again
    if (lane == j) {
      sel_v = bv;
      sel_e = be;
    }
  }
  const float mx = __shfl_sync(0xffffffffu, sel_v, 0);
  const float ex = (lane < k) ? expf(sel_v - mx) : 0.f;
  float sum = ex;
#pragma unroll
  for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane < k) {
    scores[lane] = ex / sum;
    idx[lane] = sel_e;
  }
}

// ------------------------------------------------------------------ 1. route
// xq: rows (4 t + term) of H/2 bytes (two codes per byte, low nibble first);
// xs: rows (4 t + term) of gp bytes (one e8m0 scale per 32 values).
template <typename WT>
__global__ void __launch_bounds__(256) decode_route_kernel(
    const __nv_bfloat16* __restrict__ x, const WT* __restrict__ W, const WT* __restrict__ b,
    int T, int H, int E, int k, int bf16_logits, float* __restrict__ logits,
    float* __restrict__ scores, int32_t* __restrict__ idx, int* __restrict__ offsets,
    int* __restrict__ row_of_slot, int* __restrict__ slot_of_row, int2* __restrict__ groups,
    uint8_t* __restrict__ xq, uint8_t* __restrict__ xs, int gp, DecodeMeta* meta, int* status) {
  __shared__ float red[8][kRTok];
  __shared__ int cnt[1024];
  __shared__ int off[1025];
  __shared__ int is_last;
  pdl_wait();  // x comes from the previous kernel in the stream
  pdl_launch();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

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

  if (W) {  // logits of expert blockIdx.x for 16 tokens
    const int e = blockIdx.x, t0 = blockIdx.y * kRTok;
    if (e < E) {
      const int nt = min(kRTok, T - t0);
      float acc[kRTok];
#pragma unroll
      for (int t = 0; t < kRTok; ++t) acc[t] = 0.f;
      const WT* w = W + (int64_t)e * H;
      for (int h = tid * 4; h < H; h += 256 * 4) {
        const float w0 = ldf(w + h), w1 = ldf(w + h + 1), w2 = ldf(w + h + 2), w3 = ldf(w + h + 3);
#pragma unroll
        for (int t = 0; t < kRTok; ++t) {
          if (t < nt) {
            const uint2 xv = *reinterpret_cast<const uint2*>(x + (int64_t)(t0 + t) * H + h);
            float a = acc[t];
            a = fmaf(bf16lo(xv.x), w0, a);
            a = fmaf(bf16hi(xv.x), w1, a);
            a = fmaf(bf16lo(xv.y), w2, a);
            a = fmaf(bf16hi(xv.y), w3, a);
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
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&meta->ticket, 1u) == gridDim.x * gridDim.y - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (W) {
    for (int t = warp; t < T; t += 8)
      warp_topk([&](int e2) { return __ldcg(logits + (int64_t)t * E + e2); }, E, k,
                scores + (int64_t)t * k, idx + (int64_t)t * k);
    __threadfence();
    __syncthreads();
  }
  // dispatch: rows grouped by expert, (token, slot) order within an expert
  const int n = T * k;
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const int e = __ldcg(idx + i);
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    else record_status(status, BS_ERR_INVALID_ARGUMENT);
  }
  __syncthreads();
  if (tid == 0) {
    // groups: (expert | tokens << 16, first row), up to kGroupTok tokens each
    int run = 0, ng = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = run;
      offsets[e] = run;
      for (int c = 0; c < cnt[e]; c += kGroupTok) groups[ng++] = make_int2(e | (min(kGroupTok, cnt[e] - c) << 16), run + c);
      run += cnt[e];
    }
    off[E] = run;
    offsets[E] = run;
    meta->n_groups = ng;
  }
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const int e = __ldcg(idx + i);
    if (e < 0 || e >= E) {
      row_of_slot[i] = -1;
      continue;
    }
    int r = 0;
    for (int j = 0; j < i; ++j) r += (__ldcg(idx + j) == e);
    const int pos = off[e] + r;
    row_of_slot[i] = pos;
    slot_of_row[pos] = i;
  }
}

// ------------------------------------------------------------------ 2/3. experts
struct MxArgs {
  CUtensorMap tm_a;       // weight codes [E*Nw rows][K/2 bytes], box {128 B, 128 rows}, 128B swizzle
  CUtensorMap tm_b;       // B term rows [rows][K/2 bytes], box {128 B, tokbox rows}, 128B swizzle
  const uint8_t* scales;  // [E][Nw][K/32] e8m0
  const void* bias;       // [E][Nw]
  int bias_f32;
  const uint8_t* bsf;     // B scales: rows (4 r + term) of gp bytes
  int gp;
  const int2* groups;     // (expert | tokens << 16, first row) per group
  const int* slot_of_row;
  const DecodeMeta* meta;
  const float* scores;
  int E, Nw, K, k;
  int nb;                 // B rows a stage holds (multiple of 16, >= 4 x tokens of any expert)
  int stages, nsc, nacc;  // pipeline stages, per-item scale buffers, accumulator buffers
  float alpha, limit;
  uint8_t* hq;            // MODE 0 out: rows (4 r + term) of Nw/4 bytes (codes of h, Nw/2 values)
  uint8_t* hs;            //             rows (4 r + term) of gp_out bytes
  int gp_out;
  float* y;               // MODE 1 out: [rows][Nw] fp32
  int* status;
};

// MODE 0: B rows are gathered per token (4 term rows each, one TMA box per
// token); MODE 1: the expert's rows are contiguous (one box of nb rows).
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) decode_mx_kernel(const __grid_constant__ MxArgs p) {
  extern __shared__ uint8_t smem_raw[];
  // data[s]: the stage's copies landed (TMA transaction count); empty[s]: the
  // MMAs are done with it; scfull[b]: an item's scale rows landed in staging
  // buffer b (one barrier per buffer, so a waiter is never two phases ahead);
  // sfready[b]: its repacked scales are ready; accfull[b] / accempty[b]:
  // accumulator handoff; drain: teardown
  __shared__ uint64_t bars[3 * kMaxStages + 7];
  __shared__ uint32_t tmem_holder;
  __shared__ volatile int abort_flag;
  __shared__ float red[2][4][4];
  __shared__ int2 s_grp[kMaxGroups];  // (expert | tokens << 16, first row)
  __shared__ int s_ngrp;
  uint8_t* smem = smem_raw + ((1024u - (ptx::smem_addr(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = p.stages;
  const int K = p.K, G = K / 32, Nw = p.Nw;
  const int a_bytes = kBM * 128, stage_bytes = a_bytes + p.nb * 128;
  // per-item scale blocks (ring of p.nsc): A rows [128][G], B rows [nb][gp];
  // then two buffers of repacked scales: per group q of four k-blocks, a
  // 512-byte block for A and one for B (row r -> word (r % 32, r / 32))
  const int sa_bytes = (kBM * G + 15) & ~15, sc_bytes = sa_bytes + p.nb * p.gp;
  const int G4 = (G + 3) / 4;
  const int sf_src_bytes = G4 * 1024;
  uint8_t* scbuf = smem + S * stage_bytes;
  uint8_t* sfsrc = scbuf + p.nsc * sc_bytes;
  auto data = [&](int s) { return ptx::smem_addr(bars + s); };
  auto empty = [&](int s) { return ptx::smem_addr(bars + kMaxStages + s); };
  auto accfull = [&](int b) { return ptx::smem_addr(bars + 2 * kMaxStages + b); };
  auto accempty = [&](int b) { return ptx::smem_addr(bars + 2 * kMaxStages + 2 + b); };
  auto sfready = [&](int b) { return ptx::smem_addr(bars + 2 * kMaxStages + 4 + b); };
  const uint32_t drain = ptx::smem_addr(bars + 2 * kMaxStages + 6);
  auto scfull = [&](int b) { return ptx::smem_addr(bars + 2 * kMaxStages + 7 + b); };
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(data(s), 1);
      ptx::mbar_init(empty(s), 1);
    }
    for (int b = 0; b < p.nsc; ++b) ptx::mbar_init(scfull(b), 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(accfull(b), 1);
      ptx::mbar_init(accempty(b), 4);
      ptx::mbar_init(sfready(b), 1);
    }
    ptx::mbar_init(drain, 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 5) {
    ptx::tmem_alloc(ptx::smem_addr(&tmem_holder), kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    ptx::tma_prefetch_desc(&p.tm_a);
    ptx::tma_prefetch_desc(&p.tm_b);
  }
  pdl_wait();  // routing and the B operands come from the previous kernels
  pdl_launch();
  if (tid == 0) s_ngrp = p.meta->n_groups;
  __syncthreads();
  for (int i = tid; i < s_ngrp; i += kThreads) s_grp[i] = p.groups[i];
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = tmem_holder;

  const int per_e = (Nw + kBM - 1) / kBM;
  const int n_items = s_ngrp * per_e;
  const int nkc = (K + kKC - 1) / kKC;
  const int n_my = n_items > (int)blockIdx.x ? (n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t smem0 = ptx::smem_addr(smem);
  const uint32_t sf_base = (uint32_t)(p.nacc * p.nb);  // TMEM column of stage 0's scale factors
  auto item_of = [&](int it) { return (int)blockIdx.x + it * (int)gridDim.x; };

  if (warp == 4) {
    // ---------------------------------------------------------- TMA producer (one thread)
    if (lane == 0) {
      int g = 0, n_issued = 0;
      for (int it = 0; it < n_my; ++it) {
        const int item = item_of(it);
        const int2 gr = s_grp[item / per_e];
        const int e = gr.x & 0xFFFF, ntok = gr.x >> 16, row_lo = gr.y, r0 = (item % per_e) * kBM;
        const int nrows = min(kBM, Nw - r0);
        const uint32_t sca = ptx::smem_addr(scbuf + (it % p.nsc) * sc_bytes);
        bool ok = true;
        for (int kc = 0; kc < nkc; ++kc, ++g) {
          const int s = g % S;
          if (g >= S && !ptx::mbar_wait(empty(s), ((g / S) - 1) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem0 + s * stage_bytes, sb = sa + a_bytes;
          if (kc == 0) {
            // the item's scale rows: A contiguous [rows][G], B [4 x tokens][gp]
            const uint32_t scb = scfull(it % p.nsc);
            ptx::mbar_arrive_expect_tx(scb, (uint32_t)(nrows * G + ntok * kTerms * p.gp));
            ptx::bulk_load(sca, p.scales + ((int64_t)e * Nw + r0) * G, (uint32_t)(nrows * G), scb);
            if (MODE == 0) {
              for (int j = 0; j < ntok; ++j) {
                const int t = p.slot_of_row[row_lo + j] / p.k;
                ptx::bulk_load(sca + sa_bytes + j * kTerms * p.gp, p.bsf + (int64_t)t * kTerms * p.gp,
                               (uint32_t)(kTerms * p.gp), scb);
              }
            } else {
              ptx::bulk_load(sca + sa_bytes, p.bsf + (int64_t)row_lo * kTerms * p.gp,
                             (uint32_t)(ntok * kTerms * p.gp), scb);
            }
            ++n_issued;
          }
          ptx::mbar_arrive_expect_tx(data(s), a_bytes + (MODE == 0 ? ntok * kTerms * 128 : p.nb * 128));
          ptx::tma_load_2d(sa, &p.tm_a, data(s), kc * 128, e * Nw + r0);
          if (MODE == 0) {
            for (int j = 0; j < ntok; ++j)
              ptx::tma_load_2d(sb + j * kTerms * 128, &p.tm_b, data(s), kc * 128,
                               (p.slot_of_row[row_lo + j] / p.k) * kTerms);
          } else {
            ptx::tma_load_2d(sb, &p.tm_b, data(s), kc * 128, row_lo * kTerms);
          }
        }
        if (!ok) break;
      }
      if (abort_flag) {
        // after a timeout elsewhere: let this CTA's copies in flight land
        // (bounded) before it exits
        volatile int quiet = 0;
        for (int gg = max(0, g - S); gg < g; ++gg)
          ptx::mbar_wait(data(gg % S), (gg / S) & 1, &quiet, 100000000LL);
        for (int it2 = max(0, n_issued - p.nsc); it2 < n_issued; ++it2)
          ptx::mbar_wait(scfull(it2 % p.nsc), (it2 / p.nsc) & 1, &quiet, 100000000LL);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issue (one thread)
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int it = 0; it < n_my && ok; ++it) {
        const int item = item_of(it);
        const int ntok = s_grp[item / per_e].x >> 16;
        const int N = ((kTerms * ntok + 15) / 16) * 16;
        const int ab = it % p.nacc;
        if (!ptx::mbar_wait(sfready(it & 1), (it >> 1) & 1, &abort_flag)) break;
        if (it >= p.nacc) {
          if (!ptx::mbar_wait(accempty(ab), ((it / p.nacc) - 1) & 1, &abort_flag)) break;
        }
        ptx::tc_fence_after();
        const uint32_t acc = tmem + ab * p.nb;
        const uint32_t src = ptx::smem_addr(sfsrc + (it & 1) * sf_src_bytes);
        for (int kc = 0; kc < nkc; ++kc, ++g) {
          const int s = g % S;
          if (!ptx::mbar_wait(data(s), (g / S) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sa = smem0 + s * stage_bytes;
          const uint64_t ad = ptx::sdesc_kmajor_sw128(sa), bd = ptx::sdesc_kmajor_sw128(sa + a_bytes);
          const uint32_t sf = tmem + sf_base + s * kSfStageCols;
          // the stage's scale factors: groups 2 kc, 2 kc + 1 of four k-blocks;
          // SFA at columns 4q, SFB at 8 + 4q
          for (int q = 0; q < 2 && 4 * (2 * kc + q) < G; ++q) {
            const int gq = 2 * kc + q;
            ptx::tc_cp_32x128b_warpx4(sf + 4 * q, ptx::sdesc_rows16(src + gq * 512));
            ptx::tc_cp_32x128b_warpx4(sf + 8 + 4 * q, ptx::sdesc_rows16(src + (G4 + gq) * 512));
          }
          for (int i = 0; i < 4 && kc * kKC + i * 64 < K; ++i) {
            const uint32_t id = 2 * (i & 1);
            ptx::mma_mxf4_ss(acc, ad + 2 * i, bd + 2 * i, ptx::idesc_mxf4(N, id, id), sf + 4 * (i >> 1),
                             sf + 8 + 4 * (i >> 1), (kc | i) != 0);
          }
          ptx::tc_commit(empty(s));
        }
        if (ok) ptx::tc_commit(accfull(ab));
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- scale factors + epilogue
    const uint32_t lanes = (uint32_t)(32 * warp) << 16;
    bool ok = true;
    // repack item `it`'s scales (landed with its first stage) into the blocks
    // tcgen05.cp reads; the MMA thread copies them into TMEM stage by stage
    auto repack = [&](int it) {
      const int item = item_of(it);
      const int2 gr = s_grp[item / per_e];
      const int r0 = (item % per_e) * kBM;
      const int nrows = min(kBM, Nw - r0);
      const int nbv = kTerms * (gr.x >> 16);
      bool w = true;
      if (lane == 0) w = ptx::mbar_wait(scfull(it % p.nsc), (it / p.nsc) & 1, &abort_flag);
      if (!named_and(2, 128, __shfl_sync(0xffffffffu, w, 0))) {
        ok = false;
        return;
      }
      const uint8_t* sca = scbuf + (it % p.nsc) * sc_bytes;
      const uint8_t* scb = sca + sa_bytes;
      uint8_t* dst = sfsrc + (it & 1) * sf_src_bytes;
      {
        // A: thread r = row; rows are 2-byte aligned runs of G bytes
        const int r = tid;
        const uint16_t* row = reinterpret_cast<const uint16_t*>(sca + r * G);
        for (int q = 0; q < G4; ++q) {
          uint32_t v = 0;
          if (r < nrows) v = row[2 * q] | ((4 * q + 2 < G) ? (uint32_t)row[2 * q + 1] << 16 : 0u);
          *reinterpret_cast<uint32_t*>(dst + q * 512 + (r & 31) * 16 + (r >> 5) * 4) = v;
        }
      }
      // B: rows n < nbv (pitch gp, 16-byte aligned words)
      for (int idx = tid; idx < nbv * G4; idx += 128) {
        const int n = idx / G4, q = idx - n * G4;
        const uint32_t v = *reinterpret_cast<const uint32_t*>(scb + n * p.gp + 4 * q);
        *reinterpret_cast<uint32_t*>(dst + (G4 + q) * 512 + (n & 31) * 16 + (n >> 5) * 4) = v;
      }
      ptx::fence_proxy_async_smem();
      named_sync(2, 128);
      if (tid == 0) ptx::mbar_arrive(sfready(it & 1));
    };
    auto epilogue = [&](int it) {
      const int item = item_of(it);
      const int2 gr = s_grp[item / per_e];
      const int e = gr.x & 0xFFFF, ntok = gr.x >> 16, row_lo = gr.y, r0 = (item % per_e) * kBM;
      const int nrows = min(kBM, Nw - r0);
      const int N = ((kTerms * ntok + 15) / 16) * 16;
      const int ab = it % p.nacc;
      const int lrow = 32 * warp + lane;
      const bool rv = lrow < nrows;
      const int64_t grow = (int64_t)e * Nw + r0 + lrow;
      float bv = 0.f;
      if (rv && p.bias)
        bv = p.bias_f32 ? static_cast<const float*>(p.bias)[grow]
                        : __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[grow]);
      float wt0 = 0.f, wt1 = 0.f;  // MODE 1: routing weights of tokens lane, lane + 32
      if (MODE == 1) {
        if (lane < ntok) wt0 = p.scores[p.slot_of_row[row_lo + lane]];
        if (lane + 32 < ntok) wt1 = p.scores[p.slot_of_row[row_lo + lane + 32]];
      }
      bool got = ok;
      if (got) got = ptx::mbar_wait(accfull(ab), (it / p.nacc) & 1, &abort_flag);
      if (!named_and(1, 128, got)) {
        ok = false;
        return;
      }
      ptx::tc_fence_after();
      const uint32_t tl = tmem + lanes + ab * p.nb;
      for (int c = 0; c < N / 16; ++c) {
        float v[16];
        {
          uint32_t u[16];
          ptx::tmem_ld_32x32b_x16(tl + c * 16, u);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(u[j]);
        }
        if (c == N / 16 - 1) {
          // accumulator drained: the MMAs of a later item may use it
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(accempty(ab));
        }
        float acc[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[jj] = v[4 * jj] + v[4 * jj + 1] + v[4 * jj + 2] + v[4 * jj + 3] + bv;
        if (MODE == 1) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int tok = c * 4 + jj;
            const float wt = __shfl_sync(0xffffffffu, tok < 32 ? wt0 : wt1, tok & 31);
            if (tok < ntok && rv) p.y[(int64_t)(row_lo + tok) * Nw + r0 + lrow] = acc[jj] * wt;
          }
        } else {
          // rows alternate gate / up: h_i (i = row / 2) sits in lanes 2m, 2m+1;
          // a 32-block of h is 64 rows = warps (0,1) or (2,3); the byte of
          // codes (h_i, h_i+1), i even, is written by lane 4m'
          float r[4];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float other = __shfl_xor_sync(0xffffffffu, acc[jj], 1);
            const float gate = (lane & 1) ? other : acc[jj], up = (lane & 1) ? acc[jj] : other;
            r[jj] = swiglu(gate, up, p.alpha, p.limit);
          }
          const int i = (r0 + lrow) >> 1, I = Nw >> 1;
#pragma unroll
          for (int term = 0; term < kTerms; ++term) {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const float m = group_max<32>(fabsf(r[jj]));
              if (lane == 0) red[term & 1][warp][jj] = m;
            }
            named_sync(1, 128);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const int tok = c * 4 + jj;
              const uint32_t sb = e8m0_for_max(fmaxf(red[term & 1][warp][jj], red[term & 1][warp ^ 1][jj]));
              const float q = r[jj] * exp2_neg(sb);
              const float qn = __shfl_down_sync(0xffffffffu, q, 2);  // h_{i+1}
              const uint32_t byte = ptx::e2m1x2_from_f32(q, qn);
              r[jj] -= ptx::e2m1_lo_to_f32(byte) * exp2_pos(sb);
              if (tok < ntok && rv) {
                const int64_t hr = (int64_t)(row_lo + tok) * kTerms + term;
                if ((lane & 3) == 0) p.hq[hr * (I / 2) + (i >> 1)] = (uint8_t)byte;
                if (lane == 0 && !(warp & 1)) p.hs[hr * p.gp_out + (i >> 5)] = (uint8_t)sb;
              }
            }
          }
        }
      }
    };
    // The epilogue of item it-1 runs after the repack of item it when two
    // accumulators alternate (the MMAs of item it overlap it); with one,
    // item it's MMAs need that epilogue first.
    for (int it = 0; it < n_my && ok; ++it) {
      if (p.nacc == 1 && it > 0) epilogue(it - 1);
      if (!ok) break;
      repack(it);
      if (p.nacc == 2 && it > 0 && ok) epilogue(it - 1);
    }
    if (ok && n_my > 0) epilogue(n_my - 1);
  }
  __syncthreads();
  if (warp == 5) {
    if (lane == 0 && abort_flag) {
      // MMAs and copies may still be in flight after a timeout: let the MMAs
      // finish (bounded) before the tensor memory is released.
      record_status(p.status, BS_ERR_TIMEOUT);
      ptx::tc_commit(drain);
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
    out[i] = make_uint2(pack_bf16x2(a0, a1), pack_bf16x2(a2, a3));
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

// Pipeline shape of one expert projection: stages, scale buffers and
// accumulator buffers that fit in shared and tensor memory.
int plan_mx(MxArgs& a) {
  const int64_t K = a.K, G = K / 32, nkc = cdiv(K, (int64_t)kKC);
  const size_t stage = (size_t)(kBM + a.nb) * 128;
  const size_t sc = align_up((size_t)kBM * G, 16) + (size_t)a.nb * a.gp;
  const size_t a4 = 2 * (size_t)cdiv(G, (int64_t)4) * 1024;  // repacked scales
  const size_t budget = 200 * 1024;  // dynamic shared memory (the static arrays take ~9 KB)
  a.stages = 0;
  for (int S = kMaxStages; S >= 2; --S) {
    const int nsc = (int)std::max<int64_t>(2, cdiv((int64_t)S - 1, nkc) + 1);
    if (S * stage + nsc * sc + a4 + 1024 <= budget) {
      a.stages = S;
      a.nsc = nsc;
      break;
    }
  }
  BS_REQUIRE(a.stages >= 2, BS_ERR_UNSUPPORTED, "decode path: B tile of %d rows does not fit", a.nb);
  a.nacc = (2 * a.nb + a.stages * kSfStageCols <= kTmemCols) ? 2 : 1;
  BS_REQUIRE(a.nacc * a.nb + a.stages * kSfStageCols <= kTmemCols, BS_ERR_UNSUPPORTED,
             "decode path: tensor memory plan does not fit");
  return BS_OK;
}

size_t mx_smem_bytes(const MxArgs& a) {
  const int64_t G = a.K / 32;
  const size_t stage = (size_t)(kBM + a.nb) * 128;
  const size_t sc = align_up((size_t)kBM * G, 16) + (size_t)a.nb * a.gp;
  const size_t a4 = 2 * (size_t)cdiv(G, (int64_t)4) * 1024;
  return a.stages * stage + a.nsc * sc + a4 + 1024;
}

template <int MODE>
int launch_mx(const MxArgs& a, cudaStream_t st) {
  const size_t smem = mx_smem_bytes(a);
  BS_CUDA(cudaFuncSetAttribute(decode_mx_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return launch_pdl(decode_mx_kernel<MODE>, dim3((unsigned)sm_count()), dim3(kThreads), smem, st, a);
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
  w.total = o;
  return w;
}

size_t decode_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  return decode_carve(nullptr, T, H, I, E, k).total;
}

bool decode_supported(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  return T >= 1 && T <= kMaxDecodeT && E <= 1024 && k <= 32 && H % 64 == 0 && I % 64 == 0 &&
         (2 * I) % kBM == 0;
}

// The four-launch decode forward.  router_weight NULL: scores/indices are inputs.
int decode_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                   const void* rw, const void* rb, int rdt, float* scores, int32_t* indices,
                   const void* gu_b, const void* gu_s, const void* gu_bias, const void* dn_b,
                   const void* dn_s, const void* dn_bias, int bias_f32, float alpha, float limit,
                   void* out, void* ws, cudaStream_t st) {
  BS_ARG(decode_supported(T, H, I, E, k),
         "decode path: need 1 <= T <= %d, E <= 1024, k <= 32, H and I multiples of 64", kMaxDecodeT);
  BS_REQUIRE(((uintptr_t)gu_b | (uintptr_t)dn_b | (uintptr_t)gu_s | (uintptr_t)dn_s) % 16 == 0,
             BS_ERR_MISALIGNED, "decode path: expert blocks and scales must be 16-byte aligned");
  const DecodeWS w = decode_carve(ws, T, H, I, E, k);
  int* status = device_status_ptr();
  BS_CUDA(cudaMemsetAsync(w.meta, 0, sizeof(DecodeMeta), st));
  const int64_t G = H / 32;
  const dim3 rgrid((unsigned)std::max<int64_t>(rw ? E : 1, std::min<int64_t>(G, 128)),
                   (unsigned)cdiv(T, (int64_t)kRTok));
  if (!rw || rdt == BS_F32) {
    BS_TRY(launch_pdl(decode_route_kernel<float>, rgrid, dim3(256), 0, st,
                      static_cast<const __nv_bfloat16*>(x), static_cast<const float*>(rw),
                      static_cast<const float*>(rb), (int)T, (int)H, (int)E, (int)k, 0, w.logits,
                      scores, indices, w.offsets, w.row_of_slot, w.slot_of_row, w.groups, w.xq, w.xs,
                      gp_of(H), w.meta, status));
  } else {
    BS_TRY(launch_pdl(decode_route_kernel<__nv_bfloat16>, rgrid, dim3(256), 0, st,
                      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(rw),
                      static_cast<const __nv_bfloat16*>(rb), (int)T, (int)H, (int)E, (int)k, 1,
                      w.logits, scores, indices, w.offsets, w.row_of_slot, w.slot_of_row, w.groups,
                      w.xq, w.xs, gp_of(H), w.meta, status));
  }
  const int nb = (int)((std::min<int64_t>(kTerms * T, kTerms * kGroupTok) + 15) / 16 * 16);
  MxArgs a{};
  a.groups = w.groups;
  a.slot_of_row = w.slot_of_row;
  a.meta = w.meta;
  a.scores = scores;
  a.E = (int)E;
  a.k = (int)k;
  a.nb = nb;
  a.alpha = alpha;
  a.limit = limit;
  a.bias_f32 = bias_f32;
  a.status = status;
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  // gate_up: A = [E][2I][H/32][16], B = x terms (4 rows per token), out = h terms
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
  BS_TRY(make_map_2d(&a.tm_b, u8, w.xq, (uint64_t)(H / 2), (uint64_t)(T * kTerms), (uint64_t)(H / 2), 128,
                     kTerms, sw));
  BS_TRY(plan_mx(a));
  BS_TRY(launch_mx<0>(a, st));
  // down: A = [E][H][I/32][16], B = h terms (contiguous per expert), out = weighted fp32 rows
  a.scales = static_cast<const uint8_t*>(dn_s);
  a.bias = dn_bias;
  a.bsf = w.hs;
  a.gp = gp_of(I);
  a.Nw = (int)H;
  a.K = (int)I;
  a.y = w.y;
  BS_TRY(make_map_2d(&a.tm_a, u8, dn_b, (uint64_t)(I / 2), (uint64_t)(E * H), (uint64_t)(I / 2), 128, kBM, sw));
  BS_TRY(make_map_2d(&a.tm_b, u8, w.hq, (uint64_t)(I / 2), (uint64_t)(T * k * kTerms), (uint64_t)(I / 2), 128,
                     (uint32_t)nb, sw));
  BS_TRY(plan_mx(a));
  BS_TRY(launch_mx<1>(a, st));
  const int vecs = (int)(H / 4);
  const int cgrid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(T * vecs, (int64_t)256), sm_count() * 4));
  BS_TRY(launch_pdl(decode_combine_kernel, dim3(cgrid), dim3(256), 0, st, (const float4*)w.y,
                    (const int*)w.row_of_slot, (int)T, (int)k, vecs, static_cast<uint2*>(out)));
  return BS_OK;
}

}  // namespace bs
