// Shared host/device helpers of the B200 gpt-oss MoE library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "bs_moe.h"

namespace bs {

// ---------------------------------------------------------------- host side
void set_error(const char* fmt, ...);
const char* last_error();
// Device address of the per-device status word (see bs_device_status).
int* device_status_ptr();
int sm_count();
int check_device();  // BS_OK on sm_100, else BS_ERR_UNSUPPORTED (message set)

#define BS_REQUIRE(cond, code, ...)   \
  do {                                \
    if (!(cond)) {                    \
      ::bs::set_error(__VA_ARGS__);   \
      return (code);                  \
    }                                 \
  } while (0)

#define BS_ARG(cond, ...) BS_REQUIRE(cond, BS_ERR_INVALID_ARGUMENT, __VA_ARGS__)
#define BS_ALIGNED16(p, name) \
  BS_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15) == 0, BS_ERR_MISALIGNED, "%s must be 16-byte aligned", name)

#define BS_CUDA(expr)                                                                   \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess) {                                                            \
      ::bs::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                      __LINE__);                                                        \
      return BS_ERR_CUDA;                                                               \
    }                                                                                   \
  } while (0)

#define BS_LAUNCHED()                                                                       \
  do {                                                                                      \
    cudaError_t e_ = cudaGetLastError();                                                    \
    if (e_ != cudaSuccess) {                                                                \
      ::bs::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(e_), __FILE__, \
                      __LINE__);                                                            \
      return BS_ERR_CUDA;                                                                   \
    }                                                                                       \
  } while (0)

#define BS_TRY(expr)          \
  do {                        \
    int s_ = (expr);          \
    if (s_ != BS_OK) return s_; \
  } while (0)

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
inline size_t align_up(size_t a, size_t b) { return (a + b - 1) / b * b; }

// ---------------------------------------------------------------- device side

// bf16 bits of FP4_VALUES[code] * 2^(scale-127): exact product, +-inf when the
// magnitude reaches 2^128, bf16 subnormals kept.  (transformers
// integrations/mxfp4.py:29-46 table, 305-322 LUT + ldexp.)  General for every
// byte; the GEMM/GEMV paths use the faster form below when 2 <= scale <= 252.
__host__ __device__ __forceinline__ uint16_t e2m1_to_bf16_bits(uint32_t code, uint32_t scale) {
  const uint32_t sign = (code & 8u) << 12;
  const uint32_t m = code & 7u;
  if (m == 0) return (uint16_t)sign;
  // value = (1 + mant/2) * 2^E,  E = (scale-127) + eo(m)
  const int eo = (m == 1) ? -1 : (int)(m >> 1) - 1;
  const uint32_t mant = (m >= 2) ? (m & 1u) : 0u;
  const int E = (int)scale - 127 + eo;
  if (E >= 128) return (uint16_t)(sign | 0x7F80u);
  if (E >= -126) return (uint16_t)(sign | ((uint32_t)(E + 127) << 7) | (mant << 6));
  // subnormal: (2 + mant) * 2^(E-1) = frac * 2^-133  -> frac = (2+mant) << (E + 132)
  return (uint16_t)(sign | ((2u + mant) << (E + 132)));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// Fast path: eight e2m1 codes (one 32-bit word, low nibble first) under one scale
// in [2, 252] -> four bf16x2 words.  Magnitude bits are ((s-1)<<7) + (m>=2 ? m<<6 : 0)
// (m=0 -> 0), which equals the exact product whenever it stays a normal bf16,
// i.e. for 2 <= s <= 252.  Byte tables are built per scale and indexed with prmt.
struct E2M1Pool {
  uint32_t lo_a, lo_b, hi_a, hi_b;
};

// prmt.b32 (default mode): byte i of the result is byte (sel nibble i & 7) of
// the pool {b:a}; a set bit 3 replicates that byte's sign bit.  The host form
// lets the decode below be checked on the CPU.
__host__ __device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
#ifdef __CUDA_ARCH__
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
#else
  const uint64_t pool = ((uint64_t)b << 32) | a;
  uint32_t r = 0;
  for (int i = 0; i < 4; ++i) {
    const uint32_t s = (sel >> (4 * i)) & 0xFu;
    uint32_t byte = (uint32_t)(pool >> ((s & 7u) * 8)) & 0xFFu;
    if (s & 8u) byte = (byte & 0x80u) ? 0xFFu : 0u;
    r |= byte << (8 * i);
  }
  return r;
#endif
}

__host__ __device__ __forceinline__ E2M1Pool make_e2m1_pool(uint32_t scale) {
  const uint32_t base = (scale - 1u) << 7;
  const uint32_t B = base * 0x10001u;
  const uint32_t p01 = base << 16;        // m=0 -> 0, m=1 -> base
  const uint32_t p23 = B + 0x00C00080u;   // m=2 -> base+128, m=3 -> base+192
  const uint32_t p45 = B + 0x01400100u;   // m=4,5
  const uint32_t p67 = B + 0x01C00180u;   // m=6,7
  E2M1Pool p;
  p.lo_a = prmt(p01, p23, 0x6420u);
  p.lo_b = prmt(p45, p67, 0x6420u);
  p.hi_a = prmt(p01, p23, 0x7531u);
  p.hi_b = prmt(p45, p67, 0x7531u);
  return p;
}

// w: 8 codes (bytes b0..b3, each low nibble = even element).  out[0] = (e0,e1), ...
__host__ __device__ __forceinline__ void e2m1x8_to_bf16x8(uint32_t w, const E2M1Pool& p, uint32_t out[4]) {
  const uint32_t mags = w & 0x77777777u;
  const uint32_t sel_a = mags & 0xFFFFu;   // e0..e3
  const uint32_t sel_b = mags >> 16;       // e4..e7
  const uint32_t loA = prmt(p.lo_a, p.lo_b, sel_a);
  const uint32_t hiA = prmt(p.hi_a, p.hi_b, sel_a);
  const uint32_t loB = prmt(p.lo_a, p.lo_b, sel_b);
  const uint32_t hiB = prmt(p.hi_a, p.hi_b, sel_b);
  out[0] = prmt(loA, hiA, 0x5140u);
  out[1] = prmt(loA, hiA, 0x7362u);
  out[2] = prmt(loB, hiB, 0x5140u);
  out[3] = prmt(loB, hiB, 0x7362u);
  // signs: element 2i's sign is w bit (8i+3) -> bit 15; element 2i+1's is bit (8i+7) -> bit 31
  const uint32_t w4 = w << 4;
  out[0] |= prmt(w4, w, 0x4000u) & 0x80008000u;
  out[1] |= prmt(w4, w, 0x5010u) & 0x80008000u;
  out[2] |= prmt(w4, w, 0x6020u) & 0x80008000u;
  out[3] |= prmt(w4, w, 0x7030u) & 0x80008000u;
}

// Same result for any scale (slow general path).
__host__ __device__ __forceinline__ void e2m1x8_to_bf16x8_any(uint32_t w, uint32_t scale, uint32_t out[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t byte = (w >> (8 * i)) & 0xFFu;
    out[i] = (uint32_t)e2m1_to_bf16_bits(byte & 15u, scale) |
             ((uint32_t)e2m1_to_bf16_bits(byte >> 4, scale) << 16);
  }
}

__host__ __device__ __forceinline__ void e2m1x8_decode(uint32_t w, uint32_t scale, const E2M1Pool& p,
                                              uint32_t out[4]) {
  if (scale - 2u <= 250u) {
    e2m1x8_to_bf16x8(w, p, out);
  } else {
    e2m1x8_to_bf16x8_any(w, scale, out);
  }
}

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// bf16(residual + bf16(v)) for two packed values: the decoder layer's
// `residual + mlp(...)` (modeling_gpt_oss.py, GptOssDecoderLayer.forward), where
// the MLP output is itself a bf16 tensor.
__device__ __forceinline__ uint32_t add_residual_bf16x2(uint32_t res, float v_lo, float v_hi) {
  const float lo = __bfloat162float(__float2bfloat16_rn(v_lo)) + bf16lo(res);
  const float hi = __bfloat162float(__float2bfloat16_rn(v_hi)) + bf16hi(res);
  return pack_bf16x2(lo, hi);
}

// SwiGLU of the reference (block_streamer/gptoss.py:130-135) in fp32.
__device__ __forceinline__ float swiglu(float gate, float up, float alpha, float limit) {
  gate = fminf(gate, limit);
  up = fminf(fmaxf(up, -limit), limit);
  const float glu = gate / (1.0f + expf(-alpha * gate));
  return (up + 1.0f) * glu;
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace bs
