// Host-side check of the library's e2m1 -> bf16 decode (bs_common.cuh), built
// and run by tests/test_host_logic.py.  Prints the bf16 bits of every (scale,
// byte) pair through the general decode, then the number of words where the
// fast prmt decode disagrees with it.
#include <stdio.h>
#include <stdint.h>

#include "bs_common.cuh"

int main() {
  // 1) table [scale][byte] -> (lo bits, hi bits) through the general path
  for (uint32_t s = 0; s < 256; ++s)
    for (uint32_t b = 0; b < 256; ++b)
      printf("%04x %04x\n", bs::e2m1_to_bf16_bits(b & 15u, s), bs::e2m1_to_bf16_bits(b >> 4, s));
  // 2) fast vs general over every byte in every position, all scales, random fill
  uint64_t rng = 0x9E3779B97F4A7C15ull;
  long mismatches = 0, checked = 0;
  for (uint32_t s = 0; s < 256; ++s) {
    const bs::E2M1Pool pool = bs::make_e2m1_pool(s);
    for (uint32_t b = 0; b < 256; ++b)
      for (int pos = 0; pos < 4; ++pos)
        for (int rep = 0; rep < 4; ++rep) {
          rng ^= rng << 13; rng ^= rng >> 7; rng ^= rng << 17;
          uint32_t w = (uint32_t)rng;
          w = (w & ~(0xFFu << (8 * pos))) | (b << (8 * pos));
          uint32_t f[4], g[4], d[4];
          bs::e2m1x8_to_bf16x8_any(w, s, g);
          bs::e2m1x8_decode(w, s, pool, d);
          if (s >= 2 && s <= 252) bs::e2m1x8_to_bf16x8(w, pool, f);
          for (int i = 0; i < 4; ++i) {
            if (d[i] != g[i]) ++mismatches;
            if (s >= 2 && s <= 252 && f[i] != g[i]) ++mismatches;
          }
          ++checked;
        }
  }
  printf("MISMATCHES %ld CHECKED %ld\n", mismatches, checked);
  return mismatches ? 1 : 0;
}
