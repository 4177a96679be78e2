// Host check of the kernels' multiply-shift division (spkv2::FastDiv, the
// host branch of the same arithmetic the device runs with __umulhi): for
// every divisor below 4097, the pixel / tile / unit counts of the named
// networks, powers of two and their neighbours, and seeded random divisors,
// FastDiv(d).div(n) must equal n / d for edge numerators (0, multiples of d
// and their neighbours, 2^31 - 1, 2^32 - 1) and seeded random ones.
// Prints "ok <checks>" and exits 0, or prints the first mismatch and exits 1.
#include <stdint.h>
#include <stdio.h>

#include <vector>

#include "common.cuh"

namespace {

uint64_t g_state = 0x9E3779B97F4A7C15ull;

uint32_t next_u32() {
  g_state ^= g_state << 13;
  g_state ^= g_state >> 7;
  g_state ^= g_state << 17;
  return uint32_t(g_state >> 16);
}

bool check(uint32_t d, uint32_t n, uint64_t *checks) {
  const spkv2::FastDiv f(d);
  ++*checks;
  if (f.div(n) != n / d) {
    printf("mismatch: d=%u n=%u got %u want %u\n", d, n, f.div(n), n / d);
    return false;
  }
  return true;
}

}  // namespace

int main() {
  std::vector<uint32_t> divs;
  for (uint32_t d = 1; d <= 4096; ++d) divs.push_back(d);
  // Output pixels per image and per batch (ResNet 112^2..7^2, the detector's
  // 320^2..20^2 at batches 1..256), K-step and tile counts.
  const uint32_t named[] = {3136, 12544, 50176, 200704, 802816, 3211264, 25088, 6272, 784, 196, 49,
                            102400, 409600, 1600, 6400, 25600, 8400, 1179648, 2359296, 72, 144, 288};
  for (uint32_t d : named) divs.push_back(d);
  for (int b = 12; b < 32; ++b) {
    const uint32_t p = 1u << b;
    divs.push_back(p - 1);
    divs.push_back(p);
    divs.push_back(p + 1);
  }
  divs.push_back(0x7FFFFFFFu);
  for (int i = 0; i < 2000; ++i) divs.push_back(1 + (next_u32() & 0x7FFFFFFEu));

  uint64_t checks = 0;
  for (uint32_t d : divs) {
    const uint32_t edges[] = {0u, 1u, d - 1, d, d + 1, 2 * d - 1, 2 * d, 0x7FFFFFFFu, 0x80000000u, 0xFFFFFFFFu};
    for (uint32_t n : edges)
      if (!check(d, n, &checks)) return 1;
    // Multiples of d and their neighbours up to 2^32.
    for (uint64_t k = 1; k * d <= 0xFFFFFFFFull; k = k * 3 + 1) {
      const uint32_t q = uint32_t(k * d);
      if (!check(d, q - 1, &checks) || !check(d, q, &checks) || !check(d, q + 1, &checks)) return 1;
    }
    for (int i = 0; i < 4000; ++i)
      if (!check(d, next_u32(), &checks)) return 1;
  }
  printf("ok %llu\n", static_cast<unsigned long long>(checks));
  return 0;
}
