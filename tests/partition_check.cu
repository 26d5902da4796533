// Host-side check of the launch partitions (alveare_b200/csrc/stream.cuh):
// the 32-bit FastDiv / Partition arithmetic against the 64-bit formulas it
// replaced, over shapes of every kernel family and several grid sizes.
#include <cstdint>
#include <cstdio>
#include <random>
#include "stream.cuh"
using namespace alv;
static uint64_t old_range_start(uint64_t w, uint64_t U, uint64_t W) { return w * U / W; }
int main() {
  std::mt19937_64 rng(1);
  long bad = 0, n = 0;
  for (uint32_t d = 1; d < 5000; ++d) {
    FastDiv f = FastDiv::make(d);
    for (int i = 0; i < 2000; ++i) {
      uint32_t x = (i < 1000) ? static_cast<uint32_t>(rng()) : static_cast<uint32_t>(rng() % (1u << 24));
      if (i < 10) x = d * i + (i & 1 ? d - 1 : 0);
      if (f.div(x) != x / d) { if (bad++ < 5) printf("fastdiv bad d=%u x=%u\n", d, x); }
      ++n;
    }
    for (uint32_t x : {0u, 1u, d - 1, d, d + 1, 0xFFFFFFFFu, 0xFFFFFFFEu}) if (f.div(x) != x / d) { if (bad++ < 5) printf("fastdiv edge d=%u x=%u\n", d, x); }
  }
  printf("fastdiv: %ld checks, %ld bad\n", n, bad);
  long pbad = 0, pn = 0;
  const uint32_t shapes[][2] = {{432, 18}, {960, 60}, {240, 240}, {128, 32}, {192, 32}, {8016, 32}, {1, 1}, {3, 5},
                                {36, 100}, {37, 4}, {16384, 256}, {200, 7}, {960, 60}, {1920, 60}, {240, 120}};
  for (auto& sh : shapes)
    for (uint32_t nctas : {148u, 132u, 1u, 2u, 7u})
      for (int al = 0; al < 2; ++al) {
        const uint32_t RT = sh[0], KT = sh[1];
        Partition p = Partition::make(RT, KT, nctas, al);
        const uint64_t U = uint64_t(RT) * KT;
        const uint64_t per = (uint64_t(RT) + nctas - 1) / nctas;
        const bool aligned = al || (RT >= nctas && per * nctas * 32 <= uint64_t(RT) * 33);
        const uint64_t mu = (KT + 15) / 16;
        uint64_t W = U / mu; if (W < 1) W = 1; if (W > uint64_t(nctas) * kWarpsPerCtaS) W = uint64_t(nctas) * kWarpsPerCtaS;
        if (p.aligned != aligned || p.W != W) { printf("make mismatch\n"); ++pbad; }
        for (uint32_t c = 0; c <= nctas; ++c) {
          uint64_t ob;
          if (aligned) ob = uint64_t(c) * RT / nctas * KT;
          else { uint64_t gw = uint64_t(c) * kWarpsPerCtaS; ob = old_range_start(gw < W ? gw : W, U, W); }
          if (p.cta_begin(c) != ob) { if (pbad++ < 5) printf("cta_begin RT=%u KT=%u n=%u c=%u\n", RT, KT, nctas, c); }
          ++pn;
          if (c == nctas) continue;
          for (uint32_t w = 0; w < kWarpsPerCtaS; ++w) {
            uint32_t u0, u1; p.warp_range(c, w, u0, u1);
            uint64_t o0, o1;
            if (aligned) { uint64_t c0 = ob, len = (c + 1 <= nctas ? (uint64_t(c + 1) * RT / nctas * KT) : U) - c0; o0 = c0 + len * w / kWarpsPerCtaS; o1 = c0 + len * (w + 1) / kWarpsPerCtaS; }
            else { uint64_t gw = uint64_t(c) * kWarpsPerCtaS + w; if (gw >= W) o0 = o1 = U; else { o0 = old_range_start(gw, U, W); o1 = old_range_start(gw + 1, U, W); } }
            if (u0 != o0 || u1 != o1) { if (pbad++ < 5) printf("warp_range RT=%u KT=%u n=%u c=%u w=%u\n", RT, KT, nctas, c, w); }
            ++pn;
          }
        }
        if (!aligned)
          for (uint64_t u = 0; u < U; u += (U > 100000 ? 97 : 1)) {
            uint32_t ow = uint32_t(((u + 1) * W - 1) / U);
            if (p.warp_of_unit(uint32_t(u)) != ow) { if (pbad++ < 5) printf("warp_of_unit RT=%u KT=%u u=%lu\n", RT, KT, (unsigned long)u); }
            ++pn;
          }
      }
  printf("partition: %ld checks, %ld bad\n", pn, pbad);
  return (bad || pbad) ? 1 : 0;
}
