// Compares the restated expf / expm1f / tanhf (small-lm-rs_b200/csrc/
// slmkv_libm.h, host build) with the C library's, bit for bit, over every
// float whose bits are congruent to `phase` modulo `stride`, every float of
// magnitude in [0.5, 8] (where SiTU's activations and softmax's larger
// exponents fall) and the softmax range [-104, 0] at 1/4096 of its floats.
// Prints the mismatch counts; exit status 0 when there are none.
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "slmkv_libm.h"

using namespace slmkv::libm;

int main(int argc, char** argv) {
  const uint64_t stride = argc > 1 ? std::strtoull(argv[1], nullptr, 10) : 1;
  const uint64_t phase = argc > 2 ? std::strtoull(argv[2], nullptr, 10) : 0;
  long n = 0, bad_exp = 0, bad_tanh = 0, bad_expm1 = 0;
  auto check = [&](float x) {
    if (std::isnan(x)) return;
    ++n;
    if (f2u(expf(x)) != f2u(slm_expf(x))) {
      if (bad_exp++ < 3) std::printf("expf %a: %a vs %a\n", x, expf(x), slm_expf(x));
    }
    if (f2u(tanhf(x)) != f2u(slm_tanhf(x))) {
      if (bad_tanh++ < 3) std::printf("tanhf %a: %a vs %a\n", x, tanhf(x), slm_tanhf(x));
    }
    if (f2u(expm1f(x)) != f2u(slm_expm1f(x))) {
      if (bad_expm1++ < 3) std::printf("expm1f %a: %a vs %a\n", x, expm1f(x), slm_expm1f(x));
    }
  };
  for (uint64_t u = phase; u <= 0xffffffffull; u += stride) check(u2f(static_cast<uint32_t>(u)));
  for (uint32_t u = f2u(0.5f); u <= f2u(8.0f); ++u) {
    check(u2f(u));
    check(-u2f(u));
  }
  for (uint32_t u = f2u(-104.f); u > 0x80000000u; u -= 4096) check(u2f(u));
  std::printf("checked %ld floats: expf %ld, tanhf %ld, expm1f %ld mismatches\n", n, bad_exp,
              bad_tanh, bad_expm1);
  return (bad_exp || bad_tanh || bad_expm1) ? 1 : 0;
}
