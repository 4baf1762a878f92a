// Host build of the kernels' float sine/cosine (cufk_b200/csrc/nerf_math.cuh), compared with double
// sin/cos.  Prints the largest absolute errors on [-pi-0.2, pi+0.2] and on [-8192, 8192].
#include "nerf_math.cuh"

#include <cmath>
#include <cstdio>
#include <random>

int main() {
  double near_s = 0, near_c = 0, wide_s = 0, wide_c = 0;
  auto check = [](float x, double& ms, double& mc) {
    float s, c;
    cufkb::sincos_fast(x, s, c);
    ms = std::fmax(ms, std::fabs(double(s) - std::sin(double(x))));
    mc = std::fmax(mc, std::fabs(double(c) - std::cos(double(x))));
  };
  for (int i = -1000000; i <= 1000000; ++i) check(i * (3.35f / 1000000), near_s, near_c);
  std::mt19937 g(7);
  std::uniform_real_distribution<float> u(-cufkb::kSinCosFastRange, cufkb::kSinCosFastRange);
  for (int i = 0; i < 2000000; ++i) check(u(g), wide_s, wide_c);
  std::printf("%.6e %.6e %.6e %.6e\n", near_s, near_c, wide_s, wide_c);
  return 0;
}
