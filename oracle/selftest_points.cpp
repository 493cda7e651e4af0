// selftest_points -- writes the reference selftest's input points as raw float32.
//
// TEST INFRASTRUCTURE ONLY.  The reference's selftest (src/main.cu:904-920) draws three
// Gaussian blobs (centres (0,0), (10,0), (0,10), sigma 0.5) from std::mt19937(seed) through
// std::normal_distribution<float>, x then y for each point, cluster by cluster, and leaves
// every coordinate beyond the first two at zero.  Its recorded answers (clusters, noise per
// configuration, official-campaign-v1/.../validation/selftest-cuvs.log:30-38) are only
// reproducible from the same random stream, so the points are drawn here with the same
// standard-library engine and distribution.
//
// usage: selftest_points N_PER_CLUSTER D SEED OUT.f32
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

int main(int argc, char** argv)
{
  if (argc != 5) {
    std::fprintf(stderr, "usage: %s N_PER_CLUSTER D SEED OUT.f32\n", argv[0]);
    return 2;
  }
  const int per = std::atoi(argv[1]);
  const int d = std::atoi(argv[2]);
  const unsigned seed = static_cast<unsigned>(std::strtoul(argv[3], nullptr, 10));
  if (per <= 0 || d < 2) return 2;
  const float cx[3] = {0.0f, 10.0f, 0.0f};
  const float cy[3] = {0.0f, 0.0f, 10.0f};
  std::mt19937 rng(seed);
  std::normal_distribution<float> noise(0.0f, 0.5f);
  std::vector<float> pts(static_cast<size_t>(3) * per * d, 0.0f);
  for (int c = 0; c < 3; ++c) {
    for (int i = 0; i < per; ++i) {
      const size_t row = static_cast<size_t>(c) * per + i;
      pts[row * d + 0] = cx[c] + noise(rng);
      pts[row * d + 1] = cy[c] + noise(rng);
    }
  }
  FILE* f = std::fopen(argv[4], "wb");
  if (!f) return 1;
  const size_t w = std::fwrite(pts.data(), sizeof(float), pts.size(), f);
  std::fclose(f);
  return w == pts.size() ? 0 : 1;
}
