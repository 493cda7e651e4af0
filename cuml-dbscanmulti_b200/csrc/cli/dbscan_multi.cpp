// dbscan_multi -- command-line front end of libdbm.so with the reference CLI's contract.
//
// Same flags, files and last-line JSON as the reference executable (src/main.cu:233-269,
// 1361-1643), so the reference's Python tools (tools/bench_vs_cuml.py:414-490,
// tools/run_validation_matrix.py:51-137, tools/benchmark_campaign.py:1145-1283) can drive it
// unchanged:
//
//   dbscan_multi --input points.f32 --n N --d D (--eps E[,E2..] | --eps-min A --eps-max B --eps-step S)
//                --min-samples M[,M2..] [--output labels.i32] [--max-mbytes-per-batch MB]
//                [--backend cuvs|codes] [--index auto|int32|int64] [--route auto|annotated|dense]
//                [--neigh-per-row V] [--warmup W] [--repeat R] [--solo] [--perfil] [--json]
//   dbscan_multi --selftest [--backend cuvs|codes] [--json]
//   dbscan_multi --build-info
//
// points.f32: row-major float32, no header.  labels.i32: one int32 per point per
// configuration, configuration-major, configurations eps-major (config = e*l + m).
// fit_ms is the median over --repeat fits with the points already on the device
// (CUDA events around dbm_fit_multi); reading, copies and the label write are outside it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <limits>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "dbm.h"

namespace {

struct Options {
  std::string input, output;
  long long n = 0, d = 0;
  std::vector<float> eps;
  float eps_min = 0, eps_max = 0, eps_step = 0;
  bool has_eps_range = false, has_eps_list = false;
  std::vector<int> min_samples;
  unsigned long long max_bytes_per_batch = 0;
  int warmup = 0, repeat = 1;
  std::string backend = "cuvs", index = "auto", route = "auto";
  long long neigh_per_row = 0;
  bool solo = false, json = false, selftest = false, perfil = false, build_info = false;
};

[[noreturn]] void die(int code, const std::string& msg)
{
  std::cerr << "error: " << msg << "\n";
  std::exit(code);
}

void usage()
{
  std::cerr
    << "usage: dbscan_multi --input points.f32 --n N --d D\n"
       "                    (--eps E[,E2,...] | --eps-min A --eps-max B --eps-step S)\n"
       "                    --min-samples M[,M2,...]\n"
       "                    [--output labels.i32] [--max-mbytes-per-batch MB]\n"
       "                    [--backend cuvs|codes] [--index auto|int32|int64]\n"
       "                    [--route auto|annotated|dense] [--neigh-per-row V]\n"
       "                    [--warmup W] [--repeat R] [--solo] [--perfil] [--json]\n"
       "       dbscan_multi --selftest [--backend cuvs|codes] [--json]\n"
       "       dbscan_multi --build-info\n"
       "  k eps values x l min-samples values give k*l configurations, eps-major\n"
       "  (config = e*l + m); at most 16 eps values.  fit_ms is the median of --repeat\n"
       "  fits with the points resident on the device, after --warmup discarded fits.\n";
}

long long parse_int(const std::string& raw, const char* flag)
{
  try {
    size_t used = 0;
    const long long v = std::stoll(raw, &used, 10);
    if (used != raw.size()) throw std::invalid_argument("suffix");
    return v;
  } catch (const std::exception&) {
    die(2, std::string(flag) + " needs a valid integer, got '" + raw + "'");
  }
}

int parse_int32(const std::string& raw, const char* flag)
{
  const long long v = parse_int(raw, flag);
  if (v < std::numeric_limits<int>::min() || v > std::numeric_limits<int>::max())
    die(2, std::string(flag) + " is outside the int range: '" + raw + "'");
  return static_cast<int>(v);
}

float parse_float(const std::string& raw, const char* flag)
{
  try {
    size_t used = 0;
    const float v = std::stof(raw, &used);
    if (used != raw.size() || !std::isfinite(v)) throw std::invalid_argument("not finite");
    return v;
  } catch (const std::exception&) {
    die(2, std::string(flag) + " needs a valid finite number, got '" + raw + "'");
  }
}

std::vector<std::string> split_list(const std::string& raw, const char* flag)
{
  if (raw.empty() || raw.front() == ',' || raw.back() == ',' || raw.find(",,") != std::string::npos)
    die(2, std::string(flag) + " has an empty item");
  std::vector<std::string> out;
  std::stringstream ss(raw);
  std::string item;
  while (std::getline(ss, item, ',')) out.push_back(item);
  return out;
}

// The range includes eps_max when it belongs to the progression (src/main.cu:278-294).
std::vector<float> expand_eps_range(float lo, float hi, float step)
{
  if (step <= 0.0f) die(2, "--eps-step must be positive");
  if (hi < lo) die(2, "--eps-max must be >= --eps-min");
  std::vector<float> out;
  const double tol = 1e-9 * std::max(1.0, static_cast<double>(std::fabs(hi)));
  for (int i = 0;; ++i) {
    const double v = static_cast<double>(lo) + i * static_cast<double>(step);
    if (v > static_cast<double>(hi) + tol) break;
    out.push_back(static_cast<float>(v));
    if (out.size() > DBM_MAX_EPS) break;
  }
  return out;
}

Options parse_args(int argc, char** argv)
{
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&](const char* name) -> std::string {
      if (i + 1 >= argc) die(2, std::string(name) + " needs a value");
      return argv[++i];
    };
    if (a == "--input") o.input = next("--input");
    else if (a == "--output") o.output = next("--output");
    else if (a == "--n") o.n = parse_int32(next("--n"), "--n");
    else if (a == "--d") o.d = parse_int32(next("--d"), "--d");
    else if (a == "--eps") {
      o.eps.clear();
      for (auto& s : split_list(next("--eps"), "--eps")) o.eps.push_back(parse_float(s, "--eps"));
      o.has_eps_list = true;
    } else if (a == "--eps-min") { o.eps_min = parse_float(next("--eps-min"), "--eps-min"); o.has_eps_range = true; }
    else if (a == "--eps-max") { o.eps_max = parse_float(next("--eps-max"), "--eps-max"); o.has_eps_range = true; }
    else if (a == "--eps-step") { o.eps_step = parse_float(next("--eps-step"), "--eps-step"); o.has_eps_range = true; }
    else if (a == "--min-samples") {
      o.min_samples.clear();
      for (auto& s : split_list(next("--min-samples"), "--min-samples"))
        o.min_samples.push_back(parse_int32(s, "--min-samples"));
    } else if (a == "--max-mbytes-per-batch") {
      const long long mb = parse_int(next("--max-mbytes-per-batch"), "--max-mbytes-per-batch");
      if (mb < 0 || static_cast<unsigned long long>(mb) > UINT64_MAX / 1000000ull)
        die(2, "--max-mbytes-per-batch must be >= 0 and fit in size_t");
      o.max_bytes_per_batch = static_cast<unsigned long long>(mb) * 1000000ull;
    } else if (a == "--backend") o.backend = next("--backend");
    else if (a == "--index") o.index = next("--index");
    else if (a == "--route") o.route = next("--route");
    else if (a == "--neigh-per-row") o.neigh_per_row = parse_int32(next("--neigh-per-row"), "--neigh-per-row");
    else if (a == "--warmup") o.warmup = parse_int32(next("--warmup"), "--warmup");
    else if (a == "--repeat") o.repeat = parse_int32(next("--repeat"), "--repeat");
    else if (a == "--solo") o.solo = true;
    else if (a == "--perfil") o.perfil = true;
    else if (a == "--json") o.json = true;
    else if (a == "--selftest") o.selftest = true;
    else if (a == "--build-info") o.build_info = true;
    else if (a == "--help" || a == "-h") { usage(); std::exit(0); }
    else { std::cerr << "error: unknown argument '" << a << "'\n"; usage(); std::exit(2); }
  }
  if (o.has_eps_list && o.has_eps_range) die(2, "--eps and the --eps-min/--eps-max/--eps-step range are mutually exclusive");
  if (o.repeat < 1) die(2, "--repeat must be >= 1");
  if (o.warmup < 0) die(2, "--warmup must be >= 0");
  if (o.neigh_per_row < 0) die(2, "--neigh-per-row must be >= 0");
  if (o.has_eps_range) o.eps = expand_eps_range(o.eps_min, o.eps_max, o.eps_step);
  return o;
}

template <typename T>
void normalize_list(std::vector<T>& v, const char* flag)
{
  const std::vector<T> orig = v;
  std::sort(v.begin(), v.end());
  v.erase(std::unique(v.begin(), v.end()), v.end());
  if (v != orig)
    std::cerr << "warning: " << flag << " was sorted/de-duplicated; the configuration order follows the "
                 "\"eps\" and \"min_samples\" fields of the JSON\n";
}

int backend_code(const std::string& b)
{
  if (b == "cuvs") return DBM_BACKEND_CUVS;
  if (b == "codes") return DBM_BACKEND_CODES;
  die(2, "--backend must be 'cuvs' or 'codes', got '" + b + "'");
}
int index_bits(const std::string& s)
{
  if (s == "auto") return 0;
  if (s == "int32") return 32;
  if (s == "int64") return 64;
  die(2, "--index must be 'auto', 'int32' or 'int64', got '" + s + "'");
}
int route_code(const std::string& s)
{
  if (s == "auto") return DBM_ROUTE_AUTO;
  if (s == "annotated") return DBM_ROUTE_ANNOTATED;
  if (s == "dense") return DBM_ROUTE_DENSE;
  die(2, "--route must be 'auto', 'annotated' or 'dense', got '" + s + "'");
}

std::string json_escape(const std::string& s)
{
  std::ostringstream o;
  for (unsigned char c : s) {
    switch (c) {
      case '"': o << "\\\""; break;
      case '\\': o << "\\\\"; break;
      case '\n': o << "\\n"; break;
      case '\r': o << "\\r"; break;
      case '\t': o << "\\t"; break;
      default:
        if (c < 0x20) { char b[8]; std::snprintf(b, sizeof b, "\\u%04x", c); o << b; }
        else o << static_cast<char>(c);
    }
  }
  return o.str();
}

template <typename T>
std::string join(const std::vector<T>& v)
{
  std::ostringstream o;
  o.precision(9);
  for (size_t i = 0; i < v.size(); ++i) o << (i ? "," : "") << v[i];
  return o.str();
}

float median_of(std::vector<float> v)
{
  std::sort(v.begin(), v.end());
  const size_t m = v.size() / 2;
  return (v.size() % 2) ? v[m] : 0.5f * (v[m - 1] + v[m]);
}

#define CK(call)                                                                              \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess) die(1, std::string(#call) + ": " + cudaGetErrorString(e_));        \
  } while (0)

// ---- one device-resident fitting session (handle + buffers reused across calls) ------------
struct Session {
  dbm_handle* h = nullptr;
  cudaStream_t stream = nullptr;
  float* x = nullptr;
  int32_t* labels = nullptr;
  size_t x_cap = 0, l_cap = 0;

  Session()
  {
    CK(cudaSetDevice(0));
    CK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    char err[512] = {0};
    h = dbm_create(0, stream, err, sizeof err);
    if (!h) die(1, std::string("dbm_create: ") + err);
  }
  ~Session()
  {
    if (h) dbm_destroy(h);
    if (x) cudaFree(x);
    if (labels) cudaFree(labels);
    if (stream) cudaStreamDestroy(stream);
  }
  void upload(const std::vector<float>& pts)
  {
    if (pts.size() > x_cap) {
      if (x) cudaFree(x);
      CK(cudaMalloc(&x, pts.size() * sizeof(float)));
      x_cap = pts.size();
    }
    CK(cudaMemcpyAsync(x, pts.data(), pts.size() * sizeof(float), cudaMemcpyHostToDevice, stream));
    CK(cudaStreamSynchronize(stream));
  }
  void ensure_labels(size_t count)
  {
    if (count > l_cap) {
      if (labels) cudaFree(labels);
      CK(cudaMalloc(&labels, count * sizeof(int32_t)));
      l_cap = count;
    }
  }
};

struct FitOut {
  std::vector<int32_t> labels;  // k*l*n
  std::vector<float> timings;   // ms, one per measured repeat
  dbm_stats stats{};
  std::vector<uint8_t> routes;
};

FitOut fit(Session& s, const std::vector<float>& pts, long long n, long long d, const std::vector<float>& eps,
           const std::vector<int>& ms, const dbm_options& opt, int warmup, int repeat, bool upload = true)
{
  FitOut out;
  const size_t total = static_cast<size_t>(n) * eps.size() * ms.size();
  if (upload) s.upload(pts);
  s.ensure_labels(total);
  std::vector<int32_t> mp(ms.begin(), ms.end());
  out.routes.assign(static_cast<size_t>(n) + 1, 0);
  char err[1024] = {0};
  auto once = [&]() {
    const int rc = dbm_fit_multi(s.h, s.x, n, d, eps.data(), static_cast<int>(eps.size()), mp.data(),
                                 static_cast<int>(mp.size()), s.labels, nullptr, &opt, &out.stats,
                                 out.routes.data(), static_cast<int>(out.routes.size()), s.stream, err,
                                 sizeof err);
    if (rc != DBM_OK) die(1, std::string("fit_multi failed: ") + err);
  };
  for (int i = 0; i < warmup; ++i) once();
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  for (int i = 0; i < repeat; ++i) {
    CK(cudaEventRecord(a, s.stream));
    once();
    CK(cudaEventRecord(b, s.stream));
    CK(cudaEventSynchronize(b));
    float msec = 0;
    CK(cudaEventElapsedTime(&msec, a, b));
    out.timings.push_back(msec);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  out.labels.resize(total);
  CK(cudaMemcpyAsync(out.labels.data(), s.labels, total * sizeof(int32_t), cudaMemcpyDeviceToHost, s.stream));
  CK(cudaStreamSynchronize(s.stream));
  for (size_t i = 0; i < total; ++i)
    if (out.labels[i] < -1 || out.labels[i] >= n)
      die(1, "invalid CUDA label at position " + std::to_string(i) + ": " + std::to_string(out.labels[i]));
  out.routes.resize(static_cast<size_t>(out.stats.batches));
  return out;
}

std::vector<float> read_points(const std::string& path, long long n, long long d)
{
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) die(1, "cannot open '" + path + "'");
  const std::streamsize bytes = f.tellg();
  const size_t want = static_cast<size_t>(n) * static_cast<size_t>(d) * sizeof(float);
  if (static_cast<size_t>(bytes) != want)
    die(1, "'" + path + "' has " + std::to_string(bytes) + " bytes, expected " + std::to_string(want) +
             " for n=" + std::to_string(n) + " d=" + std::to_string(d) + " in float32");
  f.seekg(0);
  std::vector<float> v(static_cast<size_t>(n) * static_cast<size_t>(d));
  f.read(reinterpret_cast<char*>(v.data()), bytes);
  if (!f) die(1, "failed to read '" + path + "'");
  return v;
}

void write_labels(const std::string& path, const std::vector<int32_t>& labels)
{
  std::ofstream f(path, std::ios::binary);
  if (!f) die(1, "cannot write '" + path + "'");
  f.write(reinterpret_cast<const char*>(labels.data()), static_cast<std::streamsize>(labels.size() * 4));
  if (!f) die(1, "failed to write '" + path + "'");
}

const char* route_name(uint8_t r)
{
  return r == DBM_BATCH_ANNOTATED ? "annotated" : r == DBM_BATCH_DENSE ? "dense" : "not-applicable";
}

std::string cuda_json()
{
  int rt = 0, drv = 0, dev = -1;
  cudaDeviceProp prop{};
  const bool rok = cudaRuntimeGetVersion(&rt) == cudaSuccess;
  const bool dok = cudaDriverGetVersion(&drv) == cudaSuccess;
  const bool pok = cudaGetDevice(&dev) == cudaSuccess && cudaGetDeviceProperties(&prop, dev) == cudaSuccess;
  std::ostringstream o;
  o << "{\"runtime_version\":" << (rok ? rt : 0) << ",\"driver_version\":" << (dok ? drv : 0)
    << ",\"device\":" << (pok ? dev : -1);
  if (pok)
    o << ",\"gpu_name\":\"" << json_escape(prop.name) << "\",\"compute_capability\":\"" << prop.major << "."
      << prop.minor << "\",\"total_global_memory\":" << static_cast<unsigned long long>(prop.totalGlobalMem);
  o << "}";
  return o.str();
}

// ---- selftest (the reference's checks, src/main.cu:958-1357) ---------------------------------
std::vector<float> make_blobs(int per, int d, unsigned seed = 42)
{
  const float cx[3] = {0.0f, 10.0f, 0.0f}, cy[3] = {0.0f, 0.0f, 10.0f};
  std::mt19937 rng(seed);
  std::normal_distribution<float> noise(0.0f, 0.5f);
  std::vector<float> p(static_cast<size_t>(3) * per * d, 0.0f);
  for (int c = 0; c < 3; ++c)
    for (int i = 0; i < per; ++i) {
      const size_t r = static_cast<size_t>(c) * per + i;
      p[r * d + 0] = cx[c] + noise(rng);
      p[r * d + 1] = cy[c] + noise(rng);
    }
  return p;
}

void summarize(const std::vector<int32_t>& lab, long long n, size_t cfg, int& clusters, int& noise)
{
  clusters = noise = 0;
  const int32_t* p = lab.data() + cfg * static_cast<size_t>(n);
  for (long long i = 0; i < n; ++i) {
    if (p[i] < 0) ++noise;
    else clusters = std::max(clusters, p[i] + 1);
  }
}

std::vector<int> canonical(const std::vector<int32_t>& lab, long long n, size_t cfg)
{
  const int32_t* p = lab.data() + cfg * static_cast<size_t>(n);
  std::vector<int> out(static_cast<size_t>(n), -1), map(static_cast<size_t>(n), -1);
  int next = 0;
  for (long long i = 0; i < n; ++i) {
    if (p[i] < 0) continue;
    if (map[static_cast<size_t>(p[i])] < 0) map[static_cast<size_t>(p[i])] = next++;
    out[static_cast<size_t>(i)] = map[static_cast<size_t>(p[i])];
  }
  return out;
}

int mismatching_configs(const std::vector<int32_t>& a, const std::vector<int32_t>& b, long long n, size_t cfgs)
{
  int bad = 0;
  for (size_t c = 0; c < cfgs; ++c) bad += canonical(a, n, c) != canonical(b, n, c);
  return bad;
}

dbm_options make_opt(int backend, int bits, int route, long long npr, unsigned long long budget,
                     unsigned long long cap = 0)
{
  dbm_options o;
  std::memset(&o, 0, sizeof o);
  o.backend = backend;
  o.index_bits = bits;
  o.route = route;
  o.neigh_per_row = npr;
  o.max_bytes_per_batch = budget;
  o.csr_cap_bytes = cap;
  return o;
}

int run_selftest(bool json, int backend)
{
  Session s;
  const bool cuvs = backend == DBM_BACKEND_CUVS;
  const int per = 1000, n = 3 * per, d = 2;
  const std::vector<float> eps{0.3f, 0.5f, 0.8f};
  const std::vector<int> ms{4, 8, 16};
  const size_t k = eps.size(), l = ms.size(), ncfg = k * l;
  const std::vector<float> pts = make_blobs(per, d);
  const FitOut base = fit(s, pts, n, d, eps, ms, make_opt(backend, 32, 0, 0, 0), 0, 1);
  bool ok = true;
  std::vector<int> clusters(ncfg), noise(ncfg);
  std::ostringstream cfgs;
  for (size_t e = 0; e < k; ++e)
    for (size_t m = 0; m < l; ++m) {
      const size_t c = e * l + m;
      summarize(base.labels, n, c, clusters[c], noise[c]);
      std::cerr << "[selftest] eps=" << eps[e] << " minPts=" << ms[m] << " clusters=" << clusters[c]
                << " noise=" << noise[c] << "\n";
      cfgs << (c ? "," : "") << "{\"eps\":" << eps[e] << ",\"min_samples\":" << ms[m]
           << ",\"n_clusters\":" << clusters[c] << ",\"n_noise\":" << noise[c] << "}";
    }
  // part 1: the other backend, three repetitions, deterministic and identical
  bool compared = false;
  int backend_mm = 0, repeat_mm = 0;
  if (cuvs) {
    compared = true;
    std::vector<int32_t> first;
    for (int r = 0; r < 3; ++r) {
      const FitOut c = fit(s, pts, n, d, eps, ms, make_opt(DBM_BACKEND_CODES, 32, 0, 0, 0), 0, 1, false);
      backend_mm = std::max(backend_mm, mismatching_configs(base.labels, c.labels, n, ncfg));
      if (r == 0) first = c.labels;
      else repeat_mm = std::max(repeat_mm, mismatching_configs(first, c.labels, n, ncfg));
    }
    if (backend_mm || repeat_mm) ok = false;
    std::cerr << "[selftest] backends: " << ncfg - backend_mm << "/" << ncfg << " identical between cuvs and codes; "
              << ncfg - repeat_mm << "/" << ncfg << " deterministic over 3 codes runs\n";
  }
  const size_t easiest = (k - 1) * l;
  if (clusters[easiest] != 3) { std::cerr << "[selftest] FAIL: expected 3 clusters at the largest eps\n"; ok = false; }
  for (size_t e = 0; e < k; ++e)
    for (size_t m = 1; m < l; ++m)
      if (noise[e * l + m] < noise[e * l + m - 1]) { std::cerr << "[selftest] FAIL: noise fell as minPts grew\n"; ok = false; }
  for (size_t m = 0; m < l; ++m)
    for (size_t e = 1; e < k; ++e)
      if (noise[e * l + m] > noise[(e - 1) * l + m]) { std::cerr << "[selftest] FAIL: noise grew as eps grew\n"; ok = false; }
  // part 2: forced batches
  const uint64_t budget = dbm_max_bytes_for_batch_size(n, static_cast<int>(k), static_cast<int>(l), n / 4, backend, 0, 32);
  uint64_t bsz = 0;
  char err[512];
  dbm_batch_size(n, static_cast<int>(k), static_cast<int>(l), budget, backend, 0, 32, &bsz, err, sizeof err);
  const int nbat = static_cast<int>((n + bsz - 1) / bsz);
  const FitOut batched = fit(s, pts, n, d, eps, ms, make_opt(backend, 32, 0, 0, budget), 0, 1, false);
  const int batched_mm = mismatching_configs(base.labels, batched.labels, n, ncfg);
  if (batched_mm) ok = false;
  if (nbat < 2) { std::cerr << "[selftest] FAIL: the tight budget did not produce several batches\n"; ok = false; }
  std::cerr << "[selftest] batches: " << nbat << " x " << bsz << " points, " << ncfg - batched_mm << "/" << ncfg
            << " identical to one batch\n";
  // part 3: dimensions and eps counts
  const int dims[] = {2, 8, 16, 32, 33};
  const std::vector<std::vector<float>> eps_sets{{0.8f}, {0.3f, 0.5f, 0.8f}, {0.2f, 0.3f, 0.5f, 0.65f, 0.8f}};
  for (int dt : dims) {
    const std::vector<float> p = make_blobs(500, dt);
    bool dim_ok = true;
    for (const auto& es : eps_sets) {
      const FitOut r = fit(s, p, 1500, dt, es, {4}, make_opt(backend, 32, 0, 0, 0), 0, 1);
      int c = 0, z = 0, prev = -1;
      summarize(r.labels, 1500, es.size() - 1, c, z);
      if (c != 3) { dim_ok = ok = false; }
      for (size_t e = 0; e < es.size(); ++e) {
        summarize(r.labels, 1500, e, c, z);
        if (prev >= 0 && z > prev) dim_ok = ok = false;
        prev = z;
      }
    }
    std::cerr << "[selftest] D=" << dt << (dim_ok ? " ok" : " FAILED") << " for k = 1, 3 and 5\n";
  }
  // part 3b: D=33 vs D=8193
  const std::vector<float> eps_high{0.5f, 1.0f, 2.0f, 3.0f, 4.0f};
  const FitOut h33 = fit(s, make_blobs(16, 33), 48, 33, eps_high, {2}, make_opt(DBM_BACKEND_CODES, 32, 0, 0, 0), 0, 1);
  const FitOut hbig = fit(s, make_blobs(16, 8193), 48, 8193, eps_high, {2}, make_opt(DBM_BACKEND_CODES, 32, 0, 0, 0), 0, 1);
  const int high_mm = mismatching_configs(h33.labels, hbig.labels, 48, eps_high.size());
  if (high_mm) ok = false;
  std::cerr << "[selftest] high dimension: " << (high_mm ? "DIFFERENT" : "identical") << " between D=33 and D=8193\n";
  // part 4: index type
  const FitOut i64 = fit(s, pts, n, d, eps, ms, make_opt(backend, 64, 0, 0, 0), 0, 1);
  const int idx_mm = mismatching_configs(base.labels, i64.labels, n, ncfg);
  if (idx_mm) ok = false;
  std::cerr << "[selftest] index: " << ncfg - idx_mm << "/" << ncfg << " identical between int32 and int64\n";
  // part 5: batch correction under a 1 MB CSR cap with neigh_per_row lying (1)
  const FitOut fixup = fit(s, pts, n, d, eps, ms, make_opt(backend, 32, 0, 1, 0, 1024ull * 1024ull), 0, 1, false);
  const int fix_mm = mismatching_configs(base.labels, fixup.labels, n, ncfg);
  if (fix_mm || fixup.stats.batch_corrections == 0) ok = false;
  std::cerr << "[selftest] corrected batch (" << fixup.stats.batch_corrections << "x): " << ncfg - fix_mm << "/"
            << ncfg << " identical\n";
  // part 6: both routes
  int route_mm = 0;
  if (cuvs) {
    const FitOut ra = fit(s, pts, n, d, eps, ms, make_opt(backend, 32, DBM_ROUTE_ANNOTATED, 0, 0), 0, 1, false);
    const FitOut rd = fit(s, pts, n, d, eps, ms, make_opt(backend, 32, DBM_ROUTE_DENSE, 0, 0), 0, 1, false);
    route_mm = mismatching_configs(ra.labels, rd.labels, n, ncfg);
    if (route_mm) ok = false;
    std::cerr << "[selftest] routes: " << ncfg - route_mm << "/" << ncfg << " identical between annotated and dense\n";
  }
  std::cerr << "[selftest] " << (ok ? "PASSED" : "FAILED") << "\n";
  if (json) {
    std::cout << "{\"selftest\":" << (ok ? "true" : "false") << ",\"backend\":\"" << (cuvs ? "cuvs" : "codes")
              << "\",\"fit_ms\":" << base.timings.front() << ",\"n\":" << n << ",\"d\":" << d << ",\"eps\":["
              << join(eps) << "],\"min_samples\":[" << join(ms) << "],\"configuration_count\":" << ncfg
              << ",\"config_order\":\"eps_major\",\"batches\":" << nbat << ",\"batch_size\":" << bsz
              << ",\"batched_mismatches\":" << batched_mm << ",\"index_mismatches\":" << idx_mm
              << ",\"batch_fixup_mismatches\":" << fix_mm << ",\"route_mismatches\":" << route_mm
              << ",\"route_tested\":" << (cuvs ? "true" : "false")
              << ",\"backend_comparison_performed\":" << (compared ? "true" : "false")
              << ",\"backend_mismatches\":" << backend_mm << ",\"backend_repeat_mismatches\":" << repeat_mm
              << ",\"high_dim_mismatches\":" << high_mm << ",\"configurations\":[" << cfgs.str()
              << "],\"build\":" << dbm_build_info_json() << ",\"cuda\":" << cuda_json() << "}" << std::endl;
  }
  return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv)
{
  Options o = parse_args(argc, argv);
  if (o.build_info) {
    std::cout << "{\"build\":" << dbm_build_info_json() << "}" << std::endl;
    return 0;
  }
  const int backend = backend_code(o.backend);
  const int bits = index_bits(o.index);
  const int route = route_code(o.route);
  if (route != DBM_ROUTE_AUTO && backend != DBM_BACKEND_CUVS) die(2, "--route only applies to the cuvs backend");
  if (o.selftest && route != DBM_ROUTE_AUTO) die(2, "--route must not be combined with --selftest; the test forces both routes");
  if (o.selftest) return run_selftest(o.json, backend);
  if (o.input.empty() || o.n <= 0 || o.d <= 0 || o.eps.empty() || o.min_samples.empty()) {
    std::cerr << "error: --input, --n, --d, --eps (or the range) and --min-samples are required\n";
    usage();
    return 2;
  }
  normalize_list(o.eps, "--eps");
  normalize_list(o.min_samples, "--min-samples");
  const float safe = std::sqrt(std::numeric_limits<float>::max());
  for (float e : o.eps)
    if (!std::isfinite(e) || e <= 0.0f || e > safe) die(2, "eps values must be finite, positive and not overflow eps^2");
  for (int m : o.min_samples)
    if (m <= 0) die(2, "min-samples values must be positive");
  if (o.eps.size() > DBM_MAX_EPS) die(2, "at most 16 eps values per run");
  const std::vector<float> pts = read_points(o.input, o.n, o.d);
  for (float v : pts)
    if (!std::isfinite(v)) die(2, "the input file contains NaN or infinity");

  const dbm_options opt = make_opt(backend, bits, route, o.neigh_per_row, o.max_bytes_per_batch);
  Session s;
  const FitOut r = fit(s, pts, o.n, o.d, o.eps, o.min_samples, opt, o.warmup, o.repeat);
  const float fit_ms = median_of(r.timings);
  if (!o.output.empty()) write_labels(o.output, r.labels);
  const size_t ncfg = o.eps.size() * o.min_samples.size();

  if (o.perfil) {
    // one extra fit outside the measurement with per-phase device timers
    dbm_set_phase_timing(s.h, 1);
    const FitOut p = fit(s, pts, o.n, o.d, o.eps, o.min_samples, opt, 0, 1, false);
    dbm_set_phase_timing(s.h, 0);
    const dbm_stats& st = p.stats;
    const double tot = st.ms_distance + st.ms_graph + st.ms_label + st.ms_relabel;
    std::fprintf(stderr, "\n[perfil] %d batch(es), %lld neighbour pairs, %zu configurations\n", st.batches,
                 static_cast<long long>(st.edges), ncfg);
    std::fprintf(stderr, "[perfil] %-34s %9s %6s   %s\n", "phase", "ms", "%", "when");
    const struct { const char* name; double ms; const char* when; } rows[] = {
      {"distance pass (all pairs, once)", st.ms_distance, "shared by all configurations"},
      {"degrees, core masks, CSR", st.ms_graph, "shared by all configurations"},
      {"per-eps slabs + connected components", st.ms_label, "per batch, eps and configuration"},
      {"final relabel", st.ms_relabel, "all configurations at once"}};
    for (const auto& row : rows)
      std::fprintf(stderr, "[perfil] %-34s %9.2f %5.1f%%   %s\n", row.name, row.ms, tot > 0 ? 100.0 * row.ms / tot : 0.0,
                   row.when);
    std::fprintf(stderr, "[perfil] %-34s %9.2f\n", "total", tot);
  }

  std::vector<float> solo_ms;
  std::ostringstream solo_all;
  if (o.solo) {
    for (size_t e = 0; e < o.eps.size(); ++e)
      for (size_t m = 0; m < o.min_samples.size(); ++m) {
        const FitOut one = fit(s, pts, o.n, o.d, {o.eps[e]}, {o.min_samples[m]}, opt, o.warmup, o.repeat, false);
        solo_all << (solo_ms.empty() ? "" : ",") << "[" << join(one.timings) << "]";
        solo_ms.push_back(median_of(one.timings));
      }
  }

  if (o.json) {
    const dbm_stats& st = r.stats;
    int annotated = 0, dense = 0;
    for (uint8_t x : r.routes) { annotated += x == DBM_BATCH_ANNOTATED; dense += x == DBM_BATCH_DENSE; }
    const char* observed = "not-applicable";
    if (backend == DBM_BACKEND_CUVS && o.eps.size() > 1)
      observed = (annotated && dense) ? "mixed" : annotated ? "annotated" : dense ? "dense" : "unknown";
    std::ostringstream routes;
    for (size_t i = 0; i < r.routes.size(); ++i) routes << (i ? "," : "") << "\"" << route_name(r.routes[i]) << "\"";
    std::ostringstream argvj;
    for (int i = 0; i < argc; ++i) argvj << (i ? "," : "") << "\"" << json_escape(argv[i]) << "\"";
    std::cout << "{\"fit_ms\":" << fit_ms << ",\"fit_ms_all\":[" << join(r.timings) << "],\"backend\":\""
              << o.backend << "\",\"index\":\"" << (st.index_bits == 64 ? "int64" : "int32")
              << "\",\"neigh_per_row\":" << o.neigh_per_row << ",\"warmup\":" << o.warmup << ",\"repeat\":" << o.repeat
              << ",\"configuration_count\":" << ncfg << ",\"eps_count\":" << o.eps.size()
              << ",\"min_samples_count\":" << o.min_samples.size() << ",\"eps\":[" << join(o.eps)
              << "],\"min_samples\":[" << join(o.min_samples) << "],\"config_order\":\"eps_major\",\"n\":" << o.n
              << ",\"d\":" << o.d;
    if (o.solo) std::cout << ",\"solo_ms\":[" << join(solo_ms) << "],\"solo_ms_all\":[" << solo_all.str() << "]";
    std::cout << ",\"input\":\"" << json_escape(o.input) << "\",\"input_bytes\":"
              << static_cast<unsigned long long>(o.n) * static_cast<unsigned long long>(o.d) * 4ull
              << ",\"max_bytes_per_batch\":" << o.max_bytes_per_batch << ",\"requested_index\":\"" << o.index
              << "\",\"requested_route\":\"" << o.route << "\",\"execution\":{\"effective_max_bytes_per_batch\":"
              << st.max_bytes_per_batch << ",\"batch_size\":" << st.batch_size << ",\"batches\":" << st.batches
              << ",\"attempts\":" << st.attempts << ",\"batch_corrections\":" << st.batch_corrections
              << ",\"dense_batches\":" << dense << ",\"annotated_batches\":" << annotated << ",\"batch_routes\":["
              << routes.str() << "],\"route_observed\":\"" << observed
              << "\",\"stats_scope\":\"last_measured_repeat\",\"max_nnz\":" << st.max_nnz
              << ",\"total_nnz_max_eps\":" << st.total_nnz_max_eps << ",\"mean_degree_max_eps\":"
              << static_cast<double>(st.total_nnz_max_eps) / static_cast<double>(o.n)
              << ",\"neighbour_pairs\":" << st.edges << ",\"distance_passes\":" << st.distance_passes
              << ",\"kernel_launches\":" << st.launches << "},\"build\":" << dbm_build_info_json()
              << ",\"cuda\":" << cuda_json() << ",\"argv\":[" << argvj.str() << "]}" << std::endl;
  }
  return 0;
}
