// noalloc.cu -- per-eps neighbour counts without any device allocation.
//
// Some callers cannot call cudaMalloc: code living under an allocator that owns all of the
// device's memory (a framework's caching allocator, a hard memory budget), and latency-critical
// callers that cannot afford the implicit device-wide synchronisation of cudaMalloc/cudaFree.
// For them, dbm_neighbor_counts_noalloc computes the same per-eps degrees as
// dbm_neighbor_counts but takes every byte of scratch from one file-scope device array of fixed
// size, so the call allocates nothing.  The caller still passes the points and the output
// buffer.
//
// The array (kNoAllocScratchBytes, 32 MiB) is part of the library image: every GPU on which
// the library is used keeps it until the process exits.  Its device address is looked up
// once per device, on the first call made with that device current.  All calls share the
// array and it keeps the previous call's contents, so the parts that must start at zero are
// cleared on every call, and two calls that overlap on the GPU (different streams or threads)
// race on it.  The call ends by reading its status word back to the host and synchronising the
// stream.
//
// Cost: the exact tile kernel over every tile pair (O(N^2 D)); the spatial order, tile-pair
// pruning and tensor-core screen of dbm_neighbor_counts need buffers sized by N and by the
// surviving tile pairs, which this entry point does not have.
#include "dbm_internal.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

namespace dbm {

Status launch_distance(const DistLaunch& a, cudaStream_t s);
Status transpose_pad(const float* x, float* xt, int64_t n, int32_t d, int32_t* err, cudaStream_t s,
                     const int32_t* perm = nullptr, int32_t rows = 0, float* box_lo = nullptr,
                     float* box_hi = nullptr);
int32_t padded_dims(int32_t d);
int64_t padded_points(int64_t n);

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mutex;
static void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array for the current device (looked up once per device).
static Status noalloc_scratch(void** out)
{
  int dev = -1;
  DBM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return Status::Err(DBM_ERR_INVALID, "device ordinal out of range for the static scratch table");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return Status::Err(DBM_ERR_CUDA, std::string("cudaGetSymbolAddress of the static scratch failed: ") +
                                          cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return Status::Ok();
}

// deg[e][i] = 1 + sum_{c <= e} hist[c][i]
__global__ void noalloc_degrees_kernel(const int32_t* __restrict__ hist, int64_t n, int k,
                                       int32_t* __restrict__ deg)
{
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int32_t run = 1;
  for (int e = 0; e < k; ++e) {
    run += hist[static_cast<int64_t>(e) * n + i];
    deg[static_cast<int64_t>(e) * n + i] = run;
  }
}

static Status neighbor_counts_noalloc(const float* x, int64_t n, int64_t d, const float* eps, int k,
                                      int32_t* deg_out, cudaStream_t s)
{
  if (n < 1 || d < 1 || !x || !deg_out || !eps)
    return Status::Err(DBM_ERR_INVALID, "x, eps and deg must be given, with n >= 1 and d >= 1");
  if (k < 1 || k > kMaxEps) return Status::Err(DBM_ERR_INVALID, "the number of eps values must be between 1 and 16");
  for (int e = 0; e < k; ++e) {
    if (!(eps[e] > 0.0f) || !std::isfinite(eps[e]) || (e > 0 && !(eps[e] > eps[e - 1])))
      return Status::Err(DBM_ERR_INVALID, "eps values must be finite, positive and strictly ascending");
  }
  if (n >= (int64_t(1) << kCodeShift)) return Status::Err(DBM_ERR_TOO_LARGE, "N must be below 2^28");

  // scratch plan: [counters 256][err 256][edge slot 256][hist k*n int32][XT dp*npad float]
  const int32_t di = static_cast<int32_t>(d);
  const int64_t npad = padded_points(n);
  const size_t hist_bytes = align_up(sizeof(int32_t) * static_cast<size_t>(k) * n, 256);
  const size_t xt_bytes = align_up(sizeof(float) * static_cast<size_t>(padded_dims(di)) * npad, 256);
  const size_t need = 3 * 256 + hist_bytes + xt_bytes;
  if (d > (int64_t(1) << 20) || need > kNoAllocScratchBytes)
    return Status::Err(DBM_ERR_TOO_LARGE,
                       "this call needs " + std::to_string(need) + " bytes of scratch; the static scratch "
                       "holds " + std::to_string(kNoAllocScratchBytes) + " bytes (use dbm_neighbor_counts)");

  void* base = nullptr;
  DBM_TRY(noalloc_scratch(&base));
  unsigned char* p = static_cast<unsigned char*>(base);
  auto* counters = reinterpret_cast<unsigned long long*>(p);
  auto* err = reinterpret_cast<int32_t*>(p + 256);
  auto* edges = reinterpret_cast<uint64_t*>(p + 512);
  auto* hist = reinterpret_cast<int32_t*>(p + 768);
  auto* xt = reinterpret_cast<float*>(p + 768 + hist_bytes);

  float eps2[kMaxEps];
  for (int e = 0; e < k; ++e) {
    volatile float v = eps[e] * eps[e];
    eps2[e] = v;
  }
  // the counters, the error word and the histogram must start at zero on every call
  DBM_CUDA(cudaMemsetAsync(p, 0, 768 + hist_bytes, s));
  DBM_TRY(transpose_pad(x, xt, n, di, err, s));
  int dev = 0, sms = 148;
  DBM_CUDA(cudaGetDevice(&dev));
  DBM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  DistLaunch a{n, di, k, xt, eps2, counters, edges, 0, hist, err, sms};
  DBM_TRY(launch_distance(a, s));
  count_launch();
  noalloc_degrees_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, s>>>(hist, n, k, deg_out);
  DBM_CUDA(cudaGetLastError());
  int32_t flags = 0;
  DBM_CUDA(cudaMemcpyAsync(&flags, err, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  DBM_CUDA(cudaStreamSynchronize(s));
  if (flags & kErrNonFinite) return Status::Err(DBM_ERR_NONFINITE, "the input contains NaN or infinity");
  if (flags & kErrTmaTimeout)
    return Status::Err(DBM_ERR_NOT_CONVERGED, "a bounded TMA wait in the distance kernel ran out");
  return Status::Ok();
}

}  // namespace dbm

extern "C" int dbm_neighbor_counts_noalloc(const float* x_dev, int64_t n, int64_t d,
                                           const float* eps_host, int k, int32_t* deg_dev,
                                           void* stream, char* err, size_t err_len)
{
  const dbm::Status r = dbm::neighbor_counts_noalloc(x_dev, n, d, eps_host, k, deg_dev,
                                                     static_cast<cudaStream_t>(stream));
  if (err && err_len) {
    const size_t c = std::min(err_len - 1, r.msg.size());
    std::memcpy(err, r.msg.data(), c);
    err[c] = '\0';
  }
  return r.code;
}
