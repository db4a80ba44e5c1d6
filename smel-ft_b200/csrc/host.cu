// Host-side helpers: error text, per-device status word, SM count, tensor-map encoding.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <vector>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "host.h"

namespace smelb {

static thread_local char g_last_error[512] = {0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_last_error; }

static std::mutex g_mu;
static int* g_status[64] = {nullptr};
static int g_sms[64] = {0};

int* device_status(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, kStatusWords * sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, kStatusWords * sizeof(int)) != cudaSuccess) return nullptr;
    g_status[dev] = p;
  }
  return g_status[dev];
}

int num_sms(int dev) {
  if (dev < 0 || dev >= 64) return 148;
  if (!g_sms[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

// ---------------------------------------------------------------------------------------------- instrumentation
static std::atomic<long long> g_launches{0};
static std::atomic<bool> g_timing{false};
static std::mutex g_tmu;
static std::vector<cudaEvent_t> g_ev_pool;
static std::vector<std::pair<cudaEvent_t, cudaEvent_t>> g_ev_used;
static cudaEvent_t g_ev_open = nullptr;

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(); }
bool gemm_timing_enabled() { return g_timing.load(std::memory_order_relaxed); }

static cudaEvent_t take_event() {
  if (g_ev_pool.empty()) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
  }
  cudaEvent_t e = g_ev_pool.back();
  g_ev_pool.pop_back();
  return e;
}

void gemm_timing_begin(cudaStream_t st) {
  std::lock_guard<std::mutex> lk(g_tmu);
  g_ev_open = take_event();
  if (g_ev_open) cudaEventRecord(g_ev_open, st);
}

void gemm_timing_end(cudaStream_t st) {
  std::lock_guard<std::mutex> lk(g_tmu);
  if (!g_ev_open) return;
  cudaEvent_t e = take_event();
  if (!e) return;
  cudaEventRecord(e, st);
  g_ev_used.emplace_back(g_ev_open, e);
  g_ev_open = nullptr;
}

void set_gemm_timing(bool on) {
  std::lock_guard<std::mutex> lk(g_tmu);
  g_timing.store(on);
}

// Sum of the recorded GEMM launch durations (synchronizes on the recorded events), then recycles the events.
int read_gemm_timing(double* ms, long long* n) {
  std::lock_guard<std::mutex> lk(g_tmu);
  double tot = 0.0;
  for (auto& pr : g_ev_used) {
    SMELB_CUDA(cudaEventSynchronize(pr.second));
    float t = 0.f;
    SMELB_CUDA(cudaEventElapsedTime(&t, pr.first, pr.second));
    tot += t;
    g_ev_pool.push_back(pr.first);
    g_ev_pool.push_back(pr.second);
  }
  *ms = tot;
  *n = (long long)g_ev_used.size();
  g_ev_used.clear();
  return kOk;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, int swizzle_bytes) {
  auto fn = encode_fn();
  SMELB_CHECK_ARG(fn != nullptr, kErrCuda, "cuTensorMapEncodeTiled is not available from the driver");
  SMELB_CHECK_ARG(base != nullptr, kErrArg, "tensor map over a null pointer");
  SMELB_CHECK_ARG((reinterpret_cast<uintptr_t>(base) & 15) == 0, kErrShape, "tensor map base not 16-byte aligned");
  SMELB_CHECK_ARG(row_bytes % 16 == 0, kErrShape, "tensor map row pitch %llu not a multiple of 16 bytes",
                  (unsigned long long)row_bytes);
  SMELB_CHECK_ARG((box_cols * elem_bytes) % 16 == 0, kErrShape, "tensor map box inner extent not 16-byte multiple");
  SMELB_CHECK_ARG(swizzle_bytes == 0 || (int)(box_cols * elem_bytes) == swizzle_bytes, kErrShape,
                  "tensor map swizzle span %d for a %u-byte box row", swizzle_bytes, box_cols * elem_bytes);
  const CUtensorMapSwizzle swz = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                       : CU_TENSOR_MAP_SWIZZLE_NONE;
  if (rows == 0) rows = 1;  // an empty matrix still needs a valid (never read) map
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  SMELB_CHECK_ARG(r == CUDA_SUCCESS, kErrShape,
                  "cuTensorMapEncodeTiled failed (%d): rows=%llu cols=%llu pitch=%llu box=%ux%u", (int)r,
                  (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)row_bytes, box_cols,
                  box_rows);
  return kOk;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, const uint64_t dims[3],
                 const uint64_t strides_bytes[2], const uint32_t box[3], int swizzle_bytes) {
  auto fn = encode_fn();
  SMELB_CHECK_ARG(fn != nullptr, kErrCuda, "cuTensorMapEncodeTiled is not available from the driver");
  SMELB_CHECK_ARG(base != nullptr, kErrArg, "tensor map over a null pointer");
  SMELB_CHECK_ARG((reinterpret_cast<uintptr_t>(base) & 15) == 0, kErrShape, "tensor map base not 16-byte aligned");
  SMELB_CHECK_ARG(strides_bytes[0] % 16 == 0 && strides_bytes[1] % 16 == 0, kErrShape,
                  "tensor map strides %llu, %llu not multiples of 16 bytes", (unsigned long long)strides_bytes[0],
                  (unsigned long long)strides_bytes[1]);
  const CUtensorMapSwizzle swz = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                       : CU_TENSOR_MAP_SWIZZLE_NONE;
  cuuint64_t d[3] = {dims[0], dims[1] ? dims[1] : 1, dims[2] ? dims[2] : 1};
  cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  SMELB_CHECK_ARG(r == CUDA_SUCCESS, kErrShape, "cuTensorMapEncodeTiled (3-d) failed (%d): dims=%llux%llux%llu box=%ux%ux%u",
                  (int)r, (unsigned long long)d[0], (unsigned long long)d[1], (unsigned long long)d[2], bx[0], bx[1],
                  bx[2]);
  return kOk;
}

}  // namespace smelb
