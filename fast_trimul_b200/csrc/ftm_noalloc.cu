// ftm_trimul_fwd_static_scratch: the whole forward without any device allocation.
//
// Some callers cannot hand this library a workspace: hosts that receive a fixed
// device-memory budget at start-up and may not grow it, or that must not call
// cudaMalloc while running because it can synchronise the device and stall the
// other streams. For them the intermediate a, b, x planes and the error word live in
// one file-scope device array, reserved when the library is loaded and held by every
// GPU that loads it until the process exits.
//
// Limit: batch * rows * cols <= FTM_STATIC_SCRATCH_MAX_POSITIONS (65,536 positions,
// e.g. N = 256 at B = 1), i.e. 3 * 65,536 * 128 * 2 + 65,536 * 8 bytes (48.5 MiB) per GPU.
// Larger problems are rejected with FTM_BAD_WORKSPACE.
//
// The array is shared by every call on a device and keeps the previous call's
// contents; the error word is cleared at the start of each call and a, b, x are fully
// rewritten before they are read. Calls whose kernels overlap on the GPU (e.g. on two
// streams) race on the array and must be serialised by the caller.
//
// The device address of the array is looked up once per device, on the first call
// made with that device current (cudaGetSymbolAddress); make that first call before
// any stream capture. The cached address belongs to the device's primary context: a
// process that resets the device (cudaDeviceReset) must not call this entry point
// afterwards, because the cached address no longer names the array.
//
// ftm_static_scratch_error_word() returns the device's error word inside the array,
// for ftm_check_error: a bounded device wait that expired in a call is reported
// there, not through the call's return value (the call returns once it has queued
// the kernels).
#include <mutex>

#include "../../include/fast_trimul_b200.h"
#include "ftm_kernels.h"

namespace {

constexpr size_t kPlaneBytes = size_t(FTM_STATIC_SCRATCH_MAX_POSITIONS) * ftm::kC * 2;
constexpr size_t kStatsBytes = size_t(FTM_STATIC_SCRATCH_MAX_POSITIONS) * 8;
constexpr size_t kScratchBytes = 3 * kPlaneBytes + kStatsBytes + 256;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// device address of g_scratch on the current device (nullptr on failure)
void* scratch_address(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess) return nullptr;
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int ftm_trimul_fwd_static_scratch(const ftm_problem* p, const void* z,
                                             const float* mask, const void* packed, void* out,
                                             ftm_stream_t stream) {
  ftm::set_last_launch_count(0);
  // every argument is checked before anything is queued, so a rejected call leaves the
  // shared array as it was
  int st = ftm::check_forward_args(p, z, mask, packed, out);
  if (st != FTM_OK) return st;
  const double positions = double(p->batch) * p->rows * p->cols;
  if (positions > double(FTM_STATIC_SCRATCH_MAX_POSITIONS)) return FTM_BAD_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FTM_LAUNCH_FAILED;
  if (ftm_device_supported(dev) != 1) return FTM_UNSUPPORTED_ARCH;
  unsigned char* base = static_cast<unsigned char*>(scratch_address(dev));
  if (!base) return FTM_LAUNCH_FAILED;

  unsigned char* a = base;
  unsigned char* b = base + kPlaneBytes;
  unsigned char* x = base + 2 * kPlaneBytes;
  float* zstats = reinterpret_cast<float*>(base + 3 * kPlaneBytes);
  int* err = reinterpret_cast<int*>(base + 3 * kPlaneBytes + kStatsBytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(err, 0, sizeof(int), s) != cudaSuccess) return FTM_LAUNCH_FAILED;
  st = ftm_input_stage(p, z, mask, packed, a, b, zstats, err, stream);
  if (st != FTM_OK) return st;
  st = ftm_contraction(a, b, x, p->batch * ftm::kC, p->rows, p->cols, p->cols, 1, err, stream);
  if (st != FTM_OK) return st;
  st = ftm_output_stage(p, z, mask, x, zstats, packed, out, err, stream);
  if (st != FTM_OK) return st;
  ftm::set_last_launch_count(3);
  return FTM_OK;
}

extern "C" int* ftm_static_scratch_error_word(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  unsigned char* base = static_cast<unsigned char*>(scratch_address(dev));
  if (!base) return nullptr;
  return reinterpret_cast<int*>(base + 3 * kPlaneBytes + kStatsBytes);
}
