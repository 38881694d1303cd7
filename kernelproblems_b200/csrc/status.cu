// status.cu — version, status strings, per-thread CUDA error record and the
// cached device queries used to size launches.
#include <mutex>

#include "common.cuh"

namespace frag {

static thread_local int g_last_cuda_error = 0;

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return d;
}

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int d = current_device();
  if (d < 0 || d >= 64) return 0;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[d] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    cache[d] = n;
  }
  return cache[d];
}

// Error word kernels report into (FRAG_DEVFLAG_* bits), one per device.
__device__ int g_error_word;

int* device_error_word() {
  static std::mutex mu;
  static int* cache[64] = {nullptr};
  const int d = current_device();
  if (d < 0 || d >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[d] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cache[d] = static_cast<int*>(p);
  }
  return cache[d];
}

bool allow_dynamic_smem(const void* kernel, int bytes) {
  // Largest dynamic shared memory size set so far, per device and kernel.
  static std::mutex mu;
  static const void* kern[64][32] = {};
  static int set_bytes[64][32] = {};
  const int d = current_device();
  if (d < 0 || d >= 64) return false;
  std::lock_guard<std::mutex> lk(mu);
  int slot = -1;
  for (int i = 0; i < 32; ++i) {
    if (kern[d][i] == kernel) {
      if (set_bytes[d][i] >= bytes) return true;
      slot = i;
      break;
    }
    if (kern[d][i] == nullptr && slot < 0) slot = i;
  }
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (slot >= 0) {
    kern[d][slot] = kernel;
    set_bytes[d][slot] = bytes;
  }
  return true;
}

namespace {

// One thread waits, with the library's bounded wait, on an mbarrier that
// nothing arrives on: the wait must give up after `limit` cycles and set
// FRAG_DEVFLAG_WAIT_TIMEOUT in the error word, as every kernel's waits do.
__global__ void bounded_wait_probe(int* err, long long limit) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  mbar_init_fence();
  mbar_wait_for(&bar, 0, err, limit);
}

}  // namespace
}  // namespace frag

extern "C" {

int frag_selftest_bounded_wait(int64_t limit_cycles, frag_stream_t stream) {
  if (limit_cycles <= 0 || limit_cycles > frag::kWaitCycles) return FRAG_ERR_INVALID_ARG;
  int* err = frag::device_error_word();
  if (!err) return FRAG_ERR_CUDA;
  frag::bounded_wait_probe<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      err, static_cast<long long>(limit_cycles));
  return frag::check_launch();
}

const char* frag_version(void) { return "libfrag 0.1.0 (sm_100a)"; }

const char* frag_status_string(int status) {
  switch (status) {
    case FRAG_OK: return "ok";
    case FRAG_ERR_INVALID_ARG: return "invalid argument (null pointer or negative size)";
    case FRAG_ERR_SHAPE: return "unsupported shape";
    case FRAG_ERR_ALIGN: return "misaligned pointer or stride";
    case FRAG_ERR_WORKSPACE: return "workspace missing or too small";
    case FRAG_ERR_CUDA: return "CUDA runtime error";
    case FRAG_ERR_NO_DEVICE: return "no CUDA device";
    case FRAG_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the no-alloc entry point's static buffer holds";
    default: return "unknown status";
  }
}

int frag_last_cuda_error(void) { return frag::g_last_cuda_error; }

int frag_device_sm_count(void) { return frag::sm_count(); }

int frag_device_errors(int clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, frag::g_error_word, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(frag::g_error_word, &zero, sizeof(int));
  }
  if (e != cudaSuccess) {
    frag::set_last_cuda_error(e);
    cudaGetLastError();
    return -FRAG_ERR_CUDA;
  }
  return v;
}

}  // extern "C"
