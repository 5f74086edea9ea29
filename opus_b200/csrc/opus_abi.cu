// Library-wide state of libopus_b200.so: error reporting, the per-device
// error word that bounded device waits write into, device properties and
// TMA descriptor encoding.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "opus_common.cuh"

namespace opus {

namespace {
thread_local char g_last_error[1024] = {0};

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_dev_err[kMaxDevices] = {nullptr};
int g_sm_count[kMaxDevices] = {0};
int g_smem_optin[kMaxDevices] = {0};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
PFN_cuCtxGetCurrent_v4000 g_ctx_get_current = nullptr;
std::atomic<int64_t> g_launches{0};

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return set_error(OPUS_ERR_CUDA, "%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int* device_error_word() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_dev_err[dev] == nullptr) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int) * 4) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int) * 4) != cudaSuccess) return nullptr;
    g_dev_err[dev] = p;
  }
  return g_dev_err[dev];
}

int sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  }
  return g_sm_count[dev];
}

int max_smem_optin() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 232448;
  if (g_smem_optin[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    g_smem_optin[dev] = n > 0 ? n : 232448;
  }
  return g_smem_optin[dev];
}

int current_context(CUcontext* ctx) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_ctx_get_current == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
        return set_error(OPUS_ERR_CUDA, "cannot resolve cuCtxGetCurrent");
      g_ctx_get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    }
  }
  if (g_ctx_get_current(ctx) != CUDA_SUCCESS) return set_error(OPUS_ERR_CUDA, "cuCtxGetCurrent failed");
  return OPUS_OK;
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
        return set_error(OPUS_ERR_CUDA, "cannot resolve cuTensorMapEncodeTiled");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(OPUS_ERR_INVALID, "TMA base address %p is not 16-byte aligned", base);
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0)
      return set_error(OPUS_ERR_INVALID, "TMA stride %llu is not a multiple of 16 bytes",
                       static_cast<unsigned long long>(strides_bytes[i]));
  cuuint32_t estrides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                        reinterpret_cast<const cuuint64_t*>(dims), reinterpret_cast<const cuuint64_t*>(strides_bytes),
                        reinterpret_cast<const cuuint32_t*>(box), estrides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OPUS_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return OPUS_OK;
}

namespace {

// One thread waits on an mbarrier that nothing arrives on, through the same
// bounded wait as the pipelined kernels: after kWaitLimitNs it records
// kDevTimeoutSelftest in the device error word and the kernel returns.
__global__ void stalled_wait_kernel(int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
    (void)mbar_wait(&bar, 0, &abort_flag, err, kDevTimeoutSelftest);
  }
}

}  // namespace
}  // namespace opus

extern "C" {

int opus_selftest_stalled_wait(void* stream) {
  int* err = opus::device_error_word();
  if (err == nullptr) return opus::set_error(OPUS_ERR_CUDA, "device error word unavailable");
  opus::stalled_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(err);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int opus_abi_version(void) { return OPUS_ABI_VERSION; }

int64_t opus_kernel_launches(void) { return opus::g_launches.load(std::memory_order_relaxed); }

const char* opus_last_error(void) { return opus::g_last_error; }

int opus_device_error(int* code) {
  if (code == nullptr) return opus::set_error(OPUS_ERR_INVALID, "opus_device_error: code is NULL");
  *code = 0;
  int* w = opus::device_error_word();
  if (w == nullptr) return opus::set_error(OPUS_ERR_CUDA, "device error word unavailable");
  OPUS_CUDA_TRY(cudaDeviceSynchronize());
  int v = 0;
  OPUS_CUDA_TRY(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) {
    OPUS_CUDA_TRY(cudaMemset(w, 0, sizeof(int)));
    *code = v;
    return opus::set_error(OPUS_ERR_DEVICE, "device error word set: 0x%x", v);
  }
  return OPUS_OK;
}

}  // extern "C"
