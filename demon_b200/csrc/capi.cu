// capi.cu -- C-ABI utilities: thread-local error messages, device checks,
// the per-device status word written by bounded device-side waits, and TMA
// tensor-map encoding through the CUDA driver entry point (no -lcuda needed).
#include <atomic>
#include <cstring>
#include <cudaTypedefs.h>
#include <mutex>

#include "demon_common.cuh"
#include "demon_host.h"

// Per-device status word: [0] = DEMON_DEV_* bits, [1] = first failing site.
__device__ unsigned int g_demon_status[2];

namespace demon {

namespace {
thread_local char g_err[1024] = {0};
constexpr int kMaxDev = 64;
std::atomic<int> g_dev_ok[kMaxDev];           // 0 unknown, 1 ok, 2 unsupported
std::atomic<unsigned int*> g_status_ptr[kMaxDev];
std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
}

int check_device() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("cudaGetDevice failed: %s", cudaGetErrorString(e));
    return DEMON_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDev) {
    set_error("device ordinal %d out of range", dev);
    return DEMON_ERR_INVALID;
  }
  int s = g_dev_ok[dev].load(std::memory_order_acquire);
  if (s == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
      set_error("cannot query compute capability of device %d", dev);
      return DEMON_ERR_CUDA;
    }
    s = (major == 10 && minor == 0) ? 1 : 2;
    g_dev_ok[dev].store(s, std::memory_order_release);
  }
  if (s != 1) {
    set_error("device %d is not sm_100 (B200); this library is built for sm_100a only", dev);
    return DEMON_ERR_UNSUPPORTED;
  }
  return DEMON_OK;
}

unsigned int* status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  unsigned int* p = g_status_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_demon_status) != cudaSuccess) return nullptr;
    p = static_cast<unsigned int*>(addr);
    g_status_ptr[dev].store(p, std::memory_order_release);
  }
  return p;
}

static uint64_t device_bit() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 0;
  return 1ull << dev;
}

bool device_pending(const std::atomic<uint64_t>& flags) {
  return (flags.load(std::memory_order_acquire) & device_bit()) == 0;
}

void mark_device_done(std::atomic<uint64_t>& flags) { flags.fetch_or(device_bit(), std::memory_order_acq_rel); }

static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols, uint64_t rows,
                 uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  if (!encoder()) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return DEMON_ERR_CUDA;
  }
  if (((uintptr_t)base & 15) != 0 || (ld_bytes & 15) != 0) {
    set_error("TMA operand must be 16-byte aligned with a 16-byte multiple row pitch (ld=%llu)",
              (unsigned long long)ld_bytes);
    return DEMON_ERR_INVALID;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): dims %llux%llu ld %llu box %ux%u", (int)r,
              (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)ld_bytes, box_cols, box_rows);
    return DEMON_ERR_INVALID;
  }
  return DEMON_OK;
}

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t depth,
                      uint64_t ld_bytes, uint64_t depth_bytes, uint32_t box_cols, uint32_t box_rows) {
  if (!encoder()) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return DEMON_ERR_CUDA;
  }
  if (((uintptr_t)base & 15) != 0 || (ld_bytes & 15) != 0 || (depth_bytes & 15) != 0) {
    set_error("TMA operand must be 16-byte aligned with 16-byte multiple pitches (ld=%llu, depth pitch=%llu)",
              (unsigned long long)ld_bytes, (unsigned long long)depth_bytes);
    return DEMON_ERR_INVALID;
  }
  const cuuint64_t dims[3] = {cols, rows, depth};
  const cuuint64_t strides[2] = {ld_bytes, depth_bytes};
  const cuuint32_t box[3] = {box_cols, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): dims %llux%llux%llu pitches %llu/%llu box %ux%u", (int)r,
              (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)depth,
              (unsigned long long)ld_bytes, (unsigned long long)depth_bytes, box_cols, box_rows);
    return DEMON_ERR_INVALID;
  }
  return DEMON_OK;
}

}  // namespace demon

extern "C" int demon_abi_version(void) { return DEMON_ABI_VERSION; }

extern "C" int demon_struct_sizes(int64_t* gemm_args, int64_t* ode_slot) {
  if (!gemm_args || !ode_slot) return DEMON_ERR_INVALID;
  *gemm_args = (int64_t)sizeof(DemonGemmArgs);
  *ode_slot = (int64_t)sizeof(DemonOdeSlot);
  return DEMON_OK;
}

extern "C" int demon_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return DEMON_ERR_INVALID;
  strncpy(buf, demon::g_err, n - 1);
  buf[n - 1] = '\0';
  return DEMON_OK;
}

extern "C" int demon_device_status(unsigned int* out_host, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(out_host != nullptr, "device_status: null output");
  unsigned int* p = demon::status_word();
  DEMON_CHECK_ARG(p != nullptr, "device_status: status word unavailable");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  DEMON_CUDA(cudaMemcpyAsync(out_host, p, 2 * sizeof(unsigned int), cudaMemcpyDeviceToHost, st));
  DEMON_CUDA(cudaMemsetAsync(p, 0, 2 * sizeof(unsigned int), st));
  DEMON_CUDA(cudaStreamSynchronize(st));
  return DEMON_OK;
}
