// demon_host.h -- host-side helpers shared by the C-ABI entry points:
// thread-local error message, argument checks, CUDA error mapping, device
// capability check, and TMA tensor-map encoding through the driver entry point.
#pragma once
#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/demon_b200.h"

namespace demon {

void set_error(const char* fmt, ...);
int check_device();  // DEMON_OK if the current device is sm_100, else DEMON_ERR_UNSUPPORTED/CUDA
unsigned int* status_word();  // device address of the per-device status word (nullptr on failure)

// True until mark_device_done(flags) ran on the current device (per-device once-flags
// for function attributes, which the runtime keeps per device).
bool device_pending(const std::atomic<uint64_t>& flags);
void mark_device_done(std::atomic<uint64_t>& flags);

// 2-D row-major tiled tensor map: `rows` x `cols` elements of `elem_bytes`,
// row pitch `ld_bytes`, box `box_rows` x `box_cols`, given swizzle (default 128-byte).
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols, uint64_t rows,
                 uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// 3-D bf16 tiled tensor map with 128-byte swizzle: `depth` blocks of `rows` x `cols`
// elements (row pitch `ld_bytes`, block pitch `depth_bytes`), box `box_rows` x `box_cols` x 1.
int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t depth,
                      uint64_t ld_bytes, uint64_t depth_bytes, uint32_t box_cols, uint32_t box_rows);

// Host-only argument checks of demon_nvfp4_quantize / demon_nvfp4_gemm (no CUDA call, no
// launch): DEMON_OK, or DEMON_ERR_INVALID with the message set.  The entry points run them
// first; callers that chain both kernels run both before launching either.
int quantize_check(const void* x, int64_t M, int64_t K, int64_t ldx, int gs_mode, const float* gs,
                   const uint8_t* codes, const uint8_t* sf);
int gemm_check(const DemonGemmArgs* a);

}  // namespace demon

#define DEMON_API_BEGIN()                   \
  do {                                      \
    int _dev_rc = ::demon::check_device();  \
    if (_dev_rc != DEMON_OK) return _dev_rc; \
  } while (0)

#define DEMON_CHECK_ARG(cond, ...)      \
  do {                                  \
    if (!(cond)) {                      \
      ::demon::set_error(__VA_ARGS__);  \
      return DEMON_ERR_INVALID;         \
    }                                   \
  } while (0)

#define DEMON_CUDA(call)                                                               \
  do {                                                                                 \
    cudaError_t _e = (call);                                                           \
    if (_e != cudaSuccess) {                                                           \
      ::demon::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(_e), __FILE__, __LINE__); \
      return DEMON_ERR_CUDA;                                                           \
    }                                                                                  \
  } while (0)
