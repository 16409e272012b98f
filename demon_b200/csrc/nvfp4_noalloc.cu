// nvfp4_noalloc.cu -- NVFP4 linear (quantise + block-scaled GEMM) that allocates nothing.
//
// Some callers cannot call cudaMalloc while they run this layer: a TensorRT
// plugin's enqueue() must not allocate device memory (TensorRT hands out the
// only workspace it allows), and a real-time audio thread must not block on
// the CUDA allocator (cudaMalloc / cudaFree can synchronise the device).  The
// regular path needs three intermediate buffers between its two kernels (the
// activation's E2M1 codes, block scales and per-row global scales), which the
// caller normally provides.  This entry point keeps them instead in one
// file-scope device array of fixed size, so the caller passes only the inputs
// (x and the packed weight) and the output.
//
// Limits and behaviour:
//   - the array is 4.875 MiB (demon_nvfp4_noalloc_scratch_bytes()).  It belongs to this
//     library's device code: with CUDA's default lazy module loading it is set up in a
//     device's context when the library's module is first loaded there (at the latest on
//     the first call of this entry point on that device) and stays until the context ends;
//   - it holds at most M * K <= 8,388,608 activation elements (4 MiB of codes),
//     block scales of up to 640 KiB and per-row scales for up to 65,536 rows;
//     larger calls are rejected with DEMON_ERR_INVALID before anything runs;
//   - every argument check of both kernels (shape, strides, alignment, null pointers)
//     runs on the host before the first launch, so a rejected call launches nothing and
//     leaves the array untouched;
//   - the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current); that lookup can
//     also be where the module gets loaded, so make the first call before any stream
//     capture;
//   - every call on a device shares the array and leaves the last call's
//     contents in it.  Nothing in it has to start at zero: the per-row
//     quantiser rewrites every code, block scale (padding rows included) and
//     row scale that the GEMM then reads.  Calls whose work overlaps on the
//     GPU (two streams, or two host threads without ordering) race on the
//     array; serialise them on one stream.
#include <atomic>
#include <cstring>

#include "demon_common.cuh"
#include "demon_host.h"

static constexpr int64_t kCodesBytes = 4ll << 20;  // E2M1 codes: M * K / 2
static constexpr int64_t kSfBytes = 640ll << 10;   // block scales: ceil(M/128)*128 * K/16
static constexpr int64_t kGsRows = 65536;          // per-row global scales (fp32)
static constexpr int64_t kScratchBytes = kCodesBytes + kSfBytes + kGsRows * 4;

// The scratch itself.  In host code this name is only a stand-in for the
// device symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

namespace {

constexpr int kMaxDev = 64;
std::atomic<uint8_t*> g_scratch_ptr[kMaxDev];

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_ptr(uint8_t** out) {
  int dev = 0;
  DEMON_CUDA(cudaGetDevice(&dev));
  DEMON_CHECK_ARG(dev >= 0 && dev < kMaxDev, "noalloc: device ordinal %d out of range", dev);
  uint8_t* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
    if (e != cudaSuccess || addr == nullptr) {
      demon::set_error("noalloc: cudaGetSymbolAddress of the scratch array failed: %s", cudaGetErrorString(e));
      return DEMON_ERR_CUDA;
    }
    p = static_cast<uint8_t*>(addr);
    g_scratch_ptr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return DEMON_OK;
}

}  // namespace

extern "C" int64_t demon_nvfp4_noalloc_scratch_bytes(void) { return kScratchBytes; }

extern "C" int demon_nvfp4_linear_noalloc(const void* x, int64_t M, int64_t K, int64_t ldx, const uint8_t* w_codes,
                                          const uint8_t* w_sf, const float* w_gs, int64_t N, const void* bias,
                                          void* out, int64_t ldo, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(M >= 0 && K > 0 && N > 0 && K % 256 == 0, "noalloc: bad shape M=%lld K=%lld N=%lld (K %% 256 == 0)",
                  (long long)M, (long long)K, (long long)N);
  DEMON_CHECK_ARG(M * (K / 2) <= kCodesBytes,
                  "noalloc: M*K = %lld exceeds the scratch limit of %lld activation elements", (long long)(M * K),
                  (long long)(2 * kCodesBytes));
  DEMON_CHECK_ARG(demon_nvfp4_sf_bytes(M, K) <= kSfBytes,
                  "noalloc: block scales need %lld bytes, the scratch holds %lld", (long long)demon_nvfp4_sf_bytes(M, K),
                  (long long)kSfBytes);
  DEMON_CHECK_ARG(M <= kGsRows, "noalloc: M=%lld exceeds the %lld-row limit", (long long)M, (long long)kGsRows);
  uint8_t* base = nullptr;
  const int rc0 = scratch_ptr(&base);
  if (rc0 != DEMON_OK) return rc0;
  uint8_t* codes = base;
  uint8_t* sf = base + kCodesBytes;
  float* gs = reinterpret_cast<float*>(base + kCodesBytes + kSfBytes);
  DemonGemmArgs g;
  memset(&g, 0, sizeof g);
  g.a_codes = codes;
  g.a_sf = sf;
  g.a_gs = gs;
  g.a_gs_per_row = 1;
  g.w_codes = w_codes;
  g.w_sf = w_sf;
  g.w_gs = w_gs;
  g.M = M;
  g.N = N;
  g.K = K;
  g.out = out;
  g.ldo = ldo;
  g.bias = bias;
  // both kernels' argument checks before either launches: a rejected call leaves the array alone
  int rc = demon::quantize_check(x, M, K, ldx, DEMON_GS_PER_ROW, gs, codes, sf);
  if (rc != DEMON_OK) return rc;
  rc = demon::gemm_check(&g);
  if (rc != DEMON_OK) return rc;
  if (M == 0) return DEMON_OK;
  rc = demon_nvfp4_quantize(x, M, K, ldx, DEMON_GS_PER_ROW, gs, codes, sf, stream);
  if (rc != DEMON_OK) return rc;
  return demon_nvfp4_gemm(&g, stream);
}
