// nvfp4_quant.cu -- NVFP4 activation quantiser for sm_100a.
//
// bf16 [M, K] -> E2M1 codes [M, K/2] + E4M3 block scales (16 elements along K,
// tcgen05 128x4-chunk layout) + fp32 global scale(s).
//
// Arithmetic, step by step (identical to the CPU restatement the tests check
// against; every step is one IEEE binary32 round-to-nearest-even operation):
//   g     = max(amax, 1e-12) / 2688                 (per row, per tensor or given)
//   s_b   = e4m3_rne(min(amax_b / (6 g), 448))       clamp before the cast, as the
//                                                   reference's FP8 re-quantiser does
//                                                   (acestep/engine/trt/lora_refit.py:598-601)
//   code  = e2m1_rne(x * (1 / (f32(s_b) * g)))      saturating at 6, zero -> code 0
// The absmax floor 1e-12 is the reference's FP8 floor (acestep/engine/trt/fp8_onnx.py:67).
//
// Layout of the work (fast path): each lane owns whole 16-element blocks (two 128-bit
// loads); a block's codes are one 64-bit store (a warp writes 256 contiguous bytes) and
// the four block scales that are contiguous in the scale layout are gathered by
// shuffles into one 32-bit store.  Other widths: one warp per row, lanes (2i, 2i+1)
// share a block.
#include <algorithm>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "demon_common.cuh"
#include "demon_host.h"
#include "nvfp4_row.cuh"

namespace demon {

constexpr int kQuantWarps = 8;

// Row absmax over the whole tensor -> atomicMax on the float bits in *amax_out
// (valid because every candidate is a non-negative float).
__global__ void __launch_bounds__(256) amax_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int64_t K,
                                                   int64_t ldx, float* amax_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * kQuantWarps + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * kQuantWarps;
  float a = 0.0f;
  for (int64_t m = warp; m < M; m += nwarps) {
    const uint4* row = reinterpret_cast<const uint4*>(x + m * ldx);
    for (int64_t c = lane; c < K / 8; c += 32) a = fmaxf(a, amax8(__ldg(row + c)));
  }
  a = warp_max(a);
  __shared__ float red[kQuantWarps];
  if (lane == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = red[0];
    for (int i = 1; i < kQuantWarps; ++i) b = fmaxf(b, red[i]);
    atomicMax(reinterpret_cast<int*>(amax_out), __float_as_int(b));
  }
}

__global__ void finalize_gs_kernel(float* gs) { gs[0] = global_scale(gs[0]); }

// GS_MODE: 0 static (gs[0] is g), 1 dynamic (gs[0] holds amax, g derived), 2 per row.
// Generic path (any K % 64 == 0): one warp per row, the row streamed in
// 32-chunk steps (per-row mode reads it twice, the second time from L1/L2).
template <int GS_MODE>
__global__ void __launch_bounds__(256) quantize_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int64_t K,
                                                       int64_t ldx, int64_t Mpad, float* __restrict__ gs,
                                                       uint8_t* __restrict__ codes, uint8_t* __restrict__ sf) {
  const int lane = threadIdx.x & 31;
  const int64_t m = (int64_t)blockIdx.x * kQuantWarps + (threadIdx.x >> 5);
  if (m >= Mpad) return;
  const int64_t nchunk = K / 8;      // 8-element chunks per row
  const int64_t kchunks64 = K / 64;  // scale chunks per 128-row block
  const int64_t r = m & 127;
  uint8_t* sf_rowbase = sf + (m >> 7) * kchunks64 * 512 + (r & 31) * 16 + (r >> 5) * 4;
  if (m >= M) {  // padding rows of the scale layout: zero scales
    for (int64_t c = lane; c < K / 64; c += 32) *reinterpret_cast<uint32_t*>(sf_rowbase + c * 512) = 0u;
    return;
  }
  const uint4* row = reinterpret_cast<const uint4*>(x + m * ldx);
  uint32_t* code_row = reinterpret_cast<uint32_t*>(codes + m * (K / 2));
  float g;
  if (GS_MODE == 0) {
    g = gs[0];
  } else if (GS_MODE == 1) {
    g = global_scale(gs[0]);
  } else {
    float a = 0.0f;
    for (int64_t c = lane; c < nchunk; c += 32) a = fmaxf(a, amax8(__ldg(row + c)));
    g = global_scale(warp_max(a));
    if (lane == 0) gs[m] = g;
  }
  const float denom = __fmul_rn(6.0f, g);
  // K % 64 == 0 makes the valid lanes of the last iteration whole groups of 8.
  for (int64_t base = 0; base < nchunk; base += 32) {
    const int64_t c = base + lane;
    const bool valid = c < nchunk;
    const uint4 v = valid ? __ldg(row + c) : make_uint4(0u, 0u, 0u, 0u);
    quant_chunk(v, valid, c, lane, g, denom, code_row, sf_rowbase);
  }
}

// Fast path for the row widths of the DiT (K in {512, 1024, 2048, 3072, 4096, 6144, 8192}):
// each lane owns whole 16-element scale blocks (two 128-bit loads per block, all loads of
// the lane in flight at once), so a block's scale is computed once; a row is held by W
// warps whose per-row absmax meets in shared memory; 8 / W rows per 256-thread CTA.
// Warps per row of the quantiser: one warp per row (4 blocks per lane, 8 rows per CTA, no
// shared-memory reduction) at K = 2048, where it measured faster on B200 than the wider split.
template <int K>
constexpr int quant_warps() {
  return K == 2048 ? 1 : 0;
}

template <int GS_MODE, int K>
__global__ void __launch_bounds__(256) quantize_blocks_kernel(const __nv_bfloat16* __restrict__ x, int64_t M,
                                                              int64_t ldx, int64_t Mpad, float* __restrict__ gs,
                                                              uint8_t* __restrict__ codes, uint8_t* __restrict__ sf) {
  using G = RowQ<K, quant_warps<K>()>;
  __shared__ float red[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wr = warp % G::W;
  const int64_t m = (int64_t)blockIdx.x * G::R + warp / G::W;
  const int64_t r = m & 127;
  uint8_t* sf_rowbase = sf + (m >> 7) * (K / 64) * 512 + (r & 31) * 16 + (r >> 5) * 4;
  const bool pad = m >= M;
  const uint4* row = reinterpret_cast<const uint4*>(x + (pad ? 0 : m) * ldx);
  const bool lane_ok = G::kBPR >= 32 || lane < G::kBPR;
  uint4 a[G::NB], b[G::NB];
#pragma unroll
  for (int j = 0; j < G::NB; ++j) {
    const int64_t kb = (int64_t)(wr * G::NB + j) * 32 + lane;
    if (!pad && lane_ok) {
      a[j] = __ldg(row + 2 * kb);
      b[j] = __ldg(row + 2 * kb + 1);
    } else {
      a[j] = b[j] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  uint32_t ma[G::NB], mb[G::NB];
#pragma unroll
  for (int j = 0; j < G::NB; ++j) {
    ma[j] = absmax_bits8(a[j]);
    mb[j] = absmax_bits8(b[j]);
  }
  float g = 0.0f;
  if (GS_MODE == 0) {
    g = gs[0];
  } else if (GS_MODE == 1) {
    g = global_scale(gs[0]);
  } else {
    const float am = fmaxf(lane_absmax(a, ma), lane_absmax(b, mb));
    g = global_scale(row_reduce<G::W, true>(am, red, warp, lane));
    if (wr == 0 && lane == 0 && !pad) gs[m] = g;
  }
  if (m >= Mpad) return;
  if (pad) {  // padding rows of the scale layout: zero scales
    for (int64_t c = wr * 32 + lane; c < K / 64; c += 32 * G::W) *reinterpret_cast<uint32_t*>(sf_rowbase + c * 512) = 0u;
    return;
  }
  const float denom = __fmul_rn(6.0f, g);
  uint8_t* code_row = codes + m * (K / 2);
#pragma unroll
  for (int j = 0; j < G::NB; ++j) {
    const int64_t kb = (int64_t)(wr * G::NB + j) * 32 + lane;
    store_block(quant_block_m(a[j], b[j], ma[j], mb[j], g, denom), lane_ok, kb, lane, code_row, sf_rowbase);
  }
}

template <int GS_MODE, int K>
void launch_blocks(cudaStream_t st, const __nv_bfloat16* x, int64_t M, int64_t ldx, int64_t Mpad, float* gs,
                   uint8_t* codes, uint8_t* sf) {
  constexpr int R = RowQ<K, quant_warps<K>()>::R;
  quantize_blocks_kernel<GS_MODE, K><<<(unsigned)((Mpad + R - 1) / R), 256, 0, st>>>(x, M, ldx, Mpad, gs, codes, sf);
}

template <int GS_MODE>
void launch_quantize(cudaStream_t st, const __nv_bfloat16* x, int64_t M, int64_t K, int64_t ldx, int64_t Mpad,
                     float* gs, uint8_t* codes, uint8_t* sf) {
  switch (K) {
    case 512: launch_blocks<GS_MODE, 512>(st, x, M, ldx, Mpad, gs, codes, sf); return;
    case 1024: launch_blocks<GS_MODE, 1024>(st, x, M, ldx, Mpad, gs, codes, sf); return;
    case 2048: launch_blocks<GS_MODE, 2048>(st, x, M, ldx, Mpad, gs, codes, sf); return;
    case 3072: launch_blocks<GS_MODE, 3072>(st, x, M, ldx, Mpad, gs, codes, sf); return;
    case 4096: launch_blocks<GS_MODE, 4096>(st, x, M, ldx, Mpad, gs, codes, sf); return;
    case 6144: launch_blocks<GS_MODE, 6144>(st, x, M, ldx, Mpad, gs, codes, sf); return;
    case 8192: launch_blocks<GS_MODE, 8192>(st, x, M, ldx, Mpad, gs, codes, sf); return;
    default: {
      const dim3 grid((unsigned)((Mpad + kQuantWarps - 1) / kQuantWarps));
      quantize_kernel<GS_MODE><<<grid, 256, 0, st>>>(x, M, K, ldx, Mpad, gs, codes, sf);
    }
  }
}

}  // namespace demon

using namespace demon;

extern "C" int64_t demon_nvfp4_sf_bytes(int64_t rows, int64_t K) {
  if (rows < 0 || K < 0) return -1;
  return ((rows + 127) / 128) * 128 * (K / 16);
}

namespace demon {
int quantize_check(const void* x, int64_t M, int64_t K, int64_t ldx, int gs_mode, const float* gs,
                   const uint8_t* codes, const uint8_t* sf) {
  DEMON_CHECK_ARG(M >= 0 && K > 0 && K % 64 == 0, "quantize: need K > 0, K %% 64 == 0 (K=%lld)", (long long)K);
  DEMON_CHECK_ARG(ldx >= K && ldx % 8 == 0, "quantize: ldx must be >= K and a multiple of 8 (ldx=%lld)",
                  (long long)ldx);
  DEMON_CHECK_ARG(gs_mode >= 0 && gs_mode <= 2, "quantize: bad gs_mode %d", gs_mode);
  DEMON_CHECK_ARG(gs != nullptr && (M == 0 || (x && codes && sf)), "quantize: null pointer");
  DEMON_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)codes & 3) == 0 && ((uintptr_t)sf & 3) == 0,
                  "quantize: x must be 16-byte aligned, codes/sf 4-byte aligned");
  return DEMON_OK;
}
}  // namespace demon

extern "C" int demon_nvfp4_quantize(const void* x, int64_t M, int64_t K, int64_t ldx, int gs_mode, float* gs,
                                    uint8_t* codes, uint8_t* sf, void* stream) {
  DEMON_API_BEGIN();
  const int rc0 = demon::quantize_check(x, M, K, ldx, gs_mode, gs, codes, sf);
  if (rc0 != DEMON_OK) return rc0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t Mpad = (M + 127) / 128 * 128;
  if (Mpad == 0) return DEMON_OK;
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  if (gs_mode == DEMON_GS_STATIC) {
    launch_quantize<0>(st, xb, M, K, ldx, Mpad, gs, codes, sf);
  } else if (gs_mode == DEMON_GS_DYNAMIC) {
    DEMON_CUDA(cudaMemsetAsync(gs, 0, sizeof(float), st));
    if (M > 0) {
      const int blocks = (int)std::min<int64_t>((M + kQuantWarps - 1) / kQuantWarps, 148 * 8);
      amax_kernel<<<blocks, 256, 0, st>>>(xb, M, K, ldx, gs);
    }
    launch_quantize<1>(st, xb, M, K, ldx, Mpad, gs, codes, sf);
    finalize_gs_kernel<<<1, 1, 0, st>>>(gs);
  } else {
    launch_quantize<2>(st, xb, M, K, ldx, Mpad, gs, codes, sf);
  }
  DEMON_CUDA(cudaGetLastError());
  return DEMON_OK;
}
