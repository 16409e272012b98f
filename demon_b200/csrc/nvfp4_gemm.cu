// nvfp4_gemm.cu -- tcgen05 block-scaled NVFP4 GEMM with fused epilogue (sm_100a),
// and the bf16 tcgen05 GEMM used for the LoRA down-projection.
//
// One CTA computes a 128 x BN output tile.  Warp roles (192 threads):
//   warp 0      TMA producer: A/B tiles with tiled TMA loads (128-byte swizzle,
//               no multicast) and the block scales of the stage with untiled
//               bulk copies -- the quantiser writes scales directly in the
//               tcgen05 128x4-chunk layout, so a stage's scales are contiguous.
//   warp 1      TMEM allocation + a single MMA-issuing thread: per stage it
//               copies the scales SMEM -> TMEM (tcgen05.cp 32x128b.warpx4,
//               replicated into the four lane quadrants), then issues four
//               tcgen05.mma.kind::mxf4nvf4.block_scale.block16 (K = 64 each),
//               and commits to the stage's "empty" barrier.
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (one row per
//               thread), alpha * acc + bias, optional gate * y and residual +,
//               bf16 stores.
// Hot LoRA: the rank-r product xa . B^T is one extra group of kind::f16 MMAs
// into the same TMEM accumulator before the FP4 K-loop; xa is pre-divided by
// alpha and pre-multiplied by the strength (demon_lora_down), so changing the
// strength never touches the packed weights.
//
// Every mbarrier wait is bounded (demon_common.cuh); on expiry the CTA records
// DEMON_DEV_TIMEOUT, stops issuing, drains what it issued and frees TMEM.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "demon_common.cuh"
#include "demon_host.h"

namespace demon {

struct GemmParams {
  const uint8_t* a_sf;
  const uint8_t* w_sf;
  const float* a_gs;
  const float* w_gs;
  const float* col_scale;  // bf16 mode: per-output-column scale
  __nv_bfloat16* out;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* gate;
  unsigned int* status;
  int64_t ldo, ldr, gate_rows, ld_gate;
  int M, N, K;
  int a_gs_per_row;
  int lora_rank;
};

constexpr int kBM = 128;
constexpr int kRowBytes = 128;  // one 128-byte swizzle row per stage (256 fp4 / 64 bf16)

template <int BN, int STAGES, bool FP4, int LBOX>
struct GemmCfg {
  static constexpr int kA = kBM * kRowBytes;
  static constexpr int kB = BN * kRowBytes;
  static constexpr int kSFA = FP4 ? 2048 : 0;
  static constexpr int kSFB = FP4 ? (BN / 128) * 2048 : 0;
  static constexpr int kLoraBoxes = LBOX;  // LoRA boxes of 64 bf16 along the rank
  static constexpr int kLA = kBM * kRowBytes;
  static constexpr int kLB = BN * kRowBytes;
  static constexpr int offA = 0;
  static constexpr int offB = offA + STAGES * kA;
  static constexpr int offLA = offB + STAGES * kB;
  static constexpr int offLB = offLA + kLoraBoxes * kLA;
  static constexpr int offSFA = offLB + kLoraBoxes * kLB;
  static constexpr int offSFB = offSFA + STAGES * kSFA;
  static constexpr int offBar = offSFB + STAGES * kSFB;
  static constexpr int kBars = 2 * STAGES + 2;
  static constexpr int offMisc = offBar + kBars * 8;
  static constexpr int kSmem = offMisc + 16 + 1024;  // + alignment slack
  static constexpr int kAccCols = BN;
  static constexpr int kSfaCol = BN;            // 4 columns per K=64 step, 4 steps
  static constexpr int kSfbCol = BN + 16;       // BN/32 columns per step, 4 steps
  static constexpr int kUsedCols = FP4 ? BN + 16 + (BN / 32) * 4 : BN;
  static constexpr uint32_t kTmemCols = kUsedCols <= 32 ? 32 : kUsedCols <= 64 ? 64 : kUsedCols <= 128 ? 128
                                        : kUsedCols <= 256 ? 256 : 512;
  static constexpr int kStepElems = FP4 ? 256 : 64;  // K elements per stage
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
};

__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
  // K-major, 128-byte swizzle: 8-row core groups 1024 bytes apart.
  return smem_desc(smem_u32(p), 16, 1024, 2);
}
__device__ __forceinline__ uint64_t sf_desc(const void* p) {
  // 32 rows x 16 bytes, no swizzle: 8-row core matrices 128 bytes apart.
  return smem_desc(smem_u32(p), 0, 128, 0);
}

template <int BN, int STAGES, bool FP4, int LBOX>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmLB,
                const GemmParams p) {
  using C = GemmCfg<BN, STAGES, FP4, LBOX>;
  constexpr bool LORA = LBOX > 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::offBar);
  uint64_t* empty = full + STAGES;
  uint64_t* lora_full = empty + STAGES;
  uint64_t* acc_full = lora_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::offMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::offMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_blk = blockIdx.x, m_blk = blockIdx.y;
  const int m0 = m_blk * kBM, n0 = n_blk * BN;
  const int KT = p.K / C::kStepElems;
  const uint64_t t0 = globaltimer();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(lora_full, 1);
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (LORA) {
      prefetch_tmap(&tmLA);
      prefetch_tmap(&tmLB);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int issued = 0;
      const int lboxes = LORA ? (p.lora_rank + 63) / 64 : 0;
      if (LORA) {
        mbar_arrive_expect_tx(lora_full, (uint32_t)lboxes * (C::kLA + C::kLB));
        for (int b = 0; b < lboxes; ++b) {
          tma_load_2d(smem + C::offLA + b * C::kLA, &tmLA, lora_full, b * 64, m0);
          tma_load_2d(smem + C::offLB + b * C::kLB, &tmLB, lora_full, b * 64, n0);
        }
      }
      // scale halves of the B tile that exist in the (128-row padded) scale buffer
      const int sfb_halves = FP4 ? std::min(BN / 128, (p.N - n0 + 127) / 128) : 0;
      const uint32_t tx = (uint32_t)(C::kA + C::kB + C::kSFA + sfb_halves * 2048);
      const int64_t kchunks = p.K / 64;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, t0, p.status, 1)) break;
        mbar_arrive_expect_tx(&full[s], tx);
        const int kx = FP4 ? kt * kRowBytes : kt * 64;
        tma_load_2d(smem + C::offA + s * C::kA, &tmA, &full[s], kx, m0);
        tma_load_2d(smem + C::offB + s * C::kB, &tmB, &full[s], kx, n0);
        if (FP4) {
          bulk_load(smem + C::offSFA + s * C::kSFA, p.a_sf + ((int64_t)m_blk * kchunks + kt * 4) * 512, 2048,
                    &full[s]);
          for (int h = 0; h < sfb_halves; ++h)
            bulk_load(smem + C::offSFB + s * C::kSFB + h * 2048,
                      p.w_sf + ((int64_t)(n_blk * (BN / 128) + h) * kchunks + kt * 4) * 512, 2048, &full[s]);
        }
        ++issued;
      }
      // drain: never leave the CTA with copies in flight (no-op on the normal path)
      for (int i = std::max(0, issued - STAGES); i < issued; ++i) {
        volatile int never = 0;
        mbar_wait(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u, &never, globaltimer(), p.status, 2);
      }
      if (LORA) {
        volatile int never = 0;
        mbar_wait(lora_full, 0, &never, globaltimer(), p.status, 3);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      const uint32_t idesc = FP4 ? idesc_mxf4nvf4(kBM, BN) : idesc_bf16(kBM, BN);
      const uint32_t d_acc = tmem;
      uint32_t accum = 0;
      bool ok = true;
      if (LORA) {
        ok = mbar_wait(lora_full, 0, abort_flag, t0, p.status, 4);
        if (ok) {
          tc_fence_after();
          const uint32_t ib = idesc_bf16(kBM, BN);
          for (int b = 0; b < LBOX; ++b) {
            const uint64_t la = sw128_desc(smem + C::offLA + b * C::kLA);
            const uint64_t lb = sw128_desc(smem + C::offLB + b * C::kLB);
            for (int j = 0; j < 4; ++j) {
              if (b * 64 + j * 16 < p.lora_rank) {
                mma_bf16(d_acc, la + 2 * j, lb + 2 * j, ib, accum);
                accum = 1;
              }
            }
          }
        }
      }
      for (int kt = 0; ok && kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (uint32_t)(kt / STAGES) & 1u;
        if (!mbar_wait(&full[s], ph, abort_flag, t0, p.status, 5)) break;
        tc_fence_after();
        const uint64_t adesc = sw128_desc(smem + C::offA + s * C::kA);
        const uint64_t bdesc = sw128_desc(smem + C::offB + s * C::kB);
        if (FP4) {
          const uint8_t* sfa = smem + C::offSFA + s * C::kSFA;
          const uint8_t* sfb = smem + C::offSFB + s * C::kSFB;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            tc_cp_32x128b_warpx4(tmem + C::kSfaCol + 4 * j, sf_desc(sfa + j * 512));
#pragma unroll
            for (int h = 0; h < BN / 128; ++h)
              tc_cp_32x128b_warpx4(tmem + C::kSfbCol + (BN / 32) * j + 4 * h, sf_desc(sfb + h * 2048 + j * 512));
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            mma_mxf4nvf4(d_acc, adesc + 2 * j, bdesc + 2 * j, idesc, tmem + C::kSfaCol + 4 * j,
                         tmem + C::kSfbCol + (BN / 32) * j, accum);
            accum = 1;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            mma_bf16(d_acc, adesc + 2 * j, bdesc + 2 * j, idesc, accum);
            accum = 1;
          }
        }
        tc_commit(&empty[s]);
      }
      tc_commit(acc_full);
      // wait for our own MMAs before anyone frees TMEM (returns at once normally)
      volatile int never = 0;
      mbar_wait(acc_full, 0, &never, globaltimer(), p.status, 6);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant accessible to this warp
    const int64_t row = (int64_t)m0 + q * 32 + lane;
    const bool ok = mbar_wait(acc_full, 0, abort_flag, t0, p.status, 7);
    tc_fence_after();
    if (ok && !*abort_flag) {
      const bool row_ok = row < p.M;
      const float ga = row_ok ? p.a_gs[p.a_gs_per_row ? row : 0] : 0.0f;
      const float alpha = ga * p.w_gs[0];
      const __nv_bfloat16* gate_row = (FP4 && p.gate && row_ok) ? p.gate + (row / p.gate_rows) * p.ld_gate : nullptr;
#pragma unroll 1
      for (int c = 0; c < (BN + 31) / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
        tmem_ld_wait();
        const int n = n0 + c * 32;
        if (!row_ok) continue;
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
          const int nn = n + g8 * 8;
          if (nn >= p.N || c * 32 + g8 * 8 >= BN) break;
          float y[8];
          if (FP4) {
            uint4 bb = make_uint4(0u, 0u, 0u, 0u);
            if (p.bias) bb = *reinterpret_cast<const uint4*>(p.bias + nn);
            const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              y[2 * i] = fmaf(alpha, __uint_as_float(v[g8 * 8 + 2 * i]), bf16_lo(bw[i]));
              y[2 * i + 1] = fmaf(alpha, __uint_as_float(v[g8 * 8 + 2 * i + 1]), bf16_hi(bw[i]));
            }
            if (gate_row) {
              const uint4 gg = *reinterpret_cast<const uint4*>(gate_row + nn);
              const uint32_t gw[4] = {gg.x, gg.y, gg.z, gg.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                y[2 * i] *= bf16_lo(gw[i]);
                y[2 * i + 1] *= bf16_hi(gw[i]);
              }
            }
            if (p.residual) {
              const uint4 rr = *reinterpret_cast<const uint4*>(p.residual + row * p.ldr + nn);
              const uint32_t rw[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                y[2 * i] += bf16_lo(rw[i]);
                y[2 * i + 1] += bf16_hi(rw[i]);
              }
            }
          } else {
            const float inv_alpha = 1.0f / alpha;
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = __uint_as_float(v[g8 * 8 + i]) * (p.col_scale[nn + i] * inv_alpha);
          }
          uint4 o;
          o.x = pack_bf16x2(y[0], y[1]);
          o.y = pack_bf16x2(y[2], y[3]);
          o.z = pack_bf16x2(y[4], y[5]);
          o.w = pack_bf16x2(y[6], y[7]);
          *reinterpret_cast<uint4*>(p.out + row * p.ldo + nn) = o;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int BN, int STAGES, bool FP4, int LBOX>
int launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& la, const CUtensorMap& lb,
                const GemmParams& p, cudaStream_t st) {
  using C = GemmCfg<BN, STAGES, FP4, LBOX>;
  auto kern = gemm_kernel<BN, STAGES, FP4, LBOX>;
  static std::atomic<uint64_t> attr_done{0};
  if (device_pending(attr_done)) {
    DEMON_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    mark_device_done(attr_done);
  }
  const dim3 grid((unsigned)((p.N + BN - 1) / BN), (unsigned)((p.M + kBM - 1) / kBM));
  kern<<<grid, 192, C::kSmem, st>>>(a, b, la, lb, p);
  DEMON_CUDA(cudaGetLastError());
  return DEMON_OK;
}

}  // namespace demon

using namespace demon;

#define DEMON_RC(x)             \
  do {                          \
    int _rc = (x);              \
    if (_rc != DEMON_OK) return _rc; \
  } while (0)

extern "C" int demon_nvfp4_gemm(const DemonGemmArgs* a, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(a != nullptr, "gemm: null args");
  const int64_t M = a->M, N = a->N, K = a->K;
  DEMON_CHECK_ARG(M >= 0 && N > 0 && K > 0, "gemm: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N,
                  (long long)K);
  DEMON_CHECK_ARG(K % 256 == 0, "gemm: K must be a multiple of 256 (K=%lld)", (long long)K);
  DEMON_CHECK_ARG(N % 128 == 0, "gemm: N must be a multiple of 128 (N=%lld)", (long long)N);
  DEMON_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm: dimension too large");
  DEMON_CHECK_ARG(a->a_codes && a->a_sf && a->a_gs && a->w_codes && a->w_sf && a->w_gs && a->out,
                  "gemm: null operand");
  DEMON_CHECK_ARG(a->ldo >= N && a->ldo % 8 == 0 && ((uintptr_t)a->out & 15) == 0,
                  "gemm: out needs ldo >= N, ldo %% 8 == 0, 16-byte alignment");
  DEMON_CHECK_ARG(!a->residual || (a->ldr >= N && a->ldr % 8 == 0 && ((uintptr_t)a->residual & 15) == 0),
                  "gemm: residual needs ldr >= N, ldr %% 8 == 0, 16-byte alignment");
  DEMON_CHECK_ARG(!a->bias || ((uintptr_t)a->bias & 15) == 0, "gemm: bias must be 16-byte aligned");
  DEMON_CHECK_ARG(!a->gate || (a->gate_rows > 0 && a->ld_gate >= N && a->ld_gate % 8 == 0 &&
                               ((uintptr_t)a->gate & 15) == 0),
                  "gemm: gate needs gate_rows > 0, ld_gate >= N, ld_gate %% 8 == 0, 16-byte alignment");
  DEMON_CHECK_ARG(((uintptr_t)a->a_sf & 15) == 0 && ((uintptr_t)a->w_sf & 15) == 0,
                  "gemm: scale buffers must be 16-byte aligned");
  const bool lora = a->lora_xa != nullptr;
  DEMON_CHECK_ARG(!lora || (a->lora_b && a->lora_rank > 0 && a->lora_rank % 16 == 0 && a->lora_rank <= 128),
                  "gemm: LoRA needs lora_b and rank %% 16 == 0, 0 < rank <= 128 (rank=%lld)",
                  (long long)a->lora_rank);
  if (M == 0) return DEMON_OK;
  unsigned int* status = status_word();

  const bool bn256 = (N % 256 == 0) && !(lora && a->lora_rank > 64);
  const uint32_t BN = bn256 ? 256 : 128;
  CUtensorMap ta, tb, tla, tlb;
  memset(&tla, 0, sizeof tla);
  memset(&tlb, 0, sizeof tlb);
  DEMON_RC(make_tmap_2d(&ta, a->a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)K / 2, (uint64_t)M,
                        (uint64_t)K / 2, 128, 128));
  DEMON_RC(make_tmap_2d(&tb, a->w_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)K / 2, (uint64_t)N,
                        (uint64_t)K / 2, 128, BN));
  if (lora) {
    const uint64_t r = (uint64_t)a->lora_rank;
    DEMON_RC(make_tmap_2d(&tla, a->lora_xa, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, r, (uint64_t)M, r * 2, 64, 128));
    DEMON_RC(make_tmap_2d(&tlb, a->lora_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, r, (uint64_t)N, r * 2, 64, BN));
  }
  GemmParams p{};
  p.a_sf = a->a_sf;
  p.w_sf = a->w_sf;
  p.a_gs = a->a_gs;
  p.w_gs = a->w_gs;
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a->bias);
  p.residual = reinterpret_cast<const __nv_bfloat16*>(a->residual);
  p.gate = reinterpret_cast<const __nv_bfloat16*>(a->gate);
  p.status = status;
  p.ldo = a->ldo;
  p.ldr = a->ldr;
  p.gate_rows = a->gate_rows > 0 ? a->gate_rows : 1;
  p.ld_gate = a->ld_gate;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.a_gs_per_row = a->a_gs_per_row;
  p.lora_rank = lora ? (int)a->lora_rank : 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (lora) {
    if (bn256) return launch_gemm<256, 3, true, 1>(ta, tb, tla, tlb, p, st);
    return launch_gemm<128, 3, true, 2>(ta, tb, tla, tlb, p, st);
  }
  if (bn256) return launch_gemm<256, 4, true, 0>(ta, tb, tla, tlb, p, st);
  return launch_gemm<128, 4, true, 0>(ta, tb, tla, tlb, p, st);
}

extern "C" int demon_lora_down(const void* x, int64_t M, int64_t K, int64_t ldx, const void* lora_a, int64_t rank,
                               const float* col_scale, const float* a_gs, int a_gs_per_row, const float* w_gs,
                               void* xa, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(M >= 0 && K > 0 && K % 64 == 0, "lora_down: need K %% 64 == 0 (K=%lld)", (long long)K);
  DEMON_CHECK_ARG(rank > 0 && rank % 16 == 0 && rank <= 128, "lora_down: rank %% 16 == 0, rank <= 128 (%lld)",
                  (long long)rank);
  DEMON_CHECK_ARG(ldx >= K && ldx % 8 == 0, "lora_down: ldx must be >= K and a multiple of 8");
  DEMON_CHECK_ARG(x && lora_a && col_scale && a_gs && w_gs && xa, "lora_down: null pointer");
  DEMON_CHECK_ARG(((uintptr_t)xa & 15) == 0, "lora_down: xa must be 16-byte aligned");
  if (M == 0) return DEMON_OK;
  CUtensorMap ta, tb, tz;
  memset(&tz, 0, sizeof tz);
  DEMON_RC(make_tmap_2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, 64,
                        128));
  GemmParams p{};
  p.a_gs = a_gs;
  p.w_gs = w_gs;
  p.col_scale = col_scale;
  p.out = reinterpret_cast<__nv_bfloat16*>(xa);
  p.status = status_word();
  p.ldo = rank;
  p.M = (int)M;
  p.N = (int)rank;
  p.K = (int)K;
  p.a_gs_per_row = a_gs_per_row;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rank <= 64) {
    DEMON_RC(make_tmap_2d(&tb, lora_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)rank,
                          (uint64_t)K * 2, 64, 64));
    return launch_gemm<64, 6, false, 0>(ta, tb, tz, tz, p, st);
  }
  DEMON_RC(make_tmap_2d(&tb, lora_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)rank,
                        (uint64_t)K * 2, 64, 128));
  return launch_gemm<128, 6, false, 0>(ta, tb, tz, tz, p, st);
}
