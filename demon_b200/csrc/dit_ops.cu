// dit_ops.cu -- the row kernels of the DiT decoder that sit between its NVFP4 GEMMs (sm_100a).
//
//   demon_adanorm_quantize   RMSNorm (+ AdaLN scale/shift) of the residual stream, written
//                            straight into the NVFP4 operand of the next GEMM (and/or bf16)
//   demon_silu_mul_quantize  MLP: silu(gate) * up -> NVFP4 operand of down_proj
//   demon_head_norm_rope     per-head RMSNorm of q / k (+ rotary embedding), in place
//
// Each output row is computed by a fixed set of lanes in a fixed order, independent of how
// many rows the launch has, so a slot's result never depends on the batch it shares
// (the streaming ring and the single-request path give identical bits).
//
// bf16 rounding follows the reference's eager ops one by one (Qwen3RMSNorm, the AdaLN
// modulation and the rotary embedding of acestep/models/modeling_acestep_v15_turbo.py):
// every tensor the reference materialises in bf16 is rounded to bf16 here too.
#include <algorithm>

#include "demon_common.cuh"
#include "demon_host.h"
#include "nvfp4_row.cuh"

namespace demon {

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) { return pack_bf16x2(lo, hi); }

// Row-block geometry shared by the fused row kernels: a row of D = W * 256 * NCH elements is
// held by W warps; lane l of row-warp w owns the 8-element chunks c = w*32*NCH + 32 j + l, so
// lanes (2i, 2i+1) own one 16-element scale block, as in the activation quantiser.
template <int W, int NCH>
struct RowGeo {
  static constexpr int kRowsPerCta = 8 / W;
  static constexpr int kD = W * 256 * NCH;
};

// Cross-warp reduction of one value per row (sum or max) through shared memory.
template <int W, bool MAX>
__device__ __forceinline__ float row_reduce(float v, float* red, int warp, int lane) {
  v = MAX ? warp_max(v) : warp_sum(v);
  if (W == 1) return v;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int w0 = warp - warp % W;
  float r = red[w0];
#pragma unroll
  for (int i = 1; i < W; ++i) r = MAX ? fmaxf(r, red[w0 + i]) : r + red[w0 + i];
  return r;
}

struct NormArgs {
  const __nv_bfloat16* x;
  int64_t M, ldx, Mpad;
  const __nv_bfloat16* norm_w;  // [D]
  const __nv_bfloat16* scale1;  // [M / rows_per_mod, ld_mod] = 1 + scale, or NULL
  const __nv_bfloat16* shift;   // same layout, or NULL
  int64_t rows_per_mod, ld_mod;
  float eps;
  float* gs;                    // [M] per-row global scales (codes != NULL)
  uint8_t* codes;               // [M, D/2] or NULL
  uint8_t* sf;
  __nv_bfloat16* y;             // bf16 [M, ldy] or NULL
  int64_t ldy;
};

// y = ((w * bf16(x * rsqrt(mean(x^2) + eps))) * (1 + scale)) + shift, each product / sum
// rounded to bf16 as Qwen3RMSNorm and the AdaLN lines of AceStepDiTLayer.forward
// (turbo.py:508-510, 531-538) and AceStepDiTModel.forward (turbo.py:1495-1500) do.
template <int W, int NCH>
__global__ void __launch_bounds__(256) adanorm_quant_kernel(const NormArgs a) {
  using G = RowGeo<W, NCH>;
  constexpr int64_t D = G::kD;
  __shared__ float red[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wr = warp % W;
  const int64_t m = (int64_t)blockIdx.x * G::kRowsPerCta + warp / W;
  const bool pad = m >= a.M;
  const int64_t cbase = (int64_t)wr * 32 * NCH;
  uint4 v[NCH];
  float ss = 0.0f;
  if (!pad) {
    const uint4* row = reinterpret_cast<const uint4*>(a.x + m * a.ldx);
#pragma unroll
    for (int j = 0; j < NCH; ++j) v[j] = __ldg(row + cbase + 32 * j + lane);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ss = __fadd_rn(ss, __fmul_rn(bf16_lo(w4[i]), bf16_lo(w4[i])));
        ss = __fadd_rn(ss, __fmul_rn(bf16_hi(w4[i]), bf16_hi(w4[i])));
      }
    }
  }
  ss = row_reduce<W, false>(ss, red, warp, lane);
  const float rinv = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps));
  float am = 0.0f;
  if (!pad) {
    const uint4* wrow = reinterpret_cast<const uint4*>(a.norm_w);
    const int64_t mb = a.scale1 ? (m / a.rows_per_mod) * a.ld_mod : 0;
    const uint4* srow = a.scale1 ? reinterpret_cast<const uint4*>(a.scale1 + mb) : nullptr;
    const uint4* hrow = a.shift ? reinterpret_cast<const uint4*>(a.shift + mb) : nullptr;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int64_t c = cbase + 32 * j + lane;
      const uint4 wv = __ldg(wrow + c);
      const uint32_t xw[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t sw[4] = {0u, 0u, 0u, 0u}, hw[4] = {0u, 0u, 0u, 0u};
      if (srow) {
        const uint4 sv = __ldg(srow + c);
        sw[0] = sv.x, sw[1] = sv.y, sw[2] = sv.z, sw[3] = sv.w;
      }
      if (hrow) {
        const uint4 hv = __ldg(hrow + c);
        hw[0] = hv.x, hw[1] = hv.y, hw[2] = hv.z, hw[3] = hv.w;
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float lo = bf16r(__fmul_rn(bf16_lo(xw[i]), rinv));
        float hi = bf16r(__fmul_rn(bf16_hi(xw[i]), rinv));
        lo = bf16r(__fmul_rn(bf16_lo(ww[i]), lo));
        hi = bf16r(__fmul_rn(bf16_hi(ww[i]), hi));
        if (srow) {
          lo = bf16r(__fmul_rn(lo, bf16_lo(sw[i])));
          hi = bf16r(__fmul_rn(hi, bf16_hi(sw[i])));
        }
        if (hrow) {
          lo = bf16r(__fadd_rn(lo, bf16_lo(hw[i])));
          hi = bf16r(__fadd_rn(hi, bf16_hi(hw[i])));
        }
        o[i] = pack_bf16(lo, hi);
      }
      v[j] = make_uint4(o[0], o[1], o[2], o[3]);
      am = fmaxf(am, amax8(v[j]));
      if (a.y) reinterpret_cast<uint4*>(a.y + m * a.ldy)[c] = v[j];
    }
  }
  if (!a.codes) return;
  am = row_reduce<W, true>(am, red, warp, lane);
  if (m >= a.Mpad) return;
  const int64_t r = m & 127;
  uint8_t* sf_rowbase = a.sf + (m >> 7) * (D / 64) * 512 + (r & 31) * 16 + (r >> 5) * 4;
  if (pad) {  // padding rows of the scale layout: zero scales
    for (int64_t c = wr * 32 + lane; c < D / 64; c += 32 * W) *reinterpret_cast<uint32_t*>(sf_rowbase + c * 512) = 0u;
    return;
  }
  const float g = global_scale(am);
  if (wr == 0 && lane == 0) a.gs[m] = g;
  const float denom = __fmul_rn(6.0f, g);
  uint32_t* code_row = reinterpret_cast<uint32_t*>(a.codes + m * (D / 2));
#pragma unroll
  for (int j = 0; j < NCH; ++j) quant_chunk(v[j], true, cbase + 32 * j + lane, lane, g, denom, code_row, sf_rowbase);
}

struct SiluArgs {
  const __nv_bfloat16* gu;  // [M, ld]: gate in columns [0, F), up in [F, 2F)
  int64_t M, ld, Mpad;
  float* gs;
  uint8_t* codes;           // [M, F/2]
  uint8_t* sf;
};

// h = bf16(bf16(silu(gate)) * up) (Qwen3MLP: act_fn(gate_proj(x)) * up_proj(x), turbo.py:34-35),
// quantised per row for down_proj.
template <int W, int NCH>
__global__ void __launch_bounds__(256) silu_mul_quant_kernel(const SiluArgs a) {
  using G = RowGeo<W, NCH>;
  constexpr int64_t F = G::kD;
  __shared__ float red[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wr = warp % W;
  const int64_t m = (int64_t)blockIdx.x * G::kRowsPerCta + warp / W;
  const bool pad = m >= a.M;
  const int64_t cbase = (int64_t)wr * 32 * NCH;
  uint4 v[NCH];
  float am = 0.0f;
  if (!pad) {
    const uint4* grow = reinterpret_cast<const uint4*>(a.gu + m * a.ld);
    const uint4* urow = reinterpret_cast<const uint4*>(a.gu + m * a.ld + F);
    uint4 gv[NCH], uv[NCH];
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      gv[j] = __ldg(grow + cbase + 32 * j + lane);
      uv[j] = __ldg(urow + cbase + 32 * j + lane);
    }
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const uint32_t gw[4] = {gv[j].x, gv[j].y, gv[j].z, gv[j].w};
      const uint32_t uw[4] = {uv[j].x, uv[j].y, uv[j].z, uv[j].w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float g0 = bf16_lo(gw[i]), g1 = bf16_hi(gw[i]);
        const float s0 = bf16r(__fdiv_rn(g0, __fadd_rn(1.0f, expf(-g0))));
        const float s1 = bf16r(__fdiv_rn(g1, __fadd_rn(1.0f, expf(-g1))));
        o[i] = pack_bf16(__fmul_rn(s0, bf16_lo(uw[i])), __fmul_rn(s1, bf16_hi(uw[i])));
      }
      v[j] = make_uint4(o[0], o[1], o[2], o[3]);
      am = fmaxf(am, amax8(v[j]));
    }
  }
  am = row_reduce<W, true>(am, red, warp, lane);
  if (m >= a.Mpad) return;
  const int64_t r = m & 127;
  uint8_t* sf_rowbase = a.sf + (m >> 7) * (F / 64) * 512 + (r & 31) * 16 + (r >> 5) * 4;
  if (pad) {
    for (int64_t c = wr * 32 + lane; c < F / 64; c += 32 * W) *reinterpret_cast<uint32_t*>(sf_rowbase + c * 512) = 0u;
    return;
  }
  const float g = global_scale(am);
  if (wr == 0 && lane == 0) a.gs[m] = g;
  const float denom = __fmul_rn(6.0f, g);
  uint32_t* code_row = reinterpret_cast<uint32_t*>(a.codes + m * (F / 2));
#pragma unroll
  for (int j = 0; j < NCH; ++j) quant_chunk(v[j], true, cbase + 32 * j + lane, lane, g, denom, code_row, sf_rowbase);
}

struct HeadArgs {
  __nv_bfloat16* x;            // [M, ld], heads of 128 starting at column col0
  int64_t M, ld, col0;
  int heads;
  const __nv_bfloat16* w;      // [128] q_norm / k_norm weight
  const __nv_bfloat16* cos;    // [S, 128] or NULL (no rotary embedding)
  const __nv_bfloat16* sin;
  int64_t S;                   // rows per sequence (position = row % S)
  float eps;
};

// One warp per (row, head): Qwen3RMSNorm over head_dim 128, then
// x * cos + rotate_half(x) * sin with each product and the sum rounded to bf16
// (apply_rotary_pos_emb as called in AceStepAttention.forward, turbo.py:311-345).
__global__ void __launch_bounds__(256) head_norm_rope_kernel(const HeadArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t m = gw / a.heads;
  const int h = (int)(gw % a.heads);
  if (m >= a.M) return;
  __nv_bfloat16* p = a.x + m * a.ld + a.col0 + h * 128 + 4 * lane;
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  float x[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  ss = warp_sum(ss);
  const float rinv = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), a.eps));
  const uint2 wr = __ldg(reinterpret_cast<const uint2*>(a.w) + lane);
  const float wv[4] = {bf16_lo(wr.x), bf16_hi(wr.x), bf16_lo(wr.y), bf16_hi(wr.y)};
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = bf16r(__fmul_rn(wv[i], bf16r(__fmul_rn(x[i], rinv))));
  if (a.cos) {
    const int64_t pos = m % a.S;
    const uint2 cr = __ldg(reinterpret_cast<const uint2*>(a.cos + pos * 128) + lane);
    const uint2 sr = __ldg(reinterpret_cast<const uint2*>(a.sin + pos * 128) + lane);
    const float cv[4] = {bf16_lo(cr.x), bf16_hi(cr.x), bf16_lo(cr.y), bf16_hi(cr.y)};
    const float sv[4] = {bf16_lo(sr.x), bf16_hi(sr.x), bf16_lo(sr.y), bf16_hi(sr.y)};
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // rotate_half: element i < 64 takes -x[i + 64], element i >= 64 takes x[i - 64]
      const float partner = __shfl_xor_sync(0xffffffffu, x[i], 16);
      const float rot = lane < 16 ? -partner : partner;
      y[i] = bf16r(__fadd_rn(bf16r(__fmul_rn(x[i], cv[i])), bf16r(__fmul_rn(rot, sv[i]))));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = y[i];
  }
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]));
}

#define DEMON_ROW_CASE(KERN, W, NCH)                                                   \
  case (W) * 256 * (NCH): {                                                            \
    const dim3 grid((unsigned)((Mpad + RowGeo<W, NCH>::kRowsPerCta - 1) / RowGeo<W, NCH>::kRowsPerCta)); \
    KERN<W, NCH><<<grid, 256, 0, st>>>(a);                                             \
    return DEMON_OK;                                                                   \
  }

int launch_adanorm(int64_t D, int64_t Mpad, const NormArgs& a, cudaStream_t st) {
  switch (D) {
    DEMON_ROW_CASE(adanorm_quant_kernel, 1, 1)
    DEMON_ROW_CASE(adanorm_quant_kernel, 2, 1)
    DEMON_ROW_CASE(adanorm_quant_kernel, 4, 1)
    DEMON_ROW_CASE(adanorm_quant_kernel, 4, 2)
    DEMON_ROW_CASE(adanorm_quant_kernel, 4, 3)
    DEMON_ROW_CASE(adanorm_quant_kernel, 4, 4)
    DEMON_ROW_CASE(adanorm_quant_kernel, 4, 6)
    DEMON_ROW_CASE(adanorm_quant_kernel, 4, 8)
    default: return DEMON_ERR_INVALID;
  }
}

int launch_silu(int64_t F, int64_t Mpad, const SiluArgs& a, cudaStream_t st) {
  switch (F) {
    DEMON_ROW_CASE(silu_mul_quant_kernel, 1, 1)
    DEMON_ROW_CASE(silu_mul_quant_kernel, 2, 1)
    DEMON_ROW_CASE(silu_mul_quant_kernel, 4, 1)
    DEMON_ROW_CASE(silu_mul_quant_kernel, 4, 2)
    DEMON_ROW_CASE(silu_mul_quant_kernel, 4, 3)
    DEMON_ROW_CASE(silu_mul_quant_kernel, 4, 4)
    DEMON_ROW_CASE(silu_mul_quant_kernel, 4, 6)
    DEMON_ROW_CASE(silu_mul_quant_kernel, 4, 8)
    default: return DEMON_ERR_INVALID;
  }
}

bool row_width_ok(int64_t D) {
  return D == 256 || D == 512 || D == 1024 || D == 2048 || D == 3072 || D == 4096 || D == 6144 || D == 8192;
}

}  // namespace demon

using namespace demon;

extern "C" int demon_adanorm_quantize(const void* x, int64_t M, int64_t D, int64_t ldx, const void* norm_w,
                                      const void* scale1, const void* shift, int64_t rows_per_mod, int64_t ld_mod,
                                      float eps, float* gs, uint8_t* codes, uint8_t* sf, void* y, int64_t ldy,
                                      void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(M >= 0 && row_width_ok(D), "adanorm: D must be one of 256, 512, 1024, 2048, 3072, 4096, 6144, "
                                             "8192 (D=%lld)", (long long)D);
  DEMON_CHECK_ARG(x && norm_w && (codes || y), "adanorm: null pointer");
  DEMON_CHECK_ARG(!codes || (gs && sf), "adanorm: codes need gs and sf");
  DEMON_CHECK_ARG(ldx >= D && ldx % 8 == 0 && (!y || (ldy >= D && ldy % 8 == 0)), "adanorm: bad leading dimension");
  DEMON_CHECK_ARG((!scale1 && !shift) || (rows_per_mod > 0 && ld_mod >= D && ld_mod % 8 == 0),
                  "adanorm: modulation needs rows_per_mod > 0 and ld_mod >= D, ld_mod %% 8 == 0");
  DEMON_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)norm_w & 15) == 0 && ((uintptr_t)scale1 & 15) == 0 &&
                      ((uintptr_t)shift & 15) == 0 && ((uintptr_t)y & 15) == 0,
                  "adanorm: operands must be 16-byte aligned");
  NormArgs a{};
  a.x = reinterpret_cast<const __nv_bfloat16*>(x);
  a.M = M;
  a.ldx = ldx;
  a.Mpad = codes ? (M + 127) / 128 * 128 : M;
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w);
  a.scale1 = reinterpret_cast<const __nv_bfloat16*>(scale1);
  a.shift = reinterpret_cast<const __nv_bfloat16*>(shift);
  a.rows_per_mod = rows_per_mod > 0 ? rows_per_mod : 1;
  a.ld_mod = ld_mod;
  a.eps = eps;
  a.gs = gs;
  a.codes = codes;
  a.sf = sf;
  a.y = reinterpret_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  if (a.Mpad == 0) return DEMON_OK;
  DEMON_CHECK_ARG(launch_adanorm(D, a.Mpad, a, reinterpret_cast<cudaStream_t>(stream)) == DEMON_OK,
                  "adanorm: unsupported width %lld", (long long)D);
  DEMON_CUDA(cudaGetLastError());
  return DEMON_OK;
}

extern "C" int demon_silu_mul_quantize(const void* gu, int64_t M, int64_t F, int64_t ld, float* gs, uint8_t* codes,
                                       uint8_t* sf, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(M >= 0 && row_width_ok(F), "silu_mul: F must be one of 256 ... 8192 (F=%lld)", (long long)F);
  DEMON_CHECK_ARG(gu && gs && codes && sf, "silu_mul: null pointer");
  DEMON_CHECK_ARG(ld >= 2 * F && ld % 8 == 0 && ((uintptr_t)gu & 15) == 0,
                  "silu_mul: ld >= 2F, ld %% 8 == 0, 16-byte aligned input");
  SiluArgs a{};
  a.gu = reinterpret_cast<const __nv_bfloat16*>(gu);
  a.M = M;
  a.ld = ld;
  a.Mpad = (M + 127) / 128 * 128;
  a.gs = gs;
  a.codes = codes;
  a.sf = sf;
  if (a.Mpad == 0) return DEMON_OK;
  DEMON_CHECK_ARG(launch_silu(F, a.Mpad, a, reinterpret_cast<cudaStream_t>(stream)) == DEMON_OK,
                  "silu_mul: unsupported width %lld", (long long)F);
  DEMON_CUDA(cudaGetLastError());
  return DEMON_OK;
}

extern "C" int demon_head_norm_rope(void* x, int64_t M, int64_t ld, int64_t col0, int64_t heads, const void* w,
                                    const void* cos, const void* sin, int64_t S, float eps, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(M >= 0 && heads > 0 && col0 >= 0 && col0 % 8 == 0 && ld % 8 == 0 && col0 + heads * 128 <= ld,
                  "head_norm: need col0 %% 8 == 0, ld %% 8 == 0, col0 + 128 * heads <= ld");
  DEMON_CHECK_ARG(x && w && (!cos || (sin && S > 0)), "head_norm: null pointer");
  DEMON_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 && ((uintptr_t)cos & 15) == 0 &&
                      ((uintptr_t)sin & 15) == 0,
                  "head_norm: operands must be 16-byte aligned");
  HeadArgs a{};
  a.x = reinterpret_cast<__nv_bfloat16*>(x);
  a.M = M;
  a.ld = ld;
  a.col0 = col0;
  a.heads = (int)heads;
  a.w = reinterpret_cast<const __nv_bfloat16*>(w);
  a.cos = reinterpret_cast<const __nv_bfloat16*>(cos);
  a.sin = reinterpret_cast<const __nv_bfloat16*>(sin);
  a.S = S > 0 ? S : 1;
  a.eps = eps;
  const int64_t warps = M * heads;
  if (warps == 0) return DEMON_OK;
  head_norm_rope_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  DEMON_CUDA(cudaGetLastError());
  return DEMON_OK;
}
