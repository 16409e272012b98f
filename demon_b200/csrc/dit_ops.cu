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

// sum / D rounded to fp32; for a power-of-two D the product with 1 / D is the same exact
// quotient rounded once (scaling by a power of two), without the division's instruction
// sequence.
template <int D>
__device__ __forceinline__ float mean_of_sum(float sum) {
  if constexpr ((D & (D - 1)) == 0) return __fmul_rn(sum, 1.0f / (float)D);
  return __fdiv_rn(sum, (float)D);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) { return pack_bf16x2(lo, hi); }

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

// Eight bf16 (x) -> bf16(bf16(bf16(w * bf16(x * rinv)) * s1) + sh) (product / sum skipped when
// s1 / sh are absent), as Qwen3RMSNorm followed by the AdaLN modulation, in packed arithmetic:
// x * rinv in fp32 then rounded; the products and the sum of two bf16 operands by the bf16x2
// instructions, whose single rounding of the exact result equals the reference's fp32
// operation followed by rounding to bf16 (the fp32 result is exact, or the smaller operand is
// far below half an ulp of the larger).
template <bool MUL, bool ADD>
__device__ __forceinline__ uint4 norm8(uint4 x, uint4 w, uint4 s1, uint4 sh, float rinv) {
  const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, ww[4] = {w.x, w.y, w.z, w.w};
  const uint32_t sw[4] = {s1.x, s1.y, s1.z, s1.w}, hw[4] = {sh.x, sh.y, sh.z, sh.w};
  const float2 r2 = make_float2(rinv, rinv);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t v = mul_bf2(ww[i], f2_bf2(mul_f2(bf2_f2(xw[i]), r2)));
    if (MUL) v = mul_bf2(v, sw[i]);
    if (ADD) v = add_bf2(v, hw[i]);
    o[i] = v;
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Sum of squares of eight bf16 values onto acc: even elements in one fp32 chain, odd ones in
// another, summed at the end (sq_acc_bf2: the same bits as widening first).
__device__ __forceinline__ float sumsq8(uint4 v, float acc) {
  float se = acc, so = 0.0f;
  sq_acc_bf2(v.x, se, so);
  sq_acc_bf2(v.y, se, so);
  sq_acc_bf2(v.z, se, so);
  sq_acc_bf2(v.w, se, so);
  return se + so;
}

// y = ((w * bf16(x * rsqrt(mean(x^2) + eps))) * (1 + scale)) + shift, each product / sum
// rounded to bf16 as Qwen3RMSNorm and the AdaLN lines of AceStepDiTLayer.forward
// (turbo.py:508-510, 531-538) and AceStepDiTModel.forward (turbo.py:1495-1500) do, then
// quantised per row.  Block-per-lane geometry of RowQ<D>: every load of the lane (x, norm
// weight, modulation) is issued before the first reduction.
template <int D, bool MUL, bool ADD>
__global__ void __launch_bounds__(256) adanorm_quant_kernel(const NormArgs a) {
  using G = RowQ<D>;
  __shared__ float red[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wr = warp % G::W;
  const int64_t m = (int64_t)blockIdx.x * G::R + warp / G::W;
  const bool pad = m >= a.M;
  const bool lane_ok = G::kBPR >= 32 || lane < G::kBPR;
  const bool live = !pad && lane_ok;
  const uint4* row = reinterpret_cast<const uint4*>(a.x + (pad ? 0 : m) * a.ldx);
  const int64_t mb = (pad ? 0 : m / a.rows_per_mod) * a.ld_mod;
  const uint4* srow = reinterpret_cast<const uint4*>(a.scale1 + mb);
  const uint4* hrow = reinterpret_cast<const uint4*>(a.shift + mb);
  const uint4* wrow = reinterpret_cast<const uint4*>(a.norm_w);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  uint4 xv[2 * G::NB], wv[2 * G::NB], sv[2 * G::NB], hv[2 * G::NB];
#pragma unroll
  for (int j = 0; j < G::NB; ++j) {
    const int64_t c = 2 * ((int64_t)(wr * G::NB + j) * 32 + lane);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      xv[2 * j + h] = live ? __ldg(row + c + h) : z;
      wv[2 * j + h] = live ? __ldg(wrow + c + h) : z;
      sv[2 * j + h] = (MUL && live) ? __ldg(srow + c + h) : z;
      hv[2 * j + h] = (ADD && live) ? __ldg(hrow + c + h) : z;
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 2 * G::NB; ++j) ss = sumsq8(xv[j], ss);
  ss = row_reduce<G::W, false>(ss, red, warp, lane);
  const float rinv = __frsqrt_rn(__fadd_rn(mean_of_sum<D>(ss), a.eps));
  uint32_t vmax[2 * G::NB];
#pragma unroll
  for (int j = 0; j < 2 * G::NB; ++j) {
    xv[j] = norm8<MUL, ADD>(xv[j], wv[j], sv[j], hv[j], rinv);
    vmax[j] = absmax_bits8(xv[j]);
  }
  float am = lane_absmax(xv, vmax);
  if (a.y && live) {
    uint4* yrow = reinterpret_cast<uint4*>(a.y + m * a.ldy);
#pragma unroll
    for (int j = 0; j < G::NB; ++j) {
      const int64_t c = 2 * ((int64_t)(wr * G::NB + j) * 32 + lane);
      yrow[c] = xv[2 * j];
      yrow[c + 1] = xv[2 * j + 1];
    }
  }
  if (!a.codes) return;
  am = row_reduce<G::W, true>(am, red, warp, lane);
  if (m >= a.Mpad) return;
  const int64_t r = m & 127;
  uint8_t* sf_rowbase = a.sf + (m >> 7) * (D / 64) * 512 + (r & 31) * 16 + (r >> 5) * 4;
  if (pad) {  // padding rows of the scale layout: zero scales
    for (int64_t c = wr * 32 + lane; c < D / 64; c += 32 * G::W) *reinterpret_cast<uint32_t*>(sf_rowbase + c * 512) = 0u;
    return;
  }
  const float g = global_scale(am);
  if (wr == 0 && lane == 0) a.gs[m] = g;
  const float denom = __fmul_rn(6.0f, g);
  uint8_t* code_row = a.codes + m * (D / 2);
  if (!warp_any_nan(vmax)) {
#pragma unroll
    for (int j = 0; j < G::NB; ++j) {
      const int64_t kb = (int64_t)(wr * G::NB + j) * 32 + lane;
      store_block(quant_block_finite(xv[2 * j], xv[2 * j + 1], vmax[2 * j], vmax[2 * j + 1], g, denom), lane_ok, kb,
                  lane, code_row, sf_rowbase);
    }
  } else {
#pragma unroll
    for (int j = 0; j < G::NB; ++j) {
      const int64_t kb = (int64_t)(wr * G::NB + j) * 32 + lane;
      store_block(quant_block_m(xv[2 * j], xv[2 * j + 1], vmax[2 * j], vmax[2 * j + 1], g, denom), lane_ok, kb,
                  lane, code_row, sf_rowbase);
    }
  }
}

// The same row operation in the quantiser's geometry at D = 2048: one warp per row (4 blocks
// of 16 per lane), so both row reductions are warp shuffles with no shared-memory round trip.
// A CTA takes 8 * RPW rows (each warp RPW of them, one after another) and stages the norm
// weight and the (at most two) modulation rows of its rows in shared memory once; the launch
// uses this form only when the CTA's rows span at most two modulation rows
// (rows_per_mod >= 8 * RPW - 1).  The first row's x is loaded before the staging barrier, so
// its latency overlaps the staging.  Staged vectors are stored half-major (vector 2k + h at
// h * V/2 + k), so the 32 lanes of a warp read 32 consecutive 16-byte vectors (no bank
// conflicts).
constexpr int kAdaRowsPerWarp = 2;

template <int D, bool MUL, bool ADD>
__global__ void __launch_bounds__(256, 3) adanorm_warp_kernel(const NormArgs a) {
  using G = RowQ<D, 1>;
  static_assert(G::W == 1 && G::R == 8, "one warp per row");
  constexpr int V = D / 8;  // 16-byte vectors per row
  constexpr int RPW = kAdaRowsPerWarp;
  __shared__ __align__(16) uint4 s_w[V];
  __shared__ __align__(16) uint4 s_mod[2][2][(MUL || ADD) ? V : 1];  // [modulation row][scale1, shift]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t m_first = (int64_t)blockIdx.x * G::R * RPW;
  const bool cta_live = m_first < a.M;
  const int64_t b0 = cta_live ? m_first / a.rows_per_mod : 0;
  const int64_t b1 = cta_live ? min(m_first + G::R * RPW - 1, a.M - 1) / a.rows_per_mod : 0;
  const int64_t m_b1 = (b0 + 1) * a.rows_per_mod;  // first row of modulation row b0 + 1
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  uint4 xv[2 * G::NB];
  auto load_row = [&](int64_t m) {
    const bool pad = m >= a.M;
    const uint4* row = reinterpret_cast<const uint4*>(a.x + (pad ? 0 : m) * a.ldx);
#pragma unroll
    for (int j = 0; j < G::NB; ++j) {
      const int kb = j * 32 + lane;
      xv[2 * j] = pad ? z : __ldg(row + 2 * kb);
      xv[2 * j + 1] = pad ? z : __ldg(row + 2 * kb + 1);
    }
  };
  load_row(m_first + warp);  // in flight across the staging below
  if (cta_live) {
    const uint4* wsrc = reinterpret_cast<const uint4*>(a.norm_w);
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const int si = (i & 1) * (V / 2) + (i >> 1);
      s_w[si] = __ldg(wsrc + i);
      if (MUL || ADD) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int64_t b = k ? b1 : b0;
          if (k && b1 == b0) break;
          if (MUL) s_mod[k][0][si] = __ldg(reinterpret_cast<const uint4*>(a.scale1 + b * a.ld_mod) + i);
          if (ADD) s_mod[k][1][si] = __ldg(reinterpret_cast<const uint4*>(a.shift + b * a.ld_mod) + i);
        }
      }
    }
  }
  __syncthreads();
#pragma unroll 1
  for (int rw = 0; rw < RPW; ++rw) {
    const int64_t m = m_first + rw * G::R + warp;
    if (rw > 0) load_row(m);
    const bool pad = m >= a.M;
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 2 * G::NB; ++j) ss = sumsq8(xv[j], ss);
    ss = warp_sum(ss);
    const float rinv = __frsqrt_rn(__fadd_rn(mean_of_sum<D>(ss), a.eps));
    // m >= m_first >= b0 * rows_per_mod, so m / rows_per_mod != b0 is m >= m_b1 (a compare, not
    // a 64-bit division per row)
    const int sel = (!pad && (MUL || ADD) && m >= m_b1) ? 1 : 0;
    uint32_t mb[2 * G::NB];
#pragma unroll
    for (int j = 0; j < G::NB; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = h * (V / 2) + j * 32 + lane;  // vector 2 (j * 32 + lane) + h, half-major
        const uint4 sv = MUL ? s_mod[sel][0][c] : z, hv = ADD ? s_mod[sel][1][c] : z;
        xv[2 * j + h] = norm8<MUL, ADD>(xv[2 * j + h], s_w[c], sv, hv, rinv);
        mb[2 * j + h] = absmax_bits8(xv[2 * j + h]);
      }
    }
    float am = lane_absmax(xv, mb);
    if (a.y && !pad) {
      uint4* yrow = reinterpret_cast<uint4*>(a.y + m * a.ldy);
#pragma unroll
      for (int j = 0; j < G::NB; ++j) {
        const int kb = j * 32 + lane;
        yrow[2 * kb] = xv[2 * j];
        yrow[2 * kb + 1] = xv[2 * j + 1];
      }
    }
    if (!a.codes) continue;
    am = warp_max(am);
    if (m >= a.Mpad) continue;
    const int64_t r = m & 127;
    uint8_t* sf_rowbase = a.sf + (m >> 7) * (D / 64) * 512 + (r & 31) * 16 + (r >> 5) * 4;
    if (pad) {  // padding rows of the scale layout: zero scales
      for (int c = lane; c < D / 64; c += 32) *reinterpret_cast<uint32_t*>(sf_rowbase + c * 512) = 0u;
      continue;
    }
    const float g = global_scale(am);
    if (lane == 0) a.gs[m] = g;
    const float denom = __fmul_rn(6.0f, g);
    uint8_t* code_row = a.codes + m * (D / 2);
    if (!warp_any_nan(mb)) {
#pragma unroll
      for (int j = 0; j < G::NB; ++j)
        store_block(quant_block_finite(xv[2 * j], xv[2 * j + 1], mb[2 * j], mb[2 * j + 1], g, denom), true,
                    (int64_t)j * 32 + lane, lane, code_row, sf_rowbase);
    } else {
#pragma unroll
      for (int j = 0; j < G::NB; ++j)
        store_block(quant_block_m(xv[2 * j], xv[2 * j + 1], mb[2 * j], mb[2 * j + 1], g, denom), true,
                    (int64_t)j * 32 + lane, lane, code_row, sf_rowbase);
    }
  }
}

struct SiluArgs {
  const __nv_bfloat16* gu;  // [M, ld]: gate in columns [0, F), up in [F, 2F)
  int64_t M, ld, Mpad;
  float* gs;
  uint8_t* codes;           // [M, F/2]
  uint8_t* sf;
  __nv_bfloat16* y;         // optional bf16 h [M, ldy]
  int64_t ldy;
};

__device__ __forceinline__ uint4 silu_mul8(uint4 g, uint4 u) {
  return make_uint4(silu_mul_bf2(g.x, u.x), silu_mul_bf2(g.y, u.y), silu_mul_bf2(g.z, u.z),
                    silu_mul_bf2(g.w, u.w));
}

// h = bf16(bf16(silu(gate)) * up) (Qwen3MLP: act_fn(gate_proj(x)) * up_proj(x), turbo.py:34-35),
// quantised per row for down_proj.
template <int F>
__global__ void __launch_bounds__(256) silu_mul_quant_kernel(const SiluArgs a) {
  using G = RowQ<F>;
  __shared__ float red[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wr = warp % G::W;
  const int64_t m = (int64_t)blockIdx.x * G::R + warp / G::W;
  const bool pad = m >= a.M;
  const bool lane_ok = G::kBPR >= 32 || lane < G::kBPR;
  const bool live = !pad && lane_ok;
  const uint4* grow = reinterpret_cast<const uint4*>(a.gu + (pad ? 0 : m) * a.ld);
  const uint4* urow = reinterpret_cast<const uint4*>(a.gu + (pad ? 0 : m) * a.ld + F);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  uint4 gv[2 * G::NB], uv[2 * G::NB];
#pragma unroll
  for (int j = 0; j < G::NB; ++j) {
    const int64_t c = 2 * ((int64_t)(wr * G::NB + j) * 32 + lane);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      gv[2 * j + h] = live ? __ldg(grow + c + h) : z;
      uv[2 * j + h] = live ? __ldg(urow + c + h) : z;
    }
  }
  uint32_t mb[2 * G::NB];
#pragma unroll
  for (int j = 0; j < 2 * G::NB; ++j) {
    gv[j] = silu_mul8(gv[j], uv[j]);
    mb[j] = absmax_bits8(gv[j]);
  }
  float am = lane_absmax(gv, mb);
  if (a.y && live) {
    uint4* yrow = reinterpret_cast<uint4*>(a.y + m * a.ldy);
#pragma unroll
    for (int j = 0; j < G::NB; ++j) {
      const int64_t c = 2 * ((int64_t)(wr * G::NB + j) * 32 + lane);
      yrow[c] = gv[2 * j];
      yrow[c + 1] = gv[2 * j + 1];
    }
  }
  am = row_reduce<G::W, true>(am, red, warp, lane);
  if (m >= a.Mpad) return;
  const int64_t r = m & 127;
  uint8_t* sf_rowbase = a.sf + (m >> 7) * (F / 64) * 512 + (r & 31) * 16 + (r >> 5) * 4;
  if (pad) {
    for (int64_t c = wr * 32 + lane; c < F / 64; c += 32 * G::W) *reinterpret_cast<uint32_t*>(sf_rowbase + c * 512) = 0u;
    return;
  }
  const float g = global_scale(am);
  if (wr == 0 && lane == 0) a.gs[m] = g;
  const float denom = __fmul_rn(6.0f, g);
  uint8_t* code_row = a.codes + m * (F / 2);
  if (!warp_any_nan(mb)) {
#pragma unroll
    for (int j = 0; j < G::NB; ++j) {
      const int64_t kb = (int64_t)(wr * G::NB + j) * 32 + lane;
      store_block(quant_block_finite(gv[2 * j], gv[2 * j + 1], mb[2 * j], mb[2 * j + 1], g, denom), lane_ok, kb,
                  lane, code_row, sf_rowbase);
    }
  } else {
#pragma unroll
    for (int j = 0; j < G::NB; ++j) {
      const int64_t kb = (int64_t)(wr * G::NB + j) * 32 + lane;
      store_block(quant_block_m(gv[2 * j], gv[2 * j + 1], mb[2 * j], mb[2 * j + 1], g, denom), lane_ok, kb, lane,
                  code_row, sf_rowbase);
    }
  }
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

template <int D>
void launch_adanorm_d(const NormArgs& a, cudaStream_t st) {
  if constexpr (D == 2048) {
    // the staged form needs the CTA's rows to span at most two modulation rows
    if ((!a.scale1 && !a.shift) || a.rows_per_mod >= 8 * kAdaRowsPerWarp - 1) {
      const dim3 grid((unsigned)((a.Mpad + 8 * kAdaRowsPerWarp - 1) / (8 * kAdaRowsPerWarp)));
      if (a.scale1 && a.shift) adanorm_warp_kernel<D, true, true><<<grid, 256, 0, st>>>(a);
      else if (a.scale1) adanorm_warp_kernel<D, true, false><<<grid, 256, 0, st>>>(a);
      else if (a.shift) adanorm_warp_kernel<D, false, true><<<grid, 256, 0, st>>>(a);
      else adanorm_warp_kernel<D, false, false><<<grid, 256, 0, st>>>(a);
      return;
    }
  }
  const dim3 grid((unsigned)((a.Mpad + RowQ<D>::R - 1) / RowQ<D>::R));
  if (a.scale1 && a.shift) adanorm_quant_kernel<D, true, true><<<grid, 256, 0, st>>>(a);
  else if (a.scale1) adanorm_quant_kernel<D, true, false><<<grid, 256, 0, st>>>(a);
  else if (a.shift) adanorm_quant_kernel<D, false, true><<<grid, 256, 0, st>>>(a);
  else adanorm_quant_kernel<D, false, false><<<grid, 256, 0, st>>>(a);
}

int launch_adanorm(int64_t D, const NormArgs& a, cudaStream_t st) {
  switch (D) {
    case 256: launch_adanorm_d<256>(a, st); return DEMON_OK;
    case 512: launch_adanorm_d<512>(a, st); return DEMON_OK;
    case 1024: launch_adanorm_d<1024>(a, st); return DEMON_OK;
    case 2048: launch_adanorm_d<2048>(a, st); return DEMON_OK;
    case 3072: launch_adanorm_d<3072>(a, st); return DEMON_OK;
    case 4096: launch_adanorm_d<4096>(a, st); return DEMON_OK;
    case 6144: launch_adanorm_d<6144>(a, st); return DEMON_OK;
    case 8192: launch_adanorm_d<8192>(a, st); return DEMON_OK;
    default: return DEMON_ERR_INVALID;
  }
}

template <int F>
void launch_silu_f(const SiluArgs& a, cudaStream_t st) {
  silu_mul_quant_kernel<F><<<(unsigned)((a.Mpad + RowQ<F>::R - 1) / RowQ<F>::R), 256, 0, st>>>(a);
}

int launch_silu(int64_t F, const SiluArgs& a, cudaStream_t st) {
  switch (F) {
    case 256: launch_silu_f<256>(a, st); return DEMON_OK;
    case 512: launch_silu_f<512>(a, st); return DEMON_OK;
    case 1024: launch_silu_f<1024>(a, st); return DEMON_OK;
    case 2048: launch_silu_f<2048>(a, st); return DEMON_OK;
    case 3072: launch_silu_f<3072>(a, st); return DEMON_OK;
    case 4096: launch_silu_f<4096>(a, st); return DEMON_OK;
    case 6144: launch_silu_f<6144>(a, st); return DEMON_OK;
    case 8192: launch_silu_f<8192>(a, st); return DEMON_OK;
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
  DEMON_CHECK_ARG(launch_adanorm(D, a, reinterpret_cast<cudaStream_t>(stream)) == DEMON_OK,
                  "adanorm: unsupported width %lld", (long long)D);
  DEMON_CUDA(cudaGetLastError());
  return DEMON_OK;
}

extern "C" int demon_silu_mul_quantize(const void* gu, int64_t M, int64_t F, int64_t ld, float* gs, uint8_t* codes,
                                       uint8_t* sf, void* y, int64_t ldy, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(M >= 0 && row_width_ok(F), "silu_mul: F must be one of 256 ... 8192 (F=%lld)", (long long)F);
  DEMON_CHECK_ARG(gu && gs && codes && sf, "silu_mul: null pointer");
  DEMON_CHECK_ARG(ld >= 2 * F && ld % 8 == 0 && ((uintptr_t)gu & 15) == 0,
                  "silu_mul: ld >= 2F, ld %% 8 == 0, 16-byte aligned input");
  DEMON_CHECK_ARG(!y || (ldy >= F && ldy % 8 == 0 && ((uintptr_t)y & 15) == 0),
                  "silu_mul: y needs ldy >= F, ldy %% 8 == 0, 16-byte alignment");
  SiluArgs a{};
  a.gu = reinterpret_cast<const __nv_bfloat16*>(gu);
  a.M = M;
  a.ld = ld;
  a.Mpad = (M + 127) / 128 * 128;
  a.gs = gs;
  a.codes = codes;
  a.sf = sf;
  a.y = reinterpret_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  if (a.Mpad == 0) return DEMON_OK;
  DEMON_CHECK_ARG(launch_silu(F, a, reinterpret_cast<cudaStream_t>(stream)) == DEMON_OK,
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
