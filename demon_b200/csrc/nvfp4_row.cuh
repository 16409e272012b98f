// nvfp4_row.cuh -- device helpers shared by the row kernels that end in NVFP4
// quantisation (the activation quantiser and the fused DiT row kernels).
// The arithmetic of each step is documented in nvfp4_quant.cu.
#pragma once
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "demon_common.cuh"

namespace demon {

// E4M3FN byte -> float (format definition: bias 7, subnormals m * 2^-9).
__device__ __forceinline__ float e4m3_value(uint32_t b) {
  const uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
  const float v = (e == 0u) ? __int2float_rn((int)m) * 0.001953125f
                            : __int2float_rn((int)(8u + m)) * __uint_as_float((e + 117u) << 23);  // 2^(e-10)
  return (b & 0x80u) ? -v : v;
}

__device__ __forceinline__ uint32_t e4m3_rne_sat(float s) {
  return (uint32_t)__nv_cvt_float_to_fp8(s, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float global_scale(float amax) {
  return __fdiv_rn(fmaxf(amax, 1e-12f), 2688.0f);
}

// Block absmax of 8 bf16 values with packed bf16x2 abs/max (exact: no rounding).
__device__ __forceinline__ float amax8(uint4 v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  const __nv_bfloat162 m = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])), __hmax2(__habs2(h[2]), __habs2(h[3])));
  return fmaxf(__low2float(m), __high2float(m));
}

// Packed fp32 multiply (two IEEE round-to-nearest products per instruction).
__device__ __forceinline__ float2 mul2(float2 a, float b) {
  uint64_t r;
  const uint64_t av = (uint64_t)__float_as_uint(a.x) | ((uint64_t)__float_as_uint(a.y) << 32);
  const uint64_t bv = (uint64_t)__float_as_uint(b) | ((uint64_t)__float_as_uint(b) << 32);
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(av), "l"(bv));
  return make_float2(__uint_as_float((uint32_t)r), __uint_as_float((uint32_t)(r >> 32)));
}

// Two elements -> one byte of E2M1 codes (low nibble = first element) with
// the hardware round-to-nearest-even, saturating conversion; NaN is mapped to
// zero first (the format spec gives NaN code 0).
__device__ __forceinline__ uint32_t cvt2(float lo, float hi) {
  lo = (lo == lo) ? lo : 0.0f;
  hi = (hi == hi) ? hi : 0.0f;
  return (uint32_t)__nv_cvt_float2_to_fp4x2(make_float2(lo, hi), __NV_E2M1, cudaRoundNearest);
}

// Eight elements -> 32 bits of codes.  A value that rounds to magnitude 0
// keeps no sign bit (canonical zero, code 0).
__device__ __forceinline__ uint32_t pack2(uint32_t w, float rs) {
  const float2 p = mul2(make_float2(bf16_lo(w), bf16_hi(w)), rs);
  return cvt2(p.x, p.y);
}
__device__ __forceinline__ uint32_t pack8(uint4 v, float rs) {
  const uint32_t c = pack2(v.x, rs) | (pack2(v.y, rs) << 8) | (pack2(v.z, rs) << 16) | (pack2(v.w, rs) << 24);
  const uint32_t mag = c & 0x77777777u;
  const uint32_t nz = (mag | (mag >> 1) | (mag >> 2)) & 0x11111111u;
  return mag | (c & (nz << 3));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One 8-element chunk of a row: block absmax (lanes 2i, 2i+1), scale, codes,
// and the 32-bit scale-group store (lanes with lane % 8 == 0).  Every lane of
// the warp calls this (the shuffles need the full warp); `valid` masks stores.
__device__ __forceinline__ void quant_chunk(uint4 v, bool valid, int64_t c, int lane, float g, float denom,
                                            uint32_t* code_row, uint8_t* sf_rowbase) {
  const float mine = amax8(v);
  const float am = fmaxf(mine, __shfl_xor_sync(0xffffffffu, mine, 1));
  const float s = fminf(__fdiv_rn(am, denom), 448.0f);
  const uint32_t sb = e4m3_rne_sat(s);
  const float sbf = e4m3_value(sb);
  uint32_t packed = 0u;
  if (sbf != 0.0f) packed = pack8(v, __frcp_rn(__fmul_rn(sbf, g)));
  const uint32_t s1 = __shfl_down_sync(0xffffffffu, sb, 2);
  const uint32_t s2 = __shfl_down_sync(0xffffffffu, sb, 4);
  const uint32_t s3 = __shfl_down_sync(0xffffffffu, sb, 6);
  if (valid) {
    code_row[c] = packed;
    if ((lane & 7) == 0)
      *reinterpret_cast<uint32_t*>(sf_rowbase + ((c >> 1) >> 2) * 512) = sb | (s1 << 8) | (s2 << 16) | (s3 << 24);
  }
}

// E4M3 byte -> float through the hardware conversion (exact: every E4M3 value, subnormals
// included, is an FP16 value).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  uint32_t h2;
  asm("{\n\t.reg .b16 s;\n\tcvt.u16.u32 s, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, s;\n\t}" : "=r"(h2) : "r"(b & 0xFFu));
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}

// One 16-element scale block held by one lane (two 8-element chunks): block scale byte
// and 64 bits of codes (same arithmetic as quant_chunk, without the pair exchange).
struct QBlock {
  uint2 codes;
  uint32_t sb;
};
// Eight elements -> 32 bits of codes, for blocks known to hold no NaN (no per-element
// NaN test; otherwise identical to pack8).
__device__ __forceinline__ uint32_t pack2_finite(uint32_t w, float rs) {
  const float2 p = mul2(make_float2(bf16_lo(w), bf16_hi(w)), rs);
  return (uint32_t)__nv_cvt_float2_to_fp4x2(p, __NV_E2M1, cudaRoundNearest);
}
__device__ __forceinline__ uint32_t pack8_finite(uint4 v, float rs) {
  const uint32_t c = pack2_finite(v.x, rs) | (pack2_finite(v.y, rs) << 8) | (pack2_finite(v.z, rs) << 16) |
                     (pack2_finite(v.w, rs) << 24);
  const uint32_t mag = c & 0x77777777u;
  const uint32_t nz = (mag | (mag >> 1) | (mag >> 2)) & 0x11111111u;
  return mag | (c & (nz << 3));
}

// Largest |x| bit patterns of 8 bf16 values, one per half-word (still packed): for
// non-negative IEEE values the bit patterns order like the values, so an unsigned SIMD max
// gives the absmax exactly; a half above 0x7F80 (infinity) means a NaN among its values.
// The row kernels compute these once per 16-byte vector and use them for both the row's
// global scale and the 16-element block scales.
__device__ __forceinline__ uint32_t absmax_bits8(uint4 v) {
  const uint32_t k = 0x7FFF7FFFu;
  return __vmaxu2(__vmaxu2(v.x & k, v.y & k), __vmaxu2(v.z & k, v.w & k));
}
__device__ __forceinline__ uint32_t halves_max(uint32_t m) { return max(m & 0xFFFFu, m >> 16); }

// Absolute maximum of a lane's N vectors (NaN ignored, as the packed max does) from their
// packed maxima; a lane holding a NaN takes the NaN-ignoring max of every vector instead.
template <int N>
__device__ __forceinline__ float lane_absmax(const uint4 (&v)[N], const uint32_t (&mb)[N]) {
  uint32_t acc = 0u;
#pragma unroll
  for (int j = 0; j < N; ++j) acc = __vmaxu2(acc, mb[j]);
  const uint32_t bits = halves_max(acc);
  if (bits <= 0x7F80u) return __uint_as_float(bits << 16);
  float am = 0.0f;
#pragma unroll
  for (int j = 0; j < N; ++j) am = fmaxf(am, amax8(v[j]));
  return am;
}

// One 16-element block (vectors a, b with packed maxima ma, mb) -> scale byte + codes.
__device__ __forceinline__ QBlock quant_block_m(uint4 a, uint4 b, uint32_t ma, uint32_t mbits, float g,
                                                float denom) {
  const uint32_t mb = halves_max(__vmaxu2(ma, mbits));
  const bool nan = mb > 0x7F80u;
  // NaN elements do not count towards the block absmax (the packed max ignores them)
  const float am = nan ? fmaxf(amax8(a), amax8(b)) : __uint_as_float(mb << 16);
  const float s = fminf(__fdiv_rn(am, denom), 448.0f);
  QBlock q;
  q.sb = e4m3_rne_sat(s);
  q.codes = make_uint2(0u, 0u);
  const float sbf = e4m3_to_f32(q.sb);
  if (sbf != 0.0f) {
    const float rs = __frcp_rn(__fmul_rn(sbf, g));
    q.codes = nan ? make_uint2(pack8(a, rs), pack8(b, rs)) : make_uint2(pack8_finite(a, rs), pack8_finite(b, rs));
  }
  return q;
}
__device__ __forceinline__ QBlock quant_block(uint4 a, uint4 b, float g, float denom) {
  return quant_block_m(a, b, absmax_bits8(a), absmax_bits8(b), g, denom);
}
// The same for a block known to hold no NaN, without a branch: an all-zero block (scale byte
// 0) gets rs = 0, so every product is (+-)0 and every code the canonical 0, as above.
__device__ __forceinline__ QBlock quant_block_finite(uint4 a, uint4 b, uint32_t ma, uint32_t mbits, float g,
                                                     float denom) {
  const float am = __uint_as_float(halves_max(__vmaxu2(ma, mbits)) << 16);
  const float s = fminf(__fdiv_rn(am, denom), 448.0f);
  QBlock q;
  q.sb = e4m3_rne_sat(s);
  const float sbf = e4m3_to_f32(q.sb);
  const float rs = sbf != 0.0f ? __frcp_rn(__fmul_rn(sbf, g)) : 0.0f;
  q.codes = make_uint2(pack8_finite(a, rs), pack8_finite(b, rs));
  return q;
}
// True when some lane of the warp holds a NaN among the vectors with packed maxima mb[]
// (warp-uniform, so the block loops that follow, which shuffle, stay converged).
template <int N>
__device__ __forceinline__ bool warp_any_nan(const uint32_t (&mb)[N]) {
  uint32_t acc = 0u;
#pragma unroll
  for (int j = 0; j < N; ++j) acc = __vmaxu2(acc, mb[j]);
  return __any_sync(0xffffffffu, halves_max(acc) > 0x7F80u);
}

// Lane owns scale block kb of row m (K/16 blocks per row): store its 8 code bytes and, from
// lanes with kb % 4 == 0, the four consecutive scale bytes of the tcgen05 layout as one word.
// All 32 lanes must call it (shuffles); `valid` masks the stores.
__device__ __forceinline__ void store_block(const QBlock& q, bool valid, int64_t kb, int lane, uint8_t* code_row,
                                            uint8_t* sf_rowbase) {
  const uint32_t s1 = __shfl_down_sync(0xffffffffu, q.sb, 1);
  const uint32_t s2 = __shfl_down_sync(0xffffffffu, q.sb, 2);
  const uint32_t s3 = __shfl_down_sync(0xffffffffu, q.sb, 3);
  if (valid) {
    reinterpret_cast<uint2*>(code_row)[kb] = q.codes;
    if ((lane & 3) == 0)
      *reinterpret_cast<uint32_t*>(sf_rowbase + (kb >> 2) * 512) = q.sb | (s1 << 8) | (s2 << 16) | (s3 << 24);
  }
}

// Geometry of the block-per-lane row kernels for a row of K elements: W warps per row, NB
// blocks per lane; lane l of row-warp w owns blocks kb = (w * NB + j) * 32 + l (j < NB).
// Rows shorter than 512 use the first K/16 lanes of one warp.  WF != 0 fixes W.
template <int K, int WF = 0>
struct RowQ {
  static constexpr int kBPR = K / 16;
  static constexpr int W = WF ? WF : (kBPR % 128 == 0) ? 4 : (kBPR % 64 == 0) ? 2 : 1;
  static constexpr int NB = kBPR >= 32 * W ? kBPR / (32 * W) : 1;
  static constexpr int R = 8 / W;  // rows per 256-thread CTA
  static_assert(kBPR % 4 == 0 && (kBPR < 32 || kBPR % (32 * W) == 0), "row width");
};

// Cross-warp reduction of one value per row (sum or max): full-warp shuffle, then the W
// warps of a row combine through shared memory (all threads of the CTA must call it).
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


}  // namespace demon
