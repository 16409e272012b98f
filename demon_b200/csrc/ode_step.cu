// ode_step.cu -- fused per-slot ODE/SDE step of the DEMON streaming tick (sm_100a).
//
// One launch advances every slot of the ring by one denoising step.  A slot is
// a [T, 64] bf16 latent; its step is the post-forward section of the
// reference's StreamPipeline._tick_pt (acestep/engine/stream.py:1060-1276):
//   velocity assembly   blend_velocities        (acestep/engine/ode_steps.py:150-183)
//   APG guidance        MomentumBuffer.update, apg_forward, apg_project (:276-362)
//   CFG rescale         cfg_rescale             (:365-392)
//   integration         x0_from_vel, mask_post_blend_x0, blend_x0_target,
//                       step_ode_euler, step_sde_curve, step_sde_renoise (:72-266)
// and it also writes the next tick's decoder input: mask_pre_blend at t_next
// times the [T, 64] channel gain (stream.py:983-998), so the next forward reads
// a ready batch row.
//
// APG and cfg_rescale reduce over T for each (slot, channel) (dims=(1,), the
// reference's default, ode_steps.py:328-336 and :365-370).  The T axis of a
// slot is split over a 4-, 8- or 16-CTA thread-block cluster.  A first pass over a CTA's
// rows streams v_pos, v_neg and the old momentum, stores the new momentum and
// accumulates per-channel moments in registers; the cluster exchanges the
// partial moments through distributed shared memory; the second pass streams
// the state and re-reads v_pos and the new momentum, which the same thread
// touched microseconds before (L2 hits: DRAM sees every byte once).
//
// The norm of the guided velocity is obtained in closed form from moments of
// the first pass (w_t = g_t - 1, d = k r):
//   v_g = (1 - w_t a) v_pos + w_t k r,  a = k <r, v_pos> / max(|v_pos|, 1e-12)^2
//   |v_g|^2 = P0 - 2a P1 + a^2 P2 + 2k Q1 - 2ka Q2 + k^2 R2
// with P_i = sum w^i v_pos^2, Q_i = sum w^i v_pos r, R2 = sum w^2 r^2, so the
// step needs no second pass over T.  Moments are summed in fp32 per thread over
// its rows and in fp64 across threads and CTAs, in a fixed order: results are
// deterministic and independent of which other slots share the launch.
//
// Numerics: arithmetic is fp32 (fp64 for the moments); values are rounded to
// bf16 where the reference materialises a bf16 tensor that the step reuses
// (momentum, guided velocity, scaled velocity, x0, v_blended, the new state,
// the masked state, the decoder input).
#include <cooperative_groups.h>

#include <algorithm>

#include "demon_common.cuh"
#include "demon_host.h"

namespace cg = cooperative_groups;

namespace demon {

// CTAs per slot cluster: up to 16, chosen per launch (see ode_cluster)
constexpr int kOdeClusterMax = 16;
constexpr int kOdeThreads = 256;
constexpr int kOdeWarps = kOdeThreads / 32;
constexpr int kOdeMinBlocks = 4;                // CTAs per SM: 64 registers per thread
constexpr int kOdeD = 64;
constexpr int kOdeRowsPass = kOdeThreads / 8;   // 8 lanes x 8 channels per row
constexpr int kOdeMaxT = 6400;

__device__ __forceinline__ float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Rows of a slot per CTA of its cluster: even, so the row pairs (2k, 2k+1) of the DCW wavelet
// step never straddle two CTAs.
__host__ __device__ __forceinline__ int ode_rows_per_cta(int T, int cluster) {
  return (T + 2 * cluster - 1) / (2 * cluster) * 2;
}

__device__ __forceinline__ float curve(const float* c, float s, int t) { return c ? __ldg(c + t) : s; }

// Per-step Gaussian noise, counter-based so that a slot's draws depend only on (seed, step,
// element): the SplitMix64 output function (Vigna; Steele, Lea, Flood, OOPSLA'14) of
// seed_key + counter * 0x9e3779b97f4a7c15 gives 64 uniform bits per counter, and Box-Muller
// turns its two 32-bit halves into two normals.  The counter of an element pair is
// step * 2^36 + (element index) / 2, distinct for every pair of every step of a slot.
__device__ __forceinline__ uint64_t splitmix64_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t noise_key(uint64_t seed) { return splitmix64_mix(seed + 0x9e3779b97f4a7c15ull); }

// two normals from the 64 bits of one counter
__device__ __forceinline__ float2 normal2(uint64_t key, uint64_t counter) {
  const uint64_t z = splitmix64_mix(key + counter * 0x9e3779b97f4a7c15ull);
  const float u1 = __uint2float_rn((uint32_t)(z >> 40)) * 5.9604644775390625e-08f + 2.98023223876953125e-08f;
  const float u2 = __uint2float_rn((uint32_t)(z >> 8) & 0xFFFFFFu) * 5.9604644775390625e-08f;
  // hardware log / sqrt / sin / cos approximations: the draws are rounded to bf16 (8 significant
  // bits), far coarser than their error
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(-2.0f * __logf(u1)));
  float sn, cs;
  __sincosf(6.2831853071795865f * (u2 - 0.5f), &sn, &cs);  // a uniform angle in [-pi, pi)
  return make_float2(rnd(r * cs), rnd(r * sn));
}

struct OdeShared {
  union {
    float gpart[kOdeWarps][8][kOdeD];  // per-warp moment partials (fp32 over the warp's rows)
    double tot[8][kOdeD];              // then: the slot's moments, summed over the cluster
  };
  double cta_part[8][kOdeD];           // this CTA's moments (read by the cluster)
  float na[kOdeD], k[kOdeD], sm1[kOdeD];  // per channel: -a, k, sigma - 1
};

// ---------------------------------------------------------------------------
// Packed arithmetic on pairs of channels.  A bf16x2 product or sum of two bf16 operands
// (mul_bf2 / add_bf2 / sub_bf2) rounds the exact result once, which equals the reference's
// fp32 operation followed by rounding to bf16; an fp32 scalar times a bf16 tensor goes
// through fp32 (mul_f2) and is rounded afterwards (f2_bf2), as torch's opmath does.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t sub_bf2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2_dup(float v) { return pack_bf16x2(v, v); }  // v already bf16-exact
__device__ __forceinline__ float2 f2_dup(float v) { return make_float2(v, v); }
// bf16(s * x) for an fp32 scalar s and a bf16 pair x
__device__ __forceinline__ uint32_t scal_bf2(float s, uint32_t x) { return f2_bf2(mul_f2(f2_dup(s), bf2_f2(x))); }

// mask_pre_blend (ode_steps.py:89-106): m x + (1 - m)(t noise + (1 - t) orig), each product and
// sum rounded to bf16 as the reference's eager tensors are.  m2 / om2 = bf16 pairs of m, 1 - m.
__device__ __forceinline__ uint32_t pre_blend2(uint32_t x, uint32_t nz, uint32_t o, uint32_t m2, uint32_t om2,
                                               float t) {
  const uint32_t noised = add_bf2(scal_bf2(t, nz), scal_bf2(1.0f - t, o));
  return add_bf2(mul_bf2(m2, x), mul_bf2(om2, noised));
}

__device__ __forceinline__ uint4 ldg16(const void* p, int64_t off) {
  return __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p) + off));
}
// the state rewritten in place (xt, momentum) is read through L2, never the read-only path (the
// second pass reads back the momentum that the same thread stored in the first)
__device__ __forceinline__ uint4 ldcg16(const void* p, int64_t off) {
  return __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p) + off));
}
__device__ __forceinline__ void stg16(void* p, int64_t off, uint4 v) {
  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p) + off) = v;
}

// Velocity blend over active conditions (ode_steps.py:150-183), 8 channels; one condition
// means no blend (stream.py:1068-1069).
__device__ __forceinline__ uint4 blend8(const void* const* v, const float* const* w, int n, int64_t off, int t) {
  if (n <= 1) return ldg16(v[0], off);
  float num[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, den = 0.f;
  for (int i = 0; i < n && i < DEMON_ODE_MAX_COND; ++i) {
    const uint4 x = ldg16(v[i], off);
    const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
    const float wi = w[i] ? __ldg(w[i] + t) : 1.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      num[2 * j] = fmaf(bf16_lo(xw[j]), wi, num[2 * j]);
      num[2 * j + 1] = fmaf(bf16_hi(xw[j]), wi, num[2 * j + 1]);
    }
    den += wi;
  }
  const float dd = fmaxf(den, 1e-8f);
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = pack_bf16x2(__fdiv_rn(num[2 * j], dd), __fdiv_rn(num[2 * j + 1], dd));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void words(uint4 v, uint32_t (&w)[4]) {
  w[0] = v.x;
  w[1] = v.y;
  w[2] = v.z;
  w[3] = v.w;
}

// APG guidance weight w_t = bf16(g_t) - 1 of frame t
__device__ __forceinline__ float guide_w(const DemonOdeSlot& S, int t) {
  return rnd(curve(S.guidance, S.guidance_s, t)) - 1.0f;
}
// pair of bf16 (v, 1 - v) for v already bf16-exact, and its two broadcasts
__device__ __forceinline__ uint32_t pair_1m(float v) { return pack_bf16x2(v, rnd(1.0f - v)); }
__device__ __forceinline__ uint32_t lo_dup(uint32_t p) { return __byte_perm(p, 0u, 0x1010); }
__device__ __forceinline__ uint32_t hi_dup(uint32_t p) { return __byte_perm(p, 0u, 0x3232); }

// v summed over the four lanes of a warp that hold the same channels (l, l^8, l^16, l^24);
// every one of them gets the same bits
__device__ __forceinline__ float2 lane_sum4(float2 v) {
  v.x += __shfl_xor_sync(0xffffffffu, v.x, 8);
  v.y += __shfl_xor_sync(0xffffffffu, v.y, 8);
  v.x += __shfl_xor_sync(0xffffffffu, v.x, 16);
  v.y += __shfl_xor_sync(0xffffffffu, v.y, 16);
  return v;
}

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;\n" ::: "memory"); }

// Per-frame scalars of the second pass, computed once per CTA row (not once per lane).
struct OdeRow {
  float w, rho, vs, en;     // guidance - 1, cfg_rescale blend, velocity scale, ode-noise x t_next
  float sdc;                // sde_denoise_curve
  uint32_t mm, mmn, cc;     // bf16 pairs (v, 1 - v): mask now, mask at t_next, x0_target coefficient
  float lo, hi;             // DCW band coefficients of the frame's band (pix: lo = per-frame scale)
  float pad[2];
};
static_assert(sizeof(OdeRow) == 48, "OdeRow is three 16-byte words");

// Layout: a slot's T rows are split over a CL-CTA cluster and a CTA's rows are visited in passes
// of 32: thread = (row r in [0, 32), channel octet q in [0, 8)) with 16-byte accesses, so a warp
// holds the row pair (2k, 2k + 1) of the DCW wavelet step in lanes l and l ^ 8.  Both passes give
// a thread the same (row, octet) elements.
template <int CL>
__global__ void __launch_bounds__(kOdeThreads, kOdeMinBlocks)
    ode_step_kernel(const DemonOdeSlot* __restrict__ slots, int T, const __nv_bfloat16* __restrict__ gain,
                    int prepare_only) {
  __shared__ __align__(16) OdeShared sh;
  __shared__ __align__(16) DemonOdeSlot s_slot;
  extern __shared__ __align__(16) uint8_t ode_smem[];
  OdeRow* rows = reinterpret_cast<OdeRow*>(ode_smem);  // the CTA's frames

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int slot_id = blockIdx.x / CL;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rr = tid >> 3, c0 = (tid & 7) * 8;  // row in pass, first channel of the octet
  {  // the slot descriptor, once per CTA, into shared memory
    const uint64_t* src = reinterpret_cast<const uint64_t*>(slots + slot_id);
    uint64_t* dst = reinterpret_cast<uint64_t*>(&s_slot);
    for (int i = tid; i < (int)(sizeof(DemonOdeSlot) / 8); i += kOdeThreads) dst[i] = __ldg(src + i);
  }
  __syncthreads();
  const DemonOdeSlot& S = s_slot;
  const int flags = S.flags;
  const int Tc = ode_rows_per_cta(T, CL);
  const int t0 = crank * Tc, t1 = min(T, t0 + Tc);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);

  if (prepare_only) {  // decoder input at the current step: mask pre-blend at t_curr, times the gain
    if (!(flags & DEMON_ODE_DEC_OUT)) return;
    const bool dm = (flags & DEMON_ODE_DEC_MASK) != 0;
    for (int t = t0 + rr; t < t1; t += kOdeRowsPass) {
      const int64_t off = (int64_t)t * kOdeD + c0;
      uint32_t x[4], o[4], nz[4], g[4];
      words(ldg16(S.xt, off), x);
      if (dm) {
        words(ldg16(S.mask_orig, off), o);
        words(ldg16(S.mask_noise, off), nz);
        const float m = rnd(__ldg(S.mask + t) * S.mask_s);
        const uint32_t m2 = bf2_dup(m), om2 = bf2_dup(rnd(1.0f - m));
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = pre_blend2(x[j], nz[j], o[j], m2, om2, S.t_curr);
      }
      if (gain) {
        words(ldg16(gain, off), g);
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = mul_bf2(x[j], g[j]);
      }
      stg16(S.dec_out, off, make_uint4(x[0], x[1], x[2], x[3]));
    }
    return;
  }

  const float tc = S.t_curr, tn = S.t_next, dt = tn - tc;
  const bool cfg = (flags & DEMON_ODE_CFG) != 0;  // uniform over the slot's cluster
  const bool x0path = (flags & DEMON_ODE_X0PATH) != 0, mask = (flags & DEMON_ODE_MASK) != 0;
  const bool final_step = (flags & DEMON_ODE_FINAL) != 0;
  const bool sde_curve = (flags & DEMON_ODE_SDE_CURVE) != 0, sde_bare = (flags & DEMON_ODE_SDE_BARE) != 0;
  const bool onc_on = (flags & DEMON_ODE_ONC) != 0;
  const bool resc = (flags & DEMON_ODE_RESCALE) != 0;
  const bool vs_on = (flags & DEMON_ODE_VS) != 0;
  const bool x0t = (flags & DEMON_ODE_X0_TARGET) != 0;
  const bool dec_out = (flags & DEMON_ODE_DEC_OUT) != 0, dec_mask = (flags & DEMON_ODE_DEC_MASK) != 0;
  const bool need_noise = !final_step && (sde_curve || (sde_bare && !mask) || (onc_on && !sde_bare));
  const bool noise_in = need_noise && S.noise != nullptr;
  const bool need_mask_data = mask || dec_mask;
  const bool dcw_pix = (flags & DEMON_ODE_DCW_PIX) != 0;
  const bool dcw_band = (flags & (DEMON_ODE_DCW_LO | DEMON_ODE_DCW_HI)) != 0;

  // per-frame scalars of the CTA's rows (each rounded to bf16 where the reference's tensor is bf16)
  auto fill_rows = [&]() {
    for (int i = tid; i < t1 - t0; i += kOdeThreads) {
      const int t = t0 + i;
      OdeRow r;
      r.w = cfg ? guide_w(S, t) : 0.f;
      r.rho = resc ? rnd(curve(S.rescale, S.rescale_s, t)) : 0.f;
      r.vs = vs_on ? rnd(curve(S.vscale, S.vscale_s, t)) : 1.f;
      r.en = (onc_on ? rnd(curve(S.onc, S.onc_s, t)) : 0.f) * tn;
      r.sdc = sde_curve ? rnd(curve(S.sdc, S.sdc_s, t)) : 0.f;
      r.mm = pair_1m(mask ? rnd(__ldg(S.mask + t) * S.mask_s) : 1.f);
      r.mmn = pair_1m(dec_mask ? rnd(__ldg(S.mask + t) * S.mask_s_next) : 1.f);
      r.cc = pair_1m(x0t ? rnd(curve(S.x0_coef, S.x0_coef_s, t) * S.x0_coef_mul) : 0.f);
      if (dcw_pix) {
        r.lo = rnd(curve(S.dcw_lo, S.dcw_lo_s, t));
        r.hi = 0.f;
      } else {
        r.lo = (flags & DEMON_ODE_DCW_LO) ? curve(S.dcw_lo, S.dcw_lo_s, t >> 1) : 0.0f;
        r.hi = (flags & DEMON_ODE_DCW_HI) ? curve(S.dcw_hi, S.dcw_hi_s, t >> 1) : 0.0f;
      }
      r.pad[0] = r.pad[1] = 0.f;
      rows[i] = r;
    }
  };

  // ---------------- pass 1 (CFG slots): momentum and the per-channel moments ----------------
  if (cfg) {
    const bool mom_init = (flags & DEMON_ODE_MOM_INIT) != 0;
    const bool cache_neg = (flags & DEMON_ODE_CACHE_NEG) != 0;
    const bool w_scalar = S.guidance == nullptr;  // one guidance weight: 3 moments give all 8
    const int n_pos = S.n_pos, n_neg = S.n_neg;
    const int nmom = w_scalar ? 3 : 8;
    // 12 packed accumulators: w_scalar: [moment 0..2][channel pair 0..3] in one sweep; per-frame
    // guidance: [moment 0..7] of one channel pair per sweep, four sweeps (the later ones re-read
    // v_pos and the new momentum from L2)
    float2 acc[12];
    const int sweeps = w_scalar ? 1 : 4;
    for (int sweep = 0; sweep < sweeps; ++sweep) {
#pragma unroll
      for (int i = 0; i < 12; ++i) acc[i] = make_float2(0.f, 0.f);
      // one row: the new momentum (sweep 0; later sweeps re-read it as `umo`), then its moments
      auto row = [&](int t, int64_t off, uint4 uvp, uint4 uvn, uint4 umo) {
        uint32_t vp[4], r[4];
        words(uvp, vp);
        if (sweep == 0) {
          uint32_t vn[4], mo[4];
          words(uvn, vn);
          words(umo, mo);
          if (cache_neg) stg16(S.neg_cache, off, uvn);
          // r = bf16(bf16(v_pos - v_neg) + bf16(m_t * r_old))  (MomentumBuffer.update, ode_steps.py:276-300)
          const uint32_t mt2 = bf2_dup(rnd(curve(S.apg_mom, S.apg_mom_s, t)));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t d = sub_bf2(vp[j], vn[j]);
            r[j] = mom_init ? d : add_bf2(d, mul_bf2(mt2, mo[j]));
          }
          stg16(S.momentum, off, make_uint4(r[0], r[1], r[2], r[3]));
        } else {
          words(umo, r);
        }
        if (w_scalar) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 v2 = bf2_f2(vp[j]), r2 = bf2_f2(r[j]);
            acc[j] = fma_f2(r2, r2, acc[j]);           // sum r^2
            acc[4 + j] = fma_f2(v2, v2, acc[4 + j]);   // sum v^2
            acc[8 + j] = fma_f2(v2, r2, acc[8 + j]);   // sum v r
          }
        } else {
          const float2 w = f2_dup(guide_w(S, t)), w2 = mul_f2(w, w);
          const uint32_t vps = sweep == 0 ? vp[0] : sweep == 1 ? vp[1] : sweep == 2 ? vp[2] : vp[3];
          const uint32_t rs = sweep == 0 ? r[0] : sweep == 1 ? r[1] : sweep == 2 ? r[2] : r[3];
          const float2 v2 = bf2_f2(vps), r2 = bf2_f2(rs);
          const float2 pp = mul_f2(v2, v2), vr = mul_f2(v2, r2), qq = mul_f2(r2, r2);
          acc[0] = add_f2(acc[0], qq);
          acc[1] = add_f2(acc[1], pp);
          acc[2] = add_f2(acc[2], vr);
          acc[3] = fma_f2(w, pp, acc[3]);
          acc[4] = fma_f2(w2, pp, acc[4]);
          acc[5] = fma_f2(w, vr, acc[5]);
          acc[6] = fma_f2(w2, vr, acc[6]);
          acc[7] = fma_f2(w2, qq, acc[7]);
        }
      };
      // two rows per thread in flight: both rows' loads, then both rows' arithmetic
      for (int tA = t0 + rr; tA < t1; tA += 2 * kOdeRowsPass) {
        const int tB = tA + kOdeRowsPass;
        const bool hasB = tB < t1;
        const int tBc = hasB ? tB : tA;
        const int64_t offA = (int64_t)tA * kOdeD + c0, offB = (int64_t)tBc * kOdeD + c0;
        const uint4 vpA = blend8(S.v_pos, S.w_pos, n_pos, offA, tA);
        const uint4 vpB = blend8(S.v_pos, S.w_pos, n_pos, offB, tBc);
        const uint4 vnA = sweep == 0 ? blend8(S.v_neg, S.w_neg, n_neg, offA, tA) : z;
        const uint4 vnB = sweep == 0 ? blend8(S.v_neg, S.w_neg, n_neg, offB, tBc) : z;
        const bool no_mo = sweep == 0 && mom_init;  // later sweeps read the new momentum
        const uint4 moA = no_mo ? z : ldcg16(S.momentum, offA);
        const uint4 moB = no_mo ? z : ldcg16(S.momentum, offB);
        row(tA, offA, vpA, vnA, moA);
        if (hasB) row(tB, offB, vpB, vnB, moB);
      }
      // the four lanes of a channel octet, then one lane per octet writes the warp's partials
#pragma unroll
      for (int i = 0; i < 12; ++i) acc[i] = lane_sum4(acc[i]);
      if (lane < 8) {
        if (w_scalar) {
#pragma unroll
          for (int m = 0; m < 3; ++m) {
            float* g = &sh.gpart[warp][m][c0];
            *reinterpret_cast<float4*>(g) = make_float4(acc[4 * m].x, acc[4 * m].y, acc[4 * m + 1].x, acc[4 * m + 1].y);
            *reinterpret_cast<float4*>(g + 4) =
                make_float4(acc[4 * m + 2].x, acc[4 * m + 2].y, acc[4 * m + 3].x, acc[4 * m + 3].y);
          }
        } else {
#pragma unroll
          for (int m = 0; m < 8; ++m) *reinterpret_cast<float2*>(&sh.gpart[warp][m][c0 + 2 * sweep]) = acc[m];
        }
      }
    }
    __syncthreads();
    for (int e = tid; e < nmom * kOdeD; e += kOdeThreads) {
      const int i = e / kOdeD, cc = e % kOdeD;
      double s = 0.0;
#pragma unroll
      for (int wi = 0; wi < kOdeWarps; ++wi) s += (double)sh.gpart[wi][i][cc];
      sh.cta_part[i][cc] = s;
    }
    cluster_arrive();  // release: this CTA's partial moments
    fill_rows();       // overlaps the cluster barrier
    cluster_wait();    // acquire: every CTA's partials
    // the slot's moments: each summed over the CL CTAs in rank order (the distributed-shared-
    // memory loads of a sum are in flight together)
    for (int e = tid; e < nmom * kOdeD; e += kOdeThreads) {
      const int i = e / kOdeD, cc = e % kOdeD;
      double part[CL];
#pragma unroll
      for (int rnk = 0; rnk < CL; ++rnk) part[rnk] = *cluster.map_shared_rank(&sh.cta_part[i][cc], rnk);
      double s = 0.0;
#pragma unroll
      for (int rnk = 0; rnk < CL; ++rnk) s += part[rnk];
      sh.tot[i][cc] = s;
    }
    // this CTA has read its peers' partials; the matching wait at the end of the kernel keeps
    // every CTA resident until its peers have read its own
    cluster_arrive();
    __syncthreads();
    if (tid < kOdeD) {
      const double Srr = sh.tot[0][tid], P0 = sh.tot[1][tid], Srp = sh.tot[2][tid];
      double P1, P2, Q1, Q2, R2;
      if (w_scalar) {
        const double w = (double)(rnd(S.guidance_s) - 1.0f), w2 = w * w;
        P1 = w * P0, P2 = w2 * P0, Q1 = w * Srp, Q2 = w2 * Srp, R2 = w2 * Srr;
      } else {
        P1 = sh.tot[3][tid], P2 = sh.tot[4][tid], Q1 = sh.tot[5][tid], Q2 = sh.tot[6][tid], R2 = sh.tot[7][tid];
      }
      const double nr = sqrt(Srr);
      const double k = nr > 0.0 ? fmin(1.0, 2.5 / nr) : 1.0;  // norm_threshold 2.5 (ode_steps.py:334)
      const double nvp = sqrt(P0);
      const double nv = fmax(nvp, 1e-12);                      // F.normalize eps
      const double a = k * Srp / (nv * nv);
      const double g2 = P0 - 2.0 * a * P1 + a * a * P2 + 2.0 * k * Q1 - 2.0 * k * a * Q2 + k * k * R2;
      const double ng = fmax(sqrt(fmax(g2, 0.0)), 1e-12);
      sh.na[tid] = (float)(-a);
      sh.k[tid] = (float)k;
      sh.sm1[tid] = (float)(nvp / ng) - 1.0f;
    }
  } else {
    fill_rows();
  }
  __syncthreads();

  // ---------------- pass 2: guidance, integration, next decoder input ----------------------
  // Every lane of a warp runs the same iterations (the DCW wavelet step exchanges adjacent rows
  // between lanes): a lane past the CTA's rows computes row t1 - 1 and stores nothing.
  const int n_pos = S.n_pos;
  for (int tb = t0; tb < t1; tb += kOdeRowsPass) {
    const bool act = tb + rr < t1;
    const int t = act ? tb + rr : t1 - 1;
    const int64_t off = (int64_t)t * kOdeD + c0;
    // the row's global loads first (the rarely used x0_target and step noise where needed)
    const uint4 ux = ldcg16(S.xt, off);
    const uint4 uo = need_mask_data ? ldg16(S.mask_orig, off) : z;
    const uint4 unz = need_mask_data ? ldg16(S.mask_noise, off) : z;
    const uint4 usrc = sde_curve ? ldg16(S.source, off) : z;
    const uint4 ug = (dec_out && gain) ? ldg16(gain, off) : z;
    const uint4 uvp = blend8(S.v_pos, S.w_pos, n_pos, off, t);
    const uint4 ur = cfg ? ldcg16(S.momentum, off) : z;
    const OdeRow& R = rows[t - t0];
    uint32_t vt[4], x[4], o[4], nz[4];
    words(uvp, vt);
    words(ux, x);
    words(uo, o);
    words(unz, nz);
    if (cfg) {  // v_g = v + w (k r - a v), then cfg_rescale; rounded once (apg_forward + cfg_rescale)
      uint32_t r[4];
      words(ur, r);
      const float4 na0 = *reinterpret_cast<const float4*>(&sh.na[c0]), na1 = *reinterpret_cast<const float4*>(&sh.na[c0 + 4]);
      const float4 k0 = *reinterpret_cast<const float4*>(&sh.k[c0]), k1 = *reinterpret_cast<const float4*>(&sh.k[c0 + 4]);
      const float2 na[4] = {make_float2(na0.x, na0.y), make_float2(na0.z, na0.w), make_float2(na1.x, na1.y),
                            make_float2(na1.z, na1.w)};
      const float2 kk[4] = {make_float2(k0.x, k0.y), make_float2(k0.z, k0.w), make_float2(k1.x, k1.y),
                            make_float2(k1.z, k1.w)};
      const float2 w2 = f2_dup(R.w);
      float2 fac[4] = {f2_dup(1.0f), f2_dup(1.0f), f2_dup(1.0f), f2_dup(1.0f)};
      if (resc) {  // cfg_rescale as one factor on v_g: 1 + rho (sigma - 1)
        const float4 s0 = *reinterpret_cast<const float4*>(&sh.sm1[c0]), s1 = *reinterpret_cast<const float4*>(&sh.sm1[c0 + 4]);
        const float2 sm[4] = {make_float2(s0.x, s0.y), make_float2(s0.z, s0.w), make_float2(s1.x, s1.y),
                              make_float2(s1.z, s1.w)};
        const float2 rho2 = f2_dup(R.rho);
#pragma unroll
        for (int j = 0; j < 4; ++j) fac[j] = fma_f2(rho2, sm[j], fac[j]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 v2 = bf2_f2(vt[j]);
        const float2 inner = fma_f2(na[j], v2, mul_f2(kk[j], bf2_f2(r[j])));
        vt[j] = f2_bf2(mul_f2(fma_f2(w2, inner, v2), fac[j]));
      }
    }
    const uint32_t m2 = lo_dup(R.mm), om2 = hi_dup(R.mm);
    if (mask) {  // mask_pre_blend at t_curr
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = pre_blend2(x[j], nz[j], o[j], m2, om2, tc);
    }
    float2 eps[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    if (need_noise) {
      if (noise_in) {
        uint32_t ew[4];
        words(ldg16(S.noise, off), ew);
#pragma unroll
        for (int j = 0; j < 4; ++j) eps[j] = bf2_f2(ew[j]);
      } else {  // counters: the element pairs' indices in the slot, (t * 64 + c) / 2, per step
        const uint64_t key = noise_key(S.seed), cbase = (S.step << 36) + ((uint64_t)off >> 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) eps[j] = normal2(key, cbase + j);
      }
    }
    uint32_t xn[4];
    if (!x0path) {  // step_ode_euler (ode_steps.py:191-216): x + dt (v vs) + eps onc t_next
      const float2 vs2 = f2_dup(R.vs), dt2 = f2_dup(dt), en2 = f2_dup(R.en);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a1 = fma_f2(dt2, mul_f2(bf2_f2(vt[j]), vs2), bf2_f2(x[j]));
        xn[j] = f2_bf2(fma_f2(eps[j], en2, a1));
      }
    } else {
      uint32_t x0[4];
      const uint32_t vs2 = bf2_dup(R.vs);
#pragma unroll
      for (int j = 0; j < 4; ++j)  // x0_from_vel: bf16(x - bf16(bf16(v vs) t_curr))
        x0[j] = sub_bf2(x[j], scal_bf2(tc, mul_bf2(vt[j], vs2)));
      if (mask) {  // mask_post_blend_x0: bf16(bf16(m x0) + bf16((1 - m) orig))
#pragma unroll
        for (int j = 0; j < 4; ++j) x0[j] = add_bf2(mul_bf2(m2, x0[j]), mul_bf2(om2, o[j]));
      }
      if (x0t) {  // blend_x0_target / scalar x0 strength: bf16(bf16((1 - c) x0) + bf16(c target))
        uint32_t tg[4];
        words(ldg16(S.x0_target, off), tg);
        const uint32_t c2 = lo_dup(R.cc), oc2 = hi_dup(R.cc);
#pragma unroll
        for (int j = 0; j < 4; ++j) x0[j] = add_bf2(mul_bf2(oc2, x0[j]), mul_bf2(c2, tg[j]));
      }
      if (sde_curve) {  // step_sde_curve: sdc (t eps + (1-t) x0) + (1 - sdc)(t eps + (1-t) src)
        uint32_t src[4];
        words(usrc, src);
        const float2 tn2 = f2_dup(tn), otn2 = f2_dup(1.0f - tn), sdc2 = f2_dup(R.sdc), osdc2 = f2_dup(1.0f - R.sdc);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 te = mul_f2(tn2, eps[j]);
          const float2 full = fma_f2(otn2, bf2_f2(x0[j]), te);
          const float2 srcn = fma_f2(otn2, bf2_f2(src[j]), te);
          xn[j] = f2_bf2(fma_f2(sdc2, full, mul_f2(osdc2, srcn)));
        }
      } else if (final_step) {
#pragma unroll
        for (int j = 0; j < 4; ++j) xn[j] = x0[j];
      } else if (sde_bare) {  // step_sde_renoise: t noise + (1 - t) x0
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 nn = mask ? bf2_f2(nz[j]) : eps[j];
          xn[j] = f2_bf2(fma_f2(f2_dup(1.0f - tn), bf2_f2(x0[j]), mul_f2(f2_dup(tn), nn)));
        }
      } else {  // v_blended = bf16(bf16(x - x0) / t_curr), then the Euler step (stream.py:1269-1273)
        const float2 en2 = f2_dup(R.en);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 d = bf2_f2(sub_bf2(x[j], x0[j]));
          const float2 vb = bf2_f2(pack_bf16x2(__fdiv_rn(d.x, tc), __fdiv_rn(d.y, tc)));
          const float2 a1 = fma_f2(f2_dup(dt), vb, bf2_f2(x[j]));
          xn[j] = f2_bf2(fma_f2(eps[j], en2, a1));
        }
      }
    }
    if (dcw_pix || dcw_band) {
      // DCW (StreamPipeline._maybe_dcw, stream.py:1387-1405): denoised = bf16(x - bf16(vt t_curr))
      // from the mask-blended state and the guided velocity before velocity_scale
      uint32_t den[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) den[j] = sub_bf2(x[j], scal_bf2(tc, vt[j]));
      if (dcw_pix) {  // dcw_pix (dcw.py:164-174): bf16(x + bf16(s bf16(x - denoised)))
        const uint32_t s2 = bf2_dup(R.lo);
#pragma unroll
        for (int j = 0; j < 4; ++j) xn[j] = add_bf2(xn[j], mul_bf2(s2, sub_bf2(xn[j], den[j])));
      } else {
        // dcw_low / dcw_high / dcw_double (dcw.py:190-234) in fp32: a single-level haar DWT
        // along T of rows (2k, 2k+1), held by lanes l and l ^ 8 (a partner row past the CTA's
        // rows, the zero padding of an odd T, arrives as zero), xL += lo (xL - yL),
        // xH += hi (xH - yH), inverse DWT.  Each lane takes the difference as own - partner:
        // the odd row's high band is then the exact negative of the even row's, and
        // R (xL + xH) is the even row's output on the even lane and the odd row's on the odd lane
        const float2 lo = f2_dup(R.lo), hi = f2_dup(R.hi);
        const float2 Rt = f2_dup(0.70710678118654752f);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t px = __shfl_xor_sync(0xffffffffu, act ? xn[j] : 0u, 8);
          const uint32_t pd = __shfl_xor_sync(0xffffffffu, act ? den[j] : 0u, 8);
          const float2 mx = bf2_f2(xn[j]), md = bf2_f2(den[j]), ox = bf2_f2(px), od = bf2_f2(pd);
          float2 xl = mul_f2(add_f2(mx, ox), Rt), xh = mul_f2(sub_f2(mx, ox), Rt);
          const float2 yl = mul_f2(add_f2(md, od), Rt), yh = mul_f2(sub_f2(md, od), Rt);
          xl = add_f2(xl, mul_f2(lo, sub_f2(xl, yl)));
          xh = add_f2(xh, mul_f2(hi, sub_f2(xh, yh)));
          xn[j] = f2_bf2(mul_f2(add_f2(xl, xh), Rt));
        }
      }
    }
    if (act) stg16(S.xt, off, make_uint4(xn[0], xn[1], xn[2], xn[3]));
    if (dec_out && act) {
      uint32_t d[4] = {xn[0], xn[1], xn[2], xn[3]};
      if (dec_mask) {  // mask_pre_blend at t_next with the next step's strength
        const uint32_t mn2 = lo_dup(R.mmn), omn2 = hi_dup(R.mmn);
#pragma unroll
        for (int j = 0; j < 4; ++j) d[j] = pre_blend2(d[j], nz[j], o[j], mn2, omn2, tn);
      }
      if (gain) {
        uint32_t g[4];
        words(ug, g);
#pragma unroll
        for (int j = 0; j < 4; ++j) d[j] = mul_bf2(d[j], g[j]);
      }
      stg16(S.dec_out, off, make_uint4(d[0], d[1], d[2], d[3]));
    }
  }
  if (cfg) cluster_wait();  // peers have finished reading this CTA's partial moments
}

static size_t ode_row_smem(int64_t T, int cl) { return (size_t)ode_rows_per_cta((int)T, cl) * sizeof(OdeRow); }

static cudaLaunchConfig_t ode_launch_cfg(int n, int64_t T, int cl, cudaStream_t stream, cudaLaunchAttribute* attr) {
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n * cl));
  cfg.blockDim = dim3(kOdeThreads);
  cfg.dynamicSmemBytes = ode_row_smem(T, cl);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

template <int CL>
static int ode_prepare_kernel_attrs() {
  const int dyn_max = 227 * 1024 - (int)sizeof(OdeShared) - (int)sizeof(DemonOdeSlot) - 1024;
  DEMON_CUDA(cudaFuncSetAttribute(ode_step_kernel<CL>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_max));
  if (CL > 8) DEMON_CUDA(cudaFuncSetAttribute(ode_step_kernel<CL>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  return DEMON_OK;
}

template <int CL>
static int ode_resident_clusters(int64_t T, int* out) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = ode_launch_cfg(1, T, CL, nullptr, attr);
  DEMON_CUDA(cudaOccupancyMaxActiveClusters(out, ode_step_kernel<CL>, &cfg));
  return DEMON_OK;
}

// CTAs per slot cluster for n slots of T frames on the current device: 16 (a non-portable size)
// while the n * 16 CTAs need no more than one per SM, else 8 while all n clusters of 8 are
// resident at once, else 4 (half the CTAs, twice the rows each).  Resident-cluster counts come
// from the occupancy calculator, cached per device for the last T (T sets the row table's
// size).  Measured at T=1500: 8 slots 16.1 us in 16-CTA clusters against 19.1 in 8-CTA ones;
// 64 slots 45.9 us in 8-CTA clusters against 55.9 in 4-CTA ones.  Odd sizes between (9 or 12
// CTAs, fewer rows on the busiest SM on paper) measured no faster at 16 slots and slower at 32
// (34.0 us against 28.6), the hardware packing clusters into GPCs unevenly.
static int ode_cluster(int n, int64_t T, int* cl) {
  static std::atomic<uint64_t> attr_done{0};
  static int sms = 0;
  if (device_pending(attr_done)) {
    if (int rc = ode_prepare_kernel_attrs<4>()) return rc;
    if (int rc = ode_prepare_kernel_attrs<8>()) return rc;
    if (int rc = ode_prepare_kernel_attrs<16>()) return rc;
    int dev = 0;
    DEMON_CUDA(cudaGetDevice(&dev));
    DEMON_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    mark_device_done(attr_done);
  }
  // per device: T in the top 32 bits, then the resident 16- and 8-CTA cluster counts
  static std::atomic<uint64_t> occ_cache[64];
  int dev = 0;
  DEMON_CUDA(cudaGetDevice(&dev));
  const uint64_t cached = dev < 64 ? occ_cache[dev].load(std::memory_order_relaxed) : 0;
  int mc16 = 0, mc8 = 0;
  if (cached != 0 && (int64_t)(cached >> 32) == T) {
    mc16 = (int)((cached >> 16) & 0xFFFF);
    mc8 = (int)(cached & 0xFFFF);
  } else {
    if (int rc = ode_resident_clusters<16>(T, &mc16)) return rc;
    if (int rc = ode_resident_clusters<8>(T, &mc8)) return rc;
    mc16 = std::min(std::max(mc16, 0), 0xFFFF);
    mc8 = std::min(std::max(mc8, 0), 0xFFFF);
    if (dev < 64) occ_cache[dev].store(((uint64_t)T << 32) | ((uint64_t)mc16 << 16) | (uint64_t)mc8, std::memory_order_relaxed);
  }
  const int64_t nsm = sms > 0 ? sms : 148;
  *cl = ((int64_t)n * 16 <= nsm && n <= mc16) ? 16 : n <= mc8 ? 8 : 4;
  return DEMON_OK;
}

static int check_ode_shape(int32_t n, int64_t T, int64_t D) {
  DEMON_CHECK_ARG(n > 0, "ode: need n_slots > 0");
  DEMON_CHECK_ARG(D == kOdeD, "ode: latent width must be 64 (D=%lld)", (long long)D);
  DEMON_CHECK_ARG(T > 0 && T <= kOdeMaxT, "ode: 0 < T <= %d required (T=%lld)", kOdeMaxT, (long long)T);
  DEMON_CHECK_ARG(n <= 65535 / kOdeClusterMax, "ode: too many slots (%d)", n);
  return DEMON_OK;
}

int launch_ode(const DemonOdeSlot* slots, int32_t n, int64_t T, int64_t D, const void* gain, void* stream,
               int prepare_only) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(slots != nullptr, "ode: need a device slot table");
  if (int rc = check_ode_shape(n, T, D)) return rc;
  DEMON_CHECK_ARG(((uintptr_t)slots & 7) == 0, "ode: slot table must be 8-byte aligned");
  DEMON_CHECK_ARG(!gain || ((uintptr_t)gain & 15) == 0, "ode: gain must be 16-byte aligned");
  int cl = 0;
  if (int rc = ode_cluster(n, T, &cl)) return rc;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = ode_launch_cfg(n, T, cl, reinterpret_cast<cudaStream_t>(stream), attr);
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(gain);
  switch (cl) {
    case 16: DEMON_CUDA(cudaLaunchKernelEx(&cfg, ode_step_kernel<16>, slots, (int)T, g, prepare_only)); break;
    case 8: DEMON_CUDA(cudaLaunchKernelEx(&cfg, ode_step_kernel<8>, slots, (int)T, g, prepare_only)); break;
    default: DEMON_CUDA(cudaLaunchKernelEx(&cfg, ode_step_kernel<4>, slots, (int)T, g, prepare_only)); break;
  }
  return DEMON_OK;
}

int ode_cluster_size(int32_t n, int64_t T, int32_t* cluster) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(cluster != nullptr, "ode_cluster_size: null output");
  if (int rc = check_ode_shape(n, T, kOdeD)) return rc;
  int cl = 0;
  if (int rc = ode_cluster(n, T, &cl)) return rc;
  *cluster = cl;
  return DEMON_OK;
}

}  // namespace demon

extern "C" int demon_ode_step(const DemonOdeSlot* slots_dev, int32_t n_slots, int64_t T, int64_t D,
                              const void* gain, void* stream) {
  return demon::launch_ode(slots_dev, n_slots, T, D, gain, stream, 0);
}

extern "C" int demon_ode_prepare(const DemonOdeSlot* slots_dev, int32_t n_slots, int64_t T, int64_t D,
                                 const void* gain, void* stream) {
  return demon::launch_ode(slots_dev, n_slots, T, D, gain, stream, 1);
}

extern "C" int demon_ode_cluster_size(int32_t n_slots, int64_t T, int32_t* cluster) {
  return demon::ode_cluster_size(n_slots, T, cluster);
}
