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
// slot is split over an 8-CTA thread-block cluster; each CTA keeps its rows of
// v_pos and of the new momentum in shared memory, accumulates per-channel
// moments, and the cluster exchanges the partial moments through distributed
// shared memory.  Every input byte is read from HBM once.
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

constexpr int kOdeCluster = 8;
constexpr int kOdeThreads = 256;
constexpr int kOdeD = 64;
constexpr int kOdeMaxT = 6400;

__device__ __forceinline__ float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void ld4(const void* p, int64_t off, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(p) + off);
  v[0] = bf16_lo(u.x);
  v[1] = bf16_hi(u.x);
  v[2] = bf16_lo(u.y);
  v[3] = bf16_hi(u.y);
}
__device__ __forceinline__ void st4(void* p, int64_t off, const float (&v)[4]) {
  uint2 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p) + off) = u;
}
__device__ __forceinline__ float curve(const float* c, float s, int t) { return c ? __ldg(c + t) : s; }

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) keyed by the slot seed;
// counter = (element group, step).  Box-Muller turns it into 4 normals.
__device__ __forceinline__ void philox_normal4(uint64_t seed, uint64_t step, uint64_t group, float (&z)[4]) {
  uint32_t c0 = (uint32_t)group, c1 = (uint32_t)(group >> 32), c2 = (uint32_t)step, c3 = (uint32_t)(step >> 32);
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  const uint32_t u[4] = {c0, c1, c2, c3};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float u1 = __uint2float_rn(u[2 * i] >> 8) * 5.9604644775390625e-08f + 2.98023223876953125e-08f;
    const float u2 = __uint2float_rn(u[2 * i + 1] >> 8) * 5.9604644775390625e-08f;
    const float r = sqrtf(-2.0f * logf(u1));
    float s, c;
    sincospif(2.0f * u2, &s, &c);
    z[2 * i] = rnd(r * c);
    z[2 * i + 1] = rnd(r * s);
  }
}

struct OdeShared {
  float warp_part[kOdeThreads / 32][16][32];  // per-warp moment partials
  double cta_part[kOdeD][8];                   // this CTA's moments (read by the cluster)
  float k[kOdeD], a[kOdeD], sigma[kOdeD];
};

// Velocity blend over active conditions (ode_steps.py:150-183); one condition
// means no blend (stream.py:1068-1069).
__device__ __forceinline__ void blend(const void* const* v, const float* const* w, int n, int64_t off, int t,
                                      float (&out)[4]) {
  if (n <= 1) {
    ld4(v[0], off, out);
    return;
  }
  float num[4] = {0.f, 0.f, 0.f, 0.f}, den = 0.f;
  for (int i = 0; i < n && i < DEMON_ODE_MAX_COND; ++i) {
    float x[4];
    ld4(v[i], off, x);
    const float wi = w[i] ? __ldg(w[i] + t) : 1.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) num[j] = fmaf(x[j], wi, num[j]);
    den += wi;
  }
  const float dd = fmaxf(den, 1e-8f);
#pragma unroll
  for (int j = 0; j < 4; ++j) out[j] = rnd(__fdiv_rn(num[j], dd));
}

// mask_pre_blend (ode_steps.py:89-106): m x + (1 - m)(t noise + (1 - t) orig),
// rounded after every operation as the reference's eager bf16 tensors are
// (the products and sums of bf16 operands are exact in fp32, so this is bit-exact).
__device__ __forceinline__ void pre_blend(const DemonOdeSlot& S, int64_t off, float m, float t, float (&x)[4]) {
  float o[4], nz[4];
  ld4(S.mask_orig, off, o);
  ld4(S.mask_noise, off, nz);
  const float om = rnd(1.0f - m), ot = 1.0f - t;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float noised = rnd(rnd(t * nz[j]) + rnd(ot * o[j]));
    x[j] = rnd(rnd(m * x[j]) + rnd(om * noised));
  }
}

// (1 - c) x + c y, op by op (mask_post_blend_x0 / blend_x0_target, ode_steps.py:109-142)
__device__ __forceinline__ float lerp_eager(float x, float c, float y) {
  return rnd(rnd(rnd(1.0f - c) * x) + rnd(c * y));
}

__device__ __forceinline__ void write_dec(const DemonOdeSlot& S, const __nv_bfloat16* gain, int64_t off, int t,
                                          bool masked, float m, float tn, float (&x)[4]) {
  float d[4] = {x[0], x[1], x[2], x[3]};
  if (masked) pre_blend(S, off, m, tn, d);
  if (gain) {
    float g[4];
    ld4(gain, off, g);
#pragma unroll
    for (int j = 0; j < 4; ++j) d[j] = d[j] * g[j];
  }
  st4(S.dec_out, off, d);
}

__device__ __forceinline__ void unpack4(uint2 u, float (&v)[4]) {
  v[0] = bf16_lo(u.x);
  v[1] = bf16_hi(u.x);
  v[2] = bf16_lo(u.y);
  v[3] = bf16_hi(u.y);
}
__device__ __forceinline__ uint2 ldraw(const void* p, int64_t off) {
  return *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(p) + off);
}

constexpr int kRB = 4;  // rows per batch and thread: all loads of a batch are issued before its compute

__global__ void __launch_bounds__(kOdeThreads, 2) ode_step_kernel(const DemonOdeSlot* __restrict__ slots, int T,
                                                               const __nv_bfloat16* __restrict__ gain,
                                                               int prepare_only) {
  extern __shared__ __align__(16) uint8_t ode_smem[];
  OdeShared& sh = *reinterpret_cast<OdeShared*>(ode_smem);
  __shared__ __align__(16) DemonOdeSlot s_slot;
  __nv_bfloat16* vp_s = reinterpret_cast<__nv_bfloat16*>(ode_smem + sizeof(OdeShared));
  const int Tc = (T + kOdeCluster - 1) / kOdeCluster;
  __nv_bfloat16* r_s = vp_s + (size_t)Tc * kOdeD;

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int slot_id = blockIdx.x / kOdeCluster;
  const int tid = threadIdx.x, cgp = tid & 15, rg = tid >> 4;
  // the slot descriptor, once per CTA, into shared memory
  {
    const uint64_t* src = reinterpret_cast<const uint64_t*>(slots + slot_id);
    uint64_t* dst = reinterpret_cast<uint64_t*>(&s_slot);
    for (int i = tid; i < (int)(sizeof(DemonOdeSlot) / 8); i += kOdeThreads) dst[i] = __ldg(src + i);
  }
  __syncthreads();
  const DemonOdeSlot& S = s_slot;
  const int flags = S.flags;
  const int t0 = crank * Tc, t1 = min(T, t0 + Tc);
  const int c0 = cgp * 4;

  if (prepare_only) {
    if (!(flags & DEMON_ODE_DEC_OUT)) return;
    for (int t = t0 + rg; t < t1; t += 16) {
      const int64_t off = (int64_t)t * kOdeD + c0;
      float x[4];
      ld4(S.xt, off, x);
      const float m = (flags & DEMON_ODE_DEC_MASK) ? rnd(__ldg(S.mask + t) * S.mask_s) : 0.f;
      write_dec(S, gain, off, t, (flags & DEMON_ODE_DEC_MASK) != 0, m, S.t_curr, x);
    }
    return;
  }

  const bool cfg = (flags & DEMON_ODE_CFG) != 0;
  const bool mom_init = (flags & DEMON_ODE_MOM_INIT) != 0;
  const bool cache_neg = (flags & DEMON_ODE_CACHE_NEG) != 0;
  const int n_pos = S.n_pos, n_neg = S.n_neg;

  // ---------------- phase 1: velocity assembly, momentum, moments ----------
  float mom[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) mom[i][j] = 0.f;

  for (int tb = t0 + rg; tb < t1; tb += 16 * kRB) {
    uint2 up[kRB], un[kRB], uo[kRB];
#pragma unroll
    for (int i = 0; i < kRB; ++i) {
      const int t = min(tb + 16 * i, t1 - 1);  // clamped: rows past t1 load a valid row, never stored
      const int64_t off = (int64_t)t * kOdeD + c0;
      up[i] = n_pos <= 1 ? ldraw(S.v_pos[0], off) : make_uint2(0u, 0u);
      if (cfg) {
        un[i] = n_neg <= 1 ? ldraw(S.v_neg[0], off) : make_uint2(0u, 0u);
        uo[i] = mom_init ? make_uint2(0u, 0u) : ldraw(S.momentum, off);
      }
    }
#pragma unroll
    for (int i = 0; i < kRB; ++i) {
      const int t = tb + 16 * i;
      if (t >= t1) break;
      const int64_t off = (int64_t)t * kOdeD + c0;
      const int64_t loc = (int64_t)(t - t0) * kOdeD + c0;
      float vp[4];
      if (n_pos <= 1) unpack4(up[i], vp);
      else blend(S.v_pos, S.w_pos, n_pos, off, t, vp);
      st4(vp_s, loc, vp);
      if (cfg) {
        float vn[4], ro[4], r[4];
        if (n_neg <= 1) unpack4(un[i], vn);
        else blend(S.v_neg, S.w_neg, n_neg, off, t, vn);
        if (cache_neg) st4(S.neg_cache, off, vn);
        unpack4(uo[i], ro);
        const float mt = rnd(curve(S.apg_mom, S.apg_mom_s, t));
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = mom_init ? rnd(vp[j] - vn[j]) : rnd(rnd(vp[j] - vn[j]) + rnd(mt * ro[j]));
        st4(S.momentum, off, r);
        st4(r_s, loc, r);
        const float w = rnd(curve(S.guidance, S.guidance_s, t)) - 1.0f;
        const float w2 = w * w;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float pp = vp[j] * vp[j], pr = vp[j] * r[j], rr = r[j] * r[j];
          mom[0][j] += rr;
          mom[1][j] += pp;
          mom[2][j] += pr;
          mom[3][j] = fmaf(w, pp, mom[3][j]);
          mom[4][j] = fmaf(w2, pp, mom[4][j]);
          mom[5][j] = fmaf(w, pr, mom[5][j]);
          mom[6][j] = fmaf(w2, pr, mom[6][j]);
          mom[7][j] = fmaf(w2, rr, mom[7][j]);
        }
      }
    }
  }

  // ---------------- cluster reduction of the moments (CFG slots only) -------
  if (cfg) {
    const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float o = __shfl_xor_sync(0xffffffffu, mom[i][j], 16);
        if (lane < 16) sh.warp_part[warp][lane][i * 4 + j] = mom[i][j] + o;
      }
    __syncthreads();
    for (int e = tid; e < 16 * 32; e += kOdeThreads) {
      const int g = e >> 5, q = e & 31;  // channel group, (moment, channel-in-group)
      double sacc = 0.0;
      for (int w = 0; w < kOdeThreads / 32; ++w) sacc += (double)sh.warp_part[w][g][q];
      sh.cta_part[g * 4 + (q & 3)][q >> 2] = sacc;
    }
  }
  cluster.sync();  // partial moments of every CTA are visible cluster-wide
  if (cfg) {
    if (tid < kOdeD) {
      double tot[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int rnk = 0; rnk < kOdeCluster; ++rnk) {
        const double* peer = cluster.map_shared_rank(&sh.cta_part[tid][0], rnk);
#pragma unroll
        for (int i = 0; i < 8; ++i) tot[i] += peer[i];
      }
      const double Srr = tot[0], P0 = tot[1], Srp = tot[2], P1 = tot[3], P2 = tot[4], Q1 = tot[5], Q2 = tot[6],
                   R2 = tot[7];
      const double nr = sqrt(Srr);
      const double k = nr > 0.0 ? fmin(1.0, 2.5 / nr) : 1.0;  // norm_threshold 2.5 (ode_steps.py:334)
      const double nvp = sqrt(P0);
      const double nv = fmax(nvp, 1e-12);                      // F.normalize eps
      const double a = k * Srp / (nv * nv);
      const double g2 = P0 - 2.0 * a * P1 + a * a * P2 + 2.0 * k * Q1 - 2.0 * k * a * Q2 + k * k * R2;
      const double ng = fmax(sqrt(fmax(g2, 0.0)), 1e-12);
      sh.k[tid] = (float)k;
      sh.a[tid] = (float)a;
      sh.sigma[tid] = (float)(nvp / ng);
    }
  }
  cluster.sync();  // peers finished reading our partials; constants visible in the CTA

  // ---------------- phase 2: guidance, integration, next decoder input -----
  const float tc = S.t_curr, tn = S.t_next, dt = tn - tc;
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
  float kc[4], ac[4], sc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    kc[j] = cfg ? sh.k[c0 + j] : 0.f;
    ac[j] = cfg ? sh.a[c0 + j] : 0.f;
    sc[j] = cfg ? sh.sigma[c0 + j] : 0.f;
  }

  for (int tb = t0 + rg; tb < t1; tb += 16 * kRB) {
    uint2 ux[kRB], uor[kRB], unz[kRB], usrc[kRB], utg[kRB], ueps[kRB], ug[kRB];
#pragma unroll
    for (int i = 0; i < kRB; ++i) {
      const int t = min(tb + 16 * i, t1 - 1);
      const int64_t off = (int64_t)t * kOdeD + c0;
      ux[i] = ldraw(S.xt, off);
      if (need_mask_data) {
        uor[i] = ldraw(S.mask_orig, off);
        unz[i] = ldraw(S.mask_noise, off);
      }
      if (sde_curve) usrc[i] = ldraw(S.source, off);
      if (x0path && x0t) utg[i] = ldraw(S.x0_target, off);
      if (noise_in) ueps[i] = ldraw(S.noise, off);
      if (dec_out && gain) ug[i] = ldraw(gain, off);
    }
#pragma unroll
    for (int i = 0; i < kRB; ++i) {
      const int t = tb + 16 * i;
      if (t >= t1) break;
      const int64_t off = (int64_t)t * kOdeD + c0;
      const int64_t loc = (int64_t)(t - t0) * kOdeD + c0;
      float vt[4], x[4], o[4], nz[4];
      ld4(vp_s, loc, vt);
      if (cfg) {
        float r[4];
        ld4(r_s, loc, r);
        const float w = rnd(curve(S.guidance, S.guidance_s, t)) - 1.0f;
        const float rho = resc ? rnd(curve(S.rescale, S.rescale_s, t)) : 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float vg = vt[j] + w * (kc[j] * r[j] - ac[j] * vt[j]);
          if (resc) vg = rho * (vg * sc[j]) + (1.0f - rho) * vg;
          vt[j] = rnd(vg);
        }
      }
      unpack4(ux[i], x);
      if (need_mask_data) {
        unpack4(uor[i], o);
        unpack4(unz[i], nz);
      }
      const float m = mask ? rnd(__ldg(S.mask + t) * S.mask_s) : 1.f;
      if (mask) {  // mask_pre_blend at t_curr (ode_steps.py:89-106), op by op
        const float om = rnd(1.0f - m), ot = 1.0f - tc;
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = rnd(rnd(m * x[j]) + rnd(om * rnd(rnd(tc * nz[j]) + rnd(ot * o[j]))));
      }
      const float vs = vs_on ? rnd(curve(S.vscale, S.vscale_s, t)) : 1.f;
      const float onc = onc_on ? rnd(curve(S.onc, S.onc_s, t)) : 0.f;
      float eps[4] = {0.f, 0.f, 0.f, 0.f};
      if (need_noise) {
        if (noise_in) unpack4(ueps[i], eps);
        else philox_normal4(S.seed, S.step, (uint64_t)off >> 2, eps);
      }
      float xn[4];
      if (!x0path) {
#pragma unroll
        for (int j = 0; j < 4; ++j) xn[j] = x[j] + dt * (vt[j] * vs) + eps[j] * onc * tn;
      } else {
        float x0[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) x0[j] = rnd(x[j] - rnd(rnd(vt[j] * vs) * tc));
        if (mask) {
          const float om = rnd(1.0f - m);
#pragma unroll
          for (int j = 0; j < 4; ++j) x0[j] = rnd(rnd(m * x0[j]) + rnd(om * o[j]));
        }
        if (x0t) {
          float tg[4];
          unpack4(utg[i], tg);
          const float c = rnd(curve(S.x0_coef, S.x0_coef_s, t) * S.x0_coef_mul);
#pragma unroll
          for (int j = 0; j < 4; ++j) x0[j] = lerp_eager(x0[j], c, tg[j]);
        }
        if (sde_curve) {
          float src[4];
          unpack4(usrc[i], src);
          const float sdc = rnd(curve(S.sdc, S.sdc_s, t));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float full = tn * eps[j] + (1.0f - tn) * x0[j];
            const float srcn = tn * eps[j] + (1.0f - tn) * src[j];
            xn[j] = sdc * full + (1.0f - sdc) * srcn;
          }
        } else if (final_step) {
#pragma unroll
          for (int j = 0; j < 4; ++j) xn[j] = x0[j];
        } else if (sde_bare) {
#pragma unroll
          for (int j = 0; j < 4; ++j) xn[j] = tn * (mask ? nz[j] : eps[j]) + (1.0f - tn) * x0[j];
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float vb = rnd(__fdiv_rn(rnd(x[j] - x0[j]), tc));
            xn[j] = x[j] + dt * vb + eps[j] * onc * tn;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) xn[j] = rnd(xn[j]);
      st4(S.xt, off, xn);
      if (dec_out) {
        float d[4] = {xn[0], xn[1], xn[2], xn[3]};
        if (dec_mask) {  // mask_pre_blend at t_next with the next step's strength
          const float mn = rnd(__ldg(S.mask + t) * S.mask_s_next);
          const float om = rnd(1.0f - mn), ot = 1.0f - tn;
#pragma unroll
          for (int j = 0; j < 4; ++j) d[j] = rnd(rnd(mn * d[j]) + rnd(om * rnd(rnd(tn * nz[j]) + rnd(ot * o[j]))));
        }
        if (gain) {
          float gg[4];
          unpack4(ug[i], gg);
#pragma unroll
          for (int j = 0; j < 4; ++j) d[j] = d[j] * gg[j];
        }
        st4(S.dec_out, off, d);
      }
    }
  }
}

int launch_ode(const DemonOdeSlot* slots, int32_t n, int64_t T, int64_t D, const void* gain, void* stream,
               int prepare_only) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(slots != nullptr && n > 0, "ode: need a device slot table and n_slots > 0");
  DEMON_CHECK_ARG(D == kOdeD, "ode: latent width must be 64 (D=%lld)", (long long)D);
  DEMON_CHECK_ARG(T > 0 && T <= kOdeMaxT, "ode: 0 < T <= %d required (T=%lld)", kOdeMaxT, (long long)T);
  DEMON_CHECK_ARG(n <= 65535 / kOdeCluster, "ode: too many slots (%d)", n);
  DEMON_CHECK_ARG(((uintptr_t)slots & 7) == 0, "ode: slot table must be 8-byte aligned");
  DEMON_CHECK_ARG(!gain || ((uintptr_t)gain & 7) == 0, "ode: gain must be 8-byte aligned");
  const int Tc = (int)((T + kOdeCluster - 1) / kOdeCluster);
  const size_t smem = sizeof(OdeShared) + (size_t)Tc * kOdeD * 2 * sizeof(__nv_bfloat16);
  static std::atomic<uint64_t> attr_done{0};
  if (device_pending(attr_done)) {
    DEMON_CUDA(cudaFuncSetAttribute(ode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - 1024));
    mark_device_done(attr_done);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n * kOdeCluster));
  cfg.blockDim = dim3(kOdeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kOdeCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DEMON_CUDA(cudaLaunchKernelEx(&cfg, ode_step_kernel, slots, (int)T,
                                reinterpret_cast<const __nv_bfloat16*>(gain), prepare_only));
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
