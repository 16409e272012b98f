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
// slot is split over a 4- or 8-CTA thread-block cluster; each CTA keeps its rows of
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

// CTAs per slot cluster: 8, or 4 when 8 would need a second wave of CTAs (see launch_ode)
constexpr int kOdeClusterMax = 8;
constexpr int kOdeThreads = 256;
constexpr int kOdeD = 64;
constexpr int kOdeMaxT = 6400;

__device__ __forceinline__ float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Rows of a slot per CTA of its cluster: even, so the row pairs (2k, 2k+1) of the DCW wavelet
// step never straddle two CTAs.
__host__ __device__ __forceinline__ int ode_rows_per_cta(int T, int cluster) {
  return (T + 2 * cluster - 1) / (2 * cluster) * 2;
}

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
    // hardware log / sqrt / sin / cos approximations: the draws are rounded to bf16 (8
    // significant bits), far coarser than their error
    const float r = __fsqrt_rn(-2.0f * __logf(u1));
    float s, c;
    __sincosf(6.2831853071795865f * (u2 - 0.5f), &s, &c);  // a uniform angle in [-pi, pi)
    z[2 * i] = rnd(r * c);
    z[2 * i + 1] = rnd(r * s);
  }
}

struct OdeShared {
  union {
    float gpart[4][kOdeD][8];   // per row-group moment partials (fp32 over the group's rows)
    double tot[kOdeD][8];       // then: the slot's moments, summed over the cluster
  };
  double cta_part[kOdeD][8];    // this CTA's moments (read by the cluster)
  float k[kOdeD], a[kOdeD], sigma[kOdeD];
};

// ---------------------------------------------------------------------------
// Packed arithmetic on pairs of channels.  A bf16x2 product or sum of two bf16 operands
// (mul_bf2 / add_bf2 / sub_bf2) rounds the exact result once, which equals the reference's
// fp32 operation followed by rounding to bf16; an fp32 scalar times a bf16 tensor goes
// through fp32 (mul_f2) and is rounded afterwards (f2_bf2), as torch's opmath does.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t sub_bf2(uint32_t a, uint32_t b) { return add_bf2(a, b ^ 0x80008000u); }
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
__device__ __forceinline__ void stg16(void* p, int64_t off, uint4 v) {
  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p) + off) = v;
}
__device__ __forceinline__ void sts16(__nv_bfloat16* base, int64_t off, uint4 v) {
  st_shared_v4(smem_u32(base + off), v.x, v.y, v.z, v.w);
}
__device__ __forceinline__ uint4 lds16(const __nv_bfloat16* base, int64_t off) { return ld_shared_v4(smem_u32(base + off)); }

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

// Layout: a slot's T rows are split over a CL-CTA cluster.  Row passes: thread = (row r in
// [0, 32), channel octet q in [0, 8)) with 16-byte loads; the moment pass: thread = (channel c,
// row group g in [0, 4)) over the rows staged in shared memory.
template <int CL>
__global__ void __launch_bounds__(kOdeThreads, CL == 8 ? 3 : 2) ode_step_kernel(const DemonOdeSlot* __restrict__ slots, int T,
                                                               const __nv_bfloat16* __restrict__ gain,
                                                               int prepare_only) {
  extern __shared__ __align__(16) uint8_t ode_smem[];
  OdeShared& sh = *reinterpret_cast<OdeShared*>(ode_smem);
  __shared__ __align__(16) DemonOdeSlot s_slot;
  __nv_bfloat16* vp_s = reinterpret_cast<__nv_bfloat16*>(ode_smem + sizeof(OdeShared));
  const int Tc = ode_rows_per_cta(T, CL);
  __nv_bfloat16* r_s = vp_s + (size_t)Tc * kOdeD;
  float* w_s = reinterpret_cast<float*>(r_s + (size_t)Tc * kOdeD);  // guidance - 1 of the CTA's rows

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int slot_id = blockIdx.x / CL;
  const int tid = threadIdx.x;
  const int rr = tid >> 3, c0 = (tid & 7) * 8;  // row in pass, first channel of the octet
  {  // the slot descriptor, once per CTA, into shared memory
    const uint64_t* src = reinterpret_cast<const uint64_t*>(slots + slot_id);
    uint64_t* dst = reinterpret_cast<uint64_t*>(&s_slot);
    for (int i = tid; i < (int)(sizeof(DemonOdeSlot) / 8); i += kOdeThreads) dst[i] = __ldg(src + i);
  }
  __syncthreads();
  const DemonOdeSlot& S = s_slot;
  const int flags = S.flags;
  const int t0 = crank * Tc, t1 = min(T, t0 + Tc);

  if (prepare_only) {  // decoder input at the current step: mask pre-blend at t_curr, times the gain
    if (!(flags & DEMON_ODE_DEC_OUT)) return;
    const bool dm = (flags & DEMON_ODE_DEC_MASK) != 0;
    for (int t = t0 + rr; t < t1; t += 32) {
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

  const bool cfg = (flags & DEMON_ODE_CFG) != 0;
  if (cfg)  // the guidance curve of the CTA's rows, read by the moment pass and phase 2
    for (int i = tid; i < t1 - t0; i += kOdeThreads) w_s[i] = rnd(curve(S.guidance, S.guidance_s, t0 + i)) - 1.0f;
  const bool mom_init = (flags & DEMON_ODE_MOM_INIT) != 0;
  const bool cache_neg = (flags & DEMON_ODE_CACHE_NEG) != 0;
  const int n_pos = S.n_pos, n_neg = S.n_neg;

  // ---------------- phase 1: velocity assembly and momentum, staged in shared memory -------
  for (int tb = t0 + rr; tb < t1; tb += 64) {
    const int tA = tb, tB = tb + 32;  // two rows per thread in flight
    const bool hasB = tB < t1;
    const int64_t offA = (int64_t)tA * kOdeD + c0, offB = (int64_t)(hasB ? tB : tA) * kOdeD + c0;
    const uint4 vpA = blend8(S.v_pos, S.w_pos, n_pos, offA, tA);
    const uint4 vpB = blend8(S.v_pos, S.w_pos, n_pos, offB, hasB ? tB : tA);
    sts16(vp_s, (int64_t)(tA - t0) * kOdeD + c0, vpA);
    if (hasB) sts16(vp_s, (int64_t)(tB - t0) * kOdeD + c0, vpB);
    if (cfg) {
      const uint4 vnA = blend8(S.v_neg, S.w_neg, n_neg, offA, tA);
      const uint4 vnB = blend8(S.v_neg, S.w_neg, n_neg, offB, hasB ? tB : tA);
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      const uint4 moA = mom_init ? z : ldg16(S.momentum, offA);
      const uint4 moB = mom_init ? z : ldg16(S.momentum, offB);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h == 1 && !hasB) break;
        const int t = h ? tB : tA;
        const int64_t off = h ? offB : offA;
        uint32_t vp[4], vn[4], mo[4], r[4];
        words(h ? vpB : vpA, vp);
        words(h ? vnB : vnA, vn);
        words(h ? moB : moA, mo);
        if (cache_neg) stg16(S.neg_cache, off, h ? vnB : vnA);
        // r = bf16(bf16(v_pos - v_neg) + bf16(m_t * r_old))  (MomentumBuffer.update, ode_steps.py:276-300)
        const uint32_t mt2 = bf2_dup(rnd(curve(S.apg_mom, S.apg_mom_s, t)));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t d = sub_bf2(vp[j], vn[j]);
          r[j] = mom_init ? d : add_bf2(d, mul_bf2(mt2, mo[j]));
        }
        // the new momentum goes to global memory in phase 2 (from r_s): no global store is
        // pending when the cluster barriers (release semantics) run
        sts16(r_s, (int64_t)(t - t0) * kOdeD + c0, make_uint4(r[0], r[1], r[2], r[3]));
      }
    }
  }
  __syncthreads();

  // ---------------- moments (CFG slots): per channel over the CTA's rows -------------------
  if (cfg) {
    const int c = tid & 63, g = tid >> 6;
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f, m4 = 0.f, m5 = 0.f, m6 = 0.f, m7 = 0.f;
    const __nv_bfloat16* vpc = vp_s + c;
    const __nv_bfloat16* rc = r_s + c;
    for (int t = t0 + g; t < t1; t += 4) {
      const int64_t loc = (int64_t)(t - t0) * kOdeD;
      const float vp = __bfloat162float(vpc[loc]), r = __bfloat162float(rc[loc]);
      const float w = w_s[t - t0], w2 = w * w;
      const float pp = vp * vp, pr = vp * r, rr2 = r * r;
      m0 += rr2;
      m1 += pp;
      m2 += pr;
      m3 = fmaf(w, pp, m3);
      m4 = fmaf(w2, pp, m4);
      m5 = fmaf(w, pr, m5);
      m6 = fmaf(w2, pr, m6);
      m7 = fmaf(w2, rr2, m7);
    }
    float* gp = sh.gpart[g][c];
    gp[0] = m0;
    gp[1] = m1;
    gp[2] = m2;
    gp[3] = m3;
    gp[4] = m4;
    gp[5] = m5;
    gp[6] = m6;
    gp[7] = m7;
    __syncthreads();
    for (int e = tid; e < kOdeD * 8; e += kOdeThreads) {
      const int cc = e >> 3, i = e & 7;
      double acc = 0.0;
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) acc += (double)sh.gpart[gg][cc][i];
      sh.cta_part[cc][i] = acc;
    }
  }
  cluster.sync();  // partial moments of every CTA are visible cluster-wide
  if (cfg) {
    // the slot's 64 x 8 moments: two per thread, each summed over the CL CTAs in rank order
    // (the distributed-shared-memory loads of a sum are in flight together)
    for (int e = tid; e < kOdeD * 8; e += kOdeThreads) {
      const int cc = e >> 3, i = e & 7;
      double part[CL];
#pragma unroll
      for (int rnk = 0; rnk < CL; ++rnk) part[rnk] = *cluster.map_shared_rank(&sh.cta_part[cc][i], rnk);
      double acc = 0.0;
#pragma unroll
      for (int rnk = 0; rnk < CL; ++rnk) acc += part[rnk];
      sh.tot[cc][i] = acc;
    }
    __syncthreads();
    if (tid < kOdeD) {
      const double* tot = sh.tot[tid];
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

  // ---------------- phase 2: guidance, integration, next decoder input ----------------------
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
  const bool dcw_pix = (flags & DEMON_ODE_DCW_PIX) != 0;
  const bool dcw_band = (flags & (DEMON_ODE_DCW_LO | DEMON_ODE_DCW_HI)) != 0;

  // Every lane of a warp runs the same iterations (the DCW wavelet step exchanges adjacent rows
  // between lanes): a lane past the CTA's rows computes row t1 - 1 and stores nothing.
  for (int tb = t0; tb < t1; tb += 32) {
    const bool act = tb + rr < t1;
    const int t = act ? tb + rr : t1 - 1;
    const int64_t off = (int64_t)t * kOdeD + c0;
    const int64_t loc = (int64_t)(t - t0) * kOdeD + c0;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    // every global load of the row first
    const uint4 ux = ldg16(S.xt, off);
    const uint4 uo = need_mask_data ? ldg16(S.mask_orig, off) : z;
    const uint4 unz = need_mask_data ? ldg16(S.mask_noise, off) : z;
    const uint4 usrc = sde_curve ? ldg16(S.source, off) : z;
    const uint4 utg = (x0path && x0t) ? ldg16(S.x0_target, off) : z;
    const uint4 ueps = noise_in ? ldg16(S.noise, off) : z;
    const uint4 ug = (dec_out && gain) ? ldg16(gain, off) : z;
    uint32_t vt[4], x[4], o[4], nz[4];
    words(lds16(vp_s, loc), vt);
    words(ux, x);
    words(uo, o);
    words(unz, nz);
    if (cfg) {  // v_g = v + w (k r - a v), then cfg_rescale; rounded once (apg_forward + cfg_rescale)
      uint32_t r[4];
      const uint4 rv = lds16(r_s, loc);
      if (act) stg16(S.momentum, off, rv);
      words(rv, r);
      const float w = w_s[t - t0];
      const float rho = resc ? rnd(curve(S.rescale, S.rescale_s, t)) : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = c0 + 2 * j;
        const float2 kk = make_float2(sh.k[c], sh.k[c + 1]), aa = make_float2(sh.a[c], sh.a[c + 1]);
        const float2 v2 = bf2_f2(vt[j]), r2 = bf2_f2(r[j]);
        const float2 inner = fma_f2(make_float2(-aa.x, -aa.y), v2, mul_f2(kk, r2));
        float2 vg = fma_f2(f2_dup(w), inner, v2);
        if (resc) {
          const float2 ss = make_float2(sh.sigma[c], sh.sigma[c + 1]);
          vg = fma_f2(f2_dup(rho), mul_f2(vg, ss), mul_f2(f2_dup(1.0f - rho), vg));
        }
        vt[j] = f2_bf2(vg);
      }
    }
    const float m = mask ? rnd(__ldg(S.mask + t) * S.mask_s) : 1.f;
    const uint32_t m2 = bf2_dup(m), om2 = bf2_dup(rnd(1.0f - m));
    if (mask) {  // mask_pre_blend at t_curr
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = pre_blend2(x[j], nz[j], o[j], m2, om2, tc);
    }
    const float vs = vs_on ? rnd(curve(S.vscale, S.vscale_s, t)) : 1.f;
    const float onc = onc_on ? rnd(curve(S.onc, S.onc_s, t)) : 0.f;
    float2 eps[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    if (need_noise) {
      if (noise_in) {
        uint32_t ew[4];
        words(ueps, ew);
#pragma unroll
        for (int j = 0; j < 4; ++j) eps[j] = bf2_f2(ew[j]);
      } else {
        float z0[4], z1[4];
        philox_normal4(S.seed, S.step, (uint64_t)off >> 2, z0);
        philox_normal4(S.seed, S.step, ((uint64_t)off >> 2) + 1, z1);
        eps[0] = make_float2(z0[0], z0[1]);
        eps[1] = make_float2(z0[2], z0[3]);
        eps[2] = make_float2(z1[0], z1[1]);
        eps[3] = make_float2(z1[2], z1[3]);
      }
    }
    uint32_t xn[4];
    if (!x0path) {  // step_ode_euler (ode_steps.py:191-216): x + dt (v vs) + eps onc t_next
      const float en = onc * tn;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 v = mul_f2(bf2_f2(vt[j]), f2_dup(vs));
        const float2 a1 = fma_f2(f2_dup(dt), v, bf2_f2(x[j]));
        xn[j] = f2_bf2(fma_f2(eps[j], f2_dup(en), a1));
      }
    } else {
      uint32_t x0[4];
      const uint32_t vs2 = bf2_dup(vs);
#pragma unroll
      for (int j = 0; j < 4; ++j)  // x0_from_vel: bf16(x - bf16(bf16(v vs) t_curr))
        x0[j] = sub_bf2(x[j], scal_bf2(tc, mul_bf2(vt[j], vs2)));
      if (mask) {  // mask_post_blend_x0: bf16(bf16(m x0) + bf16((1 - m) orig))
#pragma unroll
        for (int j = 0; j < 4; ++j) x0[j] = add_bf2(mul_bf2(m2, x0[j]), mul_bf2(om2, o[j]));
      }
      if (x0t) {  // blend_x0_target / scalar x0 strength: bf16(bf16((1 - c) x0) + bf16(c target))
        uint32_t tg[4];
        words(utg, tg);
        const float c = rnd(curve(S.x0_coef, S.x0_coef_s, t) * S.x0_coef_mul);
        const uint32_t c2 = bf2_dup(c), oc2 = bf2_dup(rnd(1.0f - c));
#pragma unroll
        for (int j = 0; j < 4; ++j) x0[j] = add_bf2(mul_bf2(oc2, x0[j]), mul_bf2(c2, tg[j]));
      }
      if (sde_curve) {  // step_sde_curve: sdc (t eps + (1-t) x0) + (1 - sdc)(t eps + (1-t) src)
        uint32_t src[4];
        words(usrc, src);
        const float sdc = rnd(curve(S.sdc, S.sdc_s, t));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 te = mul_f2(f2_dup(tn), eps[j]);
          const float2 full = fma_f2(f2_dup(1.0f - tn), bf2_f2(x0[j]), te);
          const float2 srcn = fma_f2(f2_dup(1.0f - tn), bf2_f2(src[j]), te);
          xn[j] = f2_bf2(fma_f2(f2_dup(sdc), full, mul_f2(f2_dup(1.0f - sdc), srcn)));
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
        const float en = onc * tn;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 d = bf2_f2(sub_bf2(x[j], x0[j]));
          const float2 vb = bf2_f2(pack_bf16x2(__fdiv_rn(d.x, tc), __fdiv_rn(d.y, tc)));
          const float2 a1 = fma_f2(f2_dup(dt), vb, bf2_f2(x[j]));
          xn[j] = f2_bf2(fma_f2(eps[j], f2_dup(en), a1));
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
        const uint32_t s2 = bf2_dup(rnd(curve(S.dcw_lo, S.dcw_lo_s, t)));
#pragma unroll
        for (int j = 0; j < 4; ++j) xn[j] = add_bf2(xn[j], mul_bf2(s2, sub_bf2(xn[j], den[j])));
      } else {
        // dcw_low / dcw_high / dcw_double (dcw.py:190-234) in fp32: a single-level haar DWT
        // along T of rows (2k, 2k+1), held by lanes l and l ^ 8 (a missing partner row is the
        // zero padding of an odd T), xL += lo (xL - yL), xH += hi (xH - yH), inverse DWT; both
        // lanes of a pair compute the bands and keep their own output row
        const bool even = (t & 1) == 0, pact = tb + (rr ^ 1) < t1;
        const int k = t >> 1;
        const float2 lo = f2_dup((flags & DEMON_ODE_DCW_LO) ? curve(S.dcw_lo, S.dcw_lo_s, k) : 0.0f);
        const float2 hi = f2_dup((flags & DEMON_ODE_DCW_HI) ? curve(S.dcw_hi, S.dcw_hi_s, k) : 0.0f);
        const float2 R = f2_dup(0.70710678118654752f), zf = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t px = __shfl_xor_sync(0xffffffffu, xn[j], 8);
          const uint32_t pd = __shfl_xor_sync(0xffffffffu, den[j], 8);
          const float2 mx = bf2_f2(xn[j]), md = bf2_f2(den[j]);
          const float2 ox = pact ? bf2_f2(px) : zf, od = pact ? bf2_f2(pd) : zf;
          const float2 xa = even ? mx : ox, xb = even ? ox : mx, ya = even ? md : od, yb = even ? od : md;
          float2 xl = mul_f2(add_f2(xa, xb), R), xh = mul_f2(sub_f2(xa, xb), R);
          const float2 yl = mul_f2(add_f2(ya, yb), R), yh = mul_f2(sub_f2(ya, yb), R);
          xl = add_f2(xl, mul_f2(lo, sub_f2(xl, yl)));
          xh = add_f2(xh, mul_f2(hi, sub_f2(xh, yh)));
          xn[j] = f2_bf2(mul_f2(even ? add_f2(xl, xh) : sub_f2(xl, xh), R));
        }
      }
    }
    if (act) stg16(S.xt, off, make_uint4(xn[0], xn[1], xn[2], xn[3]));
    if (dec_out && act) {
      uint32_t d[4] = {xn[0], xn[1], xn[2], xn[3]};
      if (dec_mask) {  // mask_pre_blend at t_next with the next step's strength
        const float mn = rnd(__ldg(S.mask + t) * S.mask_s_next);
        const uint32_t mn2 = bf2_dup(mn), omn2 = bf2_dup(rnd(1.0f - mn));
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
}

int launch_ode(const DemonOdeSlot* slots, int32_t n, int64_t T, int64_t D, const void* gain, void* stream,
               int prepare_only) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(slots != nullptr && n > 0, "ode: need a device slot table and n_slots > 0");
  DEMON_CHECK_ARG(D == kOdeD, "ode: latent width must be 64 (D=%lld)", (long long)D);
  DEMON_CHECK_ARG(T > 0 && T <= kOdeMaxT, "ode: 0 < T <= %d required (T=%lld)", kOdeMaxT, (long long)T);
  DEMON_CHECK_ARG(n <= 65535 / kOdeClusterMax, "ode: too many slots (%d)", n);
  DEMON_CHECK_ARG(((uintptr_t)slots & 7) == 0, "ode: slot table must be 8-byte aligned");
  DEMON_CHECK_ARG(!gain || ((uintptr_t)gain & 15) == 0, "ode: gain must be 16-byte aligned");
  constexpr size_t kMaxSmem = 227 * 1024 - 1024;
  auto smem_for = [&](int cluster) {
    const int Tc = ode_rows_per_cta((int)T, cluster);
    return sizeof(OdeShared) + (size_t)Tc * kOdeD * 2 * sizeof(__nv_bfloat16) + (size_t)Tc * sizeof(float);
  };
  static std::atomic<uint64_t> attr_done{0};
  static int sms = 0;
  if (device_pending(attr_done)) {
    DEMON_CUDA(cudaFuncSetAttribute(ode_step_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem));
    DEMON_CUDA(cudaFuncSetAttribute(ode_step_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem));
    int dev = 0;
    DEMON_CUDA(cudaGetDevice(&dev));
    DEMON_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    mark_device_done(attr_done);
  }
  // 8-CTA clusters run 3 CTAs per SM; when that needs a second wave and 4-CTA clusters (2 per
  // SM, twice the rows each) fit in one, the 4-CTA form is faster (64 slots x T=1500: 81 -> 69 us)
  const int s = sms > 0 ? sms : 148;
  const int cl = ((int64_t)n * 8 > 3LL * s && (int64_t)n * 4 <= 2LL * s && smem_for(4) <= kMaxSmem) ? 4 : 8;
  const size_t smem = smem_for(cl);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n * cl));
  cfg.blockDim = dim3(kOdeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cl == 4)
    DEMON_CUDA(cudaLaunchKernelEx(&cfg, ode_step_kernel<4>, slots, (int)T,
                                  reinterpret_cast<const __nv_bfloat16*>(gain), prepare_only));
  else
    DEMON_CUDA(cudaLaunchKernelEx(&cfg, ode_step_kernel<8>, slots, (int)T,
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
